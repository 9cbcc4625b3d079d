"""Prefill hand-off on CPU: the reference's cache-file format, and the C ABI's argument
checks for mla_rows_to_pages (which return before any CUDA call)."""
import ctypes
import importlib

import numpy as np
import torch

from mla_testlib import O, fleet

native = importlib.import_module("fleet-mi300x_b200.native")
handoff = importlib.import_module("fleet-mi300x_b200.handoff")


def test_flat_cache_file_matches_reference_layout(tmp_path):
    g = torch.Generator().manual_seed(3)
    layers, max_pos, S = 3, 100, 37
    rows = [torch.randn(S, 576, generator=g).to(torch.bfloat16) for _ in range(layers)]
    flat = torch.zeros(layers, max_pos, 576, dtype=torch.bfloat16)
    for l in range(layers):
        flat[l, :S] = rows[l]
    path = tmp_path / "cache.bin"
    handoff.write_flat_cache(path, flat)
    want = O.flat_cache_file_bytes([r.float().numpy() for r in rows], max_pos)
    assert path.read_bytes() == want
    assert torch.equal(handoff.read_flat_cache(path, layers, max_pos), flat)


def test_scatter_oracle_places_rows_by_block_table():
    pages = np.zeros((6, 64, 576), np.float32)
    bt = np.array([[4, 1, 0], [2, 5, 3]])
    rows = np.arange(130 * 576, dtype=np.float32).reshape(130, 576)
    O.scatter_rows(pages, bt, rows, [0, 70, 130], first_pos=[0, 10])
    assert np.array_equal(pages[4, 0], rows[0]) and np.array_equal(pages[1, 5], rows[69])
    assert np.array_equal(pages[2, 10], rows[70]) and np.array_equal(pages[2, 63], rows[123])
    assert np.array_equal(pages[5, 0], rows[124])


def test_rows_to_pages_refuses_bad_arguments_without_launching():
    lib = native.load_library()
    r = native.new_rows()
    assert r.struct_size == ctypes.sizeof(native.MlaRowsToPages) and r.abi_version == native.ABI_VERSION
    fake = 1 << 20  # 16-byte aligned, never dereferenced: every check below fails first
    r.batch, r.total_rows, r.rows, r.rows_stride = 2, 10, fake, 576
    r.row_start, r.block_table, r.kv_cache, r.max_blocks, r.n_pages = fake, fake, fake, 4, 8
    bad = native.MlaRowsToPages.from_buffer_copy(r); bad.mode = 7
    assert lib.mla_rows_to_pages(ctypes.byref(bad), None) == -1
    bad = native.MlaRowsToPages.from_buffer_copy(r); bad.rows_stride = 575
    assert lib.mla_rows_to_pages(ctypes.byref(bad), None) == -1
    bad = native.MlaRowsToPages.from_buffer_copy(r); bad.rows_stride = 580
    assert lib.mla_rows_to_pages(ctypes.byref(bad), None) == -3
    bad = native.MlaRowsToPages.from_buffer_copy(r); bad.struct_size = 8
    assert lib.mla_rows_to_pages(ctypes.byref(bad), None) == -1
    bad = native.MlaRowsToPages.from_buffer_copy(r); bad.mode = native.ROWS_RAW  # no norm weight / tables
    assert lib.mla_rows_to_pages(ctypes.byref(bad), None) == -1
