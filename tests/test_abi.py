"""The C-ABI library loads here (no GPU) and exports exactly what include/mla_decode.h declares.

No compute is launched: only host-side entry points (version, strings, params init,
workspace sizing, argument validation) are called.
"""
import ctypes
import importlib
import re
from pathlib import Path

import pytest

native = importlib.import_module("fleet-mi300x_b200.native")
ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "mla_decode.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mla_[a-z_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return native.load_library()


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/mla_decode.h but not exported"
    assert set(names) == set(native.EXPORTED)


def test_version_and_strings(lib):
    assert lib.mla_abi_version() == native.ABI_VERSION
    for code, name in native.STATUS.items():
        assert lib.mla_status_string(code).decode() == name
    assert b"block_table" in lib.mla_device_error_string(1)
    assert lib.mla_launches_per_step() == 3


def test_params_struct_layout(lib):
    p = native.new_params()
    assert p.struct_size == ctypes.sizeof(native.MlaDecodeParams)
    assert (p.heads, p.qk_nope, p.qk_rope, p.v_head, p.kv_lora, p.page_size) == (16, 128, 64, 128, 512, 64)
    assert p.abi_version == native.ABI_VERSION


def expected_workspace(batch: int, ctas: int) -> int:
    a = lambda x: (x + 255) // 256 * 256
    off = a((batch + 1) * 4)
    off = a(off + 16 + ctas * 32)  # the split plan: header (U, G) and one 32-byte entry per CTA
    off = a(off + batch * 16 * 576 * 2)
    off = a(off + (ctas + batch) * 16 * 2 * 4)
    off = a(off + (ctas + batch) * 16 * 512 * 4)
    return off


@pytest.mark.parametrize("batch,ctas", [(1, 148), (32, 148), (256, 7), (1000, 300)])
def test_workspace_size(lib, batch, ctas):
    p = native.new_params()
    p.batch, p.num_ctas = batch, ctas
    n = ctypes.c_uint64()
    assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == 0
    assert n.value == expected_workspace(batch, ctas)
    c, s = ctypes.c_int32(), ctypes.c_int32()
    assert lib.mla_plan_info(ctypes.byref(p), ctypes.byref(c), ctypes.byref(s)) == 0
    assert (c.value, s.value) == (ctas, ctas + batch)


def test_workspace_size_with_qc_hilo(lib):
    """MLA_FLAG_QC_HILO adds the low half of q_c, [batch][16][512] bf16, after the other regions."""
    a = lambda x: (x + 255) // 256 * 256
    for batch, ctas in ((1, 296), (256, 296)):
        p = native.new_params()
        p.batch, p.num_ctas, p.flags = batch, ctas, native.FLAG_QC_HILO | native.FLAG_P_HILO
        n = ctypes.c_uint64()
        assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == 0
        assert n.value == expected_workspace(batch, ctas) + a(batch * 16 * 512 * 2)


def test_validation_errors(lib):
    n = ctypes.c_uint64()
    p = native.new_params()
    p.batch, p.num_ctas = 4, 8
    p.kv_lora = 256  # the reference's launcher refuses kv_lora != 512 too (fleet_launch.hip:573-577)
    assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == -2
    p = native.new_params()
    p.batch, p.num_ctas = 0, 8
    assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == -1
    p.batch = native.MAX_BATCH + 1
    assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == -8
    p = native.new_params()
    p.batch, p.num_ctas = 1, 1
    p.struct_size = 8
    assert lib.mla_workspace_size(ctypes.byref(p), ctypes.byref(n)) == -1
    # null pointers are refused before anything touches a device
    p = native.new_params()
    p.batch, p.num_ctas = 1, 1
    for fn in (lib.mla_decode_step, lib.mla_prologue, lib.mla_attention, lib.mla_merge_uv):
        assert fn(ctypes.byref(p), None) == -1
    with pytest.raises(native.MlaError):
        native.check(-3, "x")


def test_static_step_limit_matches_header_and_refuses_before_launch(lib):
    text = (ROOT / "include" / "mla_decode.h").read_text()
    m = re.search(r"#define MLA_STATIC_SCRATCH_BYTES \((\d+)ull << (\d+)\)", text)
    assert m and int(m.group(1)) << int(m.group(2)) == native.STATIC_SCRATCH_BYTES
    # 558 requests fit at 148 CTAs, 559 do not; at the default 296 CTAs of a B200, 463 fit and
    # 464 do not; the refusal comes before any CUDA call
    assert expected_workspace(558, 148) <= native.STATIC_SCRATCH_BYTES < expected_workspace(559, 148)
    assert expected_workspace(463, 296) <= native.STATIC_SCRATCH_BYTES < expected_workspace(464, 296)
    for batch, ctas in ((464, 296), (600, 148)):
        p = native.new_params()
        p.batch, p.num_ctas = batch, ctas
        assert lib.mla_decode_step_static(ctypes.byref(p), None) == -8  # MLA_E_LIMIT
    p = native.new_params()
    p.batch, p.num_ctas = 559, 148
    assert lib.mla_decode_step_static(ctypes.byref(p), None) == -8  # MLA_E_LIMIT
