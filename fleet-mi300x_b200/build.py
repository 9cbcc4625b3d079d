"""Build recipe for libmla_decode.so (sm_100a only).

Compiles every file under csrc/ with nvcc for `-gencode arch=compute_100a,code=sm_100a`
into one shared library next to this file, so the built library travels with the
source tree. nvcc cross-compiles without a GPU.

    python fleet-mi300x_b200/build.py            # build if stale
    python fleet-mi300x_b200/build.py --force -v # rebuild, print ptxas register/smem usage
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libmla_decode.so"
TRACE_LIB = PKG / "libmla_decode_trace.so"  # -DMLA_TRACE: per-tile clock stamps of the attention kernel

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the MLA decode library needs the CUDA toolkit to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stale(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    lib = TRACE_LIB if trace else LIB
    if not force and not stale(lib):
        return lib
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared",
        f"-I{INCLUDE}", f"-I{CSRC}",
        "-o", str(lib) + ".tmp",
        *[str(s) for s in sources()],
    ]
    if trace:  # the timeline array is shared by the kernels of several files: relocatable device code
        cmd[1:1] = ["-DMLA_TRACE", "-rdc=true"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed ({proc.returncode}) building {lib.name}")
    if verbose:
        sys.stdout.write(proc.stdout + proc.stderr)
    os.replace(str(lib) + ".tmp", lib)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build libmla_decode_trace.so with -DMLA_TRACE")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, trace=a.trace))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
