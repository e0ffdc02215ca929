"""Build ``liblithe_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

The library is a plain shared object with ``extern "C"`` entry points (declared in
``include/lithe_b200.h``); it links the CUDA runtime statically and has no dependency
on PyTorch.  Usage: ``python -m lithe_b200.build [--verbose]``.
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
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "liblithe_b200.so"
SOURCES = ["host_common.cu", "decode_packed.cu", "sgmv_index.cu", "pack_raw.cu", "lora_gemm.cu", "selftest.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every CUDA source into ``lithe_b200/_lib/liblithe_b200.so``."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static",
           f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr",
           "-DLITHE_BUILDING_LIBRARY"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(s) for s in sources()] + ["-o", str(tmp)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}): {' '.join(cmd)}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true", help="print nvcc/ptxas output (-Xptxas -v)")
    ap.add_argument("--force", action="store_true", help="rebuild even if up to date")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
