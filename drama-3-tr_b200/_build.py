"""Build recipe for libdm3.so (the C ABI in include/dm3.h), compiled with nvcc for sm_100a only."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
SOURCES = ["abi.cu", "gemm.cu", "gemv.cu", "gemv_tc.cu", "head.cu", "moe_decode.cu", "moe_prefill.cu"]
OUT = PKG_DIR / "libdm3.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles every kernel source into libdm3.so next to this file (skipped when up to date)."""
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "dm3.h"]
    if not force and OUT.exists() and OUT.stat().st_mtime > max(p.stat().st_mtime for p in deps):
        return OUT
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           f"-I{CSRC}", f"-I{ROOT / 'include'}", "-o", str(OUT), *map(str, srcs)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout + res.stderr)
    return OUT


if __name__ == "__main__":
    print(build(verbose=True, force=True))
