"""Builds libq38attn.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is compiled with -fmad=false: the reference (Rust) never fuses
a*b+c, so implicit contraction is disabled and every fused multiply-add in the
kernels is an explicit fmaf/ffma2 where the reference calls mul_add.
The CUDA runtime is linked statically so the library loads on hosts without a
GPU (symbol checks on CPU-only machines).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libq38attn.so"
SOURCES = ["q38attn.cu", "attn_decode.cu", "deltanet_decode.cu", "attn_decode_noalloc.cu",
           "attn_prefill.cu", "deltanet_prefill.cu", "q38_gguf.cpp", "proj.cu", "proj_mma.cu", "proj_planes.cu", "q38proj.cu", "q38_nccl.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nvcc_command(out: Path = LIB_PATH, extra: list[str] | None = None) -> list[str]:
    return [
        nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "static",
        "-I", str(PKG_DIR.parent / "include"),
        *(extra or []),
        "-o", str(out),
        *[str(CSRC / s) for s in SOURCES],
        "-ldl",
    ]


def needs_rebuild(out: Path = LIB_PATH) -> bool:
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    deps = list(CSRC.glob("*")) + [PKG_DIR.parent / "include" / "q38attn.h"]
    return any(p.stat().st_mtime > mtime for p in deps if p.is_file())


def build(force: bool = False, verbose: bool = True) -> Path:
    if force or needs_rebuild():
        cmd = nvcc_command()
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv)
