"""Build step for libqgemv_b200.so (the sm_100a kernels + C-ABI) -- run by
__graft_entry__.build() and, when the library is missing, by the package loader.
nvcc cross-compiles for sm_100a without a GPU."""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parents[1]          # local-ai-gpu-acceleration_b200/
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libqgemv_b200.so"
SOURCES = ["qg_gemv.cu", "qg_aux.cu", "qg_abi.cu", "qg_slice.cu", "qg_attn.cu", "qg_decode.cu",
           "qg_noalloc.cu", "qg_gemm_tc.cu", "qg_gguf.cu", "qg_gemv_batch.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_command(out: Path, extra: list[str] | None = None) -> list[str]:
    return [
        NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-rdc=true",
        "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
        "-shared", "-o", str(out), *[str(CSRC / s) for s in SOURCES],
        "-lnccl",
        *(extra or []),
    ]


def up_to_date(out: Path = LIB_PATH) -> bool:
    if not out.exists():
        return False
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(PKG_DIR.parent / "include" / "qgemv_b200.h")
    newest = max(p.stat().st_mtime for p in deps if p.exists())
    return out.stat().st_mtime >= newest


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = nvcc_command(tmp, extra)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        print(" ".join(cmd))
        print(res.stdout[-20000:])
        print(res.stderr[-20000:])
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {LIB_PATH.name}")
    tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys
    build(force=True, verbose=True, extra=sys.argv[1:])
