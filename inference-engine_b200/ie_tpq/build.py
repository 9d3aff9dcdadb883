"""Build libie_tpq.so in-tree for sm_100a.

    python -m ie_tpq.build          (from inference-engine_b200/)

nvcc cross-compiles without a GPU.  The CUDA runtime is linked statically and
the driver API is reached through cudaGetDriverEntryPoint, so the library
loads on a machine without a driver (the symbol-export test relies on that).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # inference-engine_b200/
CSRC = ROOT / "csrc"
REPO = ROOT.parent
SOURCES = ["capi.cu", "quant.cu", "gemv.cu", "qgemm_sm100.cu", "comm.cu", "norm.cu",
           "rope_kv.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def command(out: Path) -> list[str]:
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
           "-shared", "-I", str(REPO / "include"), "-o", str(out)]
    cmd += [str(CSRC / s) for s in SOURCES]
    return cmd


def stale(out: Path) -> bool:
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [REPO / "include" / "ie_tpq.h"]
    return any(d.stat().st_mtime > mtime for d in deps if d.exists())


def build(force: bool = False, verbose: bool = True) -> Path:
    out = PKG / "libie_tpq.so"
    if not force and not stale(out):
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = command(tmp)
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv)
