"""Build libtriattn.so in-tree with nvcc for sm_100a (cross-compiles without a GPU).

    python -m boltz_mlx_b200.build            # or: python boltz_mlx_b200/build.py
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libtriattn.so"
SOURCES = ["capi.cu", "kernels_f32.cu", "kernels_tc.cu", "noalloc.cu", "peer.cu", "trimul.cu"]
HEADERS = ["sm100.cuh", "triattn_internal.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "shared",
    "-Xlinker", "-rpath,/usr/local/cuda/lib64",
    "--expt-relaxed-constexpr",
    "-lcublas",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "triattn.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-I", str(ROOT / "include"), "-I", str(CSRC),
           "-o", str(LIB), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr)
    return LIB


if __name__ == "__main__":
    extra = sys.argv[1:]
    print(build(force=True, verbose=True, extra=extra))
