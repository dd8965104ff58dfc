"""Build libdsv2.so in-tree for sm_100a (nvcc, no torch extension machinery).

Usage: python flash-deepseek-v2-lite_b200/build.py [--force] [--verbose]

The library is a plain C-ABI shared object (include/dsv2.h) with the CUDA runtime
linked statically, so it loads on machines without a GPU and carries no
dependency on torch.  Output: flash-deepseek-v2-lite_b200/dsv2/libdsv2.so.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT = PKG_ROOT / "dsv2" / "libdsv2.so"
HEADER = REPO_ROOT / "include" / "dsv2.h"

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
    "-cudart", "static",
]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [HEADER]


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _sources())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, str(CSRC / "dsv2_all.cu"), "-o", str(tmp)]
    if ptxas_verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    if verbose or ptxas_verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))
