"""Build libsimsd_b200.so (sm_100a) in-tree with nvcc.

    python simsd-release_b200/build.py            # build if any source is newer
    python simsd-release_b200/build.py --force

The library lands next to the Python package (kernels/libsimsd_b200.so), where
kernels/_lib.py loads it.  nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "kernels" / "libsimsd_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [REPO / "include" / "simsd_b200.h"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def build(force: bool = False, verbose: bool = False) -> Path:
    if OUT.exists() and not force:
        newest = max(p.stat().st_mtime for p in sources())
        if OUT.stat().st_mtime >= newest:
            return OUT
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-shared",
           "-Xptxas", "-v" if verbose else "-O3",
           "-I", str(REPO / "include"), "-o", str(OUT) + ".tmp", str(CSRC / "capi.cu")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed ({r.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
