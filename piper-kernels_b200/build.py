"""Build the sm_100a shared library ``piper_kernels/_lib/libpiper_b200.so``.

Usage: ``python piper-kernels_b200/build.py [--force] [--verbose]``.

One translation unit (``csrc/piper_b200.cu``) compiled by nvcc for
``sm_100a`` only, with the C ABI of ``include/piper_b200.h``.  The CUDA
runtime is linked statically and the driver's tensor-map encoder is looked up
at run time, so the library has no dependency beyond the NVIDIA driver.
"""

from __future__ import annotations

import argparse
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
OUTPUT = PKG_ROOT / "piper_kernels" / "_lib" / "libpiper_b200.so"
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-shared",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "piper_b200.h"]


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and OUTPUT.exists():
        newest = max(p.stat().st_mtime for p in sources())
        if OUTPUT.stat().st_mtime >= newest:
            return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    cmd = [
        "nvcc", *NVCC_FLAGS,
        f"-I{INCLUDE}", f"-I{CSRC}",
        *(["-Xptxas", "-v"] if verbose else []),
        "-o", str(OUTPUT), str(CSRC / "piper_b200.cu"),
    ]
    subprocess.run(cmd, check=True)
    return OUTPUT


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose), file=sys.stderr)
