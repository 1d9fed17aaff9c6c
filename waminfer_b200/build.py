"""Builds libwamffn.so in-tree for sm_100a with nvcc (no torch headers needed).

    python -m waminfer_b200.build [--verbose]
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = [PACKAGE / "csrc" / "capi.cu"]
HEADERS = sorted((PACKAGE / "csrc").glob("*.cuh")) + [ROOT / "include" / "wamffn.h"]
OUTPUT = PACKAGE / "libwamffn.so"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
    "-cudart",
    "static",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not OUTPUT.exists():
        return True
    built = OUTPUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in SOURCES + HEADERS)


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not stale():
        return OUTPUT
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{ROOT / 'include'}", "-o", str(OUTPUT), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return OUTPUT


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
