"""Build ``libiris_b200.so`` in-tree with nvcc for sm_100a.

    python -m iris_b200.build            # from the iris-3b-metal_b200 directory

The library is one translation unit (``csrc/iris_b200.cu``); the output lands
next to this file so it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE.parent / "csrc"
INCLUDE = PACKAGE.parent.parent / "include"
LIBRARY = PACKAGE / "libiris_b200.so"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-shared",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is needed to build libiris_b200.so")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "iris_b200.h"]


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    tmp = LIBRARY.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", "-o", str(tmp), str(CSRC / "iris_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-4000:]}")
    if verbose:
        sys.stderr.write(result.stderr)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
