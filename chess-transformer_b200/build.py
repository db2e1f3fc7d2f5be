"""Builds the CUDA library in-tree: csrc/fry_b200.cu -> libfry_b200.so, for sm_100a only.

    python chess-transformer_b200/build.py [--force]

The library statically links the CUDA runtime (nvcc's default) and finds cuTensorMapEncodeTiled through
cudaGetDriverEntryPoint, so it needs no libcuda at link time and builds on a machine without a GPU.
"""
import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIBRARY = HERE / "libfry_b200.so"
INCLUDE = HERE.parent / "include"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
         "-Xptxas", "-v"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libfry_b200.so")
    return found


def write_moves_header() -> None:
    sys.path.insert(0, str(HERE))
    try:
        from encoding import moves_header
    finally:
        sys.path.remove(str(HERE))
    path = CSRC / "moves.h"
    text = moves_header()
    if not path.exists() or path.read_text() != text:
        path.write_text(text)


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(path.stat().st_mtime > built for path in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    write_moves_header()
    if not force and not stale():
        return LIBRARY
    partial = LIBRARY.with_name(f"{LIBRARY.name}.{os.getpid()}.partial")
    command = [nvcc(), *FLAGS, "-I", str(INCLUDE), str(CSRC / "fry_b200.cu"), "-o", str(partial)]
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        partial.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-6000:]}")
    if verbose:
        print(result.stderr)
    os.replace(partial, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    arguments = parser.parse_args()
    print(build(arguments.force, verbose=True))
