"""Build the C-ABI shared library ``libravel_b200.so`` for sm_100a with nvcc.

The library is plain CUDA C++ (no PyTorch headers): ``include/ravel_b200.h``
is its interface.  It is built in-tree so that it travels with the source
tree to the GPU machine.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libravel_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcompiler", "-fvisibility=default",
]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME") or "/usr/local/cuda"
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "ravel_b200.h"]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in sources())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile ``csrc/ravel_b200.cu`` into ``libravel_b200.so`` when it is stale."""
    if not force and not needs_build():
        return LIB
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-o", str(LIB), str(CSRC / "ravel_b200.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd[cmd.index(str(LIB))] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
    print(LIB)
