"""Build the C-ABI shared library ``libravel_b200.so`` for sm_100a with nvcc,
and the C++ host extension ``_ravel_host`` that the Python API calls it through.

The library is plain CUDA C++ (no PyTorch headers): ``include/ravel_b200.h``
is its interface.  The host extension (``csrc/host_ext.cpp``, g++ against
PyTorch's headers) links to it.  Both are built in-tree so that they travel
with the source tree to the GPU machine.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libravel_b200.so"
HOST_EXT = PKG / ("_ravel_host" + sysconfig.get_config_var("EXT_SUFFIX"))

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


def host_sources() -> list[Path]:
    return [CSRC / "host_ext.cpp", ROOT / "include" / "ravel_b200.h", LIB]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in sources())


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``csrc/host_ext.cpp`` into the ``_ravel_host`` extension module when it is stale."""
    if not force and HOST_EXT.exists() and all(p.stat().st_mtime <= HOST_EXT.stat().st_mtime
                                               for p in host_sources()):
        return HOST_EXT
    from torch.utils.cpp_extension import include_paths, library_paths
    cuda_inc = str(Path(os.environ.get("CUDA_HOME") or "/usr/local/cuda") / "include")
    torch_lib = library_paths()[0]
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
           "-DTORCH_EXTENSION_NAME=_ravel_host", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in include_paths()], f"-I{cuda_inc}", f"-I{sysconfig.get_paths()['include']}",
           str(CSRC / "host_ext.cpp"), "-o", str(HOST_EXT.with_suffix(".tmp")),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           f"-L{PKG}", "-lravel_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(HOST_EXT.with_suffix(".tmp"), HOST_EXT)
    return HOST_EXT


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile ``csrc/ravel_b200.cu`` into ``libravel_b200.so`` when it is stale, then the host extension."""
    if not force and not needs_build():
        build_host(force=force, verbose=verbose)
        return LIB
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-o", str(LIB), str(CSRC / "ravel_b200.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd[cmd.index(str(LIB))] = str(tmp)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    build_host(force=True, verbose=verbose)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
    print(LIB)
