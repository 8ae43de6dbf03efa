"""In-tree build of the native libraries (run by ``__graft_entry__.build()``).

Produces, next to the package so they travel with the source tree:

* ``tonari_b200/_lib/libtonari_b200.so`` -- the C-ABI library
  (include/tonari_b200.h): sm_100a kernels + host scheduler, no PyTorch types;
* ``tonari_b200/_lib/libtonari_b200_torch.so`` -- the
  ``torch.ops.tonari_b200.neighbor_list`` custom op, linked against the
  former.

Compiler flags pin the target to B200: ``-gencode arch=compute_100a,code=sm_100a``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIB = PACKAGE / "_lib"
OBJ = PACKAGE / "_build"
CORE_LIBRARY = LIB / "libtonari_b200.so"
TORCH_LIBRARY = LIB / "libtonari_b200_torch.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["tnr_kernels.cu", "tnr_static.cu"]
HOST_SOURCES = ["tnr_api.cpp", "tnr_geometry.cpp"]


def _nvcc() -> str:
    candidate = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return candidate


def _run(command: list[str]) -> None:
    print("+", " ".join(command), flush=True)
    subprocess.run(command, check=True)


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(source.stat().st_mtime > stamp for source in sources)


def build_core(force: bool = False, debug: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "tonari_b200.h"]
    objects = []
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC)]
    if debug:
        common += ["-DTNR_DEBUG=1"]
    for name in CUDA_SOURCES + HOST_SOURCES:
        source = CSRC / name
        obj = OBJ / (name + ".o")
        objects.append(obj)
        if force or _stale(obj, [source, *headers]):
            _run([_nvcc(), *ARCH, "-lineinfo", *common, "-c", str(source), "-o", str(obj)])
    if force or _stale(CORE_LIBRARY, objects):
        _run([_nvcc(), *ARCH, "-shared", "-o", str(CORE_LIBRARY), *map(str, objects),
              "-Xlinker", "-soname=libtonari_b200.so"])
    return CORE_LIBRARY


def build_torch_op(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    source = CSRC / "tnr_torch.cpp"
    if not (force or _stale(TORCH_LIBRARY, [source, CORE_LIBRARY, ROOT / "include" / "tonari_b200.h"])):
        return TORCH_LIBRARY
    includes = cpp_extension.include_paths(device_type="cuda")
    libraries = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch.compiled_with_cxx11_abi())
    command = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=tonari_b200_torch",
        str(source), "-o", str(TORCH_LIBRARY), "-I", str(ROOT / "include"),
    ]
    for path in includes:
        command += ["-isystem", path]
    for path in libraries:
        command += ["-L", path]
    command += ["-L", str(LIB), "-ltonari_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu",
                "-ltorch_cuda", "-ltorch", "-Wl,-rpath,$ORIGIN"]
    _run(command)
    return TORCH_LIBRARY


def build(force: bool = False) -> None:
    build_core(force=force)
    build_torch_op(force=force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
