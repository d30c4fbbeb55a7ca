"""In-tree build of the two native libraries.

``libconvnd_b200.so`` is the torch-free C-ABI library (``include/convnd_b200.h``): the
tcgen05 kernels, the layout kernels and the generic CUDA-core kernels, compiled by nvcc
for sm_100a only. ``_C.so`` is the PyTorch shim that registers the
``torch_convnd::conv_nd`` / ``conv_nd_backward`` CUDA, AutocastCUDA and CPU kernels and
calls the C ABI. Both land next to this file, so they travel with the source tree.

The reference JIT-builds its addon with ``torch.utils.cpp_extension.load`` on first use
(``src/torch_convnd/_build.py:76-131``); this build is explicit and ahead of time instead,
and importing the package never compiles anything.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PACKAGE / "_lib"
CORE_LIBRARY = LIB_DIR / "libconvnd_b200.so"
SHIM_LIBRARY = LIB_DIR / "_C.so"

CORE_SOURCES = ["problem.cpp", "capi.cu", "fprop.cu", "tc_conv.cu", "pack.cu", "generic.cu"]
CORE_HEADERS = ["internal.h", "ptx.cuh", "fprop.cuh", "tc_conv.cuh", "pack.cuh", "generic.cuh"]
SHIM_SOURCES = ["shim.cpp"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(home) / "bin" / "nvcc")


def _digest(paths: list[Path], extra: str) -> str:
    hasher = hashlib.sha256(extra.encode())
    for path in paths:
        hasher.update(path.name.encode())
        hasher.update(path.read_bytes())
    return hasher.hexdigest()


def _up_to_date(target: Path, digest: str) -> bool:
    stamp = target.with_suffix(target.suffix + ".sha256")
    return target.exists() and stamp.exists() and stamp.read_text().strip() == digest


def _stamp(target: Path, digest: str) -> None:
    target.with_suffix(target.suffix + ".sha256").write_text(digest + "\n")


def _run(command: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(command), file=sys.stderr)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            "native build failed:\n" + " ".join(command) + "\n" + result.stdout + result.stderr
        )
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, file=sys.stderr)


def build_core(verbose: bool = False, force: bool = False) -> Path:
    """Compile the C-ABI library with nvcc for sm_100a (cross-compiles without a GPU)."""
    LIB_DIR.mkdir(exist_ok=True)
    inputs = [CSRC / name for name in CORE_SOURCES + CORE_HEADERS] + [INCLUDE / "convnd_b200.h"]
    flags = [
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-O2,-fvisibility=hidden",
        "-shared",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        "--expt-relaxed-constexpr",
    ]
    digest = _digest(inputs, " ".join(flags))
    if not force and _up_to_date(CORE_LIBRARY, digest):
        return CORE_LIBRARY
    sources = [str(CSRC / name) for name in CORE_SOURCES]
    temporary = CORE_LIBRARY.with_suffix(".so.tmp")
    _run([_nvcc(), *flags, *sources, "-o", str(temporary)], verbose)
    temporary.replace(CORE_LIBRARY)
    _stamp(CORE_LIBRARY, digest)
    return CORE_LIBRARY


def build_shim(verbose: bool = False, force: bool = False) -> Path:
    """Compile the PyTorch dispatcher shim against the installed torch."""
    import torch
    from torch.utils import cpp_extension

    LIB_DIR.mkdir(exist_ok=True)
    inputs = [CSRC / name for name in SHIM_SOURCES] + [INCLUDE / "convnd_b200.h"]
    includes = [f"-I{path}" for path in cpp_extension.include_paths()]
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = [
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-DTORCH_EXTENSION_NAME=_C",
        *includes,
        f"-I{cuda_home}/include",
        f"-I{INCLUDE}",
    ]
    libs = [
        *[f"-L{path}" for path in cpp_extension.library_paths()],
        f"-L{LIB_DIR}",
        "-lconvnd_b200",
        "-lc10",
        "-lc10_cuda",
        "-ltorch",
        "-ltorch_cpu",
        "-Wl,-rpath,$ORIGIN",
    ]
    digest = _digest(inputs, " ".join(flags + libs) + torch.__version__)
    if not force and _up_to_date(SHIM_LIBRARY, digest) and CORE_LIBRARY.exists():
        return SHIM_LIBRARY
    compiler = os.environ.get("CXX", "g++")
    sources = [str(CSRC / name) for name in SHIM_SOURCES]
    temporary = SHIM_LIBRARY.with_suffix(".so.tmp")
    _run([compiler, *flags, *sources, "-o", str(temporary), *libs], verbose)
    temporary.replace(SHIM_LIBRARY)
    _stamp(SHIM_LIBRARY, digest)
    return SHIM_LIBRARY


def build(verbose: bool = False, force: bool = False) -> None:
    """Build both libraries (core first: the shim links against it)."""
    build_core(verbose=verbose, force=force)
    build_shim(verbose=verbose, force=force)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv)
