"""Build the reference's own native CPU implementation into oracle/_ref/.  TEST/BASELINE
INFRASTRUCTURE ONLY (the CPU baseline and the reference arm of bench.py).

Compiles src/torch_convnd/csrc/convnd.cpp of the reference checkout, where it lies, as a
CPU-only PyTorch operator library (no WITH_CUDA, so only its unfold_cpu / fold_cpu +
MKL bmm path and the CPU / AutocastCPU registrations are built). The only dependency is
the installed torch (headers and libraries), the same one the reference JIT-builds
against. No reference source is copied into this repository; the output goes to
oracle/_ref/ (git-ignored, but carried to the GPU box with the tree).

Usage: python oracle/build_ref.py REFERENCE_ROOT
(or set CONVND_REFERENCE_ROOT; without either, only an existing build is used).
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUTPUT = HERE / "_ref" / "libtorch_convnd_ref_cpu.so"


def build(reference_root: str | None = None, verbose: bool = False) -> Path | None:
    """Compile the reference's CPU operators from `reference_root` (default: the
    CONVND_REFERENCE_ROOT environment variable). Returns the library, or None when
    there is neither a source tree nor an earlier build."""
    import os

    reference_root = reference_root or os.environ.get("CONVND_REFERENCE_ROOT")
    source = (Path(reference_root) / "src" / "torch_convnd" / "csrc" / "convnd.cpp"
              if reference_root else None)
    if source is None or not source.exists():
        return OUTPUT if OUTPUT.exists() else None
    import torch
    from torch.utils import cpp_extension

    OUTPUT.parent.mkdir(exist_ok=True)
    stamp = OUTPUT.with_suffix(".stamp")
    key = f"{source.stat().st_mtime_ns}:{torch.__version__}"
    if OUTPUT.exists() and stamp.exists() and stamp.read_text() == key:
        return OUTPUT
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    command = [
        "g++", "-O3", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{p}" for p in cpp_extension.include_paths()],
        f"-I{source.parent}", str(source), "-o", str(OUTPUT),
        *[f"-L{p}" for p in cpp_extension.library_paths()],
        "-lc10", "-ltorch", "-ltorch_cpu", "-Wl,-rpath," + cpp_extension.library_paths()[0],
    ]
    if verbose:
        print(" ".join(command), file=sys.stderr)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError("reference CPU build failed:\n" + result.stderr[-4000:])
    stamp.write_text(key)
    return OUTPUT


def load(path: Path = OUTPUT):
    """Load the reference CPU operators into a process that has NOT imported the B200
    package (both register kernels for torch_convnd::conv_nd on the CPU key)."""
    import torch

    library = torch.library.Library("torch_convnd", "DEF")
    library.define(
        "conv_nd(Tensor input, Tensor weight, Tensor? bias, int[] stride, int[] padding, "
        "int[] dilation, int groups, int workspace_bytes) -> Tensor")
    library.define(
        "conv_nd_backward(Tensor grad_output, Tensor input, Tensor weight, int[] stride, "
        "int[] padding, int[] dilation, int groups, int workspace_bytes, "
        "bool[3] output_mask) -> (Tensor?, Tensor?, Tensor?)")
    torch.ops.load_library(str(path))
    return library


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
