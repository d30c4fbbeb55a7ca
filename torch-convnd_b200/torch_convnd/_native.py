"""Loading of the prebuilt native libraries (no compilation at import or call time).

``_lib/_C.so`` registers the dispatcher kernels; it links ``_lib/libconvnd_b200.so``, the
torch-free C-ABI library that also serves non-PyTorch hosts. Both are built ahead of time
by ``torch_convnd._build`` (or the repository's ``__graft_entry__.build()``). A missing
library is an error, never a silent fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_LIB_DIR = Path(__file__).resolve().parent / "_lib"
SHIM_PATH = _LIB_DIR / "_C.so"
CORE_PATH = _LIB_DIR / "libconvnd_b200.so"

_LOCK = threading.Lock()
_LOADED = False
_CORE: ctypes.CDLL | None = None

FP32_MODES = {"3xtf32": 0, "tf32": 1, "ieee": 2}


def native_unavailable_reason() -> str | None:
    """Why the native libraries cannot be loaded, or None when they can."""
    missing = [path.name for path in (CORE_PATH, SHIM_PATH) if not path.exists()]
    if missing:
        return (
            "torch_convnd's native libraries are not built (missing "
            + ", ".join(missing)
            + "); run `python -m torch_convnd._build` or __graft_entry__.build()"
        )
    return None


def load_native() -> None:
    """Register the CUDA / AutocastCUDA / CPU kernels of the torch_convnd operators."""
    global _LOADED
    if _LOADED:
        return
    with _LOCK:
        if _LOADED:
            return
        reason = native_unavailable_reason()
        if reason is not None:
            raise RuntimeError(reason)
        from ._operators import ensure_native_definitions

        ensure_native_definitions()
        torch.ops.load_library(str(SHIM_PATH))
        _LOADED = True


def is_loaded() -> bool:
    return _LOADED


def core() -> ctypes.CDLL:
    """The C-ABI library, for the few host controls that are not operators."""
    global _CORE
    if _CORE is None:
        load_native()
        library = ctypes.CDLL(str(CORE_PATH))
        library.cnd_set_default_fp32_mode.argtypes = [ctypes.c_int32]
        library.cnd_set_default_fp32_mode.restype = ctypes.c_int
        library.cnd_launch_count.argtypes = [ctypes.c_int32]
        library.cnd_launch_count.restype = ctypes.c_int64
        library.cnd_device_status.argtypes = [ctypes.c_void_p]
        library.cnd_device_status.restype = ctypes.c_int
        library.cnd_debug_stall_test.argtypes = [ctypes.c_int32, ctypes.c_void_p]
        library.cnd_debug_stall_test.restype = ctypes.c_int
        library.cnd_set_kernel_timing.argtypes = [ctypes.c_int32]
        library.cnd_set_kernel_timing.restype = ctypes.c_int
        library.cnd_collect_kernel_timings.argtypes = [
            ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float), ctypes.c_int32]
        library.cnd_collect_kernel_timings.restype = ctypes.c_int
        library.cnd_last_error.restype = ctypes.c_char_p
        library.cnd_version.restype = ctypes.c_char_p
        _CORE = library
    return _CORE


def set_fp32_precision(mode: str) -> str:
    """Choose how float32 convolutions use the tensor cores; returns the previous mode.

    ``"3xtf32"`` (default): error-compensated split products well inside fp32's
    tolerance — three TF32 products (big/small parts) per multiply-add, or, where it
    halves the MMAs (input-gradient passes over 16 or more gradient channels), three
    products of bfloat16 hi/lo parts; the weight gradient always uses bfloat16 hi/lo
    parts. ``"tf32"``: one TF32 product for the forward and input gradient (the
    reference's bmm under ``allow_tf32=True``). ``"ieee"``: exact fp32 on the CUDA cores.
    """
    if mode not in FP32_MODES:
        raise ValueError(f"Invalid fp32 precision {mode!r}; expected one of {sorted(FP32_MODES)}")
    previous = core().cnd_set_default_fp32_mode(FP32_MODES[mode])
    return {value: key for key, value in FP32_MODES.items()}[previous]


def launch_count(reset: bool = False) -> int:
    """Kernels the library launched, from any thread, since the last reset."""
    return int(core().cnd_launch_count(1 if reset else 0))


def device_status(stream: torch.cuda.Stream | None = None) -> None:
    """Raise if a bounded in-kernel wait expired since the last check (clears the flag)."""
    handle = (stream or torch.cuda.current_stream()).cuda_stream
    status = core().cnd_device_status(ctypes.c_void_p(handle))
    if status != 0:
        raise RuntimeError(core().cnd_last_error().decode())


PASS_KINDS = {1: "forward", 2: "dgrad", 3: "wgrad", 4: "pack_activations", 5: "pack_weights",
              6: "reduce", 7: "generic"}


def set_kernel_timing(enable: bool) -> bool:
    """Bracket every library pass with CUDA events on its launching stream."""
    return bool(core().cnd_set_kernel_timing(1 if enable else 0))


def collect_kernel_timings(capacity: int = 1 << 16) -> list[tuple[str, float]]:
    """(pass kind, milliseconds) of the passes timed since the last collection."""
    kinds = (ctypes.c_int32 * capacity)()
    ms = (ctypes.c_float * capacity)()
    count = core().cnd_collect_kernel_timings(kinds, ms, capacity)
    return [(PASS_KINDS.get(kinds[i], str(kinds[i])), float(ms[i])) for i in range(count)]
