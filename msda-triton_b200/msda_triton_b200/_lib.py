"""ctypes binding of ``libmsda_b200.so`` (C ABI declared in include/msda_b200.h).

The library is loaded lazily on first use. If it is missing or cannot be
loaded the op raises ``RuntimeError``: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(os.environ.get("MSDA_B200_LIB") or (Path(__file__).resolve().parent / "libmsda_b200.so"))

MSDA_OK = 0
MSDA_ERR_INVALID_ARGUMENT = 1
MSDA_ERR_UNSUPPORTED = 2
MSDA_ERR_CUDA = 3

MSDA_DTYPE_F32 = 0
MSDA_DTYPE_F16 = 1
MSDA_DTYPE_BF16 = 2

MSDA_BWD_FP32_ACCUM = 1
MSDA_BWD_FORCE_SCATTER = 2
MSDA_BWD_FORCE_COUNTED = 8
MSDA_BWD_DETERMINISTIC = 16
MSDA_BWD_GRAD_INPUT_NCHW = 32

# Every symbol include/msda_b200.h declares, with (restype, argtypes).
_VP = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
SIGNATURES = {
    "msda_version": (ctypes.c_char_p, []),
    "msda_last_error": (ctypes.c_char_p, []),
    "msda_forward": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _VP],
    ),
    "msda_backward_workspace_size": (
        ctypes.c_size_t, [_I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, ctypes.c_uint32]),
    "msda_backward": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t,
         _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, ctypes.c_uint32, _VP],
    ),
    # Fused layer prologue: reference points + offsets (level pixels) and
    # attention logits instead of locations and weights.
    "msda_forward_fused": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _VP],
    ),
    "msda_backward_fused": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t,
         _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, ctypes.c_uint32, _VP],
    ),
    # The backward for callers that cannot allocate: same as msda_backward
    # without the workspace arguments (fp32 scratch from a static device array).
    "msda_backward_noalloc": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP,
         _I64, _I64, _I64, _I32, _I32, _I32, _I32, _I32, _VP],
    ),
    # Sibling gathers on NHWC data: grid_sample and ROI-Align; the layout conversion.
    "msda_transpose": (ctypes.c_int, [_VP, _VP, _I64, _I64, _I64, _I32, _VP]),
    "msda_grid_sample_forward": (
        ctypes.c_int, [_VP, _VP, _VP, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32, _VP]),
    "msda_grid_sample_backward_workspace_size": (
        ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I64, _I64, _I32, ctypes.c_uint32]),
    "msda_grid_sample_backward": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_size_t, _I64, _I64, _I64, _I64, _I64, _I64,
         _I32, _I32, _I32, _I32, ctypes.c_uint32, _VP],
    ),
    "msda_roi_align_forward": (
        ctypes.c_int,
        [_VP, _VP, _VP, _I64, _I64, _I64, _I64, _I64, _I32, _I32, ctypes.c_float, _I32, _I32,
         _I32, _VP],
    ),
    "msda_roi_align_backward_workspace_size": (
        ctypes.c_size_t, [_I64, _I64, _I64, _I64, _I32, ctypes.c_uint32]),
    "msda_roi_align_backward": (
        ctypes.c_int,
        [_VP, _VP, _VP, _VP, ctypes.c_size_t, _I64, _I64, _I64, _I64, _I64, _I32, _I32,
         ctypes.c_float, _I32, _I32, _I32, ctypes.c_uint32, _VP],
    ),
}

# Size of the static scratch behind msda_backward_noalloc
# (MSDA_NOALLOC_SCRATCH_BYTES in include/msda_b200.h).
MSDA_NOALLOC_SCRATCH_BYTES = 16 << 20

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class MSDALibraryError(RuntimeError):
    """A call into libmsda_b200 returned a non-zero status."""

    def __init__(self, fn: str, code: int, message: str):
        super().__init__(f"{fn} failed with status {code}: {message}")
        self.code = code


def load() -> ctypes.CDLL:
    """Load the shared library (once) and declare its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"the msda_b200 CUDA library is not built ({LIB_PATH} is missing); "
                "run `python -m msda_triton_b200.build` or __graft_entry__.build()"
            )
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:  # pragma: no cover - depends on the host
            raise RuntimeError(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def check(fn_name: str, code: int) -> None:
    if code != MSDA_OK:
        msg = load().msda_last_error().decode(errors="replace")
        raise MSDALibraryError(fn_name, code, msg)


def version() -> str:
    return load().msda_version().decode()
