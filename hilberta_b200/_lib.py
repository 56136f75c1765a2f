"""ctypes binding of the C ABI declared in ``include/hilberta_b200.h``.

The shared library is built in-tree (``hilberta_b200/lib/libhilberta_b200.so``,
see ``hilberta_b200.build``).  There is no fallback: every compute entry of this
package goes through these symbols, and loading fails loudly when the library
is missing.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libhilberta_b200.so"

HB_OK = 0
HB_ERR_ARG = -1
HB_ERR_ALIGN = -2
HB_ERR_SHARED = -3
HB_ERR_CROSS = -4
HB_ERR_CUDA = -5
HB_ERR_WORKSPACE = -6
HB_ERR_UNSUPPORTED = -7
HB_ERR_DEVICE = -8
HB_ERR_TMA = -9

HB_DEV_TIMEOUT = 1
HB_DEV_BAD_COUNT = 2
HB_DEV_BAD_BLOCK = 4
HB_DEV_PEER_TIMEOUT = 8
HB_DEV_SMEM_ALIGN = 16

HB_MAX_RANKS = 8
HB_IPC_HANDLE_BYTES = 64

# Every exported symbol of include/hilberta_b200.h (checked by the CPU tests).
EXPORTS = (
    "hb_status_string",
    "hb_version",
    "hb_hilbert_order",
    "hb_plan_dims",
    "hb_plan_build",
    "hb_validate_metadata",
    "hb_pair_metadata",
    "hb_dense_mask",
    "hb_fwd_workspace_bytes",
    "hb_fwd_workspace_bytes_for",
    "hb_paired_fwd",
    "hb_paired_fwd_noalloc",
    "hb_paired_fwd_raster",
    "hb_norm_rope_pack",
    "hb_paired_fwd_allgather",
    "hb_ipc_export",
    "hb_ipc_open",
    "hb_ipc_close",
    "hb_peer_copy",
    "hb_peer_scatter",
    "hb_adaln_residual",
    "hb_expand_kv128",
)


class PlanDims(ctypes.Structure):
    _fields_ = [
        ("image_tokens", ctypes.c_int64),
        ("image_blocks", ctypes.c_int64),
        ("total_blocks", ctypes.c_int64),
        ("text_blocks", ctypes.c_int64),
        ("shared_blocks", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("row_capacity", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_int64),
    ]


class RasterOrderC(ctypes.Structure):
    """hb_raster_order_t: raster-order token layout (text prefix + image squares)."""

    _fields_ = [("text_tokens", ctypes.c_int32), ("grid", ctypes.c_int32), ("block_origin", ctypes.c_void_p)]


class PeerOut(ctypes.Structure):
    """hb_peer_out_t: every rank's output view and flag words for the fused all-gather."""

    _fields_ = [
        ("n_ranks", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("epoch", ctypes.c_int32),
        ("timeout_ms", ctypes.c_int32),
        ("out", ctypes.c_void_p * HB_MAX_RANKS),
        ("flags", ctypes.c_void_p * HB_MAX_RANKS),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SIGS = {
    "hb_status_string": (ctypes.c_char_p, [_I]),
    "hb_version": (_I, []),
    "hb_hilbert_order": (_I, [_I, _P, _P]),
    "hb_plan_dims": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(PlanDims)]),
    "hb_plan_build": (_I, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "hb_validate_metadata": (_I, [_P, _I64, _I, _P, _I, _I, _I, _P, _P]),
    "hb_pair_metadata": (_I, [_P, _I64, _P, _I, _I, _I, _I, _P, _P, _I64, _P, _P, _P]),
    "hb_dense_mask": (_I, [_P, _I64, _P, _I, _I, _I, _I, _P, _P]),
    "hb_fwd_workspace_bytes": (ctypes.c_size_t, []),
    "hb_fwd_workspace_bytes_for": (ctypes.c_size_t, [_I, _I, _I, _I, _I]),
    "hb_paired_fwd": (
        _I,
        [_P, _P, _P, _P, ctypes.POINTER(ctypes.c_int64), _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, ctypes.c_float, _I, _P,
         _P, ctypes.c_size_t, _P],
    ),
    "hb_paired_fwd_raster": (
        _I,
        [_P, _P, _P, _P, ctypes.POINTER(ctypes.c_int64), _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, ctypes.c_float, _I,
         ctypes.POINTER(RasterOrderC), _P, ctypes.c_size_t, _P],
    ),
    "hb_norm_rope_pack": (
        _I,
        [_P, _I64, _I64, _P, _I64, _I64, _I, _I, _I, _I, _I, _P, _P, ctypes.c_float, _P, _P, _P, _P, _I64, _I64,
         _I64, _I, _P, _P],
    ),
    "hb_paired_fwd_allgather": (
        _I,
        [_P, _P, _P, ctypes.POINTER(ctypes.c_int64), _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, ctypes.c_float, _I,
         ctypes.POINTER(PeerOut), _P, ctypes.c_size_t, _P],
    ),
    "hb_ipc_export": (_I, [_P, _P, ctypes.POINTER(ctypes.c_uint64)]),
    "hb_ipc_open": (_I, [_P, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "hb_ipc_close": (_I, [_P, ctypes.c_uint64]),
    "hb_peer_copy": (_I, [_P, _P, ctypes.c_size_t, _P]),
    "hb_peer_scatter": (_I, [_P, ctypes.POINTER(ctypes.c_void_p), _I, ctypes.c_size_t, _P]),
    "hb_expand_kv128": (_I, [_P, _P, _I64, _I, _P, _I, _P, _P, _I64, _P, _P]),
    "hb_adaln_residual": (
        _I,
        [_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, ctypes.c_float, _I, _P],
    ),
    "hb_paired_fwd_noalloc": (
        _I,
        [_P, _P, _P, _P, ctypes.POINTER(ctypes.c_int64), _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, ctypes.c_float, _I, _P],
    ),
}

_lib = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib():
    """The loaded library (raises NativeLibraryMissing when it is not built)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("HILBERTA_B200_LIB", LIB_PATH))
        if not path.exists():
            raise NativeLibraryMissing(
                f"hilberta_b200 native library not found at {path}; build it with "
                "`python -c 'import hilberta_b200.build as b; b.build()'`"
            )
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_text(code: int) -> str:
    return lib().hb_status_string(int(code)).decode()


def check(code: int, what: str):
    if code != HB_OK:
        raise RuntimeError(f"{what} failed: {status_text(code)} (status {code})")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(device=None) -> torch.device:
    """The CUDA device the builder runs on; there is no CPU path."""
    if not torch.cuda.is_available():
        raise RuntimeError("hilberta_b200 requires a CUDA device (sm_100a); no CPU fallback exists")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.type != "cuda":
        raise ValueError("hilberta_b200 builds metadata on a CUDA device")
    return dev
