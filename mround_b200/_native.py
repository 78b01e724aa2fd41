"""ctypes binding of ``libmround_b200.so`` (declared in ``include/mround_b200.h``).

This is the only place Python touches the native library.  Loading fails
loudly: if the shared object is missing, or lacks a symbol the header
declares, :class:`~mround_b200.exceptions.NativeLibraryError` is raised and
nothing falls back to another implementation.

Tensors cross the boundary as raw device pointers (``tensor.data_ptr()``) and
the caller's current CUDA stream; statuses come back as integers and are
turned into the package's exceptions by :func:`check`.
"""

from __future__ import annotations

import ctypes
import functools
import re
from pathlib import Path

from mround_b200.exceptions import DeviceError, NativeLibraryError, SchemeError

__all__ = ["HEADER", "LIB_PATH", "check", "declared_symbols", "lib"]

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmround_b200.so"
HEADER = HERE.parent / "include" / "mround_b200.h"

MR_OK = 0
MR_ERR_ARGUMENT = -1
MR_ERR_ALIGNMENT = -2

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_D = ctypes.c_double

# argument types of every exported entry point, in header order
_SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "mr_version": (_I, []),
    "mr_status_string": (ctypes.c_char_p, [_I]),
    "mr_device_check": (_I, []),
    "mr_last_cuda_error": (ctypes.c_char_p, []),
    "mr_fq_forward": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _I, _I, _P, _F, _P, _P, _P, _P, _P,
                           _P, _P]),
    "mr_ste_signsgd": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _P, _F, _F, _F, _F, _I,
                            _P, _P, _P, _P, _P, _P, _P]),
    "mr_ste_signsgd_codes": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _P, _F, _F, _F, _F,
                                  _P, _P, _P, _P]),
    "mr_dequant_split": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "mr_ste_signsgd_segments": (_I, [_P, _I, _I, _I, _F, _P]),
    "mr_pack_mlx": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _I, _I, _P, _F, _P, _P, _P, _P, _P]),
    "mr_loss_workspace_bytes": (ctypes.c_size_t, []),
    "mr_loss_outlier": (_I, [_P, _P, _I64, _I64, _I, _D, _F, _P, _P, _P, _P, _P]),
    "mr_loss_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "mr_loss_outlier_noalloc": (_I, [_P, _P, _I64, _I64, _I, _D, _F, _P, _P, _P, _P]),
    "mr_loss_hist_pass": (_I, [_P, _P, _I64, _I, _P, _P, _P]),
    "mr_loss_select_digit": (_I, [_P, _I64, _I, _P, _P, _P]),
    "mr_loss_apply": (_I, [_P, _P, _I64, _D, _P, _I, _P, _P, _P, _P]),
    "mr_deltaloss": (_I, [_P, _P, _I64, _I64, _I, _P, _I, _I, _P, _F, _P, _P]),
    "mr_scale_search": (_I, [_P, _I64, _I64, _I, _I, _P, _I, _P, _P, _P]),
    "mr_colsumsq_split": (_I, [_P, _P, _I64, _I64, _P, _P]),
    "mr_split_bf16": (_I, [_P, _I64, _P, _P, _P]),
    "mr_selftest_division": (_I, [_P, _P, _I64, _P, _P]),
    "mr_gemm": (_I, [_P, _P, _I64, _I, _P, _P, _I64, _I, _P, _I64, _P, _I, _I64, _I64, _I64,
                     _I, _P]),
    "mr_gemm_batched": (_I, [_P, _P, _I64, _I64, _I, _P, _P, _I64, _I64, _I, _P, _I64, _I64, _P,
                             _I, _I64, _I64, _I64, _I64, _I, _I, _I64, _P]),
    "mr_gemm_tile_n": (_I, [_I64, _I64, _I64, _I64, _I, _I, _I, _I]),
    "mr_gemm_tile_m": (_I, [_I64, _I64, _I64, _I64, _I, _I, _I, _I]),
    "mr_gemm_status": (_I, [_I]),
    "mr_gemm_rs": (_I, [_P, _P, _I64, _I, _P, _P, _I64, _I, _I64, _I64, _I64, _I, _P, _I64, _I64,
                        _P, _I, _P, ctypes.c_uint64, _P]),
    "mr_gemm_tf32": (_I, [_P, _I64, _I, _P, _I64, _I, _P, _I64, _P, _I, _I64, _I64, _I64, _P]),
    "mr_gemm_rs_tf32": (_I, [_P, _I64, _I, _P, _I64, _I, _I64, _I64, _I64, _P, _I64, _I64, _P,
                             _I, _P, ctypes.c_uint64, _P]),
    "mr_ipc_handle_bytes": (ctypes.c_size_t, []),
    "mr_ipc_export": (_I, [_P, _P, _P]),
    "mr_ipc_import": (_I, [_P, _I64, _P, _P]),
    "mr_ipc_close": (_I, [_P]),
    "mr_reduce_slots": (_I, [_P, _I64, _I64, _I, _P, ctypes.c_uint64, _P, _P]),
    "mr_peer_send": (_I, [_P, _P, _I64, _P, ctypes.c_uint64, _P]),
    "mr_peer_status": (_I, [_I]),
    "mr_rmsnorm_split": (_I, [_P, _P, _I64, _I, _F, _P, _P, _P, _P, _P]),
    "mr_rmsnorm_bwd_split": (_I, [_P, _P, _P, _P, _P, _I64, _I, _P, _P, _P, _P, _P]),
    "mr_rope_split": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "mr_rope_bwd_split": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "mr_heads_split": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "mr_swiglu_split": (_I, [_P, _I64, _I, _P, _P, _P, _P]),
    "mr_swiglu_bwd_split": (_I, [_P, _P, _I64, _I, _P, _P, _P, _P]),
    "mr_round_tf32": (_I, [_P, _I64, _P, _P]),
    "mr_ce_grad_split": (_I, [_P, _P, _I64, _I, _F, _P, _P, _P]),
    "mr_softmax_causal_split": (_I, [_P, _I64, _I, _F, _I, _P, _P, _P]),
    "mr_softmax_bwd_split": (_I, [_P, _P, _P, _I64, _I, _F, _I, _P, _P, _P]),
}


class K2Segment(ctypes.Structure):
    """``mr_k2_segment``: one matrix of an ``mr_ste_signsgd_segments`` launch."""

    _fields_ = [
        ("gq", _P), ("w_bf16", _P), ("v", _P), ("alpha", _P), ("beta", _P),
        ("init_scale", _P), ("rows", _I64), ("cols", _I64), ("bits", _I), ("lr", _F),
        ("coef_lo", _F), ("coef_hi", _F), ("wq_hi", _P), ("wq_lo", _P), ("wq_t32", _P),
        ("codes", _P), ("qscale", _P), ("qzp", _P),
    ]


def declared_symbols() -> list[str]:
    """Entry points the public header declares, in order."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(mr_[a-z0-9_]+)\s*\(", text)


@functools.cache
def lib() -> ctypes.CDLL:
    """Load the library once; refuse if it is absent or incomplete."""
    if not LIB_PATH.exists():
        raise NativeLibraryError(
            f"{LIB_PATH} is missing: build it with `python -m mround_b200.build` "
            "(there is no CPU fallback for the tuning path)"
        )
    try:
        handle = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise NativeLibraryError(f"could not load {LIB_PATH}: {exc}") from exc
    missing = []
    for name in declared_symbols():
        try:
            fn = getattr(handle, name)
        except AttributeError:
            missing.append(name)
            continue
        restype, argtypes = _SIGNATURES.get(name, (_I, None))
        fn.restype = restype
        if argtypes is not None:
            fn.argtypes = argtypes
    if missing:
        raise NativeLibraryError(f"{LIB_PATH.name} does not export {', '.join(missing)}")
    return handle


def check(status: int, what: str) -> None:
    """Raise the package exception matching a native status."""
    if status == MR_OK:
        return
    text = lib().mr_status_string(status).decode()
    if status in (MR_ERR_ARGUMENT, MR_ERR_ALIGNMENT):
        raise SchemeError(f"{what}: {text}")
    cuda = lib().mr_last_cuda_error().decode()
    raise DeviceError(f"{what}: {text}" + (f" ({cuda})" if cuda else ""))
