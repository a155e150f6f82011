"""ctypes loader for the in-tree CUDA library ``_tropical_b200.so``.

The library is the only compute path: there is no CPU fallback.  If the
library is missing this module raises at first use with the build command.
Argument and return types are declared for every export of
``include/tropical_b200.h`` so that ctypes never guesses (the reference binding,
``cuda/maxplus_binding.py:20-34``, declared none).
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_int = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_f = ctypes.c_float
_c_p = ctypes.c_void_p
_c_bool = ctypes.c_bool

# name -> (restype, [argtypes])
SIGNATURES: dict[str, tuple] = {
    "tp_status_string": (ctypes.c_char_p, [_c_int]),
    "tp_abi_version": (_c_int, []),
    "tp_set_pointer_checks": (_c_int, [_c_int]),
    "tp_maxplus_fwd": (
        _c_int,
        [_c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p,
         _c_i64, _c_p],
    ),
    "tp_maxplus_fwd_strided": (
        _c_int,
        [_c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_f, _c_p],
    ),
    "tp_maxplus_fwd_lfdual": (
        _c_int,
        [_c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64,
         _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_maxplus_fwd_sharded": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_int, _c_i64,
         _c_i64, _c_p],
    ),
    "tp_maxplus_lse_fwd_strided": (
        _c_int,
        [_c_int, _c_f, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_f, _c_p],
    ),
    "tp_maxplus_bwd_argmax_strided": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
         _c_p, _c_f, _c_p],
    ),
    "tp_maxplus_bwd_smooth_workspace_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "tp_maxplus_bwd_smooth": (
        _c_int,
        [_c_int, _c_f, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p, _c_i64, _c_p],
    ),
    "tp_maxplus_bwd_smooth_ref": (
        _c_int,
        [_c_int, _c_f, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p, _c_p, _c_i64, _c_p],
    ),
    "tp_scan_fwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_scan_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p, _c_p],
    ),
    "tp_scan_bwd_noalloc": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p],
    ),
    "tp_scan_chunked_workspace_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_int]),
    "tp_scan_chunk_length": (_c_int, [_c_i64, _c_i64, _c_i64]),
    "tp_scan_fwd_chunked": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_int, _c_p, _c_i64,
         _c_p],
    ),
    "tp_scan_bwd_chunked": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_int, _c_p, _c_i64, _c_p],
    ),
    "tp_convert_bf16_to_f32": (_c_int, [_c_i64, _c_p, _c_p, _c_p]),
    "tp_probe_addmax": (_c_int, [_c_int, _c_i64, _c_i64, _c_i64, _c_p, _c_p]),
    "maxplus_forward_cuda": (None, [_c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_bool]),
    "maxplus_backward_cuda": (
        None, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_f, _c_int, _c_int, _c_int]),
    "maxplus_matmul_cuda": (None, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int]),
    "tp_set_argmax_tma_min_terms": (_c_i64, [_c_i64]),
    "tp_set_stream_k": (_c_int, [_c_int]),
    "tp_set_smooth_fused": (_c_int, [_c_int]),
    "tp_esn_gru_fwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p,
         _c_p],
    ),
    "tp_split_tf32": (_c_int, [_c_p, _c_i64, _c_p, _c_p, _c_p]),
    "tp_split_tf32_cat": (_c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_int, _c_int, _c_p]),
    "tp_esn_gru_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64,
         _c_p, _c_i64, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_esn_leaky_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_esn_leaky_fwd": (
        _c_int, [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p]),
    "tp_esn_gru_fwd_seg": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p,
         _c_i64, _c_p, _c_i64, _c_p, _c_p],
    ),
    "tp_esn_leaky_fwd_seg": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_p]),
    "tp_memcpy2d_async": (_c_int, [_c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p]),
    "tp_tsrn_attention_prologue": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p,
         _c_f, _c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_tsrn_attention_workspace_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64]),
    "tp_tsrn_attention_fwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_int, _c_int,
         _c_p, _c_p, _c_i64, _c_p],
    ),
    "tp_layernorm_bwd_workspace_bytes": (_c_i64, [_c_i64, _c_i64]),
    "tp_layernorm_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_p, _c_p, _c_p, _c_f, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p],
    ),
    "tp_tsrn_attention_prologue_bwd_workspace_bytes": (_c_i64, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "tp_tsrn_attention_prologue_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_f, _c_p,
         _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p],
    ),
    "tp_tsrn_attention_fwd_lists": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_int, _c_int,
         _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p],
    ),
    "tp_tsrn_attention_bwd_rows": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p, _c_p],
    ),
    "tp_tsrn_attention_bwd_group": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_tsrn_attention_bwd_keys": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
         _c_p, _c_p, _c_p],
    ),
    "tp_tsrn_attention_set_path": (_c_int, [_c_int, _c_p]),
    "tp_maslov_softmax_fwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
         _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p],
    ),
    "tp_maslov_softmax_bwd": (
        _c_int,
        [_c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
         _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p],
    ),
    "tp_last_error": (_c_int, []),
    "tp_device_error": (_c_int, [_c_int]),
    "tp_set_wait_budget_ns": (_c_int, [_c_i64, ctypes.POINTER(_c_i64)]),
    "tp_selftest_bounded_wait": (_c_int, [_c_int, _c_p, _c_p]),
}

# status codes (include/tropical_b200.h)
TP_OK = 0
TP_DTYPE_F32 = 0
TP_DTYPE_BF16 = 1
TP_DTYPE_BF16_ARITH = 2
TP_BWD_STE = 1
TP_BWD_LSE = 2
TP_DEVERR_BARRIER_TIMEOUT = 1
TP_DEVERR_FLAG_TIMEOUT = 2
TP_ATT_PATH_AUTO = 0
TP_ATT_PATH_CUDA_CORES = 1
TP_ATT_PATH_TENSOR_CORES = 2
TP_ATT_LIST = 32

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class TropicalLibraryError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int, text: str):
        super().__init__(f"{what} failed: {text} (status {status})")
        self.status = status


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library (once) and declare every signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"tropical CUDA library not found at {p}; build it with "
                "`python -m mk_iii_technologies_tsrn_b200.build` (nvcc, sm_100a). "
                "There is no CPU fallback."
            )
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def status_text(status: int) -> str:
    return load().tp_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != TP_OK:
        raise TropicalLibraryError(what, status, status_text(status))


def is_available() -> bool:
    """True when the library file exists and loads (does not need a GPU)."""
    try:
        load()
        return True
    except (RuntimeError, OSError):
        return False
