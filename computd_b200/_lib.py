"""ctypes binding of ``libdwa_b200.so`` (the C ABI declared in include/dwa_retrieval.h and
include/dwa_lm.h).

The library is the only implementation of the retrieval path: there is no
CPU or PyTorch fallback.  If the shared library is missing, importing this
module raises immediately with the command that builds it.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdwa_b200.so"

DWA_OK = 0
DWA_ERR_INVALID_ARG = 1
DWA_ERR_UNSUPPORTED_SHAPE = 2
DWA_ERR_CUDA = 3
DWA_ERR_TIMEOUT = 4
DWA_ERR_DEVICE_CHECK = 5
DWA_ERR_WORKSPACE = 6
DWA_MAX_K = 128

# Every symbol include/dwa_retrieval.h and include/dwa_lm.h declare, with its ctypes signature.
_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "dwa_abi_version": (_i32, []),
    "dwa_status_string": (ctypes.c_char_p, [_i32]),
    "dwa_last_error": (ctypes.c_char_p, []),
    "dwa_score_topk_workspace": (ctypes.c_size_t, [_i64, _i64, _i32, _i32]),
    "dwa_score_topk": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i32, _i32,
                              _f32, _f32, _f32, _i32, _i64, _c_void_p, _c_void_p,
                              _c_void_p, ctypes.c_size_t, _c_void_p]),
    "dwa_score_topk_noalloc": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i32, _i32,
                                      _f32, _f32, _f32, _i32, _i64, _c_void_p, _c_void_p,
                                      _c_void_p]),
    "dwa_score_topk_dev": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i32, _i32,
                                  _c_void_p, _i32, _i64, _c_void_p, _c_void_p, _c_void_p,
                                  ctypes.c_size_t, _c_void_p]),
    "dwa_score_topk_seqmean": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i32, _i32,
                                      _c_void_p, _i32, _i64, _i64, _c_void_p, _i64, _c_void_p,
                                      _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p]),
    "dwa_project_keys_packed": (_i32, [_c_void_p, _i64, _i64, _i32, _c_void_p, _i64, _i32, _i32,
                                       _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p]),
    "dwa_seq_scores": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _i32, _c_void_p,
                              _i32, _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p]),
    "dwa_score_backward_dev": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _c_void_p,
                                      _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_merge_topk": (_i32, [_c_void_p, _c_void_p, _i32, _i64, _i32, _c_void_p, _c_void_p,
                              _c_void_p]),
    "dwa_merge_topk_strided": (_i32, [_c_void_p, _c_void_p, _i32, _i64, _i32, _i64, _i64, _i64,
                                      _c_void_p, _c_void_p, _c_void_p]),
    "dwa_weighted_gather": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, _i64, _i64,
                                   _i64, _i32, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_gather_dot": (_i32, [_c_void_p, _i32, _i64, _c_void_p, _i64, _i32, _c_void_p, _i64, _i64,
                              _i64, _i32, _c_void_p, _c_void_p]),
    "dwa_score_backward": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _f32, _f32, _f32,
                                  _i32, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_gather_rows": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, _i64, _i64, _i64, _i32,
                               _c_void_p, _i32, _c_void_p]),
    "dwa_scatter_add_rows": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, _i32, _i64, _i64,
                                    _i64, _c_void_p, _i64, _i32, _c_void_p]),
    "dwa_pool_init_normal": (_i32, [_c_void_p, _i64, _i64, _i64, _i64, ctypes.c_uint64, _f32,
                                    _c_void_p]),
    "dwa_weighted_gather_peers": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, _i64, _i64,
                                         _i64, _i32, ctypes.POINTER(_c_void_p), _i32, _i32, _i64,
                                         _c_void_p, _c_void_p]),
    "dwa_reduce_broadcast_peers": (_i32, [_c_void_p, _i32, _i32, _i64, _i64, _i32,
                                          ctypes.POINTER(_c_void_p), _c_void_p, _i32, _i64,
                                          _c_void_p, _c_void_p]),
    "dwa_peer_wait": (_i32, [_c_void_p, _i32, _i32, _i64, _c_void_p, _c_void_p]),
    "dwa_project_keys": (_i32, [_c_void_p, _i64, _i64, _i32, _c_void_p, _i64, _i32, _i32, _c_void_p,
                                _c_void_p, _i64, _c_void_p, _c_void_p]),
    "dwa_peer_alloc": (_i32, [ctypes.c_size_t, ctypes.POINTER(_c_void_p), _c_void_p]),
    "dwa_peer_open": (_i32, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "dwa_peer_close": (_i32, [_c_void_p]),
    "dwa_peer_free": (_i32, [_c_void_p]),
    "dwa_peer_signal": (_i32, [ctypes.POINTER(_c_void_p), _i32, _i32, _i32, _c_void_p]),
    "dwa_merge_topk_peers": (_i32, [ctypes.POINTER(_c_void_p), _i32, _i64, _i32, _c_void_p, _i32,
                                    _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_lowrank_delta": (_i32, [_c_void_p, _i32, _i64, _c_void_p, _c_void_p, _i64, _i32, _c_void_p,
                                 _i64, _i64, _i64, _i32, _i32, _i32, _c_void_p, _c_void_p]),
    "dwa_retrieval_backward": (_i32, [_c_void_p, _i32, _i64, _c_void_p, _i64, _c_void_p, _i64, _i32,
                                      _c_void_p, _i64, _i32, _c_void_p, _c_void_p, _i64, _i32,
                                      _i64, _i64, _f32, _f32, _f32, _c_void_p, _i32, _c_void_p,
                                      _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_row_gradient_workspace": (ctypes.c_size_t, [_i64, _i32, _i64]),
    "dwa_row_gradient": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p, _i32, _i64, _i64, _i64,
                                _c_void_p, _i32, _i64, _i32, _c_void_p, ctypes.c_size_t,
                                _c_void_p]),
    "dwa_lowrank_delta_rows_workspace": (ctypes.c_size_t, [_i64, _i32, _i64, _i32]),
    "dwa_lowrank_delta_rows": (_i32, [_c_void_p, _i32, _i64, _c_void_p, _c_void_p, _i64, _i32,
                                      _c_void_p, _i64, _i64, _i64, _i32, _i32, _i32, _c_void_p,
                                      _c_void_p, ctypes.c_size_t, _c_void_p]),
    "dwa_assemble_finish": (_i32, [_c_void_p, _i32, _i64, _c_void_p, _c_void_p, _i64, _i32, _f32,
                                   _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p]),
    "dwa_usage_ema": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _i64, _f32, _f32, _c_void_p,
                             _c_void_p]),
    "dwa_workspace_status": (_i32, [_c_void_p, _c_void_p, ctypes.POINTER(_i32)]),
    # include/dwa_lm.h: the LM block's fused elementwise steps
    "dwa_lm_rope_qk": (_i32, [_c_void_p, _i64, _i64, _i32, _i32, _i64, _c_void_p, _c_void_p,
                              _i64, _c_void_p, _c_void_p, _c_void_p]),
    "dwa_lm_aspect_queries": (_i32, [_c_void_p, _i64, _i32, _i32, _i64, _c_void_p, _c_void_p,
                                     _f32, _f32, _i32, _c_void_p, _i64, _c_void_p, _c_void_p,
                                     _c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class DWAError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, func: str, detail: str):
        self.status = status
        self.func = func
        super().__init__(f"{func} failed: {status_name(status)}: {detail}")


class DWAArgumentError(DWAError, ValueError):
    """Invalid or unsupported arguments (the call launched nothing)."""


def load() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -m computd_b200.build` "
                "(nvcc with sm_100a support required). There is no fallback implementation.")
        lib = ctypes.CDLL(os.fspath(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def status_name(status: int) -> str:
    return load().dwa_status_string(status).decode()


def last_error() -> str:
    """Detail of the last failed C-ABI call on this thread."""
    return load().dwa_last_error().decode(errors="replace")


def check(status: int, func: str) -> None:
    if status == DWA_OK:
        return
    detail = load().dwa_last_error().decode(errors="replace")
    if status in (DWA_ERR_INVALID_ARG, DWA_ERR_UNSUPPORTED_SHAPE, DWA_ERR_WORKSPACE):
        raise DWAArgumentError(status, func, detail)
    raise DWAError(status, func, detail)
