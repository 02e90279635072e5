"""ctypes binding of the C ABI declared in include/santa_b200.h.

Only plain pointers, sizes and the raw ``cudaStream_t`` cross the boundary;
torch is used on this side for device memory and streams only.  Loading fails
loudly when the shared library is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

from . import _build

SANTA_OK = 0
SANTA_ERR_INVALID_ARGUMENT = -1
SANTA_ERR_UNSUPPORTED = -2
SANTA_ERR_CUDA = -3
SANTA_ERR_WORKSPACE = -4

DTYPE_F32 = 0
DTYPE_BF16 = 1

MODE_TOPK = 0
MODE_GUIDED = 1
MODE_UNIFORM = 2
MODE_SANTA = 3
MODE_HYBRID = 4
MODES = {"topk": MODE_TOPK, "guided": MODE_GUIDED, "uniform": MODE_UNIFORM,
         "santa": MODE_SANTA, "hybrid": MODE_HYBRID}

SAMPLES_DEVICE = 0
SAMPLES_INJECTED = 1

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32


class SantaGeometry(ctypes.Structure):
    _fields_ = [("batch", _i32), ("num_kv_heads", _i32), ("group", _i32), ("head_dim", _i32),
                ("capacity", _i32), ("n_total", _i32), ("sample_end", _i32), ("kv_dtype", _i32),
                ("block_table", _vp), ("page_size", _i32), ("max_pages", _i32),
                ("num_pages", _i32), ("reserved", _i32)]


class SantaSummary(ctypes.Structure):
    _fields_ = [("members", _vp), ("positions", _vp), ("starts", _vp), ("lengths", _vp),
                ("log_n", _vp), ("centroids", _vp), ("n_groups", _vp), ("sorted_key", _vp),
                ("sorted_value", _vp), ("max_groups", _i32)]


class SantaDecodeParams(ctypes.Structure):
    _fields_ = [("mode", _i32), ("topk_clusters", _i32), ("token_budget", _i32),
                ("samples", _i32), ("scale", ctypes.c_float), ("sample_source", _i32),
                ("seed", ctypes.c_uint64), ("step", ctypes.c_uint64), ("num_splits", _i32),
                ("step_dev", _vp)]


class SantaP2P(ctypes.Structure):
    _fields_ = [("peer_buffers", _vp), ("local_buffer", _vp), ("epoch", ctypes.c_uint64),
                ("error_flag", _vp), ("rows", _i32), ("keys_per_row", _i32),
                ("partial_floats", _i32), ("wait_limit_us", _i32)]


IPC_HANDLE_BYTES = 64


class SantaShard(ctypes.Structure):
    _fields_ = [("shard_index", _i32), ("num_shards", _i32), ("cluster_base", _i32),
                ("reserved", _i32), ("candidates", _vp), ("p2p", _vp)]


MAX_SHARDS = 32
SHARD_MAX_KEYS = 512


def partial_floats(head_dim: int) -> int:
    return head_dim + 8


class SantaPrefillShape(ctypes.Structure):
    _fields_ = [("batch", _i32), ("num_query_heads", _i32), ("num_kv_heads", _i32),
                ("seq_len", _i32), ("head_dim", _i32), ("scale", ctypes.c_float),
                ("causal", _i32), ("kv_capacity", _i32)]


# Every symbol include/santa_b200.h declares, with its ctypes signature.
_P = ctypes.POINTER
SIGNATURES = {
    "santa_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "santa_last_cuda_error": (ctypes.c_int, []),
    "santa_version": (ctypes.c_char_p, []),
    "santa_build_summary_workspace_bytes": (ctypes.c_int, [_P(SantaGeometry), _i32,
                                                           _P(ctypes.c_size_t)]),
    "santa_build_summary": (ctypes.c_int, [_P(SantaGeometry), _vp, _vp, _vp, _i32,
                                           _P(SantaSummary), _vp, ctypes.c_size_t, _vp]),
    "santa_decode_workspace_bytes": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams),
                                                    _i32, _P(ctypes.c_size_t)]),
    "santa_decode": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp, _vp,
                                    _P(SantaSummary), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    ctypes.c_size_t, _vp]),
    "santa_decode_plan": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                         _vp, _P(SantaSummary), _vp, _vp, _vp, _vp,
                                         ctypes.c_size_t, _vp]),
    "santa_decode_execute": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                            _vp, _P(SantaSummary), _vp, _vp, _vp, _vp,
                                            ctypes.c_size_t, _vp]),
    "santa_decode_static_scratch": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp,
                                                   _vp, _vp, _P(SantaSummary), _vp, _vp, _vp,
                                                   _vp, _vp, _vp, _vp]),
    "santa_decode_bad_draws": (ctypes.c_int, [_P(SantaGeometry), _vp, ctypes.c_size_t,
                                              _P(ctypes.c_int32), _vp]),
    "santa_decode_select": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                           _vp, _P(SantaSummary), _vp, _vp, _vp, _vp, _vp, _vp,
                                           ctypes.c_size_t, _vp]),
    "santa_shard_candidates": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                              _vp, _P(SantaSummary), _P(SantaShard), _vp, _vp,
                                              ctypes.c_size_t, _vp]),
    "santa_shard_plan": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp, _vp,
                                        _P(SantaSummary), _P(SantaShard), _vp, _vp, _vp,
                                        ctypes.c_size_t, _vp]),
    "santa_shard_execute": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                           _vp, _P(SantaSummary), _P(SantaShard), _vp, _vp,
                                           ctypes.c_size_t, _vp]),
    "santa_shard_select": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                          _vp, _P(SantaSummary), _P(SantaShard), _vp, _vp, _vp,
                                          _vp, _vp, ctypes.c_size_t, _vp]),
    "santa_shard_attend": (ctypes.c_int, [_P(SantaGeometry), _P(SantaDecodeParams), _vp, _vp,
                                          _vp, _P(SantaSummary), _P(SantaShard), _vp, _vp, _vp,
                                          _vp, ctypes.c_size_t, _vp]),
    "santa_merge_shards": (ctypes.c_int, [_i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "santa_p2p_buffer_bytes": (ctypes.c_int, [_i32, _i32, _i32, _i32, _P(ctypes.c_size_t)]),
    "santa_p2p_alloc": (ctypes.c_int, [ctypes.c_size_t, _P(_vp)]),
    "santa_p2p_free": (ctypes.c_int, [_vp]),
    "santa_p2p_ipc_handle": (ctypes.c_int, [_vp, _vp]),
    "santa_p2p_ipc_open": (ctypes.c_int, [_vp, _P(_vp)]),
    "santa_p2p_ipc_close": (ctypes.c_int, [_vp]),
    "santa_p2p_peek": (ctypes.c_int, [_vp, _P(ctypes.c_uint64)]),
    "santa_p2p_poke": (ctypes.c_int, [_vp, ctypes.c_uint64]),
    "santa_rope_append": (ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                                         _vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "santa_rope_append_paged": (ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                                               _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp,
                                               _vp, _vp]),
    "santa_prefill_workspace_bytes": (ctypes.c_int, [_P(SantaPrefillShape),
                                                     _P(ctypes.c_size_t)]),
    "santa_prefill": (ctypes.c_int, [_P(SantaPrefillShape), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                     ctypes.c_size_t, _vp]),
    "santa_prefill_paged": (ctypes.c_int, [_P(SantaPrefillShape), _vp, _vp, _vp, _vp, _i32,
                                           _i32, _i32, _vp, _vp, _vp, _vp, ctypes.c_size_t,
                                           _vp]),
    "santa_fingerprints_workspace_bytes": (ctypes.c_int, [_i32, _P(ctypes.c_size_t)]),
    "santa_fingerprints": (ctypes.c_int, [_vp, _i32, ctypes.c_int64, _i32, _vp, ctypes.c_int64,
                                          _i32, _vp, _i32, ctypes.c_float, _i32, _vp, _vp,
                                          ctypes.c_size_t, _vp]),
    "santa_kmeans_sqnorm": (ctypes.c_int, [_vp, ctypes.c_int64, _i32, _vp, _vp]),
    "santa_kmeans_assign": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int64, _i32, _vp, _vp, _i32,
                                           _vp, _vp, _vp, _vp]),
    "santa_kmeans_update_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, _i32,
                                                           _P(ctypes.c_size_t)]),
    "santa_kmeans_update": (ctypes.c_int, [_vp, _vp, ctypes.c_int64, _i32, _vp, _i32, _vp, _vp,
                                           _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "santa_kmeans_reassign": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp,
                                             ctypes.c_float, _vp]),
    "santa_kmeans_plusplus_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, _i32,
                                                             _P(ctypes.c_size_t)]),
    "santa_kmeans_plusplus": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int64, _i32, _i32, _i32,
                                             ctypes.c_int64, _vp, _vp, _vp, _vp,
                                             ctypes.c_size_t, _vp]),
}

_lock = threading.Lock()
_handle = None


class SantaError(RuntimeError):
    """Raised when a C ABI entry point returns a non-zero status."""

    def __init__(self, fn: str, status: int):
        lib = _handle
        msg = lib.santa_status_string(status).decode() if lib is not None else str(status)
        if status == SANTA_ERR_CUDA and lib is not None:
            msg += f" (cudaError {lib.santa_last_cuda_error()})"
        super().__init__(f"{fn} failed: {msg}")
        self.status = status


def library_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load libsanta_b200.so (building it with nvcc first if it is absent)."""
    global _handle
    with _lock:
        if _handle is not None:
            return _handle
        path = _build.LIB_PATH
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(f"SANTA++ CUDA library not built: {path}")
            _build.build()
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _handle = lib
        return lib


def check(fn: str, status: int) -> None:
    if status != SANTA_OK:
        raise SantaError(fn, status)


def ptr(t) -> int | None:
    """Raw device pointer of a tensor (None for a missing optional tensor)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
