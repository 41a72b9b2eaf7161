"""ctypes binding of libkvr_b200.so, the C ABI declared in include/kvr_b200.h.

The library is built in-tree (``python -m budgeted_kv_cache_repair_b200.build``)
and loaded from ``lib/`` next to this file. There is no fallback: every
product entry point fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "lib", "libkvr_b200.so")

OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_SCRATCH_LIMIT, ERR_INJECTED = 0, 1, 2, 3, 4, 5, 6
STATIC_SCRATCH_BYTES = 16 << 20
DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
ATTN_P_SPLIT, ATTN_P_ROUNDED = 0, 1
TP_ID_BYTES = 128
MAX_LAYER_TENSORS = 256

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_PP = ctypes.POINTER(ctypes.c_void_p)

class LayerWeights(ctypes.Structure):
    """kvr_layer_weights"""
    _fields_ = [(name, ctypes.c_void_p) for name in
                ("input_norm", "qkv", "q", "k", "v", "q_norm", "k_norm", "o", "post_norm", "gate", "up", "down")]


class Model(ctypes.Structure):
    """kvr_model"""
    _fields_ = [("num_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("q_heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("vocab", ctypes.c_int64), ("eps", ctypes.c_float), ("dtype", ctypes.c_int),
                ("embed", ctypes.c_void_p), ("layers", ctypes.POINTER(LayerWeights))]


class RefreshRequest(ctypes.Structure):
    """kvr_refresh_request"""
    _fields_ = [("k_cache", ctypes.POINTER(ctypes.c_void_p)), ("v_cache", ctypes.POINTER(ctypes.c_void_p)),
                ("cache_rows", ctypes.c_int64), ("cache_head_stride", ctypes.c_int64),
                ("cache_row_stride", ctypes.c_int64), ("ids", ctypes.c_void_p), ("id_count", ctypes.c_int64),
                ("positions", ctypes.c_void_p), ("rows", ctypes.c_int64), ("max_position", ctypes.c_int64),
                ("cos_tab", ctypes.c_void_p), ("sin_tab", ctypes.c_void_p), ("attention_precision", ctypes.c_int),
                ("tp_comm", ctypes.c_void_p), ("projections", ctypes.c_int),
                ("k_src", ctypes.POINTER(ctypes.c_void_p)), ("v_src", ctypes.POINTER(ctypes.c_void_p)),
                ("src_head_stride", ctypes.c_int64), ("src_row_stride", ctypes.c_int64),
                ("graph_replay", ctypes.c_int)]


LINEAR_MAX_SEGMENTS = 4
PROJ_CUBLAS, PROJ_SM100, PROJ_FUSED = 0, 1, 2


class LinearSegment(ctypes.Structure):
    """kvr_linear_segment"""
    _fields_ = [("weight", ctypes.c_void_p), ("weight_up", ctypes.c_void_p), ("n", ctypes.c_int64),
                ("out", ctypes.c_void_p), ("out_stride", ctypes.c_int64)]


# name -> (restype, argtypes); mirrors include/kvr_b200.h one to one.
SIGNATURES = {
    "kvr_version": (ctypes.c_char_p, []),
    "kvr_status_string": (ctypes.c_char_p, [_I]),
    "kvr_last_cuda_error": (_I, []),
    "kvr_kernel_launches": (ctypes.c_uint64, []),
    "kvr_graph_replays": (ctypes.c_uint64, []),
    "kvr_release_graphs": (_I, []),
    "kvr_rope_tables": (_I, [_P, _I, _P, _L, _F, _P, _P, _I, _P]),
    "kvr_copy_layers": (_I, [_PP, _PP, _I, _I, _L, _I, _L, _L, _L, _L, _I, _P]),
    "kvr_rope_shift_layers": (_I, [_PP, _PP, _I, _I, _L, _I, _L, _L, _L, _L, _P, _I, _P]),
    "kvr_shift_cache_layers": (_I, [_PP, _PP, _PP, _PP, _I, _I, _I, _L, _L, _L, _L, _L, _L, _L, _L,
                                    _P, _I, _I, _P]),
    "kvr_scatter_rows": (_I, [_P, _P, _P, _P, _P, _L, _I, _I, _L, _L, _L, _L, _L, _P, _I, _P]),
    "kvr_embed_rows": (_I, [_P, _L, _I, _P, _L, _P, _L, _P, _P, _I, _P]),
    "kvr_add_rmsnorm": (_I, [_P, _P, _P, _P, _L, _I, _L, _L, _L, _F, _I, _P]),
    "kvr_qkv_rope_scatter": (_I, [_P, _P, _P, _L, _L, _L, _P, _P, _F, _P, _P, _P, _L, _I, _I, _I,
                                  _P, _P, _P, _L, _L, _L, _P, _I, _P]),
    "kvr_silu_mul": (_I, [_P, _P, _P, _L, _L, _L, _L, _L, _I, _P]),
    "kvr_linear_workspace_size": (ctypes.c_size_t, [_L, _L, ctypes.POINTER(LinearSegment), _I]),
    "kvr_linear": (_I, [_P, _L, _L, _L, ctypes.POINTER(LinearSegment), _I, _P, ctypes.c_size_t, _I, _P]),
    "kvr_attention_workspace_size": (ctypes.c_size_t, [_L, _I, _I, _I, _L]),
    "kvr_selected_attention": (_I, [_P, _P, _P, _P, _P, _L, _I, _I, _I, _L, _L, _L, _L, _F, _I, _P,
                                    ctypes.c_size_t, _I, _P]),
    "kvr_packed_refresh_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(Model), _L, _L]),
    "kvr_packed_refresh": (_I, [ctypes.POINTER(Model), ctypes.POINTER(RefreshRequest), _P, ctypes.c_size_t, _P]),
    "kvr_tp_unique_id": (_I, [_P]),
    "kvr_tp_comm_init": (_I, [_P, _I, _I, ctypes.POINTER(ctypes.c_void_p)]),
    "kvr_tp_comm_destroy": (_I, [_P]),
    "kvr_selected_attention_static": (_I, [_P, _P, _P, _P, _P, _L, _I, _I, _I, _L, _L, _L, _L, _F, _I, _I, _P]),
    "kvr_attention_static_status": (_I, [_P, _P]),
    "kvr_set_wait_limit": (_I, [_L]),
    "kvr_debug_fail_refresh_after_layer": (_I, [_I]),
    "kvr_query_relevance_workspace_size": (ctypes.c_size_t, [_I, _I]),
    "kvr_query_relevance": (_I, [_P, _L, _I, _I, _P, _L, _P, _I, _F, _P, _P, ctypes.c_size_t, _P]),
}

_lock = threading.Lock()
_handle = None


class KvrError(RuntimeError):
    """A native call failed after host-side validation passed."""


def library_path() -> str:
    return LIBRARY


def load():
    """Load the library once; raise if it was not built."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not os.path.exists(LIBRARY):
                raise RuntimeError(
                    f"{LIBRARY} is missing: build it with `python -m budgeted_kv_cache_repair_b200.build` "
                    "(the B200 engine has no CPU or eager fallback)")
            lib = ctypes.CDLL(LIBRARY)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _handle = lib
    return _handle


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return DTYPE_BF16
    if dtype == torch.float16:
        return DTYPE_F16
    raise ValueError("the B200 engine computes in bfloat16 or float16")


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr_array(tensors) -> ctypes.Array:
    array = ctypes.c_void_p * len(tensors)
    try:
        return array(*map(torch.Tensor.data_ptr, tensors))
    except TypeError:  # raw addresses among the entries
        return array(*[t.data_ptr() if isinstance(t, torch.Tensor) else int(t) for t in tensors])


def check(status: int, what: str) -> None:
    if status == OK:
        return
    lib = load()
    text = lib.kvr_status_string(status).decode()
    if status in (ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_SCRATCH_LIMIT):
        raise ValueError(f"{what}: {text}")
    cuda = lib.kvr_last_cuda_error()
    raise KvrError(f"{what}: {text} (cudaError {cuda})")


def call(name: str, *args) -> None:
    fn = getattr(load(), name)
    check(fn(*args), name)
