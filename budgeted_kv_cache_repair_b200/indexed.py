"""Standalone selected-row operators (kernels/indexed_attention.py:161-241 of
the reference): bitwise K/V scatter and absolute-causal selected-query
attention, on the sm_100a kernels. CUDA only; no fallback.
"""

from __future__ import annotations

import math
from numbers import Real

import torch

from . import _lib
from .plan import validate_device_plan
from .validate import nonoverlapping_layout

_DTYPES = (torch.float16, torch.bfloat16)


def _validate_tensors(tensors):
    if any(not isinstance(t, torch.Tensor) or t.ndim != 4 for t in tensors):
        raise ValueError("attention/cache tensors must have four dimensions")
    first = tensors[0]
    if not first.is_cuda or any(t.device != first.device for t in tensors):
        raise ValueError("all tensors must share one CUDA device")
    if first.dtype not in _DTYPES or any(t.dtype != first.dtype for t in tensors):
        raise ValueError("all tensors must share float16 or bfloat16 dtype")
    if any(t.shape[0] != 1 for t in tensors):
        raise ValueError("indexed kernels currently require batch size one")
    if any(t.shape[1] <= 0 or t.shape[3] not in (64, 128) for t in tensors):
        raise ValueError("head counts must be positive and head dimension must be 64 or 128")
    if any(any(s <= 0 for s in t.stride()) or not nonoverlapping_layout(t) for t in tensors):
        raise ValueError("tensor layouts must have positive provably nonoverlapping strides")
    if any(t.requires_grad for t in tensors):
        raise ValueError("indexed kernels are inference-only; detach gradient-bearing inputs")


def _kernel_view(t: torch.Tensor) -> torch.Tensor:
    """The tensor itself when rows are 16-byte aligned with unit D stride,
    else a compact copy (only for exotic caller layouts)."""
    if t.stride(3) == 1 and t.data_ptr() % 16 == 0 and t.stride(1) % 8 == 0 and t.stride(2) % 8 == 0:
        return t
    return t.contiguous()


def indexed_kv_scatter_(out_k, out_v, fresh_k, fresh_v, device_plan):
    """Copy selected K/V rows exactly, preserving every other storage byte
    (kernels/indexed_attention.py:179-204)."""
    tensors = (out_k, out_v, fresh_k, fresh_v)
    _validate_tensors(tensors)
    validate_device_plan(device_plan, out_k.device)
    _, heads, _, dim = out_k.shape
    if any((t.shape[1], t.shape[3]) != (heads, dim) for t in tensors):
        raise ValueError("scatter K/V head geometry must match")
    if any(t.shape[2] != device_plan.logical_length for t in tensors[:2]):
        raise ValueError("output sequence length must match the plan")
    if any(t.shape[2] != device_plan.selected_count for t in tensors[2:]):
        raise ValueError("fresh sequence length must match selected_count")
    if not device_plan.selected_count:
        return
    storage = [t.untyped_storage().data_ptr() for t in tensors]
    if storage[0] == storage[1] or any(a == b for a in storage[:2] for b in storage[2:]):
        raise ValueError("output K/V storage must be independent of outputs and fresh sources")
    targets = [out_k, out_v]
    direct = all(t.stride(3) == 1 and t.data_ptr() % 16 == 0 and t.stride(1) % 8 == 0 and t.stride(2) % 8 == 0
                 for t in targets) and out_k.stride()[1:3] == out_v.stride()[1:3]
    # Exotic target layouts scatter into compact staging copies, then copy back.
    staged = targets if direct else [t.contiguous() for t in targets]
    fk, fv = _kernel_view(fresh_k), _kernel_view(fresh_v)
    if fk.stride()[1:3] != fv.stride()[1:3]:
        fk, fv = fk.contiguous(), fv.contiguous()
    with torch.cuda.device(out_k.device):
        lib = _lib.load()
        _lib.check(lib.kvr_scatter_rows(
            fk.data_ptr(), fv.data_ptr(), staged[0].data_ptr(), staged[1].data_ptr(),
            device_plan.positions.data_ptr(), device_plan.selected_count, heads, dim,
            device_plan.logical_length, fk.stride(1), fk.stride(2), staged[0].stride(1), staged[0].stride(2),
            None, _lib.dtype_code(out_k.dtype), _lib.stream_handle(out_k.device)), "scatter_rows")
        if not direct:
            for target, result in zip(targets, staged):
                target.copy_(result)


def indexed_causal_attention(q, k, v, device_plan, scale=None):
    """Attend packed queries to their entire absolute causal prefix
    (kernels/indexed_attention.py:207-241).

    q=[1,Hq,B,D], k/v=[1,Hkv,N,D], result=[1,Hq,B,D]. Row b attends key
    positions <= its absolute position, including itself.
    """
    _validate_tensors((q, k, v))
    validate_device_plan(device_plan, q.device)
    if k.shape != v.shape or q.shape[3] != k.shape[3]:
        raise ValueError("attention K/V shapes and Q/K/V head dimensions must match")
    if q.shape[1] % k.shape[1]:
        raise ValueError("query head count must be divisible by KV head count")
    if q.shape[2] != device_plan.selected_count or k.shape[2] != device_plan.logical_length:
        raise ValueError("attention sequence lengths must match the plan")
    if scale is None:
        scale = q.shape[-1] ** -0.5
    if isinstance(scale, bool) or not isinstance(scale, Real) or not math.isfinite(scale):
        raise ValueError("attention scale must be a finite host real number")
    _, heads, rows, dim = q.shape
    output = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if not rows:
        return output
    kv_heads, length = k.shape[1], k.shape[2]
    with torch.cuda.device(q.device):
        packed_q = q[0].transpose(0, 1).contiguous()          # [B, Hq, D]
        kk, vv = _kernel_view(k), _kernel_view(v)
        if kk.stride()[1:3] != vv.stride()[1:3]:
            kk, vv = kk.contiguous(), vv.contiguous()
        packed_out = torch.empty_like(packed_q)
        lib = _lib.load()
        ws_bytes = lib.kvr_attention_workspace_size(rows, heads, kv_heads, dim, length)
        workspace = torch.empty(max(int(ws_bytes), 16), dtype=torch.uint8, device=q.device)
        _lib.check(lib.kvr_selected_attention(
            packed_q.data_ptr(), kk.data_ptr(), vv.data_ptr(), packed_out.data_ptr(),
            device_plan.positions.data_ptr(), rows, heads, kv_heads, dim, length, kk.stride(1), kk.stride(2),
            device_plan.host_plan.max_position, float(scale), _lib.ATTN_P_SPLIT, workspace.data_ptr(), workspace.numel(),
            _lib.dtype_code(q.dtype), _lib.stream_handle(q.device)), "selected_attention")
        output.copy_(packed_out.transpose(0, 1).unsqueeze(0))
    return output
