"""Layer-major refresh of the selected rows on one B200.

This is the device side of ``packed_interval_repair``
(kernels/packed_cache.py:225-298 of the reference). The reference drives the
transformers decoder modules through a shallow "native view" whose cache
layers scatter on update and whose attention is masked SDPA; this engine reads
the same parameters and runs, per layer:

    add_rmsnorm        residual add + input RMSNorm            (libkvr_b200)
    q/k/v projections  one cuBLAS GEMM on [Wq; Wk; Wv]          (torch.mm)
    qkv_rope_scatter   q/k-norm, RoPE, q packing, K/V scatter   (libkvr_b200)
    selected_attention GQA split-KV flash attention             (libkvr_b200)
    o projection       cuBLAS
    add_rmsnorm        residual add + post-attention RMSNorm    (libkvr_b200)
    gate/up            cuBLAS
    silu_mul           SiLU(gate) * up                          (libkvr_b200)
    down projection    cuBLAS

Rounding follows the modules op by op (one rounding per torch op). At a few
dozen rows the projections stream weights: one GEMM over the concatenated
q/k/v weights (an engine-owned copy, 1.5 GB for an 8B model, rebuilt when a
parameter changes) runs at about three times the HBM bandwidth of three
separate GEMMs whose k/v weights are only 8 MB each.

The last layer stops after its K/V scatter: its attention output, MLP and the
final norm feed nothing in the returned cache (the reference computes and
discards them).
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass

import torch

from . import _lib


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    o: torch.Tensor
    post_norm: torch.Tensor
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    qkv: torch.Tensor | None = None        # engine-owned [Wq; Wk; Wv]
    qkv_key: tuple | None = None           # identities and versions it was built from

    def fused_qkv(self) -> torch.Tensor:
        """``cat([Wq, Wk, Wv])`` for one GEMM per layer, rebuilt if any of the
        three parameters was replaced or modified in place since."""
        key = tuple((id(t), t._version) for t in (self.q, self.k, self.v))
        if self.qkv is None or self.qkv_key != key:
            self.qkv = torch.cat((self.q, self.k, self.v), dim=0).contiguous()
            self.qkv_key = key
        return self.qkv


class ModelView:
    """Borrowed parameters of a dense Llama/Qwen3 decoder; nothing is copied."""

    def __init__(self, base):
        config = base.config
        self.base = base
        self.rotary = base.rotary_emb
        self.embed = base.embed_tokens.weight
        self.hidden = config.hidden_size
        self.heads = config.num_attention_heads
        self.kv_heads = config.num_key_value_heads
        self.head_dim = getattr(config, "head_dim", None) or self.hidden // self.heads
        self.intermediate = config.intermediate_size
        self.eps = float(config.rms_norm_eps)
        self.vocab = self.embed.shape[0]
        self.dtype = self.embed.dtype
        self.layers: list[LayerWeights] = []
        for layer in base.layers:
            attn, mlp = layer.self_attn, layer.mlp
            self.layers.append(LayerWeights(
                in_norm=layer.input_layernorm.weight, q=attn.q_proj.weight, k=attn.k_proj.weight,
                v=attn.v_proj.weight, o=attn.o_proj.weight, post_norm=layer.post_attention_layernorm.weight,
                gate=mlp.gate_proj.weight, up=mlp.up_proj.weight, down=mlp.down_proj.weight,
                q_norm=getattr(getattr(attn, "q_norm", None), "weight", None),
                k_norm=getattr(getattr(attn, "k_norm", None), "weight", None),
            ))
        if self.heads % self.kv_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        if self.head_dim not in (64, 128):
            raise ValueError("the sm_100a kernels are built for head_dim 64 or 128")
        for w in self.layers:
            for t in (w.q, w.k, w.v, w.o, w.gate, w.up, w.down, w.in_norm, w.post_norm):
                if not t.is_contiguous():
                    raise ValueError("projection weights must be contiguous")

    def rope_tables(self, positions: torch.Tensor):
        """cos/sin ``[B, D]`` at absolute positions through the model's own
        rotary module, exactly as its forward builds position_embeddings."""
        probe = torch.empty(0, dtype=self.dtype, device=positions.device)
        cos, sin = self.rotary(probe, positions.unsqueeze(0))
        return cos[0].contiguous(), sin[0].contiguous()


_views: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()

# Probabilities enter P.V as P_hi + P_lo (close to fp32 P, as the reference's
# own indexed kernel keeps them); ATTN_P_ROUNDED rounds P once like fused SDPA.
ATTENTION_PRECISION = _lib.ATTN_P_SPLIT


class KernelTimer:
    """Optional CUDA-event brackets around named launches on the current stream.

    Install with ``set_kernel_timer(timer)``; the engine then records a
    (start, end) event pair around each attention launch and the ownership
    copy. Used by benchmarks to attribute time inside a timed region.
    """

    def __init__(self):
        self.events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = {}

    def start(self, name: str):
        begin = torch.cuda.Event(enable_timing=True)
        begin.record()
        return name, begin

    def stop(self, token) -> None:
        name, begin = token
        end = torch.cuda.Event(enable_timing=True)
        end.record()
        self.events.setdefault(name, []).append((begin, end))

    def totals_ms(self) -> dict[str, tuple[int, float]]:
        return {name: (len(pairs), sum(b.elapsed_time(e) for b, e in pairs)) for name, pairs in self.events.items()}


_timer: KernelTimer | None = None


def set_kernel_timer(timer: KernelTimer | None) -> None:
    global _timer
    _timer = timer


def kernel_timer() -> KernelTimer | None:
    return _timer


def model_view(base) -> ModelView:
    """Cached view; rebuilt if any parameter was replaced since."""
    view = _views.get(base)
    if view is not None:
        probe = base.layers[0].self_attn.q_proj.weight
        if probe is view.layers[0].q and base.embed_tokens.weight is view.embed:
            return view
    view = ModelView(base)
    _views[base] = view
    return view


class Workspace:
    """Per-request activation buffers ``[B, *]`` from torch's caching allocator."""

    def __init__(self, view: ModelView, rows: int, cache_rows: int, device):
        dt = view.dtype
        qd, kd = view.heads * view.head_dim, view.kv_heads * view.head_dim
        self.hidden = torch.empty((rows, view.hidden), dtype=dt, device=device)
        self.normed = torch.empty((rows, view.hidden), dtype=dt, device=device)
        self.delta = torch.empty((rows, view.hidden), dtype=dt, device=device)
        self.qkv = torch.empty((rows, qd + 2 * kd), dtype=dt, device=device)
        self.q_rot = torch.empty((rows, qd), dtype=dt, device=device)
        self.attn = torch.empty((rows, qd), dtype=dt, device=device)
        self.gate = torch.empty((rows, view.intermediate), dtype=dt, device=device)
        self.up = torch.empty((rows, view.intermediate), dtype=dt, device=device)
        self.act = torch.empty((rows, view.intermediate), dtype=dt, device=device)
        ws = _lib.load().kvr_attention_workspace_size(rows, view.heads, view.kv_heads, view.head_dim,
                                                      cache_rows)
        self.attn_ws = torch.empty(max(int(ws), 16), dtype=torch.uint8, device=device)


def refresh_rows(view: ModelView, layers, ids: torch.Tensor, positions: torch.Tensor,
                 max_position: int, cache_rows: int) -> None:
    """Recompute the selected rows through every layer, writing K/V in place.

    ``layers``: the owned output cache, ``[(K, V)]`` each ``[1, Hkv, N, D]``
    with unit D stride; ``ids``: ``[N]`` int64 on the device; ``positions``:
    ``[B]`` int64 sorted, on the device. Runs on the current stream.
    """
    lib = _lib.load()
    device = positions.device
    rows = positions.numel()
    dt = _lib.dtype_code(view.dtype)
    stream = _lib.stream_handle(device)
    ws = Workspace(view, rows, cache_rows, device)
    cos, sin = view.rope_tables(positions)
    D, H = view.head_dim, view.hidden
    qd, kd = view.heads * D, view.kv_heads * D
    elem = ws.qkv.element_size()
    scale = float(D) ** -0.5
    pos_ptr = positions.data_ptr()
    _lib.check(lib.kvr_embed_rows(view.embed.data_ptr(), view.vocab, H, ids.data_ptr(), ids.numel(),
                                  pos_ptr, rows, ws.hidden.data_ptr(), None, dt, stream), "embed_rows")
    last = len(view.layers) - 1
    for index, w in enumerate(view.layers):
        key, value = layers[index]
        c_hs, c_rs = key.stride(1), key.stride(2)
        _lib.check(lib.kvr_add_rmsnorm(ws.hidden.data_ptr(), ws.delta.data_ptr() if index else None,
                                       w.in_norm.data_ptr(), ws.normed.data_ptr(), rows, H, H, H, H,
                                       view.eps, dt, stream), "add_rmsnorm")
        final = index == last
        torch.mm(ws.normed, w.fused_qkv().t(), out=ws.qkv)
        q_ptr = ws.qkv.data_ptr()
        k_ptr = q_ptr + qd * elem
        v_ptr = k_ptr + kd * elem
        rs = ws.qkv.stride(0)
        _lib.check(lib.kvr_qkv_rope_scatter(
            q_ptr, k_ptr, v_ptr, rs, rs, rs, w.q_norm.data_ptr() if w.q_norm is not None else None,
            w.k_norm.data_ptr() if w.k_norm is not None else None, view.eps, cos.data_ptr(),
            sin.data_ptr(), pos_ptr, rows, view.heads, view.kv_heads, D,
            None if final else ws.q_rot.data_ptr(), key.data_ptr(), value.data_ptr(), cache_rows,
            c_hs, c_rs, None, dt, stream), "qkv_rope_scatter")
        if final:
            break
        token = _timer.start("selected_attention") if _timer else None
        _lib.check(lib.kvr_selected_attention(
            ws.q_rot.data_ptr(), key.data_ptr(), value.data_ptr(), ws.attn.data_ptr(), pos_ptr, rows,
            view.heads, view.kv_heads, D, cache_rows, c_hs, c_rs, max_position, scale, ATTENTION_PRECISION,
            ws.attn_ws.data_ptr(), ws.attn_ws.numel(), dt, stream), "selected_attention")
        if token:
            _timer.stop(token)
        torch.mm(ws.attn, w.o.t(), out=ws.delta)
        _lib.check(lib.kvr_add_rmsnorm(ws.hidden.data_ptr(), ws.delta.data_ptr(), w.post_norm.data_ptr(),
                                       ws.normed.data_ptr(), rows, H, H, H, H, view.eps, dt, stream),
                   "add_rmsnorm")
        torch.mm(ws.normed, w.gate.t(), out=ws.gate)
        torch.mm(ws.normed, w.up.t(), out=ws.up)
        I = view.intermediate
        _lib.check(lib.kvr_silu_mul(ws.gate.data_ptr(), ws.up.data_ptr(), ws.act.data_ptr(), rows, I, I, I,
                                    I, dt, stream), "silu_mul")
        torch.mm(ws.act, w.down.t(), out=ws.delta)
