"""Layer-major refresh of the selected rows on one B200.

This is the device side of ``packed_interval_repair``
(kernels/packed_cache.py:225-298 of the reference). The reference drives the
transformers decoder modules through a shallow "native view" whose cache
layers scatter on update and whose attention is masked SDPA; this engine reads
the same parameters and makes one native call (``kvr_packed_refresh``) whose
C++ layer loop runs, per layer:

    add_rmsnorm        residual add + input RMSNorm            (libkvr_b200)
    q/k/v projections  one cuBLAS GEMM on [Wq; Wk; Wv]
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

Repeated requests replay a CUDA graph (``GRAPH_REPLAY``): each request's ids,
positions and rotary tables are staged into buffers kept per (device, stream,
geometry), with one workspace there, so a request with the geometry and the
cache buffers of an earlier one (for example, the caller released the last
output before asking again) makes the same launches and the library replays
them from a graph captured on the second such call.
"""

from __future__ import annotations

import ctypes
import operator
import threading
import weakref
from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _lib, registry


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
        q, k, v = self.q, self.k, self.v
        key = (id(q), q.data_ptr(), q._version, id(k), k.data_ptr(), k._version, id(v), v.data_ptr(), v._version)
        if self.qkv is None or self.qkv_key != key:
            self.qkv = torch.cat((self.q, self.k, self.v), dim=0).contiguous()
            self.qkv_key = key
        return self.qkv


class ModelView:
    """Borrowed parameters of a dense Llama/Qwen3 decoder; nothing is copied."""

    def __init__(self, base):
        config = base.config
        self.base = base
        self.epoch = -1  # registry.epoch() when this view was built
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

    def rope_tables(self, positions: torch.Tensor, out=None):
        """cos/sin ``[B, D]`` at absolute positions (``kvr_rope_tables``): the
        op sequence of the model's rotary forward on its own ``inv_freq`` and
        ``attention_scaling``, in one launch. ``out``: optional ``(cos, sin)``
        contiguous ``[B, D]`` tensors of the model dtype to write."""
        inv_freq = self.rotary.inv_freq
        if inv_freq.numel() * 2 != self.head_dim:
            raise ValueError("partial rotary embeddings are outside the supported model families")
        if inv_freq.dtype != torch.float32 or inv_freq.device != positions.device or not inv_freq.is_contiguous():
            inv_freq = inv_freq.to(device=positions.device, dtype=torch.float32).contiguous()
        rows = positions.numel()
        if out is None:
            out = tuple(torch.empty(rows, self.head_dim, dtype=self.dtype, device=positions.device) for _ in range(2))
        cos, sin = out
        _lib.check(_lib.load().kvr_rope_tables(
            inv_freq.data_ptr(), self.head_dim // 2, positions.data_ptr(), rows,
            float(getattr(self.rotary, "attention_scaling", 1.0)), cos.data_ptr(), sin.data_ptr(),
            _lib.dtype_code(self.dtype), _lib.stream_handle(positions.device)), "rope_tables")
        return cos, sin


_views: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()

# Probabilities enter P.V rounded once to the element type, as the fused SDPA
# kernels of the reference's packed CUDA path do; refreshed rows agree with the
# reference's outputs as closely as with ATTN_P_SPLIT (P_hi + P_lo, close to
# fp32 P), which indexed_causal_attention keeps for its fp32-probability parity.
ATTENTION_PRECISION = _lib.ATTN_P_ROUNDED
# Projection GEMMs of the layer loop: cuBLAS, or the sm_100a weight-streaming
# kernel (kvr_linear) for requests of up to 256 rows.
PROJECTIONS = _lib.PROJ_CUBLAS
# Stage request inputs into stable buffers and let the library replay graphs of
# repeated requests (kvr_refresh_request.graph_replay).
GRAPH_REPLAY = True
_STAGING_KEEP = 8


class _Staging:
    """Per (device, stream, geometry) input buffers and workspace of a refresh.

    Host positions reach ``positions`` through ``host_positions`` (pinned), one
    stream-ordered copy; ``host_ready`` marks the end of that copy, and the
    pinned buffer is written again only after it (normally long done)."""

    def __init__(self, device, id_count: int, rows: int, dim: int, dtype, workspace_bytes: int):
        self.ids = torch.empty(id_count, dtype=torch.int64, device=device)
        self.positions = torch.empty(rows, dtype=torch.int64, device=device)
        self.cos = torch.empty(rows, dim, dtype=dtype, device=device)
        self.sin = torch.empty(rows, dim, dtype=dtype, device=device)
        self.workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=device)
        self.host_positions = None
        self.host_ready = None


# Keyed by (thread, device, stream, geometry): two threads issuing requests on
# one stream must not stage into the same buffers (the second thread's copies
# could land between the first thread's copies and its refresh).
_staging: "OrderedDict[tuple, _Staging]" = OrderedDict()
_staging_lock = threading.Lock()


def release_graphs() -> None:
    """Drop this thread's cached refresh graphs and its staged request
    buffers (their device memory returns to torch's allocator)."""
    _lib.check(_lib.load().kvr_release_graphs(), "release_graphs")
    me = threading.get_ident()
    with _staging_lock:
        for key in [k for k in _staging if k[0] == me]:
            del _staging[key]


def _staged(view: ModelView, device, ids, positions, need) -> _Staging:
    """This thread's staging buffers for the request's geometry on the current
    stream, filled with its ids, positions and rotary tables (stream-ordered).
    ``positions``: a device tensor, or host integers (copied from pinned
    memory straight into the staged buffer)."""
    stream = torch.cuda.current_stream(device)
    rows = positions.numel() if isinstance(positions, torch.Tensor) else len(positions)
    key = (threading.get_ident(), device.index, stream.cuda_stream, ids.numel(), rows, view.head_dim, view.dtype,
           need)
    with _staging_lock:
        st = _staging.pop(key, None)
        if st is None:
            st = _Staging(device, ids.numel(), rows, view.head_dim, view.dtype, need)
            while len(_staging) >= _STAGING_KEEP:
                _staging.popitem(last=False)
        _staging[key] = st
    st.ids.copy_(ids, non_blocking=True)  # device ids, or pinned host ids
    if isinstance(positions, torch.Tensor):
        st.positions.copy_(positions)
    else:
        if st.host_positions is None:
            st.host_positions = torch.empty(rows, dtype=torch.int64).pin_memory()
            st.host_ready = torch.cuda.Event()
        else:
            st.host_ready.synchronize()  # the previous request's copy out of the pinned buffer
        st.host_positions.numpy()[:] = positions
        st.positions.copy_(st.host_positions, non_blocking=True)
        st.host_ready.record(stream)
    view.rope_tables(st.positions, out=(st.cos, st.sin))
    return st


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
    """Cached view; rebuilt once a parameter, buffer or submodule of a module
    of a cached model was registered or replaced since it was built
    (registry.epoch)."""
    old = _views.get(base)
    epoch = registry.epoch()
    if old is not None and old.epoch == epoch:
        return old
    view = ModelView(base)
    view.epoch = epoch
    registry.watch(base.modules())
    if old is not None:
        # Layers whose q/k/v are the same parameter objects keep their stacked
        # copy (fused_qkv still rebuilds it if one of them changed in place).
        for new_w, old_w in zip(view.layers, old.layers):
            if new_w.q is old_w.q and new_w.k is old_w.k and new_w.v is old_w.v:
                new_w.qkv, new_w.qkv_key = old_w.qkv, old_w.qkv_key
    _views[base] = view
    return view


_version_of = operator.attrgetter("_version")


def _native_model(view: ModelView):
    """The kvr_model struct for this view, rebuilt when a weight's storage moved
    or q/k/v (whose fused copy the engine owns) changed in place."""
    watched = getattr(view, "_watched", None)
    if watched is None:
        watched = view._watched = [view.embed] + [
            t for w in view.layers
            for t in (w.in_norm, w.q, w.k, w.v, w.o, w.post_norm, w.gate, w.up, w.down, w.q_norm, w.k_norm)
            if t is not None]
        view._qkv_sources = [t for w in view.layers for t in (w.q, w.k, w.v)]
    # One pass over every weight's data pointer and over q/k/v's version
    # counters (the fused copies' keys hold the same facts per layer).
    key = tuple(map(torch.Tensor.data_ptr, watched)) + tuple(map(_version_of, view._qkv_sources))
    if getattr(view, "_native_key", None) != key:
        qkv = [w.fused_qkv() for w in view.layers]
        arr = (_lib.LayerWeights * len(view.layers))()
        for i, (w, fused) in enumerate(zip(view.layers, qkv)):
            arr[i] = _lib.LayerWeights(
                input_norm=w.in_norm.data_ptr(), qkv=fused.data_ptr(), q=w.q.data_ptr(), k=w.k.data_ptr(),
                v=w.v.data_ptr(), q_norm=w.q_norm.data_ptr() if w.q_norm is not None else None,
                k_norm=w.k_norm.data_ptr() if w.k_norm is not None else None, o=w.o.data_ptr(),
                post_norm=w.post_norm.data_ptr(), gate=w.gate.data_ptr(), up=w.up.data_ptr(),
                down=w.down.data_ptr())
        view._native_layers = arr
        view._native = _lib.Model(
            num_layers=len(view.layers), hidden=view.hidden, q_heads=view.heads, kv_heads=view.kv_heads,
            head_dim=view.head_dim, intermediate=view.intermediate, vocab=view.vocab, eps=view.eps,
            dtype=_lib.dtype_code(view.dtype), embed=view.embed.data_ptr(), layers=arr)
        view._native_key = key
    return view._native


def linear(x: torch.Tensor, weights, outs=None) -> list[torch.Tensor]:
    """``x @ W.T`` for each entry of ``weights`` in ONE ``kvr_linear`` launch.

    ``x``: ``[rows, k]`` (unit column stride); ``weights``: up to four entries,
    each an ``[n, k]`` nn.Linear weight or a ``(gate, up)`` pair, which yields
    ``silu(x @ gate.T) * (x @ up.T)`` with the MLP's roundings. Returns one
    ``[rows, n]`` tensor per entry (or writes ``outs``).
    """
    lib = _lib.load()
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be [rows, k] with a unit column stride")
    rows, k = x.shape
    segs = (_lib.LinearSegment * len(weights))()
    result = []
    for i, w in enumerate(weights):
        gate, up = (w if isinstance(w, (tuple, list)) else (w, None))
        out = outs[i] if outs is not None else torch.empty(rows, gate.shape[0], dtype=x.dtype, device=x.device)
        for t in (gate, up):
            if t is not None and (t.shape[1] != k or not t.is_contiguous() or t.dtype != x.dtype):
                raise ValueError("weights must be contiguous [n, k] tensors of the input dtype")
        if out.stride(1) != 1:
            raise ValueError("outputs need a unit column stride")
        segs[i] = _lib.LinearSegment(weight=gate.data_ptr(), weight_up=up.data_ptr() if up is not None else None,
                                     n=gate.shape[0], out=out.data_ptr(), out_stride=out.stride(0))
        result.append(out)
    need = lib.kvr_linear_workspace_size(rows, k, segs, len(weights))
    workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=x.device)
    _lib.check(lib.kvr_linear(x.data_ptr(), x.stride(0), rows, k, segs, len(weights), workspace.data_ptr(), need,
                              _lib.dtype_code(x.dtype), _lib.stream_handle(x.device)), "linear")
    linear.last_workspace = workspace
    return result


def refresh_rows(view: ModelView, layers, ids: torch.Tensor, positions,
                 max_position: int, cache_rows: int, tp_comm=None, sources=None) -> None:
    """Recompute the selected rows through every layer, writing K/V in place.

    ``layers``: the owned output cache, ``[(K, V)]`` each ``[1, Hkv, N, D]``
    with unit D stride and one (head, row) stride pair, or a contiguous
    ``[2L, 1, Hkv, N, D]`` arena holding them (``cache.allocate_arena``: K of
    layer l at 2l, V at 2l + 1), whose layer addresses follow from its base
    address so that no per-layer view is needed; ``ids``: ``[N]`` int64
    on the device, or in pinned host memory (copied once, into the request's
    staged buffer); ``positions``: ``[B]`` sorted, a device int64 tensor or
    host integers validated by the caller (an ``IndexedPlan``'s). One
    ``kvr_packed_refresh`` call runs every layer on the current stream.
    ``sources``: optional ``[(K, V)]`` of the same geometry that ``layers``
    first become a copy of (the ownership copy of clone_cache,
    kernels/packed_cache.py:287), made inside the same call so that layer l's
    copy overlaps the work on layers before l.
    """
    lib = _lib.load()
    host_positions = not isinstance(positions, torch.Tensor)
    if ids.device.type == "cpu" and not (ids.dtype == torch.int64 and ids.is_pinned()):
        raise ValueError("host ids must be pinned int64")
    rows = len(positions) if host_positions else positions.numel()
    if isinstance(layers, torch.Tensor):
        arena = layers
        if arena.dim() != 5 or arena.shape[0] % 2 or arena.shape[1] != 1 or not arena.is_contiguous():
            raise ValueError("a cache arena must be a contiguous [2L, 1, heads, rows, head_dim] tensor")
        device, dtype = arena.device, arena.dtype
        count, heads, dim = arena.shape[0] // 2, arena.shape[2], arena.shape[4]
        head_stride, row_stride = arena.stride(2), arena.stride(3)
        plane = arena.stride(0) * arena.element_size()
        base = arena.data_ptr()
        k_ptrs = (ctypes.c_void_p * count)(*range(base, base + 2 * count * plane, 2 * plane))
        v_ptrs = (ctypes.c_void_p * count)(*range(base + plane, base + 2 * count * plane, 2 * plane))
    else:
        first = layers[0][0]
        device, dtype = first.device, first.dtype
        count, heads, dim = len(layers), first.shape[1], first.shape[3]
        strides = {(t.stride(1), t.stride(2)) for pair in layers for t in pair}
        if len(strides) != 1:
            raise ValueError("every cache layer must share one (head, row) stride pair")
        head_stride, row_stride = strides.pop()
        k_ptrs = _lib.ptr_array([k for k, _ in layers])
        v_ptrs = _lib.ptr_array([v for _, v in layers])
    model = _native_model(view)
    request = _lib.RefreshRequest(
        k_cache=k_ptrs, v_cache=v_ptrs, cache_rows=cache_rows, cache_head_stride=head_stride,
        cache_row_stride=row_stride, ids=None, id_count=ids.numel(),
        positions=None if host_positions else positions.data_ptr(), rows=rows, max_position=max_position, attention_precision=ATTENTION_PRECISION, tp_comm=tp_comm,
        projections=PROJECTIONS)
    if sources is not None:
        from .cache import uniform_layout

        if len(sources) != count:
            raise ValueError("sources must give one (K, V) pair per cache layer")
        src_heads, src_rows, src_dim, src_dtype, src_device, src_hs, src_rs = uniform_layout(sources, "clone_cache")
        if (src_heads, src_dim, src_dtype, src_device) != (heads, dim, dtype, device) or src_rows < cache_rows:
            raise ValueError("sources must match the cache's heads, head_dim, dtype and device and hold its rows")
        request.k_src = _lib.ptr_array([k for k, _ in sources])
        request.v_src = _lib.ptr_array([v for _, v in sources])
        request.src_head_stride, request.src_row_stride = src_hs, src_rs
    # No rows: the call only makes the ownership copy and takes no workspace.
    need = lib.kvr_packed_refresh_workspace_size(model, rows, cache_rows) if rows else 0
    if rows and not need:
        raise ValueError("model geometry is outside the built kernels")
    if GRAPH_REPLAY and rows and tp_comm is None:
        st = _staged(view, device, ids, positions, need)
        request.ids, request.positions = st.ids.data_ptr(), st.positions.data_ptr()
        request.cos_tab, request.sin_tab = st.cos.data_ptr(), st.sin.data_ptr()
        request.graph_replay = 1
        workspace = st.workspace
    else:
        if ids.device.type == "cpu":
            ids = ids.to(device, non_blocking=True)
        request.ids = ids.data_ptr()
        if host_positions and rows:
            from .staging import upload_int64

            positions = upload_int64(list(positions), device)
            request.positions = positions.data_ptr()
        cos, sin = view.rope_tables(positions) if rows else (None, None)
        if rows:
            request.cos_tab, request.sin_tab = cos.data_ptr(), sin.data_ptr()
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    _lib.check(lib.kvr_packed_refresh(model, request, workspace.data_ptr(), need, _lib.stream_handle(device)),
               "packed_refresh")
