"""Run one engine kernel at benchmark geometry, for profilers.

    python -m budgeted_kv_cache_repair_b200.profile_kernels shift     [--reps N] [--layers L]
    python -m budgeted_kv_cache_repair_b200.profile_kernels attention [--reps N] [--precision rounded|split]
                                                                      [--geometry config2|config3]
    python -m budgeted_kv_cache_repair_b200.profile_kernels copy      [--reps N] [--tensors T]
    python -m budgeted_kv_cache_repair_b200.profile_kernels linear    [--reps N] [--only NAME]
    python -m budgeted_kv_cache_repair_b200.profile_kernels relevance [--reps N]
    python -m budgeted_kv_cache_repair_b200.profile_kernels refresh   [--reps N] [--layers L]
                                                                      [--projections cublas|sm100|fused]

Geometry: Llama-3-8B shape (32 layers, 8 KV heads, head_dim 128, bf16),
8192-token context with 256 tokens deleted at 1024 (7936 rows), 64 selected
rows in 16 intervals of 4 (`linear`: the per-layer projections of that model
at 64 rows, each timed beside torch's cuBLAS GEMMs for the same products, with
enough weight copies in rotation that no launch finds its weights in L2, and
replayed from a CUDA graph so that host launch cost is not measured).
`refresh`: packed_interval_repair over the first `--layers` layers (2 by
default: about 3 GB on the device with the embedding and head) of that model,
every launch direct (no graph replay, unless `--replay`), so a profiler sees
each kernel of the layer loop as issued.
`relevance`: select_support's query relevance at config 3 (Qwen3-8B
embedding table, 151936 x 4096 bf16; 31744 prompt tokens; 8 query tokens).
`attention --geometry config3`: one layer of the Qwen3-8B shape at 32k context
(31744 cached rows, 1383 rows in 32 intervals from 4096). Inputs are seeded
random tensors. After two
warm-up launches the command times `--reps` launches with CUDA events and
prints the average (`attention` and `linear`: replayed from a CUDA graph,
after a capture pass and one replay); under ncu, capture with `-s 2`
(`attention`: two kernels per call).
"""

from __future__ import annotations

import argparse

import torch

from . import _lib, build

LAYERS, HEADS, KV_HEADS, D, OLD, NEW, DELETE_AT, DELETED = 32, 32, 8, 128, 8192, 7936, 1024, 256


def _positions():
    gen = torch.Generator().manual_seed(1)
    slots = (NEW - DELETE_AT) // 5
    starts = sorted(DELETE_AT + s * 5 for s in torch.randperm(slots, generator=gen)[:16].tolist())
    return sorted(p + i for p in starts for i in range(4))


NEW3, DELETE_AT3, ROWS3, INTERVALS3 = 31744, 4096, 1383, 32


def _positions3():
    """1383 rows in 32 non-adjacent intervals (widths 43 and 44) from 4096."""
    width, extra = divmod(ROWS3, INTERVALS3)
    gen = torch.Generator().manual_seed(3)
    picks = sorted(torch.randperm((NEW3 - DELETE_AT3) // (width + 2), generator=gen)[:INTERVALS3].tolist())
    return [DELETE_AT3 + s * (width + 2) + i for n, s in enumerate(picks) for i in range(width + (n < extra))]


def _time(fn, reps: int) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return begin.elapsed_time(end) / reps * 1e3


def shift(reps: int, layers: int = LAYERS) -> None:
    """`layers` < 32 runs the same per-layer geometry on fewer layers (a small
    case for multi-pass profiler captures; traffic scales with the layers)."""
    lib = _lib.load()
    ko = [torch.randn(1, KV_HEADS, OLD, D, device="cuda").bfloat16() for _ in range(layers)]
    vo = [torch.randn(1, KV_HEADS, OLD, D, device="cuda").bfloat16() for _ in range(layers)]
    kn = [torch.empty(1, KV_HEADS, NEW, D, device="cuda", dtype=torch.bfloat16) for _ in range(layers)]
    vn = [torch.empty(1, KV_HEADS, NEW, D, device="cuda", dtype=torch.bfloat16) for _ in range(layers)]
    table = torch.randn(2 * D, device="cuda").bfloat16()
    stream = _lib.stream_handle()
    args = (_lib.ptr_array(ko), _lib.ptr_array(vo), _lib.ptr_array(kn), _lib.ptr_array(vn), layers, KV_HEADS, D, NEW,
            DELETE_AT, DELETE_AT + DELETED, DELETE_AT, OLD * D, D, NEW * D, D, table.data_ptr(), 1, _lib.DTYPE_BF16,
            stream)
    us = _time(lambda: _lib.check(lib.kvr_shift_cache_layers(*args), "shift"), reps)
    algo = 2 * 2 * layers * KV_HEADS * NEW * D * 2
    print(f"kvr_shift_cache_layers: {us:.1f} us/launch, {algo / us / 1e3:.0f} GB/s on {algo} algorithmic bytes")


def copy(reps: int, tensors: int = 2 * LAYERS) -> None:
    """`tensors` 2 is the per-layer copy the refresh call makes; with fewer
    than 16 tensors each launch copies a different set of the 64, so the
    timed launches do not find their source in L2."""
    lib = _lib.load()
    src = [torch.randn(1, KV_HEADS, NEW, D, device="cuda").bfloat16() for _ in range(2 * LAYERS)]
    dst = [torch.empty_like(t) for t in src]
    stream = _lib.stream_handle()
    sets = max(1, 2 * LAYERS // tensors)
    args = [(_lib.ptr_array(src[i * tensors:(i + 1) * tensors]), _lib.ptr_array(dst[i * tensors:(i + 1) * tensors]),
             tensors, KV_HEADS, NEW, D, NEW * D, D, NEW * D, D, _lib.DTYPE_BF16, stream) for i in range(sets)]
    calls = iter(range(1 << 30))
    us = _time(lambda: _lib.check(lib.kvr_copy_layers(*args[next(calls) % sets]), "copy"), reps)
    algo = 2 * tensors * KV_HEADS * NEW * D * 2
    print(f"kvr_copy_layers: {us:.1f} us/launch, {algo / us / 1e3:.0f} GB/s on {algo} algorithmic bytes")


def attention(reps: int, precision: str, geometry: str = "config2") -> None:
    lib = _lib.load()
    positions, new = (_positions3(), NEW3) if geometry == "config3" else (_positions(), NEW)
    rows = len(positions)
    pos = torch.tensor(positions, device="cuda")
    q = (torch.randn(rows, HEADS, D, device="cuda") * 0.5).bfloat16()
    k = torch.randn(1, KV_HEADS, new, D, device="cuda").bfloat16()
    v = torch.randn(1, KV_HEADS, new, D, device="cuda").bfloat16()
    out = torch.empty_like(q)
    need = lib.kvr_attention_workspace_size(rows, HEADS, KV_HEADS, D, new)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    mode = _lib.ATTN_P_SPLIT if precision == "split" else _lib.ATTN_P_ROUNDED
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), pos.data_ptr(), rows, HEADS, KV_HEADS, D, new,
            new * D, D, positions[-1], D ** -0.5, mode, ws.data_ptr(), need, _lib.DTYPE_BF16)
    # Device time per call from a CUDA graph of back-to-back calls: a call's
    # host work (tensor maps, two launches) is longer than its kernels.
    us = _graph_time(lambda i: _lib.check(lib.kvr_selected_attention(*args, _lib.stream_handle()), "attention"), reps)
    kv = 2 * KV_HEADS * (positions[-1] + 1) * D * 2
    flops = 4.0 * HEADS * D * sum(p + 1 for p in positions)
    print(f"kvr_selected_attention ({precision}, {geometry}): {us:.1f} us/call, {kv / us / 1e3:.0f} GB/s of K/V, "
          f"{flops / us / 1e6:.1f} TFLOP/s; status {int(ws[:4].view(torch.int32).item())}")


HIDDEN, INTER, ROWS = 4096, 14336, 64


def _graph_time(fn, calls: int) -> float:
    """Average device time of `calls` back-to-back calls replayed from one
    CUDA graph (no host launch overhead in the measurement)."""
    for i in range(2):
        fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(calls):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    begin.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize()
    return begin.elapsed_time(end) / calls * 1e3


def linear(reps: int, only: str | None) -> None:
    lib = _lib.load()
    x = (torch.randn(ROWS, INTER, device="cuda") * 0.5).bfloat16()
    shapes = {  # name -> (k, [(n, paired)])
        "qkv": (HIDDEN, [(HEADS * D, False), (KV_HEADS * D, False), (KV_HEADS * D, False)]),
        "o": (HIDDEN, [(HIDDEN, False)]),
        "gate_up": (HIDDEN, [(INTER, True)]),
        "down": (INTER, [(HIDDEN, False)]),
    }
    for name, (k, spec) in shapes.items():
        if only and name != only:
            continue
        per_set = sum(n * k * 2 * (2 if paired else 1) for n, paired in spec)
        sets = max(1, -(-400_000_000 // per_set))  # > 3x L2 in rotation
        weights = [[(torch.randn(n, k, device="cuda").bfloat16(), torch.randn(n, k, device="cuda").bfloat16())
                    if paired else torch.randn(n, k, device="cuda").bfloat16() for n, paired in spec]
                   for _ in range(sets)]
        xi = x[:, :k]
        outs = [torch.empty(ROWS, n, device="cuda", dtype=torch.bfloat16) for n, _ in spec]
        segs = []
        for ws_set in weights:
            arr = (_lib.LinearSegment * len(spec))()
            for i, (w, out) in enumerate(zip(ws_set, outs)):
                gate, up = w if isinstance(w, tuple) else (w, None)
                arr[i] = _lib.LinearSegment(weight=gate.data_ptr(), weight_up=up.data_ptr() if up is not None else None,
                                            n=gate.shape[0], out=out.data_ptr(), out_stride=out.stride(0))
            segs.append(arr)
        need = lib.kvr_linear_workspace_size(ROWS, k, segs[0], len(spec))
        workspace = torch.empty(need, dtype=torch.uint8, device="cuda")

        def ours(i):
            _lib.check(lib.kvr_linear(xi.data_ptr(), xi.stride(0), ROWS, k, segs[i % sets], len(spec),
                                      workspace.data_ptr(), need, _lib.DTYPE_BF16, _lib.stream_handle()), "linear")

        def cublas(i):
            for w, out in zip(weights[i % sets], outs):
                if isinstance(w, tuple):
                    torch.mul(torch.nn.functional.silu(xi @ w[0].T), xi @ w[1].T, out=out)
                else:
                    torch.matmul(xi, w.T, out=out)

        us = _graph_time(ours, reps * sets)
        ref = _graph_time(cublas, reps * sets)
        print(f"kvr_linear {name}: {us:.1f} us/launch, {per_set / us / 1e3:.0f} GB/s of weights; "
              f"cuBLAS path {ref:.1f} us ({per_set / ref / 1e3:.0f} GB/s); "
              f"status {int(workspace[:4].view(torch.int32).item())}")


def relevance(reps: int) -> None:
    lib = _lib.load()
    vocab, hidden, n, nq = 151936, 4096, 31744, 8
    gen = torch.Generator(device="cuda").manual_seed(3)
    table = (torch.randn(vocab, hidden, device="cuda", generator=gen) * 0.02).bfloat16()
    prompt = torch.randint(0, vocab, (n,), device="cuda", generator=gen)
    query = torch.randint(0, vocab, (nq,), device="cuda", generator=gen)
    scores = torch.empty(n, device="cuda")
    need = lib.kvr_query_relevance_workspace_size(hidden, nq)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    us = _graph_time(lambda i: _lib.check(lib.kvr_query_relevance(
        table.data_ptr(), vocab, hidden, _lib.DTYPE_BF16, prompt.data_ptr(), n, query.data_ptr(), nq, 0.25,
        scores.data_ptr(), ws.data_ptr(), need, _lib.stream_handle()), "relevance"), reps)
    algo = n * hidden * 2
    print(f"kvr_query_relevance: {us:.1f} us/call, {algo / us / 1e3:.0f} GB/s of embedding rows ({algo} bytes)")


def refresh(reps: int, layers: int, projections: str, replay: bool = False) -> None:
    from transformers import LlamaConfig, LlamaForCausalLM

    from . import OperatorShim, engine, packed_interval_repair
    from .cache import make_cache

    config = LlamaConfig(vocab_size=128256, hidden_size=HIDDEN, intermediate_size=INTER, num_hidden_layers=layers,
                         num_attention_heads=HEADS, num_key_value_heads=KV_HEADS, head_dim=D, rope_theta=500000.0,
                         max_position_embeddings=131072, initializer_range=0.02)
    torch.manual_seed(1)
    previous = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device("cuda"):
            model = LlamaForCausalLM(config).eval()
    finally:
        torch.set_default_dtype(previous)
    gen = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(0, 128256, (1, NEW), device="cuda", generator=gen)
    base = make_cache([(torch.randn(1, KV_HEADS, NEW, D, device="cuda", generator=gen).bfloat16(),
                        torch.randn(1, KV_HEADS, NEW, D, device="cuda", generator=gen).bfloat16())
                       for _ in range(layers)])
    positions = _positions()
    intervals = []
    for p in positions:
        if intervals and p == intervals[-1][1]:
            intervals[-1] = (intervals[-1][0], p + 1)
        else:
            intervals.append((p, p + 1))
    engine.GRAPH_REPLAY = replay
    engine.PROJECTIONS = {"cublas": _lib.PROJ_CUBLAS, "sm100": _lib.PROJ_SM100, "fused": _lib.PROJ_FUSED}[projections]
    shim = OperatorShim(model)
    with torch.no_grad():
        for _ in range(4):  # graph replay: the first calls run directly, then capture
            packed_interval_repair(shim, base, ids, intervals)
        ms = _time(lambda: packed_interval_repair(shim, base, ids, intervals), reps) / 1e3
    how = "graph replay" if replay else "direct launches"
    print(f"packed_interval_repair ({projections}, {layers} layers, {how}): {ms:.3f} ms/call, "
          f"{ms / layers * 1e3:.1f} us/layer")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("kernel", choices=["shift", "attention", "copy", "linear", "relevance", "refresh"])
    parser.add_argument("--projections", choices=["cublas", "sm100", "fused"], default="fused",
                        help="refresh: projection path of the layer loop")
    parser.add_argument("--replay", action="store_true", help="refresh: replay repeated calls from a CUDA graph")
    parser.add_argument("--only", default=None, help="linear: one of qkv, o, gate_up, down")
    parser.add_argument("--reps", type=int, default=10)
    parser.add_argument("--layers", type=int, default=None,
                        help="shift: layers (32 by default; fewer for a small capture); refresh: layers (2)")
    parser.add_argument("--tensors", type=int, default=2 * LAYERS, help="copy: K/V tensors per launch (2 to 64)")
    parser.add_argument("--precision", choices=["rounded", "split"], default="rounded")
    parser.add_argument("--geometry", choices=["config2", "config3"], default="config2", help="attention geometry")
    args = parser.parse_args()
    build.build()
    if args.kernel == "shift":
        shift(args.reps, args.layers or LAYERS)
    elif args.kernel == "refresh":
        refresh(args.reps, args.layers or 2, args.projections, args.replay)
    elif args.kernel == "copy":
        copy(args.reps, args.tensors)
    elif args.kernel == "linear":
        linear(args.reps, args.only)
    elif args.kernel == "relevance":
        relevance(args.reps)
    else:
        attention(args.reps, args.precision, args.geometry)


if __name__ == "__main__":
    main()
