"""Failure handling on the GPU, with no GPU fault involved.

* A refresh that fails part-way (an injected error status after layer k's
  cache write, as a CUDA call failing mid-call would end it) raises, returns
  no cache, and leaves the base cache, the model and a following refresh
  untouched: the reference's transaction test
  (tests/test_packed_cache.py:227-252) restated for the native loop.
* The model contract faults of the reference's fail-closed matrix
  (tests/test_packed_cache.py:255-288: class, base forward, training, rope,
  sliding) raise ValueError on a CUDA model before any kernel is launched.
* Bounded device waits: with the pipeline wait limit cut to one SM clock, the
  attention and projection kernels give up, record an error code in their
  workspace status word, drain their own copies, free tensor memory and
  return; with the default limit restored, the next calls on the same context
  are correct.
"""

import pytest
import torch

from conftest import load_golden
from helpers import bits_equal, fixture_model, layers_cpu, to_cache
from oracle import packed_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
CASE = "case_llama_fp16_d128.pt"


def _lib():
    from budgeted_kv_cache_repair_b200 import _lib as lib

    lib.load()
    return lib


def _params(model):
    return {name: p.detach().clone() for name, p in model.named_parameters()}


@pytest.mark.parametrize("layer", [0, 1])
def test_refresh_failing_part_way_leaves_base_model_and_next_call_untouched(layer):
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    lib = _lib()
    record = load_golden(CASE)
    model = fixture_model(record, DEV)
    assert layer < model.config.num_hidden_layers
    shim = OperatorShim(model)
    base = to_cache(record["shifted_layers"], DEV)
    snapshot = layers_cpu(base)
    params = _params(model)
    config = model.config.to_dict()
    ids = record["new_ids"].to(DEV)
    clean, _ = packed_interval_repair(shim, base, ids, record["intervals"])
    clean = layers_cpu(clean)

    lib.check(lib.load().kvr_debug_fail_refresh_after_layer(layer), "arm")
    try:
        with pytest.raises(RuntimeError, match="injected"):
            packed_interval_repair(shim, base, ids, record["intervals"])
    finally:
        lib.load().kvr_debug_fail_refresh_after_layer(-1)
    torch.cuda.synchronize()
    for (k, v), (sk, sv) in zip(layers_cpu(base), snapshot):
        assert bits_equal(k, sk) and bits_equal(v, sv)
    assert model.config.to_dict() == config
    for name, p in model.named_parameters():
        assert bits_equal(p.detach(), params[name]), name

    again, _ = packed_interval_repair(shim, base, ids, record["intervals"])
    for (k, v), (ck, cv) in zip(layers_cpu(again), clean):
        assert bits_equal(k, ck) and bits_equal(v, cv)


def _fault(model, fault):
    from transformers import LlamaForCausalLM

    if fault == "class":
        class CustomLlama(LlamaForCausalLM):
            pass

        model.__class__ = CustomLlama
    elif fault == "base_forward":
        model.model.forward = lambda **kwargs: None
    elif fault == "training":
        model.train()
    elif fault == "rope":
        model.config.rope_scaling = {"rope_type": "dynamic", "factor": 2.0}
    elif fault == "sliding":
        model.config.layer_types = ["full_attention"] + ["sliding_attention"] * (model.config.num_hidden_layers - 1)
    elif fault == "activation":
        model.config.hidden_act = "gelu"


@pytest.mark.parametrize("fault", ["class", "base_forward", "training", "rope", "sliding", "activation"])
def test_packed_contract_faults_fail_closed_before_any_kernel(fault):
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    lib = _lib()
    record = load_golden(CASE)
    model = fixture_model(record, DEV)
    _fault(model, fault)
    base = to_cache(record["shifted_layers"], DEV)
    snapshot = layers_cpu(base)
    torch.cuda.synchronize()
    launches = lib.load().kvr_kernel_launches()
    with pytest.raises(ValueError):
        packed_interval_repair(OperatorShim(model), base, record["new_ids"].to(DEV), record["intervals"])
    assert lib.load().kvr_kernel_launches() == launches
    for (k, v), (sk, sv) in zip(layers_cpu(base), snapshot):
        assert bits_equal(k, sk) and bits_equal(v, sv)


def _attention_call(lib, seed):
    """kvr_selected_attention at the Llama-3-8B geometry over 7936 keys (the
    key range is split, so the combine launch runs too)."""
    L = lib.load()
    rows, heads, kv, d, n = 64, 32, 8, 128, 7936
    gen = torch.Generator().manual_seed(seed)
    positions = sorted(torch.randperm(n, generator=gen)[:rows].tolist())
    q = (torch.randn(rows, heads, d, generator=gen) * 0.5).bfloat16().to(DEV)
    k = torch.randn(1, kv, n, d, generator=gen).bfloat16().to(DEV)
    v = (torch.randn(1, kv, n, d, generator=gen) * 0.5).bfloat16().to(DEV)
    pos = torch.tensor(positions, device=DEV)
    out = torch.zeros_like(q)
    need = L.kvr_attention_workspace_size(rows, heads, kv, d, n)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)

    def run():
        lib.check(L.kvr_selected_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), pos.data_ptr(),
                                           rows, heads, kv, d, n, n * d, d, positions[-1], d ** -0.5,
                                           lib.ATTN_P_ROUNDED, ws.data_ptr(), need, lib.DTYPE_BF16,
                                           lib.stream_handle()), "attention")
        torch.cuda.synchronize()
        return int(ws[:4].view(torch.int32).item())

    def expected():
        return oracle.selected_attention_fp64(q.permute(1, 0, 2)[None].cpu(), k.cpu(), v.cpu(), positions)

    return run, out, expected


def test_attention_wait_limit_gives_up_with_a_status_and_the_context_recovers():
    lib = _lib()
    L = lib.load()
    run, out, expected = _attention_call(lib, 5)
    lib.check(L.kvr_set_wait_limit(1), "wait limit")
    try:
        status = run()
    finally:
        lib.check(L.kvr_set_wait_limit(0), "wait limit")
    assert status != 0  # a pipeline wait gave up and said so
    assert run() == 0
    torch.testing.assert_close(out.permute(1, 0, 2)[None].double().cpu(), expected(), atol=0.002, rtol=0.02)
    run2, out2, expected2 = _attention_call(lib, 6)
    assert run2() == 0
    torch.testing.assert_close(out2.permute(1, 0, 2)[None].double().cpu(), expected2(), atol=0.002, rtol=0.02)


@pytest.mark.parametrize("n", [4096, 28672])
def test_linear_wait_limit_gives_up_with_a_status_and_the_context_recovers(n):
    """kvr_linear with the limit cut: split-K clusters (n = 4096: 32 tiles) or
    the persistent stream-K grid (n = 28672, a gated pair: 224 tiles)."""
    lib = _lib()
    L = lib.load()
    rows, k = 64, 4096
    gen = torch.Generator().manual_seed(n)
    x = torch.randn(rows, k, generator=gen).bfloat16().to(DEV)
    paired = n == 28672
    width = n // 2 if paired else n
    w = (torch.randn(width, k, generator=gen) * 0.02).bfloat16().to(DEV)
    w_up = (torch.randn(width, k, generator=gen) * 0.02).bfloat16().to(DEV) if paired else None
    out = torch.zeros(rows, width, dtype=torch.bfloat16, device=DEV)
    seg = lib.LinearSegment(w.data_ptr(), w_up.data_ptr() if paired else None, width, out.data_ptr(), width)
    need = L.kvr_linear_workspace_size(rows, k, seg, 1)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)

    def run():
        lib.check(L.kvr_linear(x.data_ptr(), k, rows, k, seg, 1, ws.data_ptr(), need, lib.DTYPE_BF16,
                               lib.stream_handle()), "linear")
        torch.cuda.synchronize()
        return int(ws[:4].view(torch.int32).item())

    lib.check(L.kvr_set_wait_limit(1), "wait limit")
    try:
        status = run()
    finally:
        lib.check(L.kvr_set_wait_limit(0), "wait limit")
    assert status != 0
    assert run() == 0
    ref = x.float() @ w.float().t()
    if paired:
        ref = torch.nn.functional.silu(ref.bfloat16().float()).bfloat16().float() * \
            (x.float() @ w_up.float().t()).bfloat16().float()
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
