"""Packed refresh on the B200 against the reference's own outputs and the oracle."""

import pytest
import torch

from conftest import golden_cases, load_golden
from helpers import bits_equal, fixture_model, layers_cpu, oracle_config, to_cache
from oracle import packed_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
CASES = [n for n in golden_cases() if "fp32" not in n]


def _check_rows(actual_rows, expected_rows, what, min_cos=0.999):
    cos = oracle.row_cosine(actual_rows, expected_rows)
    assert cos.min() >= min_cos, (what, cos.min().item())
    err = (actual_rows.double() - expected_rows.double()).abs()
    bound = 2e-2 + 2e-2 * expected_rows.double().abs()
    assert (err <= bound).all(), (what, err.max().item())


@pytest.fixture(params=["cublas", "sm100", "fused"])
def projections(request, monkeypatch):
    """Both projection paths of the layer loop: cuBLAS and the kvr_linear kernel."""
    from budgeted_kv_cache_repair_b200 import _lib, engine

    monkeypatch.setattr(engine, "PROJECTIONS", {"cublas": _lib.PROJ_CUBLAS, "sm100": _lib.PROJ_SM100,
                                                "fused": _lib.PROJ_FUSED}[request.param])
    return request.param


@pytest.mark.parametrize("name", CASES)
def test_packed_matches_reference_outputs(name, projections):
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    record = load_golden(name)
    model = fixture_model(record, DEV)
    shim = OperatorShim(model)
    base = to_cache(record["shifted_layers"], DEV)
    snapshot = layers_cpu(base)
    ids = record["new_ids"].to(DEV)
    out, receipt = packed_interval_repair(shim, base, ids, record["intervals"])
    torch.cuda.synchronize()
    positions = record["positions"]
    got = layers_cpu(out)
    # Base untouched, storage independent, unselected rows bit-identical.
    for (bk, bv), (sk, sv) in zip(layers_cpu(base), snapshot):
        assert bits_equal(bk, sk) and bits_equal(bv, sv)
    keep = torch.ones(got[0][0].shape[2], dtype=torch.bool)
    keep[torch.tensor(positions)] = False
    for (k, v), (bk, bv) in zip(got, snapshot):
        assert bits_equal(k[:, :, keep], bk[:, :, keep]) and bits_equal(v[:, :, keep], bv[:, :, keep])
    from budgeted_kv_cache_repair_b200.validate import cache_layers
    for (k, v), (bk, bv) in zip(cache_layers(out), cache_layers(base)):
        assert k.untyped_storage().data_ptr() != bk.untyped_storage().data_ptr()
        assert v.untyped_storage().data_ptr() != bv.untyped_storage().data_ptr()
    # Refreshed rows vs the reference's packed SDPA path (run on CPU by make_golden).
    pos = torch.tensor(positions)
    for layer, ((k, v), (ek, ev)) in enumerate(zip(got, record["packed_rows"])):
        _check_rows(k[:, :, pos], ek, f"{name} K layer {layer}")
        _check_rows(v[:, :, pos], ev, f"{name} V layer {layer}")
    # ... and vs the oracle on the same inputs.
    ref_model = oracle.OracleModel.from_state_dict(record["state_dict"], oracle_config(record), record["inv_freq"])
    expected = oracle.packed_refresh(ref_model, snapshot, record["new_ids"], positions)
    _check_rows(oracle.fresh_rows(got, positions), oracle.fresh_rows(expected, positions), f"{name} vs oracle")
    assert receipt["recomputed_tokens"] == len(positions)
    assert receipt["selected_absolute_positions"] == positions
    assert receipt["output_cache_ownership"] == "independent"


@pytest.mark.parametrize("name", CASES)
def test_up_weights_below_gate_weights(name):
    """The gate and up projections run as one strided-batched GEMM whose
    batch 0 is the lower-addressed weight; models whose up weights sit below
    their gate weights in memory take the other order, with the same rows."""
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    record = load_golden(name)
    model = fixture_model(record, DEV)
    for layer in model.model.layers:
        gate, up = layer.mlp.gate_proj.weight, layer.mlp.up_proj.weight
        block = torch.empty((2,) + tuple(gate.shape), dtype=gate.dtype, device=gate.device)
        block[0].copy_(up.data)
        block[1].copy_(gate.data)
        up.data, gate.data = block[0], block[1]
        assert up.data_ptr() < gate.data_ptr()
    shim = OperatorShim(model)
    base = to_cache(record["shifted_layers"], DEV)
    snapshot = layers_cpu(base)
    out, _ = packed_interval_repair(shim, base, record["new_ids"].to(DEV), record["intervals"])
    torch.cuda.synchronize()
    positions = record["positions"]
    got = layers_cpu(out)
    pos = torch.tensor(positions)
    for layer, ((k, v), (ek, ev)) in enumerate(zip(got, record["packed_rows"])):
        _check_rows(k[:, :, pos], ek, f"{name} K layer {layer}")
        _check_rows(v[:, :, pos], ev, f"{name} V layer {layer}")
    ref_model = oracle.OracleModel.from_state_dict(record["state_dict"], oracle_config(record), record["inv_freq"])
    expected = oracle.packed_refresh(ref_model, snapshot, record["new_ids"], positions)
    _check_rows(oracle.fresh_rows(got, positions), oracle.fresh_rows(expected, positions), f"{name} vs oracle")


@pytest.mark.parametrize("name", CASES)
def test_scatter_matches_index_copy_of_the_engines_own_rows(name):
    """K/V written by the fused epilogue equal index_copy_ of the same rows."""
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    record = load_golden(name)
    model = fixture_model(record, DEV)
    base = to_cache(record["shifted_layers"], DEV)
    out, _ = packed_interval_repair(OperatorShim(model), base, record["new_ids"].to(DEV), record["intervals"])
    pos = torch.tensor(record["positions"], device=DEV)
    from budgeted_kv_cache_repair_b200.validate import cache_layers
    for (k, v), (bk, bv) in zip(cache_layers(out), cache_layers(base)):
        for got, src in ((k, bk), (v, bv)):
            expect = src.clone()
            expect.index_copy_(2, pos, got.index_select(2, pos))
            assert bits_equal(got, expect)


@pytest.mark.parametrize("name", CASES[:1])
@torch.no_grad()
def test_in_call_ownership_copy_matches_copy_then_refresh(name):
    """``refresh_rows(..., sources=)`` (the copy made inside the native call,
    per layer on a second stream) gives the same bits as a separate copy
    followed by an in-place refresh, for a strided source; with no rows it is
    exactly the copy."""
    from budgeted_kv_cache_repair_b200 import OperatorShim
    from budgeted_kv_cache_repair_b200.cache import allocate_layers, copy_layers
    from budgeted_kv_cache_repair_b200.engine import model_view, refresh_rows
    from budgeted_kv_cache_repair_b200.packed import _base_and_dtype
    from budgeted_kv_cache_repair_b200.plan import IndexedPlan

    record = load_golden(name)
    model = fixture_model(record, DEV)
    dense = to_cache(record["shifted_layers"], DEV)
    from budgeted_kv_cache_repair_b200.validate import cache_layers
    pairs = cache_layers(dense)
    length = pairs[0][0].shape[2]
    # Strided source: each layer is a prefix view of a longer buffer.
    src = []
    for k, v in pairs:
        wide_k = torch.zeros(1, k.shape[1], length + 24, k.shape[3], dtype=k.dtype, device=DEV)
        wide_v = torch.zeros_like(wide_k)
        wide_k[:, :, :length] = k
        wide_v[:, :, :length] = v
        src.append((wide_k[:, :, :length], wide_v[:, :, :length]))
    view = model_view(_base_and_dtype(OperatorShim(model), pairs, pairs[0][0].device))
    ids = record["new_ids"].to(DEV).reshape(-1)
    plan = IndexedPlan(record["positions"], length)
    positions = plan.to(DEV).positions
    heads, dim = pairs[0][0].shape[1], pairs[0][0].shape[3]

    expect = copy_layers(src)
    refresh_rows(view, expect, ids, positions, plan.max_position, length)
    got = allocate_layers(len(src), heads, length, dim, pairs[0][0].dtype, DEV)
    refresh_rows(view, got, ids, positions, plan.max_position, length, sources=src)
    torch.cuda.synchronize()
    for (gk, gv), (ek, ev) in zip(got, expect):
        assert bits_equal(gk, ek) and bits_equal(gv, ev)

    empty = allocate_layers(len(src), heads, length, dim, pairs[0][0].dtype, DEV)
    refresh_rows(view, empty, ids, positions[:0], plan.max_position, length, sources=src)
    torch.cuda.synchronize()
    for (gk, gv), (sk, sv) in zip(empty, src):
        assert bits_equal(gk, sk) and bits_equal(gv, sv)


@pytest.mark.parametrize("name", CASES)
def test_full_support_matches_clean_prefill(name):
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair

    record = load_golden(name)
    model = fixture_model(record, DEV)
    ids = record["new_ids"].to(DEV)
    base = to_cache(record["shifted_layers"], DEV)
    out, _ = packed_interval_repair(OperatorShim(model), base, ids, [(0, ids.shape[1])])
    with torch.no_grad():
        clean = model.model(input_ids=ids, use_cache=True).past_key_values
    got, exp = layers_cpu(out), layers_cpu(clean)
    rows = list(range(ids.shape[1]))
    _check_rows(oracle.fresh_rows(got, rows), oracle.fresh_rows(exp, rows), name)


@pytest.mark.parametrize("name", CASES)
def test_shift_cache_public_api(name):
    from budgeted_kv_cache_repair_b200 import OperatorShim, build_halo_cache

    record = load_golden(name)
    model = fixture_model(record, DEV)
    old = to_cache(record["old_layers"], DEV)
    shifted, alignment = build_halo_cache(OperatorShim(model), old, record["old_ids"].to(DEV),
                                          record["new_ids"].to(DEV), 0)
    for key in ("prefix", "suffix", "position_shift", "new_suffix_start"):
        assert alignment[key] == record["alignment"][key]
    for (k, v), (ek, ev) in zip(layers_cpu(shifted), record["shifted_layers"]):
        assert bits_equal(v, ev)
        # cos/sin come from the model's rotary module on the GPU; fp32 cos on
        # the GPU and CPU may differ in the last bit before the bf16 rounding.
        assert (k != ek).float().mean() < 1e-3
        assert oracle.row_cosine(k, ek).min() > 0.9999


def test_halo_recompute_matches_clean_prefill():
    """Changed tokens and a halo are recomputed over the prefix (cache.py:117-127)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from budgeted_kv_cache_repair_b200 import OperatorShim, build_halo_cache

    torch.manual_seed(9)
    config = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         max_position_embeddings=1024)
    model = LlamaForCausalLM(config).to(DEV, torch.bfloat16).eval()
    old_ids = torch.randint(0, 64, (1, 90), device=DEV)
    new_ids = torch.cat((old_ids[:, :30], torch.tensor([[7, 9]], device=DEV), old_ids[:, 41:]), dim=1)
    with torch.no_grad():
        old = model.model(input_ids=old_ids, use_cache=True).past_key_values
        clean = model.model(input_ids=new_ids, use_cache=True).past_key_values
    replay, meta = build_halo_cache(OperatorShim(model), old, old_ids, new_ids, halo_tokens=10**6)
    assert meta["recomputed_tokens"] == new_ids.shape[1] - meta["prefix"]
    rows = list(range(new_ids.shape[1]))
    _check_rows(oracle.fresh_rows(layers_cpu(replay), rows), oracle.fresh_rows(layers_cpu(clean), rows), "replay")
    shifted, meta = build_halo_cache(OperatorShim(model), old, old_ids, new_ids, 0)
    assert meta["mandatory_changed_tokens"] >= 2
    changed = list(range(meta["prefix"], meta["new_suffix_start"]))
    _check_rows(oracle.fresh_rows(layers_cpu(shifted), changed), oracle.fresh_rows(layers_cpu(clean), changed),
                "changed boundary tokens")


@pytest.mark.parametrize("name", ["api_llama_bfloat16.pt", "api_qwen3_bfloat16.pt"])
def test_repair_after_deletion_matches_reference_api(name):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast
    from budgeted_kv_cache_repair_b200 import repair_after_deletion

    record = load_golden(name)
    backend = Tokenizer(WordLevel({w: i for i, w in enumerate(record["words"])}, unk_token="[UNK]"))
    backend.pre_tokenizer = WhitespaceSplit()
    tokenizer = PreTrainedTokenizerFast(tokenizer_object=backend, unk_token="[UNK]")
    model = fixture_model(record, DEV)
    old = to_cache(record["old_layers"], DEV)
    snapshot = layers_cpu(old)

    def selector(model, tokenizer, text, query, ids, suffix_start, budget_percent):
        return record["positions"]  # the reference's SUR choice for this request

    result = repair_after_deletion(model, tokenizer, old, record["original_text"],
                                   delete_span=tuple(record["delete_span"]), query=record["query"],
                                   budget_percent=record["budget_percent"], selector=selector)
    assert result.edited_text == record["edited_text"]
    assert torch.equal(result.input_ids.cpu(), record["edited_ids"])
    assert list(result.selection.positions) == record["positions"]
    assert [tuple(i) for i in result.selection.intervals] == [tuple(i) for i in record["intervals"]]
    assert result.metadata["alignment"]["position_shift"] == record["alignment"]["position_shift"]
    for (k, v), (sk, sv) in zip(layers_cpu(old), snapshot):
        assert bits_equal(k, sk) and bits_equal(v, sv)
    got = layers_cpu(result.cache)
    rows = list(range(got[0][0].shape[2]))
    _check_rows(oracle.fresh_rows(got, rows), oracle.fresh_rows(record["cache"], rows), name)
