"""Host-side contract of the B200 engine (no GPU needed): C-ABI exports, plan
and interval rules against the reference's golden verdicts, fail-closed errors."""

import ctypes
import os
import re
from dataclasses import FrozenInstanceError

import numpy as np
import pytest
import torch

from conftest import ROOT, load_golden


@pytest.fixture(scope="module")
def built():
    from budgeted_kv_cache_repair_b200 import build

    return build.build()


def _header_symbols():
    text = open(os.path.join(ROOT, "include", "kvr_b200.h")).read()
    return sorted(set(re.findall(r"^KVR_API [^(]*?\b(kvr_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol(built):
    from budgeted_kv_cache_repair_b200 import _lib

    lib = ctypes.CDLL(built)
    names = _header_symbols()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must mirror the header"
    assert _lib.load().kvr_version().decode().startswith("kvr_b200")
    assert _lib.load().kvr_status_string(2).decode() == "unsupported shape or dtype"


def test_native_argument_checks_run_without_a_gpu(built):
    """Bad arguments are rejected on the host before any launch."""
    from budgeted_kv_cache_repair_b200 import _lib

    lib = _lib.load()
    assert lib.kvr_copy_layers(None, None, 1, 1, 1, 8, 8, 8, 8, 8, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_rope_shift_layers(None, None, 1, 1, 1, 96, 96, 96, 96, 96, None, 0, None) == _lib.ERR_UNSUPPORTED
    assert lib.kvr_selected_attention(None, None, None, None, None, 4, 3, 2, 128, 10, 1280, 128, 3, 1.0, 0, None, 0,
                                      0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_selected_attention(None, None, None, None, None, 4, 4, 2, 128, 10, 1280, 128, 3, 1.0, 7, None, 0,
                                      0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_silu_mul(None, None, None, 0, 16, 16, 16, 16, 7, None) == _lib.ERR_UNSUPPORTED
    # Empty work is a no-op success.
    assert lib.kvr_scatter_rows(None, None, None, None, None, 0, 1, 64, 9, 0, 0, 0, 0, None, 0, None) == _lib.OK
    seg = _lib.LinearSegment(weight=256, weight_up=None, n=128, out=512, out_stride=128)
    assert lib.kvr_linear(256, 64, 4, 60, ctypes.byref(seg), 1, 1024, 1 << 20, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_linear(256, 64, 4, 64, ctypes.byref(seg), 5, 1024, 1 << 20, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_linear(256, 64, 4, 64, ctypes.byref(seg), 1, 1024, 1 << 20, 9, None) == _lib.ERR_UNSUPPORTED
    assert lib.kvr_linear(None, 64, 0, 64, ctypes.byref(seg), 1, None, 0, 0, None) == _lib.OK
    # fewer tiles than SMs: split-K in clusters, status word only
    assert lib.kvr_linear_workspace_size(64, 64, ctypes.byref(seg), 1) == 256
    # 224 gated tiles: 148 whole tiles, 76 tiles x 64 k-chunks stream-K over 148 CTAs
    # -> status + 76 counters (304 bytes -> 512) + 148 CTAs x 2 slots x 64 x 128 fp32
    gated = _lib.LinearSegment(weight=256, weight_up=256, n=14336, out=512, out_stride=14336)
    assert lib.kvr_linear_workspace_size(64, 4096, ctypes.byref(gated), 1) == 256 + 512 + 148 * 2 * 64 * 128 * 4
    assert lib.kvr_attention_workspace_size(64, 32, 8, 128, 7936) > 0
    assert lib.kvr_attention_workspace_size(20000, 32, 8, 128, 7936) == 256  # enough tiles: status word only
    assert lib.kvr_rope_tables(None, 64, None, 4, 1.0, None, None, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_rope_tables(256, 64, 256, 4, 1.0, 256, 256, 5, None) == _lib.ERR_INVALID_ARG
    assert lib.kvr_rope_tables(256, 64, 256, 0, 1.0, 256, 256, 0, None) == _lib.OK  # no rows: no launch
    # No graph was made in this process: releasing is a no-op and nothing replayed.
    assert lib.kvr_release_graphs() == _lib.OK
    assert lib.kvr_graph_replays() == 0


def test_refresh_request_source_cache_checks_run_without_a_gpu(built):
    """The ownership-copy fields of the refresh request: K and V sources come
    together, one per layer, or the call fails before any launch."""
    from budgeted_kv_cache_repair_b200 import _lib

    lib = _lib.load()
    fake = 1 << 20  # never dereferenced: every case fails host-side validation
    layers = (_lib.LayerWeights * 2)(*[_lib.LayerWeights(input_norm=fake, qkv=fake, o=fake, post_norm=fake,
                                                        gate=fake, up=fake, down=fake) for _ in range(2)])
    model = _lib.Model(num_layers=2, hidden=64, q_heads=4, kv_heads=2, head_dim=64, intermediate=128, vocab=256,
                       eps=1e-5, dtype=_lib.DTYPE_BF16, embed=fake, layers=layers)
    ptrs = _lib.ptr_array([fake, fake])

    def request(**kw):
        base = dict(k_cache=ptrs, v_cache=ptrs, cache_rows=16, cache_head_stride=16 * 64, cache_row_stride=64,
                    rows=0, projections=_lib.PROJ_CUBLAS)
        base.update(kw)
        return _lib.RefreshRequest(**base)

    def call(req):
        return lib.kvr_packed_refresh(ctypes.byref(model), ctypes.byref(req), None, 0, None)

    assert call(request()) == _lib.OK  # no rows and no sources: nothing to do
    assert call(request(k_src=ptrs)) == _lib.ERR_INVALID_ARG  # V sources missing
    assert call(request(v_src=ptrs)) == _lib.ERR_INVALID_ARG  # K sources missing
    holes = _lib.ptr_array([fake, 0])
    assert call(request(k_src=ptrs, v_src=holes)) == _lib.ERR_INVALID_ARG  # a layer without a source


def test_alignment_matches_reference():
    from budgeted_kv_cache_repair_b200 import token_alignment

    for case in load_golden("alignment.pt"):
        assert token_alignment(case["old"], case["new"]) == case["expected"]


def test_plan_tiles_and_interval_rules_match_reference():
    from budgeted_kv_cache_repair_b200 import IndexedPlan, positions_to_intervals
    from budgeted_kv_cache_repair_b200.validate import validate_intervals

    golden = load_golden("plans.pt")
    for plan in golden["plans"]:
        ours = IndexedPlan(plan["positions"], plan["length"])
        assert ours.full_prefix_tiles == tuple(plan["full"]) and ours.total_tiles == tuple(plan["total"])
        assert positions_to_intervals(plan["positions"]) == [tuple(x) for x in plan["intervals"]]
    for verdict in golden["interval_verdicts"]:
        if verdict["ok"]:
            assert [list(x) for x in validate_intervals(verdict["intervals"], verdict["length"])] == \
                   [list(x) for x in verdict["result"]]
        else:
            with pytest.raises(ValueError):
                validate_intervals(verdict["intervals"], verdict["length"])


def test_host_plan_owns_immutable_sorted_metadata():
    from budgeted_kv_cache_repair_b200 import IndexedPlan

    positions = [3, 4, 8, 9]
    plan = IndexedPlan(positions, 10)
    positions[0] = 0
    assert plan.positions == (3, 4, 8, 9) and plan.max_position == 9
    with pytest.raises(FrozenInstanceError):
        plan.logical_length = 12


@pytest.mark.parametrize("positions,length", [
    ([2, 1], 4), ([1, 1], 4), ([-1], 4), ([4], 4), ([True], 4), ([1.0], 4), (torch.tensor([1]), 4),
    ([0], -1), ([], True), ([], 4.0), ([], 1 << 63), (None, 4),
])
def test_invalid_host_plans_fail_before_any_device_operation(positions, length):
    from budgeted_kv_cache_repair_b200 import IndexedPlan

    with pytest.raises(ValueError):
        IndexedPlan(positions, length)


def test_host_plan_upload_rejects_cpu():
    from budgeted_kv_cache_repair_b200 import IndexedPlan

    with pytest.raises(ValueError, match="CUDA"):
        IndexedPlan([0], 1).to("cpu")


def test_operators_reject_cpu_without_fallback():
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention, indexed_kv_scatter_
    from budgeted_kv_cache_repair_b200.cache import copy_layers

    q = torch.zeros((1, 1, 1, 64), dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        indexed_causal_attention(q, q, q, IndexedPlan([0], 1))
    with pytest.raises(ValueError, match="CUDA"):
        indexed_kv_scatter_(q, q, q, q, IndexedPlan([0], 1))
    with pytest.raises(ValueError, match="CUDA"):
        copy_layers([(q, q)])


def _tiny_model(family="llama"):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM

    options = dict(vocab_size=97, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                   num_attention_heads=4, num_key_value_heads=2, head_dim=8, max_position_embeddings=64)
    torch.manual_seed(71)
    if family == "llama":
        return LlamaForCausalLM(LlamaConfig(**options)).eval()
    return Qwen3ForCausalLM(Qwen3Config(**options, layer_types=["full_attention"] * 2)).eval()


def _request(model, length=12):
    from budgeted_kv_cache_repair_b200 import OperatorShim

    ids = (torch.arange(length) % 60 + 4).unsqueeze(0)
    with torch.no_grad():
        base = model(input_ids=ids, use_cache=True).past_key_values
    return OperatorShim(model), ids, base


def test_empty_support_returns_base_and_does_no_work(monkeypatch):
    import budgeted_kv_cache_repair_b200.packed as packed
    from budgeted_kv_cache_repair_b200 import IndexedPlan, packed_interval_repair
    from budgeted_kv_cache_repair_b200.cache import make_cache

    def forbidden(*args, **kwargs):
        raise AssertionError("empty support must not prepare or execute work")

    monkeypatch.setattr(packed, "qualify_model", forbidden)
    monkeypatch.setattr(packed, "refresh_rows", forbidden)
    monkeypatch.setattr(packed, "allocate_arena", forbidden)
    monkeypatch.setattr(IndexedPlan, "to", forbidden)
    base = make_cache([(torch.zeros(1, 2, 0, 8), torch.zeros(1, 2, 0, 8)) for _ in range(2)])
    actual, receipt = packed_interval_repair(object(), base, torch.empty((1, 0), dtype=torch.long), [])
    assert actual is base
    assert receipt["output_cache_ownership"] == "borrowed_base"
    assert receipt["recomputed_tokens"] == 0


def test_receipt_keys_match_reference():
    from budgeted_kv_cache_repair_b200.packed import make_receipt

    golden = load_golden("case_cfg0_llama_fp32.pt")["receipt"]
    ours = make_receipt([(50, 54)], golden["logical_length"], golden["layer_count"])
    for key, value in golden.items():
        assert ours[key] == value, key
    assert ours["engine"].startswith("kvr_b200")


@pytest.mark.parametrize("fault", ["attention_backend", "writeback_backend", "interval", "ids_rank", "ids_dtype",
                                   "cache_length", "plan", "cpu_cache"])
def test_fail_closed_contract_before_device_work(fault):
    from budgeted_kv_cache_repair_b200 import IndexedPlan, packed_interval_repair

    model = _tiny_model()
    shim, ids, base = _request(model)
    kwargs, intervals = {}, [(3, 5)]
    if fault == "attention_backend":
        kwargs["attention_backend"] = "triton"
    elif fault == "writeback_backend":
        kwargs["writeback_backend"] = "triton"
    elif fault == "interval":
        intervals = [(3, 5), (5, 6)]
    elif fault == "ids_rank":
        ids = ids[0]
    elif fault == "ids_dtype":
        ids = ids.float()
    elif fault == "cache_length":
        ids = ids[:, :-1]
    elif fault == "plan":
        kwargs["plan"] = IndexedPlan((3,), 12)
    with pytest.raises(ValueError):
        packed_interval_repair(shim, base, ids, intervals, **kwargs)


def test_api_validates_before_work():
    from budgeted_kv_cache_repair_b200 import repair_after_deletion, select_support
    from budgeted_kv_cache_repair_b200.api import budget_tokens

    model = _tiny_model()
    for bad in (True, -1, 101, float("nan")):
        with pytest.raises(ValueError):
            repair_after_deletion(model, None, None, "abc", delete_span=(0, 1), query="", budget_percent=bad)
    with pytest.raises(ValueError):
        repair_after_deletion(model, None, None, "abc", delete_span=(2, 1), query="")
    with pytest.raises(ValueError):
        repair_after_deletion(model, None, None, "abc", delete_span=(0, 1), query="", executor="other")
    with pytest.raises(ValueError, match="CUDA"):
        repair_after_deletion(model, None, None, "abc", delete_span=(0, 1), query="")
    assert budget_tokens(3, 5) == 1 and budget_tokens(100, 2) == 2 and budget_tokens(72, 5) == 4
    assert budget_tokens(0, 50) == 0 and budget_tokens(10, 100) == 10


def test_shift_cache_host_path_rejects_cpu_caches():
    from budgeted_kv_cache_repair_b200 import build_halo_cache

    model = _tiny_model()
    shim, ids, base = _request(model)
    with pytest.raises(ValueError, match="CUDA"):
        build_halo_cache(shim, base, ids, ids[:, 2:], 0)


def test_rotate_half_uses_split_half_convention():
    from budgeted_kv_cache_repair_b200 import rotate_half

    assert rotate_half(torch.tensor([1.0, 2.0, 3.0, 4.0])).tolist() == [-3.0, -4.0, 1.0, 2.0]


def test_dynamic_cache_construction_keeps_storage():
    from budgeted_kv_cache_repair_b200.cache import make_cache
    from budgeted_kv_cache_repair_b200.validate import cache_layers

    pairs = [(torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8)) for _ in range(3)]
    cache = make_cache(pairs)
    assert cache.get_seq_length() == 5 and len(cache_layers(cache)) == 3
    for (k, v), (k2, v2) in zip(pairs, cache_layers(cache)):
        assert k is k2 and v is v2


def _model_fault(model, fault):
    """The reference's contract faults (tests/test_packed_cache.py:255-288),
    plus a float32 model, which the B200 engine does not compute in."""
    from transformers import LlamaForCausalLM

    if fault == "class":
        class CustomLlama(LlamaForCausalLM):
            pass

        model.__class__ = CustomLlama
    elif fault == "training":
        model.train()
    elif fault == "rope":
        model.config.rope_scaling = {"rope_type": "dynamic", "factor": 2.0}
    elif fault == "sliding":
        model.config.layer_types = ["full_attention", "sliding_attention"]
    elif fault == "base_forward":
        model.model.forward = lambda **kwargs: None
    elif fault == "activation":
        model.config.hidden_act = "gelu"
    elif fault == "dtype":
        model.float()
    return model


@pytest.mark.parametrize("fault,match", [("class", "native dense"), ("training", "eval"), ("rope", "RoPE"),
                                         ("sliding", "full attention"), ("activation", "SiLU")])
def test_api_rejects_unsupported_models_before_any_device_work(fault, match):
    """repair_after_deletion checks the model class, mode, RoPE type,
    attention kind and MLP before it tokenises, shifts or selects anything
    (api.py:135-166): the library launches nothing and the tokenizer is never
    called."""
    from budgeted_kv_cache_repair_b200 import _lib, repair_after_deletion

    model = _model_fault(_tiny_model().to(torch.bfloat16), fault)

    def tokenizer(*args, **kwargs):
        raise AssertionError("the model contract must be checked before tokenisation")

    launches = _lib.load().kvr_kernel_launches()
    with pytest.raises(ValueError, match=match):
        repair_after_deletion(model, tokenizer, None, "abcdef", delete_span=(1, 2), query="q")
    assert _lib.load().kvr_kernel_launches() == launches



def _view_model():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(5)
    config = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                         num_attention_heads=2, num_key_value_heads=1, head_dim=64, max_position_embeddings=64)
    return LlamaForCausalLM(config).to(torch.bfloat16).eval()


def test_model_view_follows_replaced_parameter_objects():
    """A parameter object swapped anywhere in the decoder (not an in-place
    change, and not only in the first layer) rebuilds the engine's cached
    view, so no call computes with the old tensor; layers whose q/k/v are
    unchanged keep their stacked q/k/v copy."""
    from budgeted_kv_cache_repair_b200.engine import model_view

    model = _view_model()
    base = model.model
    view = model_view(base)
    assert model_view(base) is view
    stacked = view.layers[0].fused_qkv()
    down = base.layers[1].mlp.down_proj
    down.weight = torch.nn.Parameter(torch.zeros_like(down.weight))
    again = model_view(base)
    assert again is not view
    assert again.layers[1].down is down.weight
    assert again.layers[0].fused_qkv() is stacked
    assert model_view(base) is again


def test_model_contract_sees_parameter_objects_replaced_between_calls():
    """The per-call model checks re-collect the parameters once one was
    replaced after an earlier call: a replacement in the wrong dtype is
    rejected."""
    from budgeted_kv_cache_repair_b200.validate import qualify_model

    model = _view_model()
    base = model.model
    qualify_model(model, base, 2, torch.device("cpu"), torch.bfloat16)
    up = base.layers[0].mlp.up_proj
    up.weight = torch.nn.Parameter(up.weight.detach().float())
    with pytest.raises(ValueError, match="dtype"):
        qualify_model(model, base, 2, torch.device("cpu"), torch.bfloat16)


def test_registration_count_ignores_unwatched_and_unhashable_modules():
    """The registration hooks count only modules of models the engine has
    cached, and never fail another module's registration (a module class
    with ``__eq__`` and no ``__hash__`` is unhashable)."""
    from budgeted_kv_cache_repair_b200 import registry

    class Unhashable(torch.nn.Module):
        def __eq__(self, other):
            return self is other

        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(2, 2)
            self.w = torch.nn.Parameter(torch.zeros(1))

    before = registry.epoch()
    Unhashable()
    torch.nn.Linear(3, 3)
    assert registry.epoch() == before


def test_module_checks_see_hooks_forwards_and_modes_set_after_a_cached_scan():
    """The per-call module checks (kernels/packed_cache.py:123-163) run on a
    scan cached across calls: a dispatch hook, a per-instance forward or train
    mode set after the scan was built (no registration, so the scan is reused)
    is still rejected, and a hook attribute that is None is not a hook."""
    from budgeted_kv_cache_repair_b200 import validate

    model = _tiny_model().to(torch.bfloat16).eval()
    base = model.model
    cpu = torch.device("cpu")
    validate._check_modules(model, base, cpu, torch.bfloat16)  # builds and caches the scan
    scan = validate._scans[model]
    mlp = base.layers[1].mlp
    mlp._hf_hook = None
    validate._check_modules(model, base, cpu, torch.bfloat16)
    mlp._hf_hook = object()
    with pytest.raises(ValueError, match="hooks"):
        validate._check_modules(model, base, cpu, torch.bfloat16)
    del mlp._hf_hook
    base.layers[0].self_attn.forward = lambda *args, **kwargs: None
    with pytest.raises(ValueError, match="forward overrides"):
        validate._check_modules(model, base, cpu, torch.bfloat16)
    del base.layers[0].self_attn.forward
    base.norm.train()
    with pytest.raises(ValueError, match="eval mode"):
        validate._check_modules(model, base, cpu, torch.bfloat16)
    base.norm.eval()
    validate._check_modules(model, base, cpu, torch.bfloat16)
    assert validate._scans[model] is scan


@pytest.mark.parametrize("shape, contiguous", [((3, 1, 2, 4, 8), True), ((4, 2, 2, 4, 8), True),
                                               ((4, 1, 2, 4, 8), False), ((2, 2, 4, 8), True)])
def test_refresh_rejects_malformed_output_arenas(shape, contiguous):
    """An output block passed as one tensor must be a contiguous
    [2L, 1, heads, rows, head_dim] arena (K of layer l at 2l, V at 2l + 1):
    anything else raises ValueError before any device work."""
    from budgeted_kv_cache_repair_b200 import _lib
    from budgeted_kv_cache_repair_b200.engine import refresh_rows

    arena = torch.empty(shape, dtype=torch.bfloat16)
    if not contiguous:
        arena = torch.empty(shape[:-1] + (2 * shape[-1],), dtype=torch.bfloat16)[..., : shape[-1]]
    ids = torch.empty(6, dtype=torch.int64, device="meta")
    launches = _lib.load().kvr_kernel_launches()
    with pytest.raises(ValueError, match="arena"):
        refresh_rows(None, arena, ids, [1, 2], 2, shape[-2])
    assert _lib.load().kvr_kernel_launches() == launches


@pytest.mark.parametrize("intervals, ok", [
    ([(1, 3), (5, 9)], True),
    ([[1, 3], [5, 9]], True),
    ([(np.int64(1), np.int64(3)), (5, np.int32(9))], True),
    ([(True, 3)], False),
    ([(1, False)], False),
    ([(1.0, 3)], False),
    ([(1, 3), (3, 5)], False),
    ([(2, 2)], False),
])
def test_interval_bound_types_follow_the_reference(intervals, ok):
    """Plain-int bounds take a fast path; NumPy integers, booleans and floats
    take the general one. Either way the verdict, the returned bounds and their
    Python int type are the reference's (kernels/executor.py:50-70)."""
    from budgeted_kv_cache_repair_b200.validate import validate_intervals
    from oracle import packed_oracle as oracle

    if ok:
        ours = validate_intervals(intervals, 16)
        assert [list(x) for x in ours] == [list(x) for x in oracle.validate_intervals(intervals, 16)]
        assert all(type(v) is int for pair in ours for v in pair)
    else:
        with pytest.raises(ValueError):
            oracle.validate_intervals(intervals, 16)
        with pytest.raises(ValueError):
            validate_intervals(intervals, 16)


def test_native_weight_struct_follows_storage_and_qkv_versions():
    """The weight struct handed to the native refresh is rebuilt exactly when
    a weight's storage moved (`.data` reassigned, the same parameter object)
    or q/k/v changed in place (their stacked copy is the engine's); other
    in-place changes keep it, since the kernels read those weights through
    their own storage."""
    from budgeted_kv_cache_repair_b200.engine import _native_model, model_view

    model = _view_model()
    view = model_view(model.model)
    first = _native_model(view)
    assert _native_model(view) is first
    layer = model.model.layers[1]
    with torch.no_grad():
        layer.mlp.up_proj.weight.mul_(2.0)  # in place, not q/k/v: same struct
    assert _native_model(view) is first
    with torch.no_grad():
        layer.self_attn.v_proj.weight.add_(1.0)  # q/k/v in place: a new stacked copy
    second = _native_model(view)
    assert second is not first
    stacked = view.layers[1].qkv
    assert torch.equal(stacked[-layer.self_attn.v_proj.weight.shape[0]:], layer.self_attn.v_proj.weight)
    layer.mlp.gate_proj.weight.data = layer.mlp.gate_proj.weight.data.clone()  # storage moved, no registration
    third = _native_model(view)
    assert third is not second
    assert third.layers[1].gate == layer.mlp.gate_proj.weight.data_ptr()


def test_arena_layers_are_views_in_layer_order():
    """allocate_arena's block holds K of layer l at 2l and V at 2l + 1; the
    pairs arena_layers returns are [1, heads, rows, dim] views of it, each
    contiguous, sharing the block's storage."""
    from budgeted_kv_cache_repair_b200.cache import allocate_arena, arena_layers

    arena = allocate_arena(3, 2, 5, 8, torch.bfloat16, torch.device("cpu"))
    assert arena.shape == (6, 1, 2, 5, 8) and arena.is_contiguous()
    pairs = arena_layers(arena)
    assert len(pairs) == 3
    plane = 2 * 5 * 8 * arena.element_size()
    for l, (k, v) in enumerate(pairs):
        assert k.shape == v.shape == (1, 2, 5, 8) and k.is_contiguous() and v.is_contiguous()
        assert k.data_ptr() == arena.data_ptr() + 2 * l * plane
        assert v.data_ptr() == arena.data_ptr() + (2 * l + 1) * plane
        assert k.untyped_storage().data_ptr() == arena.untyped_storage().data_ptr()
