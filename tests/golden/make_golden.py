"""Generate the golden fixtures in this directory from the upstream reference.

    python tests/golden/make_golden.py --reference <checkout of yh0903/budgeted-kv-cache-repair>

Runs the reference's own functions (through ``ref_compat.load_reference``) on
CPU with seeded tiny models and records inputs and outputs:

* ``alignment.pt``   token_alignment (alignment.py:21-30) on fixed and random id pairs
* ``plans.pt``       IndexedPlan tiles (kernels/indexed_attention.py:56-83) and
                     _validate_intervals verdicts (kernels/executor.py:50-70)
* ``rope_shift.pt``  shifted_suffix_keys (cache.py:47-77) on bf16/fp16 keys
* ``case_*.pt``      prefill cache, build_halo_cache (cache.py:103-144), and
                     packed_interval_repair / sequential_repair outputs
                     (kernels/packed_cache.py:225-298, execution.py:34-59)
* ``api_*.pt``       repair_after_deletion(executor="packed") (api.py:169-244)
                     with a word-level tokenizer, incl. its SUR selection

The model weights are stored with each case, so the fixtures do not depend on
torch's RNG reproducing them elsewhere. Nothing at test time reads the
reference; the tests read only these files.
"""

from __future__ import annotations

import argparse
import os
import random
import sys
from types import SimpleNamespace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from ref_compat import load_reference  # noqa: E402


def _layers(cache):
    return [(k.clone(), v.clone()) for k, v in ((layer.keys, layer.values) for layer in cache.layers)]


def _model(family, *, hidden, inter, layers, heads, kv_heads, head_dim, vocab, theta, dtype, seed):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM

    options = dict(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                   num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                   head_dim=head_dim, max_position_embeddings=4096, attention_dropout=0.0,
                   rope_theta=theta, initializer_range=0.02)
    torch.manual_seed(seed)
    if family == "llama":
        model = LlamaForCausalLM(LlamaConfig(**options))
    else:
        model = Qwen3ForCausalLM(Qwen3Config(**options, layer_types=["full_attention"] * layers))
    model = model.to(dtype=dtype).eval()
    return model


def _config_record(model):
    cfg = model.config
    return dict(family="llama" if "Llama" in type(model).__name__ else "qwen3",
                vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                head_dim=cfg.head_dim, rope_theta=float(cfg.rope_parameters["rope_theta"]),
                rms_norm_eps=cfg.rms_norm_eps)


def make_case(kvr, name, family, dtype, *, seed, hidden, inter, heads, kv_heads, head_dim,
              vocab, theta, length, delete, intervals, layers=2):
    from kv_cache_repair.cache import OperatorShim, build_halo_cache
    from kv_cache_repair.execution import sequential_repair
    from kv_cache_repair.kernels.packed_cache import packed_interval_repair

    model = _model(family, hidden=hidden, inter=inter, layers=layers, heads=heads, kv_heads=kv_heads,
                   head_dim=head_dim, vocab=vocab, theta=theta, dtype=dtype, seed=seed)
    gen = torch.Generator().manual_seed(seed + 1000)
    old_ids = torch.randint(0, vocab, (1, length), generator=gen)
    start, stop = delete
    new_ids = torch.cat((old_ids[:, :start], old_ids[:, stop:]), dim=1)
    shim = OperatorShim(model, SimpleNamespace())
    with torch.no_grad():
        old_cache = model.model(input_ids=old_ids, use_cache=True).past_key_values
    old_layers = _layers(old_cache)
    shifted, alignment = build_halo_cache(shim, old_cache, old_ids, new_ids, 0)
    packed, receipt = packed_interval_repair(shim, shifted, new_ids, intervals)
    sequential, _ = sequential_repair(shim, shifted, new_ids, intervals)
    positions = [p for a, b in intervals for p in range(a, b)]
    pos = torch.tensor(positions)
    shifted_layers, packed_layers = _layers(shifted), _layers(packed)
    for (bk, bv), (pk, pv) in zip(shifted_layers, packed_layers):
        keep = torch.ones(bk.shape[2], dtype=torch.bool)
        keep[pos] = False
        assert torch.equal(bk[:, :, keep], pk[:, :, keep]) and torch.equal(bv[:, :, keep], pv[:, :, keep])
    record = dict(
        name=name, dtype=str(dtype).replace("torch.", ""), config=_config_record(model),
        state_dict={k: v.clone() for k, v in model.model.state_dict().items()},
        inv_freq=model.model.rotary_emb.inv_freq.clone(),
        old_ids=old_ids, new_ids=new_ids, delete=delete, alignment=alignment,
        old_layers=old_layers, shifted_layers=shifted_layers, intervals=list(intervals),
        positions=positions, receipt=receipt,
        packed_rows=[(k[:, :, pos].clone(), v[:, :, pos].clone()) for k, v in packed_layers],
        sequential_rows=[(k[:, :, pos].clone(), v[:, :, pos].clone()) for k, v in _layers(sequential)],
    )
    torch.save(record, os.path.join(HERE, f"case_{name}.pt"))
    return record


def make_rope(kvr):
    from kv_cache_repair.cache import OperatorShim, shifted_suffix_keys

    records = []
    for dtype, theta, head_dim, seed in ((torch.bfloat16, 500000.0, 128, 5), (torch.float16, 10000.0, 64, 6),
                                         (torch.bfloat16, 1000000.0, 64, 7)):
        model = _model("llama", hidden=64, inter=64, layers=1, heads=2, kv_heads=1, head_dim=head_dim,
                       vocab=16, theta=theta, dtype=dtype, seed=seed)
        shim = OperatorShim(model, SimpleNamespace())
        gen = torch.Generator().manual_seed(seed)
        key = (torch.randn((1, 4, 33, head_dim), generator=gen) * 2.0).to(dtype)
        key[0, 0, 0, :4] = torch.tensor([0.0, -0.0, 1e-30, 65000.0 if dtype == torch.float16 else 3e38])
        for shift in (-256, -16, -1, 0, 7, -1024, -4096):
            positions = torch.full((1, 1), shift, dtype=torch.long)
            cos, sin = model.model.rotary_emb(key, positions)
            records.append(dict(dtype=str(dtype).replace("torch.", ""), theta=theta, head_dim=head_dim,
                                inv_freq=model.model.rotary_emb.inv_freq.clone(), shift=shift, key=key.clone(), cos=cos[0, 0].clone(), sin=sin[0, 0].clone(),
                                expected=shifted_suffix_keys(shim, key, shift).clone()))
    torch.save(records, os.path.join(HERE, "rope_shift.pt"))


def make_alignment(kvr):
    from kv_cache_repair.alignment import token_alignment

    cases = [([1, 2, 9, 3, 4], [1, 2, 3, 4]), ([1, 2], [1, 2]), ([1, 2], []), ([1, 2, 3], [1, 8, 9, 3]),
             ([], []), ([5], [6]), ([1, 1, 1, 1], [1, 1])]
    rng = random.Random(11)
    for _ in range(40):
        old = [rng.randrange(4) for _ in range(rng.randrange(0, 30))]
        a = rng.randrange(0, len(old) + 1)
        b = rng.randrange(a, len(old) + 1)
        new = old[:a] + [rng.randrange(4) for _ in range(rng.randrange(0, 3))] + old[b:]
        cases.append((old, new))
    torch.save([dict(old=o, new=n, expected=token_alignment(o, n)) for o, n in cases],
               os.path.join(HERE, "alignment.pt"))


def make_plans(kvr):
    from kv_cache_repair.execution import positions_to_intervals
    from kv_cache_repair.kernels.executor import _validate_intervals
    from kv_cache_repair.kernels.indexed_attention import IndexedPlan

    plans = []
    rng = random.Random(12)
    sets = [([3, 4, 8, 9], 10), ([], 0), ([0], 1), (list(range(63, 63 + 67 * 17, 67)), 5000)]
    for _ in range(10):
        n = rng.randrange(1, 3000)
        sets.append((sorted(rng.sample(range(n), min(n, rng.randrange(1, 80)))), n))
    for positions, length in sets:
        plan = IndexedPlan(positions, length)
        plans.append(dict(positions=positions, length=length, full=plan.full_prefix_tiles,
                          total=plan.total_tiles, intervals=positions_to_intervals(positions)))
    verdicts = []
    for intervals, length in (([], 0), ([(0, 1)], 1), ([(3, 5), (8, 10)], 12), ([(3, 5), (5, 6)], 12),
                              ([(5, 6), (3, 4)], 12), ([(0, 13)], 12), ([(-1, 2)], 12), ([(4, 4)], 12),
                              ([(True, 2)], 12), ([(1, 2, 3)], 12), ([(1.0, 2)], 12), ("x", 12),
                              ([(0, 1), (2, 3), (11, 12)], 12)):
        try:
            result, ok = list(_validate_intervals(intervals, length)), True
        except ValueError:
            result, ok = None, False
        verdicts.append(dict(intervals=intervals, length=length, ok=ok, result=result))
    torch.save(dict(plans=plans, interval_verdicts=verdicts), os.path.join(HERE, "plans.pt"))


def make_api(kvr, family, dtype, seed):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast
    from kv_cache_repair import repair_after_deletion

    words = ["[UNK]", "prefix", "obsolete", "discard", "alpha", "beta", "gamma", ".", "red", "blue", "redblue"]
    backend = Tokenizer(WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    backend.pre_tokenizer = WhitespaceSplit()
    tokenizer = PreTrainedTokenizerFast(tokenizer_object=backend, unk_token="[UNK]")
    model = _model(family, hidden=128, inter=256, layers=2, heads=4, kv_heads=2, head_dim=64,
                   vocab=32, theta=10000.0, dtype=dtype, seed=seed)
    prefix, obsolete = "prefix ", "obsolete discard "
    original = prefix + obsolete + "alpha beta gamma . " * 25
    ids = tokenizer(original, add_special_tokens=False, return_tensors="pt")["input_ids"]
    with torch.no_grad():
        old_cache = model.model(input_ids=ids, use_cache=True).past_key_values
    old_layers = _layers(old_cache)
    result = repair_after_deletion(model, tokenizer, old_cache, original,
                                   delete_span=(len(prefix), len(prefix) + len(obsolete)),
                                   query="alpha", budget_percent=10, executor="packed")
    record = dict(
        name=f"api_{family}_{str(dtype).replace('torch.', '')}", dtype=str(dtype).replace("torch.", ""),
        config=_config_record(model), state_dict={k: v.clone() for k, v in model.model.state_dict().items()},
        inv_freq=model.model.rotary_emb.inv_freq.clone(), original_text=original, delete_span=(len(prefix), len(prefix) + len(obsolete)), query="alpha",
        budget_percent=10, old_ids=ids, old_layers=old_layers, words=words,
        edited_text=result.edited_text, edited_ids=result.input_ids.clone(),
        positions=list(result.selection.positions), intervals=list(result.selection.intervals),
        suffix_start=result.selection.suffix_start, budget_tokens=result.selection.budget_tokens,
        alignment=result.metadata["alignment"], execution=result.metadata["execution"],
        cache=_layers(result.cache),
    )
    torch.save(record, os.path.join(HERE, f"{record['name']}.pt"))


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True, help="checkout of yh0903/budgeted-kv-cache-repair")
    args = parser.parse_args()
    torch.set_num_threads(1)
    kvr = load_reference(os.path.join(args.reference, "src"))
    make_alignment(kvr)
    make_plans(kvr)
    make_rope(kvr)
    # tiny Llama fp32, delete [40,56) of 128 ids, 4 rows at suffix offsets [10,14).
    make_case(kvr, "cfg0_llama_fp32", "llama", torch.float32, seed=0, hidden=64, inter=128, heads=4,
              kv_heads=2, head_dim=16, vocab=256, theta=10000.0, length=128, delete=(40, 56),
              intervals=[(50, 54)])
    make_case(kvr, "qwen3_fp32", "qwen3", torch.float32, seed=3, hidden=32, inter=64, heads=4,
              kv_heads=2, head_dim=8, vocab=97, theta=1000000.0, length=48, delete=(9, 15),
              intervals=[(0, 1), (12, 14), (20, 23), (36, 42)])
    make_case(kvr, "llama_bf16_d64", "llama", torch.bfloat16, seed=71, hidden=128, inter=256, heads=4,
              kv_heads=2, head_dim=64, vocab=97, theta=10000.0, length=150, delete=(20, 33),
              intervals=[(0, 1), (3, 5), (62, 68), (126, 132), (136, 137)])
    make_case(kvr, "qwen3_bf16_d128", "qwen3", torch.bfloat16, seed=191, hidden=128, inter=256, heads=4,
              kv_heads=1, head_dim=128, vocab=97, theta=1000000.0, length=300, delete=(50, 70),
              intervals=[(30, 31), (100, 104), (150, 166), (200, 203), (270, 280)])
    make_case(kvr, "llama_fp16_d128", "llama", torch.float16, seed=17, hidden=128, inter=128, heads=4,
              kv_heads=2, head_dim=128, vocab=97, theta=500000.0, length=200, delete=(16, 24),
              intervals=[(20, 28), (90, 92), (150, 151), (180, 192)])
    make_api(kvr, "llama", torch.bfloat16, 23)
    make_api(kvr, "qwen3", torch.bfloat16, 23)


if __name__ == "__main__":
    main()
