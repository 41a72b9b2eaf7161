"""The packed refresh at BASELINE configs[3] geometry (Qwen3-8B shape, 32k
context, 1383 selected rows) against the reference's packed SDPA path run on
the same GPU (oracle/hf_packed.py), on two of the 36 layers: unselected rows
bit-identical, refreshed rows at cosine >= 0.999 to the reference's bf16 path,
and within twice that path's own error against an fp32 control.

This is the large-batch side of the engine that the 64-row fixtures do not
reach: projections above 256 rows (cuBLAS), attention with hundreds of
(KV head, 128-entry tile) units and split key ranges, q/k RMSNorm.
"""

import pytest
import torch

from helpers import bits_equal
from oracle import packed_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
LAYERS, HIDDEN, HEADS, KV_HEADS, HEAD_DIM, INTER, VOCAB = 2, 4096, 32, 8, 128, 12288, 151936
CONTEXT, DELETE_AT, DELETE, ROWS, INTERVALS = 32768, 4096, 1024, 1383, 32


def _model():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    config = Qwen3Config(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER, num_hidden_layers=LAYERS,
                         num_attention_heads=HEADS, num_key_value_heads=KV_HEADS, head_dim=HEAD_DIM,
                         rope_theta=1e6, max_position_embeddings=131072, initializer_range=0.02, rms_norm_eps=1e-6)
    torch.manual_seed(3)
    previous = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(DEV):
            model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(previous)
    return model.eval()


def _intervals(length):
    """32 sorted, non-adjacent intervals holding 1383 rows (widths 43 and 44)."""
    width, extra = divmod(ROWS, INTERVALS)
    gen = torch.Generator().manual_seed(3)
    slot = width + 2
    picks = sorted(torch.randperm((length - DELETE_AT) // slot, generator=gen)[:INTERVALS].tolist())
    return [(DELETE_AT + s * slot, DELETE_AT + s * slot + width + (1 if i < extra else 0))
            for i, s in enumerate(picks)]


@torch.no_grad()
def test_config3_geometry_matches_reference_packed_path():
    from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair
    from budgeted_kv_cache_repair_b200.cache import make_cache
    from budgeted_kv_cache_repair_b200.validate import cache_layers
    from oracle.hf_packed import packed_refresh_hf

    model = _model()
    length = CONTEXT - DELETE
    gen = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(0, VOCAB, (1, length), device=DEV, generator=gen)
    shape = (1, KV_HEADS, length, HEAD_DIM)
    base = [(torch.randn(shape, device=DEV, generator=gen).bfloat16(),
             (0.5 * torch.randn(shape, device=DEV, generator=gen)).bfloat16()) for _ in range(LAYERS)]
    intervals = _intervals(length)
    positions = [p for a, b in intervals for p in range(a, b)]
    assert len(positions) == ROWS

    out, receipt = packed_interval_repair(OperatorShim(model), make_cache(base), ids, intervals)
    assert receipt["recomputed_tokens"] == ROWS
    got = cache_layers(out)
    expect = packed_refresh_hf(model.model, base, ids, positions)
    torch.cuda.synchronize()

    keep = torch.ones(length, dtype=torch.bool, device=DEV)
    keep[torch.tensor(positions, device=DEV)] = False
    for (k, v), (bk, bv) in zip(got, base):
        assert bits_equal(k[:, :, keep], bk[:, :, keep]) and bits_equal(v[:, :, keep], bv[:, :, keep])
    actual_rows = oracle.fresh_rows(got, positions)
    expected_rows = oracle.fresh_rows(expect, positions)
    cos = oracle.row_cosine(actual_rows, expected_rows)
    assert cos.min() >= 0.999, cos.min().item()

    # The reference's own gate at scale (test_packed_cache.py:291-376): against
    # an fp32 control of the same path, the engine's error is at most twice the
    # error of the reference's bf16 path.
    control_model = model.float()
    control = packed_refresh_hf(control_model.model, [(k.float(), v.float()) for k, v in base], ids, positions)
    control_rows = oracle.fresh_rows(control, positions).double()
    ours = (actual_rows.double() - control_rows).abs()
    theirs = (expected_rows.double() - control_rows).abs()
    assert ours.max() <= 2 * theirs.max(), (ours.max().item(), theirs.max().item())
    assert ours.mean() <= 2 * theirs.mean(), (ours.mean().item(), theirs.mean().item())
