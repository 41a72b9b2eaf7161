"""Tensor-parallel split of the packed refresh, checked on CPU with gloo.

Two ranks each hold ``tp.shard_layer_tensors`` of a seeded model and run the
oracle's layer math on their heads, all-reducing the o_proj and down_proj
partial sums as the native loop does. Each rank's refreshed K/V rows (its KV
heads) must match the unsharded oracle on the same inputs, which pins which
rows and columns every rank owns.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import load_golden
from helpers import oracle_config


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_forward(model, shards, base_layers, ids, positions, rank, world, partial_dtype=torch.float32):
    """Oracle math for one rank's shard, with all-reduced row-parallel sums.

    ``partial_dtype``: the type the o_proj and down_proj partial sums are
    rounded to and all-reduced in. The native loop rounds each rank's
    projection to the model dtype and all-reduces that (NCCL sum, bf16/fp16
    in, one rounding of the sum out); bf16 here reproduces it."""
    from oracle import packed_oracle as oracle
    from budgeted_kv_cache_repair_b200.tp import kv_head_shard

    positions = [int(p) for p in positions]
    pos = torch.tensor(positions)
    rows, dim = len(positions), model.head_dim
    heads, kv_heads = model.heads // world, model.kv_heads // world
    out = [(kv_head_shard(k, model.kv_heads, rank, world).clone(), kv_head_shard(v, model.kv_heads, rank, world).clone())
           for k, v in base_layers]
    hidden = F.embedding(ids.index_select(0, pos), model.embed)
    cos, sin = oracle.rope_cos_sin(model.inv_freq, positions, hidden.dtype)
    cos, sin = cos[:, None, :], sin[:, None, :]
    for index, w in enumerate(shards):
        residual = hidden
        x = oracle.rms_norm(hidden, w["in_norm"], model.eps)
        q = F.linear(x, w["q"]).view(rows, heads, dim)
        k = F.linear(x, w["k"]).view(rows, kv_heads, dim)
        v = F.linear(x, w["v"]).view(rows, kv_heads, dim)
        if "q_norm" in w:
            q = oracle.rms_norm(q, w["q_norm"], model.eps)
            k = oracle.rms_norm(k, w["k_norm"], model.eps)
        q, k = oracle.apply_rope(q, cos, sin), oracle.apply_rope(k, cos, sin)
        kc, vc = out[index]
        kc.index_copy_(2, pos, k.permute(1, 0, 2).unsqueeze(0))
        vc.index_copy_(2, pos, v.permute(1, 0, 2).unsqueeze(0))
        attn = oracle.selected_attention(q, kc[0], vc[0], positions, dim ** -0.5)
        partial = F.linear(attn.reshape(rows, heads * dim), w["o"]).to(partial_dtype)
        dist.all_reduce(partial)
        hidden = residual + partial.to(residual.dtype)
        residual = hidden
        x = oracle.rms_norm(hidden, w["post_norm"], model.eps)
        partial = F.linear(F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"]), w["down"]).to(partial_dtype)
        dist.all_reduce(partial)
        hidden = residual + partial.to(residual.dtype)
    return out


def _worker(rank, world, port, name, result_path, dtype=torch.float32):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        from oracle import packed_oracle as oracle
        from budgeted_kv_cache_repair_b200.tp import kv_head_shard, shard_layer_tensors

        record = load_golden(name)
        model = oracle.OracleModel.from_state_dict(record["state_dict"], oracle_config(record), record["inv_freq"])
        model.embed = model.embed.to(dtype)
        layers = [{k: v.to(dtype) for k, v in layer.items()} for layer in model.layers]
        model.layers = layers
        base = [(k.to(dtype), v.to(dtype)) for k, v in record["shifted_layers"]]
        shards = [shard_layer_tensors(layer, heads=model.heads, kv_heads=model.kv_heads, head_dim=model.head_dim,
                                      intermediate=layer["gate"].shape[0], rank=rank, world=world)
                  for layer in layers]
        got = _tp_forward(model, shards, base, record["new_ids"][0], record["positions"], rank, world, dtype)
        full = oracle.packed_refresh(model, base, record["new_ids"], record["positions"])
        pos = torch.tensor(record["positions"])
        worst, min_cos = 0.0, 1.0
        for (k, v), (fk, fv) in zip(got, full):
            for mine, ref in ((k, kv_head_shard(fk, model.kv_heads, rank, world)),
                              (v, kv_head_shard(fv, model.kv_heads, rank, world))):
                a, b = mine[:, :, pos].double(), ref[:, :, pos].double()
                worst = max(worst, (a - b).abs().max().item())
                cos = (a * b).sum(-1) / (a.norm(dim=-1) * b.norm(dim=-1)).clamp_min(1e-30)
                min_cos = min(min_cos, cos.min().item())
                keep = torch.ones(mine.shape[2], dtype=torch.bool)
                keep[pos] = False
                assert torch.equal(mine[:, :, keep], ref[:, :, keep])
        torch.save({"rank": rank, "worst": worst, "min_cos": min_cos}, f"{result_path}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", ["case_qwen3_fp32.pt", "case_cfg0_llama_fp32.pt"])
def test_head_sharded_refresh_matches_unsharded_oracle(tmp_path, name):
    world = 2
    path = str(tmp_path / "result")
    mp.start_processes(_worker, args=(world, _free_port(), name, path), nprocs=world, start_method="spawn")
    for rank in range(world):
        result = torch.load(f"{path}.{rank}")
        assert result["worst"] < 1e-5, result


@pytest.mark.parametrize("name,dtype", [("case_llama_bf16_d64.pt", torch.bfloat16),
                                        ("case_llama_fp16_d128.pt", torch.float16)])
def test_head_sharded_refresh_with_16bit_partial_sums(tmp_path, name, dtype):
    """The native loop's arithmetic: 16-bit weights, each rank's o_proj and
    down_proj output rounded to the model dtype and all-reduced in it (one
    rounding of the sum). Against the unsharded oracle in the same dtype,
    which rounds the full product once, the refreshed rows agree to the north
    star's row cosine."""
    world = 2
    path = str(tmp_path / "result")
    mp.start_processes(_worker, args=(world, _free_port(), name, path, dtype), nprocs=world, start_method="spawn")
    for rank in range(world):
        result = torch.load(f"{path}.{rank}")
        assert result["min_cos"] >= 0.999, result
