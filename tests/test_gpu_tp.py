"""Head-sharded tensor-parallel refresh on two GPUs (NCCL all-reduce inside the
native layer loop) against the single-GPU engine on the same inputs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=device)
    group = None
    try:
        from helpers import fixture_model, to_cache
        from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair
        from budgeted_kv_cache_repair_b200.cache import copy_layers
        from budgeted_kv_cache_repair_b200.plan import IndexedPlan
        from budgeted_kv_cache_repair_b200.tp import ShardView, TPGroup, kv_head_shard, refresh_rows_tp
        from budgeted_kv_cache_repair_b200.validate import cache_layers

        record = load_golden(name)
        model = fixture_model(record, device)
        base = to_cache(record["shifted_layers"], device)
        ids = record["new_ids"].to(device)
        full, _ = packed_interval_repair(OperatorShim(model), base, ids, record["intervals"])
        view = ShardView.from_model(model.model, rank, world)
        kv = model.config.num_key_value_heads
        local = copy_layers([(kv_head_shard(k, kv, rank, world).contiguous(), kv_head_shard(v, kv, rank, world).contiguous())
                             for k, v in cache_layers(base)])
        plan = IndexedPlan(record["positions"], ids.shape[1]).to(device)
        group = TPGroup(rank, world, device)
        refresh_rows_tp(view, local, ids[0], plan.positions, plan.host_plan.max_position, ids.shape[1], group)
        torch.cuda.synchronize()
        pos = torch.tensor(record["positions"], device=device)
        worst, min_cos = 0.0, 1.0
        for (k, v), (fk, fv) in zip(local, cache_layers(full)):
            for mine, ref in ((k, kv_head_shard(fk, kv, rank, world)), (v, kv_head_shard(fv, kv, rank, world))):
                a, b = mine.index_select(2, pos).double(), ref.index_select(2, pos).double()
                worst = max(worst, (a - b).abs().max().item())
                cos = (a * b).sum(-1) / (a.norm(dim=-1) * b.norm(dim=-1)).clamp_min(1e-30)
                min_cos = min(min_cos, cos.min().item())
        torch.save({"worst": worst, "min_cos": min_cos}, f"{result_path}.{rank}")
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["case_llama_bf16_d64.pt", "case_llama_fp16_d128.pt"])
def test_tensor_parallel_refresh_matches_single_gpu(tmp_path, name):
    world = 2
    path = str(tmp_path / "result")
    mp.start_processes(_worker, args=(world, _free_port(), name, path), nprocs=world, start_method="spawn")
    for rank in range(world):
        result = torch.load(f"{path}.{rank}")
        # bf16/fp16 partial sums are all-reduced after rounding, where the single
        # GPU rounds the full GEMM once: row-cosine tolerance.
        assert result["min_cos"] >= 0.999, result


def _worker_70b(rank, world, port, result_path):
    """Two layers of the Llama-3-70B shape (hidden 8192, 64 query / 8 KV
    heads, MLP 28672) at BASELINE configs[4]'s geometry: 15872 cached rows,
    1383 rows in 16 intervals. Each rank refreshes its 8 / world KV heads with
    the NCCL all-reduces inside the native loop and checks them against the
    single-GPU engine, the reference's bf16 packed path and an fp32 control of
    it, all on its own GPU."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=device)
    group = None
    try:
        import bench
        from budgeted_kv_cache_repair_b200 import OperatorShim, packed_interval_repair
        from budgeted_kv_cache_repair_b200.cache import copy_layers, make_cache
        from budgeted_kv_cache_repair_b200.plan import IndexedPlan
        from budgeted_kv_cache_repair_b200.tp import ShardView, TPGroup, kv_head_shard, refresh_rows_tp
        from budgeted_kv_cache_repair_b200.validate import cache_layers
        from oracle import packed_oracle as oracle
        from oracle.hf_packed import packed_refresh_hf

        cfg = dict(bench.CONFIG_70B, arch="llama", layers=2, eps=1e-5)
        model = bench.build_model(cfg, 4, device)
        length = cfg["context"] - cfg["delete"]
        gen = torch.Generator(device=device).manual_seed(4)
        ids = torch.randint(0, cfg["vocab"], (1, length), device=device, generator=gen)
        shape = (1, cfg["kv_heads"], length, cfg["head_dim"])
        base = [(torch.randn(shape, device=device, generator=gen).bfloat16(),
                 (0.5 * torch.randn(shape, device=device, generator=gen)).bfloat16()) for _ in range(cfg["layers"])]
        intervals = bench.budget_intervals(4, cfg["delete_at"], length, cfg["intervals"], 1383)
        positions = [p for a, b in intervals for p in range(a, b)]

        single, _ = packed_interval_repair(OperatorShim(model), make_cache(base), ids, intervals)
        view = ShardView.from_model(model.model, rank, world)
        kv = cfg["kv_heads"]
        local = copy_layers([(kv_head_shard(k, kv, rank, world).contiguous(),
                              kv_head_shard(v, kv, rank, world).contiguous()) for k, v in base])
        plan = IndexedPlan(positions, length).to(device)
        group = TPGroup(rank, world, device)
        refresh_rows_tp(view, local, ids[0], plan.positions, plan.host_plan.max_position, length, group)
        torch.cuda.synchronize()

        def mine(layers):
            return oracle.fresh_rows([(kv_head_shard(k, kv, rank, world), kv_head_shard(v, kv, rank, world))
                                      for k, v in layers], positions).double()

        ours = oracle.fresh_rows(local, positions).double()
        one_gpu = mine(cache_layers(single))
        expect = mine(packed_refresh_hf(model.model, base, ids, positions))
        control = mine(packed_refresh_hf(model.float().model, [(k.float(), v.float()) for k, v in base], ids,
                                         positions))
        result = {"cos_single": oracle.row_cosine(ours, one_gpu).min().item(),
                  "cos_reference": oracle.row_cosine(ours, expect).min().item(),
                  "ours_max": (ours - control).abs().max().item(), "ref_max": (expect - control).abs().max().item(),
                  "ours_mean": (ours - control).abs().mean().item(),
                  "ref_mean": (expect - control).abs().mean().item()}
        torch.save(result, f"{result_path}.{rank}")
    finally:
        if group is not None:
            group.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensor_parallel_refresh_at_70b_geometry(tmp_path):
    world = 2
    path = str(tmp_path / "result")
    mp.start_processes(_worker_70b, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    for rank in range(world):
        r = torch.load(f"{path}.{rank}")
        assert r["cos_single"] >= 0.999 and r["cos_reference"] >= 0.999, r
        # The reference's gate (tests/test_packed_cache.py:291-376): within
        # twice the reference bf16 path's own error against the fp32 control.
        assert r["ours_max"] <= 2 * r["ref_max"] and r["ours_mean"] <= 2 * r["ref_mean"], r
