"""The no-allocation attention entry point (kvr_selected_attention_static).

Some callers cannot allocate device memory per call: a host runtime that
reaches this library over a plain C FFI, with a fixed, pre-planned GPU memory
budget and no caching allocator, where a cudaMalloc would synchronise the
device. The static entry point takes its split-KV scratch from a fixed device
array inside the library instead of a caller workspace. These tests check,
through the C ABI, that it returns what the workspace entry point returns on
two calls in a row (the array keeps the previous call's contents), and that a
problem too large for the array is refused before any launch.

This file is named to be collected last, so that a run stopping at the first
failure has already run every other test.
"""

import pytest
import torch

from oracle import packed_oracle as oracle

DEV = "cuda"


def _lib():
    from budgeted_kv_cache_repair_b200 import _lib, build

    build.build()
    return _lib


def _problem(seed, rows, heads, kv_heads, dim, length):
    gen = torch.Generator().manual_seed(seed)
    positions = sorted(torch.randperm(length, generator=gen)[:rows].tolist())
    q = (torch.randn(rows, heads, dim, generator=gen) * 0.5).to(torch.bfloat16).to(DEV)
    k = torch.randn(1, kv_heads, length, dim, generator=gen).to(torch.bfloat16).to(DEV)
    v = (torch.randn(1, kv_heads, length, dim, generator=gen) * 0.5).to(torch.bfloat16).to(DEV)
    return positions, q, k, v


@pytest.mark.gpu
def test_static_scratch_entry_matches_workspace_entry_on_two_calls():
    lib = _lib()
    L = lib.load()
    stream = lib.stream_handle()
    # Llama-3-8B attention geometry at 7936 keys: the key range is split, so the
    # partial results go through the scratch array.
    shape = dict(rows=64, heads=32, kv_heads=8, dim=128, length=7936)
    need = L.kvr_attention_workspace_size(shape["rows"], shape["heads"], shape["kv_heads"], shape["dim"],
                                          shape["length"])
    assert 256 < need <= lib.STATIC_SCRATCH_BYTES
    for seed in (11, 12):  # second call runs over the first call's leftovers
        positions, q, k, v = _problem(seed, **shape)
        pos = torch.tensor(positions, device=DEV)
        args = (pos.data_ptr(), shape["rows"], shape["heads"], shape["kv_heads"], shape["dim"], shape["length"],
                shape["length"] * shape["dim"], shape["dim"], positions[-1], shape["dim"] ** -0.5, lib.ATTN_P_SPLIT)
        ref = torch.empty_like(q)
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        lib.check(L.kvr_selected_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), *args,
                                           ws.data_ptr(), need, lib.DTYPE_BF16, stream), "workspace entry")
        out = torch.full_like(q, float("nan"))
        lib.check(L.kvr_selected_attention_static(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), *args,
                                                  lib.DTYPE_BF16, stream), "static entry")
        # The static call's own status word, read through its accessor.
        status = torch.full((1,), -1, dtype=torch.int32).pin_memory()
        lib.check(L.kvr_attention_static_status(status.data_ptr(), stream), "static status")
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32).item()) == 0
        assert int(status.item()) == 0
        assert torch.isfinite(out.float()).all()
        torch.testing.assert_close(out.float(), ref.float(), atol=0.002, rtol=0.02)
        expected = oracle.selected_attention_fp64(q.permute(1, 0, 2)[None].cpu(), k.cpu(), v.cpu(), positions)
        torch.testing.assert_close(out.permute(1, 0, 2)[None].double().cpu(), expected, atol=0.002, rtol=0.02)


def test_static_scratch_entry_refuses_oversized_problems_before_launch():
    lib = _lib()
    L = lib.load()
    # 64 rows x 256 query heads over 32 KV heads at 131072 keys needs more
    # split-KV scratch than the array holds; the call returns before touching
    # any pointer (all NULL here) or the GPU.
    need = L.kvr_attention_workspace_size(64, 256, 32, 128, 131072)
    assert need > lib.STATIC_SCRATCH_BYTES
    status = L.kvr_selected_attention_static(None, None, None, None, None, 64, 256, 32, 128, 131072, 131072 * 128,
                                             128, 131071, 0.088, lib.ATTN_P_SPLIT, lib.DTYPE_BF16, None)
    assert status == lib.ERR_SCRATCH_LIMIT
    assert "scratch" in L.kvr_status_string(status).decode()
