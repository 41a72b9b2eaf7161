"""sm_100a kernels through the C ABI against the oracle and the reference's fixtures."""

import ctypes

import pytest
import torch

from conftest import golden_cases, load_golden
from helpers import bits_equal
from oracle import packed_oracle as oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    from budgeted_kv_cache_repair_b200 import _lib
    from budgeted_kv_cache_repair_b200 import build

    build.build()
    return _lib


def _rope_table(cos, sin):
    return torch.cat((cos.reshape(-1), sin.reshape(-1))).to(DEV).contiguous()


def test_rope_shift_is_bit_exact_with_reference_fixture(lib):
    L = lib.load()
    for record in load_golden("rope_shift.pt"):
        key = record["key"].to(DEV)
        out = torch.empty_like(key)
        table = _rope_table(record["cos"], record["sin"])
        _, heads, rows, dim = key.shape
        lib.check(L.kvr_rope_shift_layers(lib.ptr_array([key]), lib.ptr_array([out]), 1, heads, rows, dim,
                                          rows * dim, dim, rows * dim, dim, table.data_ptr(),
                                          lib.dtype_code(key.dtype), lib.stream_handle()), "rope")
        torch.cuda.synchronize()
        if record["shift"] == 0:
            continue  # the reference clones on a zero shift; the kernel still rotates by angle 0
        assert bits_equal(out.cpu(), record["expected"]), (record["dtype"], record["shift"])


def test_rope_shift_in_place_multi_layer(lib):
    L = lib.load()
    torch.manual_seed(1)
    layers = [torch.randn(1, 8, 333, 128, device=DEV).to(torch.bfloat16) for _ in range(5)]
    inv = oracle.default_inv_freq(500000.0, 128)
    cos, sin = oracle.rope_cos_sin(inv, [-256], torch.bfloat16)
    table = _rope_table(cos, sin)
    expected = [oracle.apply_rope(t.cpu(), cos[0], sin[0]) for t in layers]
    lib.check(L.kvr_rope_shift_layers(lib.ptr_array(layers), lib.ptr_array(layers), 5, 8, 333, 128,
                                      333 * 128, 128, 333 * 128, 128, table.data_ptr(), 0, lib.stream_handle()),
              "rope")
    for got, exp in zip(layers, expected):
        assert bits_equal(got.cpu(), exp)


@pytest.mark.parametrize("dtype, dim, row_pad, in_place", [(torch.bfloat16, 64, 0, False),
                                                           (torch.float16, 128, 0, True),
                                                           (torch.bfloat16, 128, 8, False),
                                                           (torch.float16, 64, 8, True)])
def test_rope_shift_head_dims_strides_and_in_place(lib, dtype, dim, row_pad, in_place):
    """Delta-RoPE over many layers equals torch's op sequence bit for bit
    (cache.py:47-77) for both head dims, rows padded beyond head_dim (16-byte
    instead of 32-byte accesses), in place and into new tensors; padding is
    never written."""
    torch.manual_seed(20 + dim + row_pad)
    layers, heads, rows = 6, 8, 1537
    full = torch.randn(layers, 1, heads, rows, dim + row_pad).to(dtype)
    cos = (torch.rand(dim) * 2 - 1).to(dtype)
    sin = (torch.rand(dim) * 2 - 1).to(dtype)
    src_full = full.to(DEV)
    src = [src_full[i, ..., :dim] for i in range(layers)]
    if in_place:
        dst_full, dst = src_full, src
    else:
        dst_full = torch.full_like(src_full, -5.0)
        dst = [dst_full[i, ..., :dim] for i in range(layers)]
    L = lib.load()
    stride = dim + row_pad
    lib.check(L.kvr_rope_shift_layers(lib.ptr_array(src), lib.ptr_array(dst), layers, heads, rows, dim,
                                      rows * stride, stride, rows * stride, stride, _rope_table(cos, sin).data_ptr(),
                                      lib.dtype_code(dtype), lib.stream_handle()), "rope")
    torch.cuda.synchronize()
    expected = oracle.apply_rope(full[..., :dim], cos, sin)
    got = dst_full.cpu()
    assert bits_equal(got[..., :dim], expected)
    if row_pad:
        pad = full[..., dim:] if in_place else torch.full_like(full[..., dim:], -5.0)
        assert bits_equal(got[..., dim:], pad)


@pytest.mark.parametrize("name", [n for n in golden_cases() if "fp32" not in n])
def test_shift_cache_is_bit_exact_with_reference_fixture(lib, name):
    record = load_golden(name)
    old = [(k.to(DEV), v.to(DEV)) for k, v in record["old_layers"]]
    al = record["alignment"]
    dtype = old[0][0].dtype
    cos, sin = oracle.rope_cos_sin(record["inv_freq"].float(), [al["position_shift"]], dtype)
    table = _rope_table(cos, sin)
    _, heads, old_rows, dim = old[0][0].shape
    new_rows = record["new_ids"].shape[1]
    k_new = [torch.empty(1, heads, new_rows, dim, dtype=dtype, device=DEV) for _ in old]
    v_new = [torch.empty(1, heads, new_rows, dim, dtype=dtype, device=DEV) for _ in old]
    L = lib.load()
    lib.check(L.kvr_shift_cache_layers(lib.ptr_array([k for k, _ in old]), lib.ptr_array([v for _, v in old]),
                                       lib.ptr_array(k_new), lib.ptr_array(v_new), len(old), heads, dim, new_rows,
                                       al["prefix"], al["old_suffix_start"], al["new_suffix_start"],
                                       old_rows * dim, dim, new_rows * dim, dim, table.data_ptr(), 1,
                                       lib.dtype_code(dtype), lib.stream_handle()), "shift")
    for k, v, (ek, ev) in zip(k_new, v_new, record["shifted_layers"]):
        assert bits_equal(k.cpu(), ek) and bits_equal(v.cpu(), ev)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_shift_cache_special_values_match_torch_ops(lib, dtype):
    """The rotated tail equals torch's op sequence bit for bit, including NaN,
    infinities and overflow to infinity (cache.py:47-77: k*cos + rotate_half(k)*sin)."""
    torch.manual_seed(11)
    layers, heads, dim, old_rows = 3, 2, 128, 300
    prefix, old_tail, new_tail = 40, 72, 40
    new_rows = old_rows - (old_tail - new_tail)
    k = (torch.randn(layers, heads, old_rows, dim) * 3).to(dtype)
    v = torch.randn(layers, heads, old_rows, dim).to(dtype)
    big = torch.finfo(dtype).max
    special = torch.tensor([float("nan"), float("inf"), -float("inf"), big, -big, 0.0, -0.0], dtype=dtype)
    k.view(-1)[torch.randint(0, k.numel(), (400,))] = special[torch.randint(0, len(special), (400,))]
    cos = (torch.rand(dim) * 2 - 1).to(dtype)
    sin = (torch.rand(dim) * 2 - 1).to(dtype)
    kd, vd = k.to(DEV), v.to(DEV)
    k_new = [torch.empty(1, heads, new_rows, dim, dtype=dtype, device=DEV) for _ in range(layers)]
    v_new = [torch.empty(1, heads, new_rows, dim, dtype=dtype, device=DEV) for _ in range(layers)]
    L = lib.load()
    lib.check(L.kvr_shift_cache_layers(lib.ptr_array([kd[i] for i in range(layers)]),
                                       lib.ptr_array([vd[i] for i in range(layers)]), lib.ptr_array(k_new),
                                       lib.ptr_array(v_new), layers, heads, dim, new_rows, prefix, old_tail, new_tail,
                                       old_rows * dim, dim, new_rows * dim, dim, _rope_table(cos, sin).data_ptr(), 1,
                                       lib.dtype_code(dtype), lib.stream_handle()), "shift")
    torch.cuda.synchronize()
    tail = k[:, :, old_tail:]
    rot = torch.cat((-tail[..., dim // 2:], tail[..., : dim // 2]), dim=-1)
    expected_tail = tail * cos + rot * sin
    for i in range(layers):
        got = k_new[i][0].cpu()
        assert bits_equal(got[:, :prefix], k[i, :, :prefix])
        g, e = got[:, new_tail:], expected_tail[i]
        # A NaN's bit pattern depends on the conversion unit that made it
        # (torch writes different NaN payloads on CPU and CUDA): compare NaN-ness
        # there and every bit everywhere else.
        nan = torch.isnan(e)
        assert torch.equal(torch.isnan(g), nan)
        assert bits_equal(g[~nan], e[~nan])
        assert bits_equal(v_new[i][0].cpu()[:, new_tail:], v[i, :, old_tail:])


@pytest.mark.parametrize("dtype, dim, row_pad", [(torch.bfloat16, 64, 0), (torch.float16, 64, 0),
                                                  (torch.bfloat16, 128, 0), (torch.bfloat16, 128, 8),
                                                  (torch.float16, 64, 8)])
def test_shift_cache_gap_rows_strides_and_large_caches(lib, dtype, dim, row_pad):
    """Rows in [prefix, new_tail) are left to the caller (never written), head
    planes padded beyond their rows (and, with row_pad, old rows padded beyond
    head_dim: 16-byte instead of 32-byte accesses) are read and written through
    their strides, and a cache of tens of thousands of CTAs matches torch's ops
    bit for bit (cache.py:47-77,103-144)."""
    torch.manual_seed(12 + dim + row_pad)
    layers, heads, old_rows = 4, 8, 3001
    prefix, old_tail, new_tail = 700, 1037, 709  # 9 rows for the caller, 328 deleted
    new_rows = old_rows - (old_tail - new_tail)
    pad_old, pad_new = 24, 40  # unused rows at the end of every head plane
    k_rows = torch.randn(layers, heads, old_rows + pad_old, dim + row_pad).to(dtype)
    v_rows = torch.randn(layers, heads, old_rows + pad_old, dim + row_pad).to(dtype)
    k, v = k_rows[..., :dim], v_rows[..., :dim]
    cos = (torch.rand(dim) * 2 - 1).to(dtype)
    sin = (torch.rand(dim) * 2 - 1).to(dtype)
    sentinel = -3.0
    kd, vd = k_rows.to(DEV)[..., :dim], v_rows.to(DEV)[..., :dim]
    k_out = torch.full((layers, heads, new_rows + pad_new, dim), sentinel, dtype=dtype, device=DEV)
    v_out = torch.full_like(k_out, sentinel)
    L = lib.load()
    lib.check(L.kvr_shift_cache_layers(lib.ptr_array([kd[i] for i in range(layers)]),
                                       lib.ptr_array([vd[i] for i in range(layers)]),
                                       lib.ptr_array([k_out[i] for i in range(layers)]),
                                       lib.ptr_array([v_out[i] for i in range(layers)]), layers, heads, dim,
                                       new_rows, prefix, old_tail, new_tail, (old_rows + pad_old) * (dim + row_pad),
                                       dim + row_pad, (new_rows + pad_new) * dim, dim,
                                       _rope_table(cos, sin).data_ptr(), 1,
                                       lib.dtype_code(dtype), lib.stream_handle()), "shift")
    torch.cuda.synchronize()
    tail = k[:, :, old_tail:old_rows]
    rot = torch.cat((-tail[..., dim // 2:], tail[..., : dim // 2]), dim=-1)
    expected_k = torch.full((layers, heads, new_rows + pad_new, dim), sentinel, dtype=dtype)
    expected_v = expected_k.clone()
    expected_k[:, :, :prefix] = k[:, :, :prefix]
    expected_k[:, :, new_tail:new_rows] = tail * cos + rot * sin
    expected_v[:, :, :prefix] = v[:, :, :prefix]
    expected_v[:, :, new_tail:new_rows] = v[:, :, old_tail:old_rows]
    assert bits_equal(k_out.cpu(), expected_k)
    assert bits_equal(v_out.cpu(), expected_v)


@pytest.mark.parametrize("dense", [True, False])
def test_copy_layers_is_bitwise(lib, dense):
    torch.manual_seed(2)
    if dense:
        src = [torch.randn(1, 4, 257, 128, device=DEV).to(torch.float16) for _ in range(6)]
    else:
        src = [torch.randn(1, 257, 4, 128, device=DEV).to(torch.float16).transpose(1, 2) for _ in range(6)]
    dst = [torch.empty(1, 4, 257, 128, dtype=torch.float16, device=DEV) for _ in src]
    L = lib.load()
    lib.check(L.kvr_copy_layers(lib.ptr_array(src), lib.ptr_array(dst), 6, 4, 257, 128, src[0].stride(1),
                                src[0].stride(2), 257 * 128, 128, 1, lib.stream_handle()), "copy")
    for s, d in zip(src, dst):
        assert bits_equal(s.contiguous(), d)


@pytest.mark.parametrize("dtype,bits", [
    (torch.float16, [0, -32768, 31744, -1024, 32257, 1]),
    (torch.bfloat16, [0, -32768, 32640, -128, 32705, 1]),
])
def test_scatter_is_bitwise_copy_including_nan_payloads(dtype, bits):
    # tests/test_indexed_attention.py:284-300 of the reference.
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_kv_scatter_

    plan = IndexedPlan([0, 3, 8], 9).to(DEV)
    raw = torch.tensor(bits, dtype=torch.int16, device=DEV).repeat(32).reshape(1, 1, 3, 64)
    fresh_key = raw.view(dtype)
    fresh_value = fresh_key.clone()
    key = torch.zeros((1, 1, 9, 64), device=DEV, dtype=dtype)
    value = key.clone()
    indexed_kv_scatter_(key, value, fresh_key, fresh_value, plan)
    assert bits_equal(key.index_select(2, plan.positions), fresh_key)
    assert bits_equal(value.index_select(2, plan.positions), fresh_value)
    assert torch.count_nonzero(key[:, :, [1, 2, 4, 5, 6, 7]].view(torch.int16)) == 0


def _positions(count, length):
    return [length - 1] if count == 1 else [i * (length - 1) // (count - 1) for i in range(count)]


def _assert_attention_close(actual, expected):
    # The reference's frozen tolerances (tests/test_indexed_attention.py:119-124).
    atol, rtol = ((0.002, 0.02) if actual.dtype == torch.bfloat16 else (0.00025, 0.003))
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual.double().cpu(), expected.cpu(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("count", [1, 15, 16, 17, 64])
def test_attention_matches_independent_fp64_oracle(count, dim, dtype):
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention

    torch.manual_seed(8200 + count + dim)
    length = 1025
    positions = _positions(count, length)
    plan = IndexedPlan(positions, length).to(DEV)
    q = torch.randn((1, 4, count, dim), device=DEV, dtype=dtype) * 0.5
    k = torch.randn((1, 2, length, dim), device=DEV, dtype=dtype) * 0.5
    v = torch.randn_like(k) * 0.5
    before = [t.clone() for t in (q, k, v)]
    actual = indexed_causal_attention(q, k, v, plan)
    assert actual.shape == q.shape and actual.dtype == dtype
    _assert_attention_close(actual, oracle.selected_attention_fp64(q.cpu(), k.cpu(), v.cpu(), positions))
    assert all(bits_equal(t, s) for t, s in zip((q, k, v), before))


@pytest.mark.parametrize("heads,kv_heads,count,length", [(32, 8, 64, 7936), (32, 8, 200, 4099), (8, 1, 37, 3000),
                                                         (64, 8, 40, 2500), (4, 4, 130, 600)])
def test_attention_split_kv_long_context(heads, kv_heads, count, length):
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention

    torch.manual_seed(heads * 7 + count)
    positions = sorted(torch.randperm(length)[:count].tolist())
    plan = IndexedPlan(positions, length).to(DEV)
    q = torch.randn((1, heads, count, 128), device=DEV, dtype=torch.bfloat16) * 0.5
    k = torch.randn((1, kv_heads, length, 128), device=DEV, dtype=torch.bfloat16) * 0.5
    v = torch.randn_like(k) * 0.5
    actual = indexed_causal_attention(q, k, v, plan)
    _assert_attention_close(actual, oracle.selected_attention_fp64(q.cpu(), k.cpu(), v.cpu(), positions))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_nonuniform_attention_with_cancelling_large_value_channels(dtype):
    # tests/test_indexed_attention.py:127-155 of the reference.
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention

    positions = [0, 1, 3, 7, 16, 31, 63, 64, 95, 127, 191, 255, 256]
    plan = IndexedPlan(positions, 257).to(DEV)
    query = torch.zeros((1, 4, len(positions), 64), device=DEV, dtype=dtype)
    key = torch.zeros((1, 2, 257, 64), device=DEV, dtype=dtype)
    for head in range(4):
        query[:, head, :, 0] = 1 + head / 4
        query[:, head, :, 1] = torch.arange(len(positions), device=DEV, dtype=torch.float32) / 16 - 0.5
    key[:, :, :, 0] = torch.linspace(-3, 3, 257, device=DEV, dtype=torch.float32)
    key[:, :, :, 1] = ((torch.arange(257, device=DEV) % 9).float() - 4) / 8
    signs = torch.where(torch.arange(257, device=DEV) % 2 == 0, 1.0, -1.0)
    magnitude = torch.tensor([64.0] * 16 + [1.0] * 16 + [0.03125] * 32, device=DEV)
    value = (signs[:, None] * magnitude[None, :]).to(dtype)[None, None].repeat(1, 2, 1, 1)
    value[:, 1].mul_(1.5)
    actual = indexed_causal_attention(query, key, value, plan, scale=1.0)
    _assert_attention_close(actual, oracle.selected_attention_fp64(query.cpu(), key.cpu(), value.cpu(),
                                                                   positions, 1.0))


@pytest.mark.parametrize("heads,kv_heads", [(1, 1), (4, 1), (4, 4), (8, 2)])
def test_grouped_query_head_mapping(heads, kv_heads):
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention

    positions = [0, 64, 130]
    plan = IndexedPlan(positions, 131).to(DEV)
    q = torch.zeros((1, heads, 3, 64), device=DEV, dtype=torch.bfloat16)
    k = torch.zeros((1, kv_heads, 131, 64), device=DEV, dtype=torch.bfloat16)
    v = torch.empty_like(k)
    for head in range(kv_heads):
        v[:, head].fill_(head + 1)
    actual = indexed_causal_attention(q, k, v, plan)
    for head in range(heads):
        torch.testing.assert_close(actual[:, head].float(),
                                   torch.full_like(actual[:, head].float(), head // (heads // kv_heads) + 1),
                                   atol=0.02, rtol=0.01)


def test_fresh_selected_visibility_and_future_exclusion():
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention, indexed_kv_scatter_

    positions = [3, 4, 8, 9]
    plan = IndexedPlan(positions, 131).to(DEV)
    key = torch.zeros((1, 2, 131, 64), device=DEV, dtype=torch.bfloat16)
    value = torch.zeros_like(key)
    fresh_key = torch.zeros((1, 2, 4, 64), device=DEV, dtype=torch.bfloat16)
    fresh_value = torch.empty_like(fresh_key)
    for row in range(4):
        fresh_value[:, :, row].fill_(10 + row)
    query = torch.zeros((1, 4, 4, 64), device=DEV, dtype=torch.bfloat16)
    indexed_kv_scatter_(key, value, fresh_key, fresh_value, plan)
    output = indexed_causal_attention(query, key, value, plan)
    assert float(output[0, 0, 2, 0]) > 3.5
    preserved = output.clone()
    key[:, :, 9:].fill_(50)
    value[:, :, 9:].fill_(500)
    changed = indexed_causal_attention(query, key, value, plan)
    assert bits_equal(changed[:, :, :3], preserved[:, :, :3])
    assert not bits_equal(changed[:, :, 3:], preserved[:, :, 3:])


def test_query_at_zero_reads_only_itself():
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention

    plan = IndexedPlan([0], 130).to(DEV)
    q = torch.randn((1, 4, 1, 64), device=DEV, dtype=torch.float16)
    k = torch.randn((1, 2, 130, 64), device=DEV, dtype=torch.float16)
    v = torch.randn_like(k)
    output = indexed_causal_attention(q, k, v, plan)
    assert bits_equal(output, v[:, :, :1].repeat_interleave(2, dim=1))


def test_kernels_use_the_callers_nondefault_stream():
    from budgeted_kv_cache_repair_b200 import IndexedPlan, indexed_causal_attention, indexed_kv_scatter_

    host = IndexedPlan([0, 3, 4, 8, 9], 130)
    plan = host.to(DEV)
    q = torch.zeros((1, 4, 5, 64), device=DEV, dtype=torch.bfloat16)
    k = torch.zeros((1, 2, 130, 64), device=DEV, dtype=torch.bfloat16)
    v = k.clone()
    fresh = torch.zeros((1, 2, 5, 64), device=DEV, dtype=torch.bfloat16)
    indexed_kv_scatter_(k, v, fresh, fresh.clone(), plan)
    indexed_causal_attention(q, k, v, plan)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        torch.cuda._sleep(2_000_000)
        plan = host.to(DEV)
        q = torch.randn_like(q) * 0.5
        k, v = torch.randn_like(k) * 0.5, torch.randn_like(v) * 0.5
        fresh_k, fresh_v = torch.randn_like(fresh), torch.randn_like(fresh)
        indexed_kv_scatter_(k, v, fresh_k, fresh_v, plan)
        output = indexed_causal_attention(q, k, v, plan)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    _assert_attention_close(output, oracle.selected_attention_fp64(q.cpu(), k.cpu(), v.cpu(), host.positions))


def test_row_kernels_match_torch_rounding(lib):
    """add_rmsnorm and silu_mul follow the transformers modules op by op."""
    L = lib.load()
    torch.manual_seed(5)
    rows, H, I = 37, 4096, 1024
    hidden = torch.randn(rows, H, device=DEV).to(torch.bfloat16)
    delta = torch.randn(rows, H, device=DEV).to(torch.bfloat16)
    weight = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    expected_h = hidden + delta
    expected = oracle.rms_norm(expected_h, weight, 1e-5)
    out = torch.empty_like(hidden)
    h = hidden.clone()
    lib.check(L.kvr_add_rmsnorm(h.data_ptr(), delta.data_ptr(), weight.data_ptr(), out.data_ptr(), rows, H, H, H,
                                H, 1e-5, 0, lib.stream_handle()), "rmsnorm")
    assert bits_equal(h, expected_h)
    diff = (out.float() - expected.float()).abs()
    assert (diff <= 2 ** -7 * expected.float().abs() + 1e-6).all()  # at most one bf16 ulp
    assert (out == expected).float().mean() > 0.99
    gate = torch.randn(rows, I, device=DEV).to(torch.bfloat16)
    up = torch.randn(rows, I, device=DEV).to(torch.bfloat16)
    act = torch.empty_like(gate)
    lib.check(L.kvr_silu_mul(gate.data_ptr(), up.data_ptr(), act.data_ptr(), rows, I, I, I, I, 0,
                             lib.stream_handle()), "silu")
    ref = torch.nn.functional.silu(gate) * up
    assert (act.float() - ref.float()).abs().max() <= 2 ** -7 * ref.float().abs().max()
    assert (act == ref).float().mean() > 0.99


@pytest.mark.parametrize("precision", [0, 1])
@pytest.mark.parametrize("dim,heads,kv_heads,count,length", [(128, 32, 8, 64, 7936), (64, 8, 2, 300, 2000),
                                                              (128, 8, 8, 5, 130), (128, 64, 8, 129, 3001)])
def test_attention_c_abi_status_word_and_precision_modes(lib, precision, dim, heads, kv_heads, count, length):
    """Direct C-ABI call: the workspace status word stays 0 and both P modes meet the fp64 oracle."""
    L = lib.load()
    torch.manual_seed(count + dim)
    positions = sorted(torch.randperm(length)[:count].tolist())
    pos = torch.tensor(positions, device=DEV)
    q = (torch.randn(count, heads, dim, device=DEV) * 0.5).to(torch.bfloat16)
    k = (torch.randn(1, kv_heads, length, dim, device=DEV) * 0.5).to(torch.bfloat16)
    v = (torch.randn(1, kv_heads, length, dim, device=DEV) * 0.5).to(torch.bfloat16)
    out = torch.empty_like(q)
    ws_bytes = L.kvr_attention_workspace_size(count, heads, kv_heads, dim, length)
    ws = torch.full((ws_bytes,), 0xFF, dtype=torch.uint8, device=DEV)
    lib.check(L.kvr_selected_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), pos.data_ptr(),
                                       count, heads, kv_heads, dim, length, length * dim, dim, positions[-1],
                                       dim ** -0.5, precision, ws.data_ptr(), ws_bytes, 0, lib.stream_handle()),
              "attention")
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    expected = oracle.selected_attention_fp64(q.permute(1, 0, 2)[None].cpu(), k.cpu(), v.cpu(), positions)
    _assert_attention_close(out.permute(1, 0, 2)[None], expected)


@pytest.mark.parametrize("arch,theta,dim", [("llama", 500000.0, 128), ("qwen3", 1000000.0, 128),
                                            ("llama", 10000.0, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rope_tables_are_bit_exact_with_the_rotary_module(arch, theta, dim, dtype):
    """kvr_rope_tables against the model's own rotary forward (transformers
    LlamaRotaryEmbedding / Qwen3RotaryEmbedding) at the same positions."""
    from transformers import LlamaConfig, Qwen3Config
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    from budgeted_kv_cache_repair_b200.engine import ModelView

    cls, rot = (Qwen3Config, Qwen3RotaryEmbedding) if arch == "qwen3" else (LlamaConfig, LlamaRotaryEmbedding)
    config = cls(hidden_size=dim * 4, num_attention_heads=4, num_key_value_heads=2, head_dim=dim, rope_theta=theta,
                 max_position_embeddings=131072)
    module = rot(config=config).to("cuda")
    gen = torch.Generator().manual_seed(dim)
    positions = torch.cat((torch.tensor([0, 1, 2, 4095, 131071]),
                           torch.randint(0, 131072, (3000,), generator=gen))).sort().values.cuda()
    view = ModelView.__new__(ModelView)  # only the fields rope_tables reads
    view.rotary, view.head_dim, view.dtype = module, dim, dtype
    cos, sin = view.rope_tables(positions)
    probe = torch.empty(0, dtype=dtype, device="cuda")
    ref_cos, ref_sin = module(probe, positions.unsqueeze(0))
    assert bits_equal(cos, ref_cos[0].contiguous()) and bits_equal(sin, ref_sin[0].contiguous())
