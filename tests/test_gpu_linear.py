"""sm_100a projection kernel (kvr_linear) against fp64 products of the same
nn.Linear / gated-MLP ops with the modules' roundings, and against torch's own
cuBLAS product as the yardstick for fp32 accumulation error."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"

# (rows, k, [(n, paired)]) -- rows 1..300 (more than 256 rows runs as two
# launches), k not a multiple of 64, n not a multiple of the tile, several
# segments in one launch, tiles cut across CTAs (stream-K fix-up).
CASES = [
    (1, 64, [(128, False)]),
    (5, 136, [(200, False)]),
    (37, 4096, [(4096, False)]),
    (64, 4096, [(4096, False), (1024, False), (1024, False)]),
    (64, 4096, [(2048, True)]),
    (64, 2048, [(4096, False)]),
    (100, 512, [(384, True), (96, False)]),
    (200, 1024, [(640, False)]),
    (256, 256, [(256, False)]),
    (300, 512, [(256, False), (64, True)]),
]


def _weights(spec, k, dtype, gen):
    out = []
    for n, paired in spec:
        make = lambda: (torch.randn(n, k, generator=gen, device=DEV) * k ** -0.5).to(dtype)
        out.append((make(), make()) if paired else make())
    return out


def _spacing(v: torch.Tensor, dtype) -> torch.Tensor:
    """Distance between adjacent 16-bit values at the magnitude of ``v``."""
    fi = torch.finfo(dtype)
    exp = torch.floor(torch.log2(v.abs().double().clamp_min(fi.smallest_normal)))
    return torch.pow(2.0, exp - {torch.bfloat16: 7, torch.float16: 10}[dtype])


def _excess(out, x, w):
    """Error of a rounded fp32-accumulated product beyond its own rounding
    (half a spacing), relative to sum |x_i w_i|: the fp32 accumulation error."""
    ref = x.double() @ w.double().T
    mag = x.double().abs() @ w.double().abs().T
    err = (out.double() - ref).abs() - 0.5 * _spacing(out, out.dtype)
    return (err.clamp_min(0) / mag.clamp_min(1e-30)).max().item()


@pytest.fixture(scope="module")
def engine():
    from budgeted_kv_cache_repair_b200 import build, engine

    build.build()
    return engine


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,spec", CASES)
def test_linear_matches_fp32_reference(engine, rows, k, spec, dtype):
    gen = torch.Generator(device=DEV).manual_seed(rows * 7919 + k)
    x = torch.randn(rows, k, generator=gen, device=DEV).to(dtype)
    weights = _weights(spec, k, dtype, gen)
    outs = engine.linear(x, weights)
    again = engine.linear(x, weights)
    torch.cuda.synchronize()
    assert int(engine.linear.last_workspace[:4].view(torch.int32).item()) == 0
    for out, rep, w in zip(outs, again, weights):
        assert torch.equal(out.view(torch.int16), rep.view(torch.int16)), "fixed summation order"
        if isinstance(w, tuple):
            # LlamaMLP on 16-bit tensors: gate and up rounded, SiLU rounded, product rounded.
            gate = (x.double() @ w[0].double().T).to(dtype)
            up = (x.double() @ w[1].double().T).to(dtype)
            act = F.silu(gate)
            expected = act * up
            # gate or up may round one spacing apart at a near-tie (fp32 sums in
            # another order); propagate such a flip through silu (|silu'| < 1.1)
            # and the product, plus the output's and act's own roundings.
            u, a = up.double(), act.double()
            # fp32 accumulation error of gate and up (as bounded for plain segments)
            acc_g = 2 ** -19 * (x.double().abs() @ w[0].double().abs().T)
            acc_u = 2 ** -19 * (x.double().abs() @ w[1].double().abs().T)
            bound = (2 * _spacing(expected, dtype)
                     + u.abs() * (1.1 * (_spacing(gate, dtype) + acc_g) + _spacing(act, dtype))
                     + a.abs() * (_spacing(up, dtype) + acc_u))
            err = (out.double() - expected.double()).abs()
            assert (err <= bound + 1e-7).all(), float((err - bound).max())
            assert (out == expected).float().mean() > 0.97
        else:
            # one rounding of an fp32 sum; the accumulation error (tensor-core
            # fp32 sums in another order than cuBLAS's) stays at fp32 scale,
            # as it does for torch's own cuBLAS product of the same tensors
            assert _excess(out, x, w) < 2 ** -19
            assert _excess(out, x, w) <= max(4 * _excess(x @ w.T, x, w), 2 ** -21)
            expected = (x.double() @ w.double().T).to(dtype)
            assert (out == expected).float().mean() > 0.97


def test_linear_writes_strided_outputs_in_place(engine):
    """q/k/v segments land in column slices of one buffer (the refresh's layout)."""
    gen = torch.Generator(device=DEV).manual_seed(3)
    rows, k = 48, 1024
    x = torch.randn(rows, 2 * k, generator=gen, device=DEV).to(torch.bfloat16)[:, :k]  # strided input
    wq, wk, wv = (torch.randn(n, k, generator=gen, device=DEV).to(torch.bfloat16) * 0.03 for n in (512, 128, 128))
    buf = torch.full((rows, 768), 7.0, device=DEV, dtype=torch.bfloat16)
    engine.linear(x, [wq, wk, wv], outs=[buf[:, :512], buf[:, 512:640], buf[:, 640:]])
    torch.cuda.synchronize()
    fused = torch.cat([wq, wk, wv])
    assert _excess(buf, x, fused) < 2 ** -19
