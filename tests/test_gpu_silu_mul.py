"""The SiLU-gated gate_up GEMM (cawq_gemm_silu_mul) on the GPU.

The reference has no fused counterpart: a gated MLP runs gate_proj and
up_proj as two AWQGEMMLinear calls (awq_gemm.rs:146-232) and applies
silu(gate) * up afterwards. The expected value is built that way from the
exact oracle, in fp64: gate = oracle.gemm_f64(x, W_gate), up =
oracle.gemm_f64(x, W_up), ref = gate / (1 + exp(-gate)) * up. The kernel's
error in gate and up is bounded by the GEMM tolerance (tol * ||gate||_inf and
tol * ||up||_inf, helpers.GEMM_TOL); since |silu'| <= 1.1, to first order
|y - ref| <= (1.1 * ||up|| * tol * ||gate|| + ||silu(gate)|| * tol * ||up||)
<= 2.1 * tol * ||gate||_inf * ||up||_inf, which is the bound asserted here,
plus the output's own rounding (half an ulp of |ref|).
"""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import GEMM_TOL, as_f64, random_awq, to_numpy, to_torch

pytestmark = pytest.mark.gpu

PATH_DECODE, PATH_PREFILL = 1, 2
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
ULP = {"f16": 2.0 ** -11, "bf16": 2.0 ** -8}


def _problem(rows, k, inter, g, dtype, seed):
    """Seeded gate and up projections (AutoAWQ layout each) and one input."""
    x, qg, zg, sg, bg = random_awq(k, inter, g, dtype, rows, seed)
    _, qu, zu, su, bu = random_awq(k, inter, g, dtype, rows, seed + 1000)
    return x, (qg, zg, sg, bg), (qu, zu, su, bu)


def _expected(x, gate, up, g, dtype, bias):
    gv = oracle.gemm_f64(x, *gate[:3], g, bias=gate[3] if bias else None, dtype=dtype,
                         deq_round=False)
    uv = oracle.gemm_f64(x, *up[:3], g, bias=up[3] if bias else None, dtype=dtype,
                         deq_round=False)
    return gv / (1.0 + np.exp(-gv)) * uv, gv, uv


def _check(y, dtype, ref, gv, uv):
    got = as_f64(to_numpy(y, dtype), dtype)
    assert got.shape == ref.shape
    bound = 2.1 * GEMM_TOL[dtype] * np.abs(gv).max() * np.abs(uv).max()
    err = np.abs(got - ref) - ULP[dtype] * np.abs(ref)
    assert err.max() <= bound, (float(err.max()), float(bound))


def _fused_tensors(gate, up, dtype, dev, bias):
    t = lambda a, d: to_torch(a, d, dev)
    cat = lambda a, b, d: cawq.interleave_gate_up(torch.cat([t(a, d), t(b, d)], dim=-1))
    qw = cat(gate[0], up[0], "u32")
    qz = cat(gate[1], up[1], "u32")
    sc = cat(gate[2], up[2], dtype)
    b = cat(gate[3], up[3], dtype) if bias else None
    return qw, qz, sc, b


def _run(dev, rows, k, inter, g, dtype, plan=None, bias=False, seed=0):
    x, gate, up = _problem(rows, k, inter, g, dtype, seed)
    qw, qz, sc, b = _fused_tensors(gate, up, dtype, dev, bias)
    y = cawq.gemm_silu_mul(to_torch(x, dtype, dev), qw, qz, sc, g, bias=b, plan=plan)
    torch.cuda.synchronize()
    assert y.shape == (rows, inter) and y.dtype == TDT[dtype]
    ref, gv, uv = _expected(x, gate, up, g, dtype, bias)
    return y, ref, gv, uv


def test_interleave_is_a_column_permutation(cuda_device):
    rng = np.random.default_rng(5)
    a = rng.integers(-2**31, 2**31, (6, 2 * 48), dtype=np.int64).astype(np.int32)
    got = cawq.interleave_gate_up(torch.from_numpy(a).to(cuda_device)).cpu().numpy()
    gate, up = a[:, :48], a[:, 48:]
    want = np.concatenate([np.concatenate([gate[:, j:j + 16], up[:, j:j + 16]], axis=1)
                           for j in range(0, 48, 16)], axis=1)
    assert np.array_equal(got, want)
    h = torch.randn(3, 2, 512, dtype=torch.bfloat16, device=cuda_device)
    got = cawq.interleave_gate_up(h)
    want = torch.stack([h[..., :256].reshape(3, 2, 2, 128), h[..., 256:].reshape(3, 2, 2, 128)],
                       dim=3).reshape(3, 2, 512)
    assert torch.equal(got, want)
    with pytest.raises(cawq.ShapeError):
        cawq.interleave_gate_up(torch.zeros(4, 384, dtype=torch.float16, device=cuda_device))


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 2, 5, 8, 16])
@pytest.mark.parametrize("k,inter,g", [(512, 256, 128), (1024, 384, 64), (4096, 1408, 128),
                                       (3584, 640, 64)])
def test_decode_default_plan(cuda_device, dtype, rows, k, inter, g):
    y, ref, gv, uv = _run(cuda_device, rows, k, inter, g, dtype, bias=rows % 2 == 1, seed=rows)
    _check(y, dtype, ref, gv, uv)


@pytest.mark.parametrize("split", [1, 2, 4, 8])
@pytest.mark.parametrize("warps", [2, 4, 8])
@pytest.mark.parametrize("rows,dtype", [(3, "f16"), (11, "bf16")])
def test_decode_every_plan(cuda_device, split, warps, rows, dtype):
    # 2 * inter = 1280 columns: five 256-column gate / up block pairs, so the
    # last band of every strip count is partly out of range
    if rows > 8 and 2 * warps > 8:
        pytest.skip("more warps than a 16-row tile allows")
    plan = {"path": PATH_DECODE, "split": split, "warps": warps, "stages": 3}
    y, ref, gv, uv = _run(cuda_device, rows, 2048, 640, 128, dtype, plan=plan, bias=True,
                          seed=split + warps)
    _check(y, dtype, ref, gv, uv)


@pytest.mark.parametrize("halves,split", [(1, 1), (1, 2), (1, 4), (1, 8), (2, 1)])
@pytest.mark.parametrize("rows", [20, 64, 200])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_prefill_every_plan(cuda_device, halves, split, rows, dtype):
    plan = {"path": PATH_PREFILL, "warps": halves, "split": split}
    y, ref, gv, uv = _run(cuda_device, rows, 1024, 384, 128, dtype, plan=plan, bias=True,
                          seed=rows + split)
    _check(y, dtype, ref, gv, uv)


def test_prefill_two_halves_refuses_split_k(cuda_device):
    # the 256-row tile's split-K hand-off has no SiLU epilogue
    with pytest.raises(cawq.CubeAwqError):
        _run(cuda_device, 64, 1024, 384, 128, "f16", plan={"path": PATH_PREFILL, "warps": 2,
                                                            "split": 2})


@pytest.mark.parametrize("rows", [64, 300, 2048])
def test_prefill_default_plan(cuda_device, rows):
    # Qwen2-7B-like gate_up shape (K 3584, 2 x 2560 columns); rows > 1024 are
    # checked on a sample so the fp64 oracle stays fast
    dtype, k, inter, g = "f16", 3584, 2560, 64
    x, gate, up = _problem(rows, k, inter, g, dtype, seed=rows)
    qw, qz, sc, b = _fused_tensors(gate, up, dtype, cuda_device, True)
    y = cawq.gemm_silu_mul(to_torch(x, dtype, cuda_device), qw, qz, sc, g, bias=b)
    torch.cuda.synchronize()
    pick = np.arange(rows) if rows <= 300 else np.r_[0:3, 1021:1027, rows - 3:rows]
    ref, gv, uv = _expected(x[pick], gate, up, g, dtype, True)
    _check(y[torch.from_numpy(pick).to(cuda_device)], dtype, ref, gv, uv)


def test_module_matches_two_linears(cuda_device):
    # AWQGateUpSiluMul against the unfused composition of two AWQGEMMLinear
    # layers and torch's silu, on a rank-3 input
    dtype, k, inter, g = "bf16", 1024, 512, 64
    x, gate, up = _problem(6, k, inter, g, dtype, seed=77)
    t = lambda a, d: to_torch(a, d, cuda_device)
    lg = cawq.AWQGEMMLinear(t(gate[0], "u32"), t(gate[1], "u32"), t(gate[2], dtype),
                            t(gate[3], dtype))
    lu = cawq.AWQGEMMLinear(t(up[0], "u32"), t(up[1], "u32"), t(up[2], dtype), t(up[3], dtype))
    fused = cawq.AWQGateUpSiluMul(lg, lu)
    xt = t(x, dtype).reshape(2, 3, k)
    y = fused(xt)
    assert y.shape == (2, 3, inter)
    ref = (torch.nn.functional.silu(lg(xt).double()) * lu(xt).double())
    torch.cuda.synchronize()
    gv = lg(xt).double().abs().max().item()
    uv = lu(xt).double().abs().max().item()
    err = (y.double() - ref).abs() - ULP[dtype] * ref.abs()
    assert err.max().item() <= 2.1 * GEMM_TOL[dtype] * gv * uv
    assert fused(xt[:, :0]).shape == (2, 0, inter)


def test_module_rejects_mismatched_projections(cuda_device):
    mk = lambda n, dt=torch.float16: cawq.AWQGEMMLinear(
        torch.zeros(256, n // 8, dtype=torch.int32, device=cuda_device),
        torch.zeros(2, n // 8, dtype=torch.int32, device=cuda_device),
        torch.ones(2, n, dtype=dt, device=cuda_device))
    with pytest.raises(cawq.ShapeError):
        cawq.AWQGateUpSiluMul(mk(256), mk(384))
    with pytest.raises(cawq.ShapeError):
        cawq.AWQGateUpSiluMul(mk(192), mk(192))  # not whole 128-column blocks
    with pytest.raises(cawq.DTypeError):
        cawq.AWQGateUpSiluMul(mk(256, torch.float32), mk(256, torch.float32))


@pytest.mark.parametrize("path", [PATH_DECODE, PATH_PREFILL])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_saturated_gates(cuda_device, path, dtype):
    # gate biases of -200 / +200 push silu to its limits (0 and the identity):
    # the exp in the denominator overflows to inf for the negative ones, and
    # the output must be 0 there, never NaN
    rows = 4 if path == PATH_DECODE else 40
    k, inter, g = 512, 256, 128
    x, gate, up = _problem(rows, k, inter, g, dtype, seed=9)
    gb = np.where(np.arange(inter) % 2 == 0, -200.0, 200.0).astype(np.float32)
    gate = gate[:3] + ((oracle.bf16_bits(gb) if dtype == "bf16" else gb.astype(np.float16)),)
    qw, qz, sc, b = _fused_tensors(gate, up, dtype, cuda_device, True)
    y = cawq.gemm_silu_mul(to_torch(x, dtype, cuda_device), qw, qz, sc, g, bias=b,
                           plan={"path": path, "split": 2, "warps": 2 if path == PATH_DECODE else 1,
                                 "stages": 3})
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert (y[:, 0::2] == 0).all()
    ref, gv, uv = _expected(x, gate, up, g, dtype, True)
    _check(y, dtype, ref, gv, uv)
