"""Numerics of the fused GEMM on inputs built to stress its fold, and the
autotuner's plan choice (on the GPU).

The decode kernel turns nibbles into magic-number operands (1024 + q for f16,
128 + q for bf16), lets the tensor core accumulate x * (offset + q) over a
quantization group together with sum(x), and per group adds
s * (D - (offset + z) * sum(x)) in fp32. With activations whose mean is far
from zero, D and (offset + z) * sum(x) are both large and nearly cancel; a few
activations 300 times larger than the rest make it worse. The reference
computes (q - z) * s per weight (awq_kernel_gemm.rs:355-362), so these inputs
are where a difference would show. Every case is checked against the exact
(fp64) oracle with the parity tests' bound, max|y - ref| <= tol * ||ref||_inf
(tol: f32 1e-3, f16 5e-3, bf16 1e-2), on the decode kernel (with and without
split K), the tensor-core prefill kernel and the generic kernel.

The f32-activation paths carry x on the tensor cores as a bf16 hi + lo pair
(16 significand bits); the error budget that gives is far inside 1e-3 (see
test_f32_split_error_budget).
"""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import GEMM_TOL, as_f64, max_rel_err, random_awq, to_numpy, to_torch

pytestmark = pytest.mark.gpu

PATH_DECODE, PATH_PREFILL, PATH_GENERIC = 1, 2, 3
TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _activations(rows, k, dtype, seed, mean=4.0, outliers=12, factor=300.0):
    rng = np.random.default_rng(seed)
    x32 = (rng.standard_normal((rows, k)) + mean).astype(np.float32)
    if outliers:
        x32[:, rng.choice(k, size=outliers, replace=False)] *= factor
    if dtype == "f16":
        return x32.astype(np.float16)
    if dtype == "bf16":
        return oracle.bf16_bits(x32)
    return x32


def _check(dev, dtype, rows, k, n, g, plan, mean=4.0, outliers=12, seed=0):
    _, qw, qz, s, _ = random_awq(k, n, g, dtype, rows, seed)
    x = _activations(rows, k, dtype, seed + 1, mean, outliers)
    t = lambda a, d: to_torch(a, d, dev)
    y = cawq.gemm(t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), g, plan=plan)
    torch.cuda.synchronize()
    got = as_f64(to_numpy(y, dtype), dtype)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype=dtype, deq_round=False)
    err = max_rel_err(got, ref)
    assert err <= GEMM_TOL[dtype], err
    return err


DECODE_PLANS = [
    None,                                                        # planner default
    {"path": PATH_DECODE, "split": 1, "warps": 2, "stages": 4},  # whole K in one CTA
    {"path": PATH_DECODE, "split": 8, "warps": 2, "stages": 2},  # split K over a cluster
]


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("g", [64, 128])
@pytest.mark.parametrize("rows", [1, 3, 9])
@pytest.mark.parametrize("plan", DECODE_PLANS, ids=["default", "split1", "split8"])
def test_decode_fold_with_offset_mean_and_outliers(cuda_device, dtype, g, rows, plan):
    _check(cuda_device, dtype, rows, 4096, 1024, g, plan)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("g", [64, 128])
def test_decode_fold_large_mean_no_outliers(cuda_device, dtype, g):
    # mean 30: the offset term is ~30x the signal before any outlier
    _check(cuda_device, dtype, 1, 11008, 512, g, None, mean=30.0, outliers=0)


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("g", [64, 128])
@pytest.mark.parametrize("rows", [40, 300])
def test_prefill_with_offset_mean_and_outliers(cuda_device, dtype, g, rows):
    _check(cuda_device, dtype, rows, 2048, 512, g, None)


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_generic_with_offset_mean_and_outliers(cuda_device, dtype):
    _check(cuda_device, dtype, 24, 1024, 256, 128, {"path": PATH_GENERIC})


def test_f32_split_error_budget(cuda_device):
    # f32 activations enter the tensor core as hi = bf16(x), lo = bf16(x - hi):
    # |x - hi - lo| <= 2^-16 |x|, so each product x * w carries a relative error
    # of at most 2^-16 and the sum at most 2^-16 * sum|x w|. With x ~ N(0, 1)
    # and K = 4096 that is ~1e-4 of ||ref||_inf in the worst case; the
    # measured error must stay inside that budget (and far inside 1e-3).
    rows, k, n, g = 1, 4096, 4096, 128
    x, qw, qz, s, _ = random_awq(k, n, g, "f32", rows, seed=5)
    t = lambda a, d: to_torch(a, d, cuda_device)
    y = cawq.gemm(t(x, "f32"), t(qw, "u32"), t(qz, "u32"), t(s, "f32"), g)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype="f32", deq_round=False)
    # sum_k |x w| per output, the scale of the worst-case split error
    w = oracle.dequant(qw, qz, s, g, "f32", "awq").astype(np.float64)
    absref = np.abs(x.astype(np.float64)) @ np.abs(w)
    budget = 2.0 ** -16 * absref + 1e-6 * np.abs(ref).max()
    assert np.all(np.abs(got - ref) <= budget)
    assert max_rel_err(got, ref) <= 1e-4


def test_autotune_plan_is_valid_cached_and_matches_the_oracle(cuda_device):
    rows, k, n, g = 2, 4096, 4096, 128
    x, qw, qz, s, _ = random_awq(k, n, g, "f16", rows, seed=9)
    t = lambda a, d: to_torch(a, d, cuda_device)
    xt, qwt, qzt, st = t(x, "f16"), t(qw, "u32"), t(qz, "u32"), t(s, "f16")
    cawq.plan_cache_clear()
    try:
        best = cawq.autotune(xt, qwt, qzt, st, g)
        assert best["path"] in (PATH_DECODE, PATH_PREFILL, PATH_GENERIC)
        # the cache now answers with the tuned plan, every time
        assert cawq.plan_get(rows, k, n, g, torch.float16) == best
        assert cawq.plan_get(rows, k, n, g, torch.float16) == best
        ref = oracle.gemm_f64(x, qw, qz, s, g, dtype="f16", deq_round=False)
        y_auto = cawq.gemm(xt, qwt, qzt, st, g)          # cached plan
        y_plan = cawq.gemm(xt, qwt, qzt, st, g, plan=best)
        torch.cuda.synchronize()
        assert torch.equal(y_auto, y_plan)
        assert max_rel_err(as_f64(to_numpy(y_auto, "f16"), "f16"), ref) <= GEMM_TOL["f16"]
    finally:
        cawq.plan_cache_clear()


@pytest.mark.parametrize("rows", [8, 16, 24, 32, 64])
def test_autotune_across_the_crossover_matches_the_oracle(cuda_device, rows):
    k, n, g = 3584, 3584, 64
    x, qw, qz, s, _ = random_awq(k, n, g, "f16", rows, seed=10 + rows)
    t = lambda a, d: to_torch(a, d, cuda_device)
    xt, qwt, qzt, st = t(x, "f16"), t(qw, "u32"), t(qz, "u32"), t(s, "f16")
    cawq.plan_cache_clear()
    try:
        best = cawq.autotune(xt, qwt, qzt, st, g)
        y = cawq.gemm(xt, qwt, qzt, st, g, plan=best)
        torch.cuda.synchronize()
        ref = oracle.gemm_f64(x, qw, qz, s, g, dtype="f16", deq_round=False)
        assert max_rel_err(as_f64(to_numpy(y, "f16"), "f16"), ref) <= GEMM_TOL["f16"]
    finally:
        cawq.plan_cache_clear()
