"""The mid-M tensor-core kernel with the dequantized weights as the MMA's A
operand in tensor memory (prefill plan warps = 4, rows <= 128): parity with
the oracle that rounds the weights to F exactly as the reference's gemm_awq
does (src/kernel/awq_kernel_gemm.rs:181-439), for every split of K, both
nibble orders, bias, fp32 output, a column slice of a wider output, the qkv
three-way output split, ragged N and rows that are not a multiple of 16."""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import GEMM_TOL, as_f64, max_rel_err, random_awq, to_numpy, to_torch

PATH_PREFILL = 2
TW = 4  # plan.warps of the weights-in-tensor-memory tile
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}

pytestmark = pytest.mark.gpu


def _run(x, qw, qz, s, g, dtype, dev, split, tile_n=256, **kw):
    t = lambda a, d: to_torch(a, d, dev)
    return cawq.gemm(t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), g,
                     plan={"path": PATH_PREFILL, "warps": TW, "split": split, "tile_n": tile_n},
                     **kw)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows,tile_n", [(1, 256), (17, 256), (32, 256), (45, 256), (64, 256),
                                         (100, 256), (128, 256), (1, 512), (17, 512), (32, 512),
                                         (45, 512), (64, 512)])
@pytest.mark.parametrize("split", [1, 2, 4, 8])
def test_tw_parity(cuda_device, dtype, rows, tile_n, split):
    # n = 800: a partial last column tile of 256 (32 columns) or 512 (288)
    k, n, g = 2048, 800, 128
    x, qw, qz, s, _ = random_awq(k, n, g, dtype, rows, seed=rows * 7 + split)
    y = _run(x, qw, qz, s, g, dtype, cuda_device, split, tile_n)
    torch.cuda.synchronize()
    got = as_f64(to_numpy(y, dtype), dtype)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype=dtype, deq_round=True)
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]
    assert cawq.device_error() == 0


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("k,n,g", [(1024, 4096, 64), (3584, 4608, 64), (4096, 1024, 128),
                                   (512, 256, 512)])
def test_tw_shapes(cuda_device, dtype, k, n, g):
    rows = 64
    x, qw, qz, s, _ = random_awq(k, n, g, dtype, rows, seed=k + n)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype=dtype, deq_round=True)
    for tile_n in (256, 512):
        for split in (1, 4):
            if split > k // 64:
                continue
            y = _run(x, qw, qz, s, g, dtype, cuda_device, split, tile_n)
            torch.cuda.synchronize()
            got = as_f64(to_numpy(y, dtype), dtype)
            assert max_rel_err(got, ref) <= GEMM_TOL[dtype], f"split {split} tile_n {tile_n}"


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("split", [1, 2])
@pytest.mark.parametrize("tile_n", [256, 512])
def test_tw_bias_natural_order_fp32_out_and_ld(cuda_device, dtype, split, tile_n):
    rows, k, n, g = 40, 1024, 512, 128
    x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed=19 + split)
    full = torch.zeros(rows, 2 * n, dtype=torch.float32, device=cuda_device)
    _run(x, qw, qz, s, g, dtype, cuda_device, split, tile_n, bias=to_torch(b, dtype, cuda_device),
         out=full[:, n:], out_dtype=torch.float32, order="natural")
    torch.cuda.synchronize()
    ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b, dtype=dtype, order="natural", deq_round=True)
    got = full.cpu().numpy()
    assert max_rel_err(got[:, n:], ref) <= 2e-3
    assert float(np.abs(got[:, :n]).max()) == 0.0


@pytest.mark.parametrize("split", [1, 4])
@pytest.mark.parametrize("tile_n", [256, 512])
def test_tw_qkv_split_outputs_match_the_plain_call(cuda_device, split, tile_n):
    # the three-way output map: every element bit-identical to the one-output
    # call with the same plan
    rows, k, g = 48, 1024, 128
    nq, nk, nv = 512, 256, 256
    n = nq + nk + nv
    x, qw, qz, s, _ = random_awq(k, n, g, "f16", rows, seed=23)
    t = lambda a, d: to_torch(a, d, cuda_device)
    plan = {"path": PATH_PREFILL, "warps": TW, "split": split, "tile_n": tile_n}
    xt, qwt, qzt, st = t(x, "f16"), t(qw, "u32"), t(qz, "u32"), t(s, "f16")
    y = cawq.gemm(xt, qwt, qzt, st, g, plan=plan)
    q = torch.empty(rows, nq, dtype=torch.float16, device=cuda_device)
    kc = torch.zeros(rows, 2 * nk, dtype=torch.float16, device=cuda_device)
    v = torch.empty(rows, nv, dtype=torch.float16, device=cuda_device)
    cawq.plan_set(rows, k, n, g, torch.float16, plan)  # the qkv call takes the cached plan
    try:
        assert cawq.plan_get(rows, k, n, g, torch.float16)["warps"] == TW
        cawq.gemm_qkv(xt, qwt, qzt, st, g, nq, nk, out=(q, kc[:, :nk], v))
        torch.cuda.synchronize()
    finally:
        cawq.plan_cache_clear()
    assert torch.equal(q, y[:, :nq])
    assert torch.equal(kc[:, :nk], y[:, nq:nq + nk])
    assert torch.equal(v, y[:, nq + nk:])
    assert float(kc[:, nk:].abs().max()) == 0.0


@pytest.mark.parametrize("tile_n", [256, 512])
def test_tw_chain_reads_the_previous_output(cuda_device, tile_n):
    # Dependent launches back to back (programmatic dependent launch): each
    # reads the previous output as X and writes the buffer the one before read.
    rows, k, g = 64, 1024, 128
    x, qw, qz, s, _ = random_awq(k, k, g, "f16", rows, seed=31)
    _, qw2, qz2, s2, _ = random_awq(k, k, g, "f16", rows, seed=32)
    t = lambda a, d: to_torch(a, d, cuda_device)
    plan = {"path": PATH_PREFILL, "warps": TW, "split": 2, "tile_n": tile_n}
    w1 = (t(qw, "u32"), t(qz, "u32"), t(s, "f16"))
    w2 = (t(qw2, "u32"), t(qz2, "u32"), t(s2, "f16"))
    a = t(x, "f16")
    b = torch.empty_like(a)
    for _ in range(2):
        a = t(x, "f16")
        cawq.gemm(a, *w1, g, out=b, plan=plan)
        cawq.gemm(b, *w2, g, out=a, plan=plan)
        cawq.gemm(a, *w1, g, out=b, plan=plan)
    torch.cuda.synchronize()
    h1 = oracle.gemm_f64(x, qw, qz, s, g, dtype="f16", deq_round=True).astype(np.float16)
    h2 = oracle.gemm_f64(h1, qw2, qz2, s2, g, dtype="f16", deq_round=True)
    assert max_rel_err(a.float().cpu().numpy(), h2) <= 2 * GEMM_TOL["f16"]
    h3 = oracle.gemm_f64(a.cpu().numpy(), qw, qz, s, g, dtype="f16", deq_round=True)
    assert max_rel_err(b.float().cpu().numpy(), h3) <= GEMM_TOL["f16"]


def test_tw_repeated_launches_are_bit_identical(cuda_device):
    rows, k, n, g = 96, 4096, 2048, 128
    x, qw, qz, s, _ = random_awq(k, n, g, "bf16", rows, seed=41)
    first = _run(x, qw, qz, s, g, "bf16", cuda_device, 4)
    for _ in range(5):
        again = _run(x, qw, qz, s, g, "bf16", cuda_device, 4)
        torch.cuda.synchronize()
        assert torch.equal(first, again)
    x, qw, qz, s, _ = random_awq(k, n, g, "bf16", 48, seed=42)
    first = _run(x, qw, qz, s, g, "bf16", cuda_device, 4, 512)
    for _ in range(3):
        again = _run(x, qw, qz, s, g, "bf16", cuda_device, 4, 512)
        torch.cuda.synchronize()
        assert torch.equal(first, again)


def test_tw_plan_is_refused_where_it_does_not_apply(cuda_device):
    x, qw, qz, s, _ = random_awq(1024, 512, 32, "f16", 64, seed=5)
    with pytest.raises(Exception):  # group size 32: stages hold whole groups only
        _run(x, qw, qz, s, 32, "f16", cuda_device, 1)
    x, qw, qz, s, _ = random_awq(1024, 512, 128, "f16", 129, seed=5)
    with pytest.raises(Exception):  # more than 128 rows
        _run(x, qw, qz, s, 128, "f16", cuda_device, 1)
    x, qw, qz, s, _ = random_awq(1024, 512, 128, "f16", 65, seed=5)
    with pytest.raises(Exception):  # 512-column tiles: at most 64 rows
        _run(x, qw, qz, s, 128, "f16", cuda_device, 1, 512)
