"""The fused qkv projection with a split epilogue (cawq_gemm_qkv) on the GPU.

The reference runs q_proj, k_proj and v_proj as three AWQGEMMLinear forwards
(awq_gemm.rs:146-232). cawq_gemm_qkv is one cawq_gemm over the concatenated
[q | k | v] weights whose epilogue sends each column to its own output, so
with the same plan every element must equal, bit for bit, the element
cawq_gemm writes into a single [rows, N] output; that GEMM's own parity with
the oracle is covered by test_gpu_gemm.py, and one oracle check is repeated
here.
"""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import GEMM_TOL, as_f64, max_rel_err, random_awq, to_numpy, to_torch

pytestmark = pytest.mark.gpu

PATH_DECODE, PATH_PREFILL, PATH_GENERIC = 1, 2, 3
K, NQ, NKV, G = 1024, 512, 128, 128


def _tensors(dev, rows, dtype, seed, nq=NQ, nkv=NKV, k=K, g=G):
    x, qw, qz, s, b = random_awq(k, nq + 2 * nkv, g, dtype, rows, seed)
    t = lambda a, d: to_torch(a, d, dev)
    return (x, qw, qz, s, b), (t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), t(b, dtype))


def _same_as_gemm(dev, rows, dtype, plan, out_dtype=None, seed=0):
    _, (x, qw, qz, s, b) = _tensors(dev, rows, dtype, seed)
    n = NQ + 2 * NKV
    cawq.plan_cache_clear()
    if plan is not None:
        cawq.plan_set(rows, K, n, G, x.dtype, plan)  # cawq_gemm_qkv takes the pinned plan
    try:
        y = cawq.gemm(x, qw, qz, s, G, bias=b, out_dtype=out_dtype, plan=plan)
        q, k, v = cawq.gemm_qkv(x, qw, qz, s, G, NQ, NKV, bias=b, out_dtype=out_dtype)
    finally:
        cawq.plan_cache_clear()
    torch.cuda.synchronize()
    assert q.shape == (rows, NQ) and k.shape == (rows, NKV) and v.shape == (rows, NKV)
    assert torch.equal(q, y[:, :NQ])
    assert torch.equal(k, y[:, NQ:NQ + NKV])
    assert torch.equal(v, y[:, NQ + NKV:])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 5, 16])
@pytest.mark.parametrize("split", [1, 2, 4])
def test_decode_plans_match_gemm(cuda_device, dtype, rows, split):
    _same_as_gemm(cuda_device, rows, dtype,
                  {"path": PATH_DECODE, "split": split, "warps": 2 if rows > 8 else 4,
                   "stages": 3}, seed=rows + split)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [40, 300])
@pytest.mark.parametrize("halves,split", [(1, 1), (1, 4), (2, 1), (2, 2)])
def test_prefill_plans_match_gemm(cuda_device, dtype, rows, halves, split):
    _same_as_gemm(cuda_device, rows, dtype, {"path": PATH_PREFILL, "warps": halves, "split": split},
                  seed=rows + split)


@pytest.mark.parametrize("rows", [3, 40])
def test_generic_path_and_f32_out_match_gemm(cuda_device, rows):
    _same_as_gemm(cuda_device, rows, "f32", {"path": PATH_GENERIC})
    _same_as_gemm(cuda_device, rows, "f16", None, out_dtype=torch.float32, seed=1)


@pytest.mark.parametrize("rows", [1, 64])
def test_outputs_can_be_cache_rows(cuda_device, rows):
    # k and v land in slot 3 of [rows, slots, n_kv] caches; q in a padded
    # buffer: nothing outside the written views may change
    dtype = "f16"
    (xn, qwn, qzn, sn, bn), (x, qw, qz, s, b) = _tensors(cuda_device, rows, dtype, seed=7)
    qbuf = torch.full((rows, NQ + 64), 7.0, dtype=torch.float16, device=cuda_device)
    kc = torch.full((rows, 5, NKV), 7.0, dtype=torch.float16, device=cuda_device)
    vc = torch.full((rows, 5, NKV), 7.0, dtype=torch.float16, device=cuda_device)
    q, k, v = cawq.gemm_qkv(x, qw, qz, s, G, NQ, NKV, bias=b,
                            out=(qbuf[:, :NQ], kc[:, 3], vc[:, 3]))
    torch.cuda.synchronize()
    assert q.data_ptr() == qbuf.data_ptr() and k.data_ptr() == kc[:, 3].data_ptr()
    assert (qbuf[:, NQ:] == 7).all()
    assert (kc[:, [0, 1, 2, 4]] == 7).all() and (vc[:, [0, 1, 2, 4]] == 7).all()
    ref = oracle.gemm_f64(xn, qwn, qzn, sn, G, bias=bn, dtype=dtype, deq_round=rows > 16)
    got = np.concatenate([as_f64(to_numpy(t, dtype), dtype) for t in (q, k, v)], axis=1)
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]


def test_module_matches_three_linears(cuda_device):
    dtype, k, nq, nkv, g = "bf16", 1024, 512, 64, 64
    x, qw, qz, s, b = random_awq(k, nq + 2 * nkv, g, dtype, 6, seed=3)
    t = lambda a, d: to_torch(a, d, cuda_device)
    cols = [(0, nq), (nq, nq + nkv), (nq + nkv, nq + 2 * nkv)]
    lin = [cawq.AWQGEMMLinear(t(qw[:, a // 8:c // 8], "u32"), t(qz[:, a // 8:c // 8], "u32"),
                              t(s[:, a:c], dtype), t(b[a:c], dtype)) for a, c in cols]
    fused = cawq.AWQQKVLinear(*lin)
    xt = t(x, dtype).reshape(2, 3, k)
    q, kk, v = fused(xt)
    assert q.shape == (2, 3, nq) and kk.shape == (2, 3, nkv) and v.shape == (2, 3, nkv)
    torch.cuda.synchronize()
    for got, layer in zip((q, kk, v), lin):
        want = layer(xt).float()
        assert (got.float() - want).abs().max().item() <= \
            2 * GEMM_TOL[dtype] * want.abs().max().item()
    with pytest.raises(cawq.ShapeError):
        cawq.AWQQKVLinear(lin[0], lin[1], lin[0])


def test_split_sizes_are_checked(cuda_device):
    _, (x, qw, qz, s, b) = _tensors(cuda_device, 2, "f16", seed=0)
    with pytest.raises(cawq.ShapeError):
        cawq.gemm_qkv(x, qw, qz, s, G, NQ - 16, NKV + 8, bias=b)  # not multiples of 32
    with pytest.raises(cawq.ShapeError):
        cawq.gemm_qkv(x, qw, qz, s, G, NQ, NKV - 32, bias=b)  # does not add up to N
