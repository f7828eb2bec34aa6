"""The fused modules after a weight tensor is replaced (on the GPU).

AWQGateUpSiluMul and AWQQKVLinear keep the raw pointers of their tensors for
a fast forward. A caller that assigns a new tensor to one of the attributes
(and lets the old one be freed) must get results computed from the new
tensor: the forward re-makes the pointers when an attribute no longer holds
the tensor they were made from. Expected values come from the functional
calls, which take the tensors as they are.
"""

import pytest
import torch

import cube_awq_b200 as cawq
from helpers import random_awq, to_torch

pytestmark = pytest.mark.gpu


def _layer(k, n, g, dtype, seed, dev):
    x, qw, qz, s, b = random_awq(k, n, g, dtype, 2, seed)
    t = lambda a, d: to_torch(a, d, dev)
    return x, cawq.AWQGEMMLinear(t(qw, "u32"), t(qz, "u32"), t(s, dtype), t(b, dtype))


@pytest.mark.parametrize("rows", [1, 40])
def test_gate_up_reassigned_scales(cuda_device, rows):
    k, inter, g, dtype = 256, 256, 64, "f16"
    x, gate = _layer(k, inter, g, dtype, 11, cuda_device)
    _, up = _layer(k, inter, g, dtype, 12, cuda_device)
    m = cawq.AWQGateUpSiluMul(gate, up)
    xt = torch.randn(rows, k, dtype=torch.float16, device=cuda_device)
    m.forward(xt)  # pointers made from the first tensors
    new = (m.scales * 1.5).contiguous()
    m.scales = new
    torch.cuda.empty_cache()
    got = m.forward(xt)
    want = cawq.gemm_silu_mul(xt, m.qweight, m.qzeros, new, g, bias=m.bias)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("rows", [1, 40])
def test_qkv_reassigned_weights(cuda_device, rows):
    k, g, dtype = 256, 64, "f16"
    _, q = _layer(k, 128, g, dtype, 21, cuda_device)
    _, kk = _layer(k, 64, g, dtype, 22, cuda_device)
    _, v = _layer(k, 64, g, dtype, 23, cuda_device)
    m = cawq.AWQQKVLinear(q, kk, v)
    xt = torch.randn(rows, k, dtype=torch.float16, device=cuda_device)
    m.forward(xt)
    m.qweight = torch.flip(m.qweight, dims=[0]).contiguous()
    m.bias = None
    torch.cuda.empty_cache()
    got = m.forward(xt)
    want = cawq.gemm_qkv(xt, m.qweight, m.qzeros, m.scales, g, m.n_q, m.n_kv)
    torch.cuda.synchronize()
    for a, b in zip(got, want):
        assert torch.equal(a, b)
