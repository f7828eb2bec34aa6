"""Dequantize kernel parity on the GPU: bit-exact against the oracle and the
reference's fixtures (awq_dequantize.rs:133-237, tests/awq_test.rs:117-221)."""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import load_npz, to_numpy, to_torch

pytestmark = pytest.mark.gpu


def _bits(a):
    return a.view(np.uint16) if a.dtype in (np.float16, np.uint16) else a.view(np.uint32)


@pytest.mark.parametrize("name", ["dequant_module_g2.npz", "dequant_integration_g128.npz"])
def test_dequant_reference_fixtures_bit_exact(cuda_device, name):
    f = load_npz(name)
    layer = cawq.AWQLinear(to_torch(f["qweight"], "u32", cuda_device),
                           to_torch(f["qzeros"], "u32", cuda_device),
                           to_torch(f["scales"], "f32", cuda_device))
    assert layer.group_size() == int(f["group_size"])
    out = layer.dequantize()
    assert list(out.shape) == list(f["expected"].shape)
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), f["expected"].view(np.uint32))
    assert np.abs(got - f["expected"]).max() <= float(f["tol"])


def test_awq_linear_forward_fixture(cuda_device):
    f = load_npz("dequant_module_g2.npz")
    layer = cawq.AWQLinear(to_torch(f["qweight"], "u32", cuda_device),
                           to_torch(f["qzeros"], "u32", cuda_device),
                           to_torch(f["scales"], "f32", cuda_device))
    y = layer.forward(to_torch(f["forward_x"], "f32", cuda_device)).cpu().numpy()
    assert np.abs(y - f["forward_expected"]).max() <= float(f["forward_tol"])
    with pytest.raises(cawq.CubeAwqError, match="RankMismatch"):
        layer.forward(torch.zeros(2, 3, 64, device=cuda_device))


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("order", ["natural", "awq"])
@pytest.mark.parametrize("k,n,g", [(64, 32, 2), (128, 256, 64), (384, 4160, 128), (4096, 4096, 128)])
def test_dequant_random_bit_exact(cuda_device, dtype, order, k, n, g):
    rng = np.random.default_rng(k * 7 + n)
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    if dtype == "f16":
        s = s.astype(np.float16)
    elif dtype == "bf16":
        s = oracle.bf16_bits(s)
    exp = oracle.dequant(qw, qz, s, g, dtype, order)
    out = cawq.dequantize_awq(to_torch(qw, "u32", cuda_device), to_torch(qz, "u32", cuda_device),
                              to_torch(s, dtype, cuda_device), g, order=order)
    torch.cuda.synchronize()
    got = to_numpy(out, dtype)
    assert np.array_equal(_bits(got), _bits(exp))


def test_dequant_unaligned_output_takes_scalar_path(cuda_device):
    k, n, g = 64, 64, 32
    rng = np.random.default_rng(5)
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    buf = torch.empty(k * n + 1, dtype=torch.float32, device=cuda_device)
    out = buf[1:].view(k, n)  # 4-byte aligned only
    cawq.dequantize_native(to_torch(qw, "u32", cuda_device), to_torch(qz, "u32", cuda_device),
                           to_torch(s, "f32", cuda_device), out, g)
    exp = oracle.dequant(qw, qz, s, g, "f32", "natural")
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))


def test_dequant_cfg5_full_size_sampled_rows(cuda_device):
    # 8192 x 57344 (Llama-3-70B gate_up) to f32 on the GPU; every 64-row group
    # block out of a strided sample is checked bit-exact against the oracle.
    from cube_awq_b200 import synth
    k, n, g = 8192, 57344, 128
    w = synth.make_weights(k, n, g, dtype=torch.float32, device=cuda_device, seed=99)
    out = cawq.dequantize_awq(w.qweight, w.qzeros, w.scales, g)
    torch.cuda.synchronize()
    qw, qz, sc = w.qweight.cpu().numpy(), w.qzeros.cpu().numpy(), w.scales.cpu().numpy()
    for grp in (0, 17, 40, 63):
        rows = slice(grp * g, (grp + 1) * g)
        exp = oracle.dequant(qw[rows], qz[grp:grp + 1], sc[grp:grp + 1], g, "f32", "natural")
        got = out[rows].cpu().numpy()
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    assert cawq.device_error() == 0


@pytest.mark.parametrize("offset_floats", [4, 8])
def test_dequant_f32_output_16_byte_aligned(cuda_device, offset_floats):
    # offset 4: 16-byte aligned only (two 128-bit stores per word); offset 8:
    # 32-byte aligned (one 256-bit store per word)
    k, n, g = 200, 256, 40
    rng = np.random.default_rng(6 + offset_floats)
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    buf = torch.full((k * n + offset_floats,), float("nan"), dtype=torch.float32,
                     device=cuda_device)
    out = buf[offset_floats:].view(k, n)
    cawq.dequantize_native(to_torch(qw, "u32", cuda_device), to_torch(qz, "u32", cuda_device),
                           to_torch(s, "f32", cuda_device), out, g)
    exp = oracle.dequant(qw, qz, s, g, "f32", "natural")
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp.view(np.uint32))
    assert torch.isnan(buf[:offset_floats]).all()
