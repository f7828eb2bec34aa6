"""The CPU oracle pinned against the reference's own known answers.

The reference cannot run here (Rust/CubeCL on wgpu), so the oracle is pinned
by (a) the closed-form answers of its kernel tests (awq_kernel_gemm.rs
:1119-1391) and (b) bit-exact agreement with the golden fixtures written by
tests/golden/make_golden.py, an independent NumPy transcription of the
reference's CPU golden functions (awq_gemm.rs:344-383,
awq_dequantize.rs:169-180, tests/awq_test.rs:138-164).
"""

import numpy as np
import pytest

import oracle
from helpers import (AWQ_ORDER, kat_expected, load_json, load_npz, uniform_kat_tensors)

KATS = load_json("kat_gemm_uniform.json")
MODULE_FIXTURES = [
    "module_forward_b2_m32_k64_n32_g32.npz",
    "module_forward_bias_b2_m32_k64_n32_g32.npz",
    "module_forward_decode_b2_m1_k64_n32_g64.npz",
    "module_forward_4d_1x16x14_k64_n32_g32.npz",
]


def test_nibble_orders_match_reference_tables():
    # AWQ_REVERSE_ORDER (awq_gemm.rs:249) and the unpack shifts (awq_kernel_gemm.rs:10-30)
    word = 0x76543210  # nibble p holds value p
    assert [oracle.nibble(word, c, "awq") for c in range(8)] == [0, 4, 1, 5, 2, 6, 3, 7]
    assert [oracle.nibble(word, c, "natural") for c in range(8)] == list(range(8))
    # packing with AWQ_ORDER then unpacking gives the logical lanes back
    vals = [3, 14, 1, 9, 0, 15, 7, 8]
    packed = 0
    for p, lane in enumerate(AWQ_ORDER):
        packed |= vals[lane] << (4 * p)
    assert [oracle.nibble(packed, c, "awq") for c in range(8)] == vals


@pytest.mark.parametrize("kat", KATS, ids=[k["name"] for k in KATS])
def test_gemm_oracle_closed_form_kats(kat):
    x, qw, qz, sc = uniform_kat_tensors(kat)
    exp = kat_expected(kat, x)
    ref = oracle.gemm_ref(x, qw, qz, sc, kat["group_size"], dtype="f32", order="awq")
    assert np.abs(ref - exp).max() <= kat["tol"]
    f64 = oracle.gemm_f64(x, qw, qz, sc, kat["group_size"], dtype="f32", order="awq")
    assert np.abs(f64 - exp).max() <= 1e-9 * max(1.0, np.abs(exp).max())


@pytest.mark.parametrize("name", MODULE_FIXTURES)
def test_gemm_oracle_matches_module_fixture_bit_exact(name):
    f = load_npz(name)
    x = f["x"].reshape(-1, f["qweight"].shape[0])
    ref = oracle.gemm_ref(x, f["qweight"], f["qzeros"], f["scales"], int(f["group_size"]),
                          bias=f.get("bias"), dtype="f32", order="awq")
    exp = f["expected"].reshape(ref.shape)
    assert np.array_equal(ref.view(np.uint32), exp.view(np.uint32))


def test_dequant_oracle_matches_module_fixture_bit_exact():
    f = load_npz("dequant_module_g2.npz")
    out = oracle.dequant(f["qweight"], f["qzeros"], f["scales"], int(f["group_size"]), "f32", "natural")
    assert np.array_equal(out.view(np.uint32), f["expected"].view(np.uint32))
    # AWQLinear::forward golden (awq_dequantize.rs:239-281): x @ W, f32, k ascending
    fwd = oracle.gemm_ref(f["forward_x"], f["qweight"], f["qzeros"], f["scales"],
                          int(f["group_size"]), dtype="f32", order="natural")
    assert np.array_equal(fwd.view(np.uint32), f["forward_expected"].view(np.uint32))


def test_dequant_oracle_matches_integration_fixture_bit_exact():
    f = load_npz("dequant_integration_g128.npz")
    out = oracle.dequant(f["qweight"], f["qzeros"], f["scales"], int(f["group_size"]), "f32", "natural")
    assert np.array_equal(out.view(np.uint32), f["expected"].view(np.uint32))


def test_f16_rounding_matches_numpy():
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.normal(0, 1, 20000), rng.normal(0, 1e-5, 5000),
                           rng.uniform(-70000, 70000, 2000), [65504.0, 65519.99, 65520.0, 6e-8, 3e-8]])
    lib = oracle.lib()
    got = np.array([lib.awqo_f64_to_f16(float(v)) for v in vals], dtype=np.uint16)
    exp = vals.astype(np.float32).astype(np.float16).view(np.uint16)
    # numpy rounds f64->f32->f16; compare only where that double rounding cannot matter
    exact = vals.astype(np.float32).astype(np.float64) == vals
    assert np.array_equal(got[exact], exp[exact])
    exp64 = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, exp64)


def test_bf16_rounding_matches_bit_formula():
    rng = np.random.default_rng(11)
    vals = rng.normal(0, 3, 20000).astype(np.float32)
    lib = oracle.lib()
    got = np.array([lib.awqo_f32_to_bf16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, oracle.bf16_bits(vals))


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_dequant_oracle_16bit_single_rounding(dtype):
    rng = np.random.default_rng(3)
    k, n, g = 64, 64, 32
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s32 = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    if dtype == "f16":
        sc = s32.astype(np.float16)
        sf = sc.astype(np.float64)
    else:
        sc = oracle.bf16_bits(s32)
        sf = oracle.bf16_to_f32(sc).astype(np.float64)
    out = oracle.dequant(qw, qz, sc, g, dtype, "natural")
    # (q - z) * s is exact in double; one rounding to the 16-bit format
    q = np.array([[(int(qw[r, c // 8]) >> (4 * (c % 8))) & 15 for c in range(n)] for r in range(k)])
    z = np.array([[(int(qz[r, c // 8]) >> (4 * (c % 8))) & 15 for c in range(n)] for r in range(k // g)])
    exact = (q - np.repeat(z, g, axis=0)) * np.repeat(sf, g, axis=0)
    if dtype == "f16":
        assert np.array_equal(out.view(np.uint16), exact.astype(np.float16).view(np.uint16))
    else:
        assert np.array_equal(out, oracle.bf16_bits(exact.astype(np.float32)))


def test_f16_reference_numerics_accumulate_in_f16():
    # The reference's generic F is also the accumulator (awq_kernel_gemm.rs:230-235):
    # a long f16 sum stalls once the ulp exceeds the addend.
    k, n, g = 4096, 32, 128
    x = np.ones((1, k), dtype=np.float16)
    word = sum(1 << (4 * i) for i in range(8))  # every nibble = 1
    qw = np.full((k, n // 8), word, dtype=np.uint32)
    qz = np.zeros((k // g, n // 8), dtype=np.uint32)
    sc = np.ones((k // g, n), dtype=np.float16)
    ref = oracle.gemm_ref(x, qw, qz, sc, g, dtype="f16")
    assert float(ref.astype(np.float32).max()) == 2048.0  # 2048 + 1 rounds back to 2048
    exact = oracle.gemm_f64(x, qw, qz, sc, g, dtype="f16")
    assert float(exact.max()) == 4096.0
