"""Generates the golden fixtures under tests/golden/ from the reference's tests.

The reference (joshuawm/cube-awq) is Rust/CubeCL on wgpu and cannot be built
or run on this machine (no cargo, no graphics stack), so the fixtures restate
its known-answer tests: the same input formulas, and expected outputs from

* closed forms the reference states in its test comments
  (src/kernel/awq_kernel_gemm.rs:1125-1391), kept as exact numbers, and
* a NumPy transcription of the reference's own CPU golden functions
  (`cpu_reference`, src/modules/awq_gemm.rs:344-383; the dequant loops of
  src/modules/awq_dequantize.rs:169-180 and tests/awq_test.rs:138-164),
  evaluated in float32 with one rounding per multiply and add, k ascending.

Run from the repository root:  python tests/golden/make_golden.py
The outputs are committed; tests only read them.
"""

from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)          # awq_gemm.rs:248
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)  # awq_gemm.rs:249


# --------------------------------------------------------------- packing
def pack_awq(vals8) -> int:
    """pack_i4 of awq_gemm.rs:270-277: logical lane AWQ_ORDER[p] -> nibble p."""
    packed = 0
    for packed_lane, logical_lane in enumerate(AWQ_ORDER):
        packed |= (int(vals8[logical_lane]) & 0xF) << (packed_lane * 4)
    return packed


def pack_natural(vals8) -> int:
    """pack_i4 of awq_dequantize.rs:121-127 / pack_u32_cpu of awq_test.rs:104-112."""
    packed = 0
    for i, v in enumerate(vals8):
        packed |= (int(v) & 0xF) << (i * 4)
    return packed


def unpack_awq(packed: int, logical_lane: int) -> float:
    """unpack_i4 of awq_gemm.rs:279-282."""
    return float((packed >> (AWQ_REVERSE_ORDER[logical_lane] * 4)) & 0xF)


# ------------------------------------------------- module GEMM fixture
def module_layer(k: int, n: int, g: int):
    """build_layer of awq_gemm.rs:284-342 (non-uniform AWQ-order fixture)."""
    npk, ng = n // 8, k // g
    qweight = np.zeros((k, npk), dtype=np.uint32)
    qzeros = np.zeros((ng, npk), dtype=np.uint32)
    scales = np.zeros((ng, n), dtype=np.float32)
    for row in range(k):
        for col in range(npk):
            qweight[row, col] = pack_awq([(row + col + lane) % 16 for lane in range(8)])
    for grp in range(ng):
        for col in range(npk):
            qzeros[grp, col] = pack_awq([(grp + col + lane) % 8 for lane in range(8)])
        for col in range(n):
            # 0.05 + group * 0.01 + col * 0.002, evaluated in f32 as the Rust code does
            scales[grp, col] = np.float32(
                np.float32(np.float32(0.05) + np.float32(grp) * np.float32(0.01))
                + np.float32(col) * np.float32(0.002))
    return qweight, qzeros, scales


def cpu_reference(inp, qweight, qzeros, scales, bias, rows, k, n, g):
    """cpu_reference of awq_gemm.rs:344-383, float32, k ascending."""
    npk = n // 8
    inp = inp.reshape(rows, k).astype(np.float32)
    # w[kk, col] = (w - z) * scale in f32 (one rounding)
    w = np.zeros((k, n), dtype=np.float32)
    for kk in range(k):
        grp = kk // g
        for col in range(n):
            wv = np.float32(unpack_awq(int(qweight[kk, col // 8]), col % 8))
            zv = np.float32(unpack_awq(int(qzeros[grp, col // 8]), col % 8))
            w[kk, col] = np.float32((wv - zv) * scales[grp, col])
    out = np.zeros((rows, n), dtype=np.float32)
    acc = np.zeros((rows, n), dtype=np.float32)
    for kk in range(k):
        prod = (inp[:, kk:kk + 1] * w[kk:kk + 1, :]).astype(np.float32)
        acc = (acc + prod).astype(np.float32)
    out[:] = acc
    if bias is not None:
        out = (out + bias.astype(np.float32)[None, :]).astype(np.float32)
    return out


def input_formula(count: int, modulo: int, center: float, step: float):
    """((idx % modulo) as f32 - center) * step, evaluated in f32."""
    idx = np.arange(count)
    return ((np.float32(1.0) * (idx % modulo).astype(np.float32) - np.float32(center))
            * np.float32(step)).astype(np.float32)


def module_cases():
    cases = {}
    # test_forward_matches_cpu_reference (awq_gemm.rs:408-450)
    b, m, k, n, g = 2, 32, 64, 32, 32
    qw, qz, sc = module_layer(k, n, g)
    x = input_formula(b * m * k, 17, 8.0, 0.1).reshape(b, m, k)
    cases["forward_b2_m32_k64_n32_g32"] = dict(
        x=x, qweight=qw, qzeros=qz, scales=sc,
        expected=cpu_reference(x, qw, qz, sc, None, b * m, k, n, g).reshape(b, m, n),
        group_size=np.int64(g), tol=np.float64(1e-2))
    # test_forward_with_bias_matches_cpu_reference (:452-503)
    bias = (np.float32(-0.2) + np.arange(n).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    x = input_formula(b * m * k, 13, 6.0, 0.07).reshape(b, m, k)
    cases["forward_bias_b2_m32_k64_n32_g32"] = dict(
        x=x, qweight=qw, qzeros=qz, scales=sc, bias=bias,
        expected=cpu_reference(x, qw, qz, sc, bias, b * m, k, n, g).reshape(b, m, n),
        group_size=np.int64(g), tol=np.float64(1e-2))
    # test_forward_decode_shape_matches_cpu_reference (:517-559)
    b, m, k, n, g = 2, 1, 64, 32, 64
    qw, qz, sc = module_layer(k, n, g)
    x = input_formula(b * m * k, 11, 5.0, 0.09).reshape(b, m, k)
    cases["forward_decode_b2_m1_k64_n32_g64"] = dict(
        x=x, qweight=qw, qzeros=qz, scales=sc,
        expected=cpu_reference(x, qw, qz, sc, None, b * m, k, n, g).reshape(b, m, n),
        group_size=np.int64(g), tol=np.float64(1e-2))
    # test_forward_4d_input_matches_cpu_reference (:561-604)
    d0, d1, d2, k, n, g = 1, 16, 14, 64, 32, 32
    qw, qz, sc = module_layer(k, n, g)
    rows = d0 * d1 * d2
    x = input_formula(rows * k, 23, 11.0, 0.03).reshape(d0, d1, d2, k)
    cases["forward_4d_1x16x14_k64_n32_g32"] = dict(
        x=x, qweight=qw, qzeros=qz, scales=sc,
        expected=cpu_reference(x, qw, qz, sc, None, rows, k, n, g).reshape(d0, d1, d2, n),
        group_size=np.int64(g), tol=np.float64(1e-2))
    return cases


# ------------------------------------------------------ dequant fixtures
def dequant_module_fixture():
    """build_test_layer of awq_dequantize.rs:133-206 (natural order, g = 2)."""
    height, out_width = 64, 32
    packed_width = out_width // 8
    group_size = height // out_width
    num_groups = height // group_size
    wq = np.zeros((height, packed_width), dtype=np.uint32)
    zq = np.zeros((num_groups, packed_width), dtype=np.uint32)
    sc = np.zeros((num_groups, out_width), dtype=np.float32)
    for r in range(height):
        for cb in range(packed_width):
            wq[r, cb] = pack_natural([(r + cb + i) % 16 for i in range(8)])
    for g in range(num_groups):
        for cb in range(packed_width):
            zq[g, cb] = pack_natural([(g + cb + i) % 8 for i in range(8)])
        for c in range(out_width):
            sc[g, c] = np.float32(np.float32(np.float32(0.5) + np.float32(g) * np.float32(0.01))
                                  + np.float32(c) * np.float32(0.001))
    expected = np.zeros((height, out_width), dtype=np.float32)
    for r in range(height):
        g = r // group_size
        for c in range(out_width):
            w = np.float32((int(wq[r, c // 8]) >> ((c % 8) * 4)) & 0xF)
            z = np.float32((int(zq[g, c // 8]) >> ((c % 8) * 4)) & 0xF)
            expected[r, c] = np.float32((w - z) * sc[g, c])
    # forward (:239-281): input (i as f32) * 0.01, batch 2, f32 k-ascending
    batch = 2
    x = (np.arange(batch * height).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    x = x.reshape(batch, height)
    fwd = np.zeros((batch, out_width), dtype=np.float32)
    for b in range(batch):
        for c in range(out_width):
            acc = np.float32(0.0)
            for k in range(height):
                acc = np.float32(acc + np.float32(x[b, k] * expected[k, c]))
            fwd[b, c] = acc
    return dict(qweight=wq, qzeros=zq, scales=sc, expected=expected,
                group_size=np.int64(group_size), tol=np.float64(1e-4),
                forward_x=x, forward_expected=fwd, forward_tol=np.float64(1e-3))


def dequant_integration_fixture():
    """test_awq_kernel of tests/awq_test.rs:117-221 (natural order, g = 128)."""
    height, out_width, group_size = 128, 32, 128
    packed_width = out_width // 8
    wq = np.zeros((height, packed_width), dtype=np.uint32)
    zq = np.zeros((height // group_size, packed_width), dtype=np.uint32)
    sc = np.zeros(((height // group_size), out_width), dtype=np.float32)
    expected = np.zeros((height, out_width), dtype=np.float32)
    for r in range(height):
        for cb in range(packed_width):
            w_vals = [(r + cb + i) % 15 for i in range(8)]
            z_vals = [(i + 1) % 8 for i in range(8)]
            wq[r, cb] = pack_natural(w_vals)
            if r == 0:
                zq[0, cb] = pack_natural(z_vals)
            for i in range(8):
                col = cb * 8 + i
                s = np.float32(np.float32(0.5) + np.float32(col) * np.float32(0.1))
                if r == 0:
                    sc[0, col] = s
                expected[r, col] = np.float32((np.float32(w_vals[i]) - np.float32(z_vals[i])) * s)
    return dict(qweight=wq, qzeros=zq, scales=sc, expected=expected,
                group_size=np.int64(group_size), tol=np.float64(1e-4))


# --------------------------------------------- closed-form kernel KATs
def uniform_kats():
    """Section B of awq_kernel_gemm.rs:1119-1391. Every nibble of qweight and
    qzeros holds one value; `expected` is the closed form stated there."""
    kats = []

    def add(name, b, m, k, n, gs, inp, w, z, scale, expected, tol):
        kats.append(dict(name=name, b=b, m=m, k=k, n=n, group_size=gs, input=inp,
                         w_nibble=w, z_nibble=z, scales=scale, expected=expected, tol=tol))

    add("kernel_zero_input_yields_zero_output", 1, 32, 32, 32, 32, 0.0, 7, 0, 1.0, 0.0, 1e-5)
    add("kernel_zero_weight_yields_zero_output", 1, 32, 32, 32, 32, 1.0, 5, 5, 2.0, 0.0, 1e-5)
    add("kernel_zero_scale_yields_zero_output", 1, 32, 32, 32, 32, 1.0, 15, 0, 0.0, 0.0, 1e-5)
    add("kernel_ones_input_uniform_weight_single_tile", 1, 32, 32, 32, 32, 1.0, 5, 0, 1.0, 160.0, 1e-3)
    add("kernel_uniform_with_nonzero_zero_point", 1, 32, 32, 32, 32, 1.0, 8, 3, 2.0, 320.0, 1e-3)
    add("kernel_negative_effective_weight", 1, 32, 32, 32, 32, 1.0, 2, 7, 1.0, -160.0, 1e-3)
    add("kernel_weight_nibble_at_max_15", 1, 32, 32, 32, 32, 1.0, 15, 0, 1.0, 480.0, 1e-3)
    add("kernel_weight_nibble_zero_zeropoint_fifteen", 1, 32, 32, 32, 32, 1.0, 0, 15, 1.0, -480.0, 1e-3)
    add("kernel_two_k_tiles", 1, 32, 64, 32, 64, 1.0, 4, 1, 1.0, 192.0, 1e-2)
    add("kernel_four_k_tiles", 1, 32, 128, 32, 128, 0.5, 6, 2, 0.25, 64.0, 1e-2)
    add("kernel_two_groups_uniform_scale", 1, 32, 64, 32, 32, 1.0, 5, 1, 1.0, 256.0, 1e-2)
    # group 0 -> 1.0, group 1 -> 0.5: 4 * (32 * 1.0 + 32 * 0.5)
    add("kernel_two_groups_different_scales", 1, 32, 64, 32, 32, 1.0, 6, 2, [1.0, 0.5], 192.0, 1e-2)
    # scales 0.25, 0.5, 0.75, 1.0: 4 * 32 * 2.5
    add("kernel_four_groups", 1, 32, 128, 32, 32, 1.0, 7, 3, [0.25, 0.5, 0.75, 1.0], 320.0, 1e-1)
    add("kernel_m_double_n_single_tile", 1, 64, 32, 32, 32, 1.0, 5, 0, 1.0, 160.0, 1e-3)
    add("kernel_m_one_partial_tile", 1, 1, 32, 32, 32, 1.0, 5, 0, 1.0, 160.0, 1e-3)
    add("kernel_n_double_m_single_tile", 1, 32, 32, 64, 32, 1.0, 3, 1, 2.0, 128.0, 1e-3)
    # input (i % 7) * 0.1, deq = (4 - 2) * 0.5 = 1: out[r, :] = sum_k x[r, k]
    add("kernel_large_m_large_n", 1, 128, 32, 128, 32, "mod7x0.1", 4, 2, 0.5, "rowsum", 1e-1)
    # batch 0 -> 1.0, batch 1 -> 2.0; deq = (5 - 1) * 0.5 = 2 -> 64 and 128
    add("kernel_two_batches_match_cpu_ref", 2, 32, 32, 32, 32, [1.0, 2.0], 5, 1, 0.5, [64.0, 128.0], 1e-3)
    return kats


# ------------------------------------------------- validation messages
def validation_cases():
    """Section A of awq_kernel_gemm.rs:961-1117: (m, n, k, tile_m, tile_n,
    inner_k, m_valid, line_size, group_size) -> panic text or null."""
    c = []

    def add(name, m, n, k, tm, tn, ik, gs, msg, m_valid=None, line_size=4):
        c.append(dict(name=name, m=m, n=n, k=k, tile_m=tm, tile_n=tn, inner_k=ik,
                      m_valid=m if m_valid is None else m_valid, line_size=line_size,
                      group_size=gs, expected=msg))

    add("validate_accepts_minimal_valid_config", 32, 32, 32, 32, 32, 32, 32, None)
    add("validate_accepts_large_multi_tile_config", 128, 256, 512, 32, 32, 32, 128, None)
    add("validate_rejects_line_size_zero", 32, 32, 32, 32, 32, 32, 32, "line_size must be > 0", line_size=0)
    add("validate_rejects_m_tile_zero", 32, 32, 32, 0, 32, 32, 32, "m_tile_size must be > 0")
    add("validate_rejects_n_tile_zero", 32, 32, 32, 32, 0, 32, 32, "n_tile_size must be > 0")
    add("validate_rejects_inner_k_zero", 32, 32, 32, 32, 32, 0, 32, "inner_k_size must be > 0")
    add("validate_rejects_group_size_zero", 32, 32, 32, 32, 32, 32, 0, "group_size must be > 0")
    add("validate_rejects_k_not_aligned_to_line_size", 32, 32, 6, 32, 32, 4, 2, "k must be divisible by line_size")
    add("validate_rejects_n_not_aligned_to_line_size", 32, 6, 32, 32, 32, 32, 32, "n must be divisible by line_size")
    add("validate_rejects_inner_k_not_aligned_to_line_size", 32, 32, 32, 32, 32, 6, 32,
        "inner_k_size must be divisible by line_size")
    add("validate_accepts_m_not_multiple_of_m_tile", 48, 32, 32, 32, 32, 32, 32, None)
    add("validate_rejects_n_not_multiple_of_n_tile", 32, 48, 32, 32, 32, 32, 32, "n must be divisible by n_tile_size")
    add("validate_rejects_k_not_multiple_of_inner_k", 32, 32, 48, 32, 32, 32, 16, "k must be divisible by inner_k_size")
    add("validate_rejects_n_tile_not_multiple_of_32", 32, 16, 32, 32, 16, 32, 32,
        "n_tile_size must be divisible by line_size*8")
    add("validate_rejects_k_not_multiple_of_group_size", 32, 32, 32, 32, 32, 32, 24, "k must be divisible by group_size")
    add("validate_rejects_m_valid_larger_than_padded_m", 32, 32, 32, 32, 32, 32, 32, "m_valid must be <= m", m_valid=33)
    add("validate_rejects_m_zero", 0, 32, 32, 32, 32, 32, 32, "m must be > 0")
    add("validate_exact_boundary_all_equal", 32, 32, 32, 32, 32, 32, 32, None)
    add("validate_group_size_equals_k", 32, 32, 64, 32, 32, 32, 64, None)
    add("validate_rejects_group_size_smaller_than_inner_k", 32, 32, 32, 32, 32, 32, 1, "fast path requires group_size")
    add("validate_rejects_group_size_not_multiple_of_inner_k", 32, 32, 96, 32, 32, 32, 48, "fast path requires group_size")
    return c


def main():
    for name, arrays in module_cases().items():
        np.savez(os.path.join(HERE, f"module_{name}.npz"), **arrays)
    np.savez(os.path.join(HERE, "dequant_module_g2.npz"), **dequant_module_fixture())
    np.savez(os.path.join(HERE, "dequant_integration_g128.npz"), **dequant_integration_fixture())
    with open(os.path.join(HERE, "kat_gemm_uniform.json"), "w") as f:
        json.dump(uniform_kats(), f, indent=1)
    with open(os.path.join(HERE, "validation_cases.json"), "w") as f:
        json.dump(validation_cases(), f, indent=1)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
