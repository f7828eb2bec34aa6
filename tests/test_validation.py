"""Shape rules and their messages through the native library (no GPU needed).

Mirrors section A of the reference's tests (awq_kernel_gemm.rs:961-1117), the
tile tables of awq_gemm.rs:251-268, the module build asserts
(awq_gemm.rs:77-95, awq_dequantize.rs:25-41, :302-336) and the host-side
asserts of awq_gemm_linear (awq_kernel_gemm.rs:636-724).
"""

import ctypes

import pytest
import torch

import cube_awq_b200 as cawq
from cube_awq_b200 import _lib
from cube_awq_b200.errors import CubeAwqError, DTypeError, ShapeError, check
from helpers import load_json

CASES = load_json("validation_cases.json")


def _shape(c):
    return cawq.ShapeConfig(m=c["m"], k=c["k"], n=c["n"], tile_m=c["tile_m"], tile_n=c["tile_n"],
                            inner_k=c["inner_k"], line_size=c["line_size"], m_valid=c["m_valid"])


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_validate_launch_params(case):
    s = _shape(case)
    if case["expected"] is None:
        cawq.validate_launch_params(s, case["group_size"])
    else:
        with pytest.raises(ShapeError, match=case["expected"].replace("*", r"\*")):
            cawq.validate_launch_params(s, case["group_size"])


def test_decode_rules_use_one_row_and_four_lines_per_thread():
    # decode: ROWS_PER_THREAD_DECODE = 1, N_LINES_PER_THREAD_DECODE = 4 (:86-87)
    s = cawq.ShapeConfig.new(8, 32, 64, 8, 32, 32)
    cawq.validate_decode_launch_params(s, 32)
    with pytest.raises(ShapeError, match="m_tile_size must be divisible by ROWS_PER_THREAD"):
        cawq.validate_launch_params(cawq.ShapeConfig.new(8, 32, 64, 7, 32, 32), 32)
    cawq.validate_decode_launch_params(cawq.ShapeConfig.new(8, 32, 64, 7, 32, 32), 32)


def test_shape_config_argument_order():
    s = cawq.ShapeConfig.new(1, 4096, 11008, 8, 128, 64)  # (m, n, k, ...) as the reference
    assert (s.m, s.n, s.k, s.m_valid, s.line_size) == (1, 4096, 11008, 1, 4)


def test_select_tile_tables():
    # awq_gemm.rs:251-268
    assert [cawq.select_tile_m(m) for m in (1, 8, 16, 17)] == [8, 8, 16, 32]
    assert [cawq.select_tile_n(n) for n in (32, 48, 64, 128, 192, 1536, 5632)] == \
        [32, 32, 64, 128, 64, 128, 128]


def test_gemm_config_build_shapes():
    # awq_gemm.rs:385-406 (parameters only; allocation on the CPU is enough here)
    layer = cawq.AWQGEMMLinearConfig(64, 32, 32).build(device="cpu")
    assert list(layer.qweight.shape) == [64, 4]
    assert list(layer.qzeros.shape) == [2, 4]
    assert list(layer.scales.shape) == [2, 32]
    assert layer.group_size() == 32
    assert layer.bias is None
    layer = cawq.AWQGEMMLinearConfig(64, 32, 32).with_bias(True).build(device="cpu")
    assert list(layer.bias.shape) == [32]


@pytest.mark.parametrize("args,msg", [
    ((64, 32, 0), "group_size must be > 0"),
    ((64, 36, 4), "d_output must be divisible by 8"),
    ((64, 40, 32), r"d_output must be divisible by TILE_N \(32\)"),
    ((96, 32, 32), r"d_input must be divisible by INNER_K \(64\)"),
    ((128, 32, 48), "d_input must be divisible by group_size"),
])
def test_gemm_config_build_asserts(args, msg):
    with pytest.raises(ShapeError, match=msg):
        cawq.AWQGEMMLinearConfig(*args).build(device="cpu")


def test_linear_config_build_asserts():
    with pytest.raises(ShapeError, match=r"d_output % 8 == 0"):
        cawq.AWQLinearConfig(64, 36, 2).build(device="cpu")
    with pytest.raises(ShapeError, match=r"d_output % 32 == 0"):
        cawq.AWQLinearConfig(64, 16, 2).build(device="cpu")
    layer = cawq.AWQLinearConfig(64, 32, 2).build(device="cpu")
    assert layer.group_size() == 2


def _desc(shape, elem=4):
    d = _lib.TensorDescC()
    d.data = None
    d.rank = len(shape)
    for i, s in enumerate(shape):
        d.shape[i] = s
    d.elem_size = elem
    return d


def _gemm_linear_host(inp, qw, qz, sc, out, shape=None, g=32, elem=4, qw_elem=4):
    a = _lib.GemmArgsC()
    a.input, a.qweight, a.qzeros = _desc(inp, elem), _desc(qw, qw_elem), _desc(qz)
    a.scales, a.bias, a.output = _desc(sc, elem), _desc([]), _desc(out, elem)
    a.bias.rank = 0
    a.dtype = _lib.CAWQ_F32
    a.group_size = g
    c = shape.to_c() if shape else None
    return _lib.lib().cawq_awq_gemm_linear(ctypes.byref(a), ctypes.byref(c) if c else None, None)


@pytest.mark.parametrize("inp,qw,qz,sc,out,msg", [
    ([64], [64, 4], [2, 4], [2, 32], [2, 32], r"input must have shape \[\.\., M, K\] or \[M, K\]"),
    ([2, 64], [64], [2, 4], [2, 32], [2, 32], r"qweight must have shape \[K, N/8\]"),
    ([2, 64], [64, 4], [2], [2, 32], [2, 32], r"qzeros must have shape \[K/G, N/8\]"),
    ([2, 64], [64, 4], [2, 4], [2], [2, 32], r"scales must have shape \[K/G, N\]"),
    ([2, 64], [64, 4], [2, 4], [2, 32], [2], r"output must have shape \[\.\., M, N\] or \[M, N\]"),
    ([2, 0], [64, 4], [2, 4], [2, 32], [2, 32], "input K must be > 0"),
    ([2, 32], [64, 4], [2, 4], [2, 32], [2, 32], "input K must match shape.k"),
    ([2, 64], [64, 4], [2, 4], [2, 32], [2, 64], "output N must match shape.n"),
    ([2, 64], [64, 4], [2, 4], [2, 32], [3, 32], "output rows must match flattened input rows"),
    ([2, 64], [32, 4], [2, 4], [2, 32], [2, 32], "qweight K must match shape.k"),
    ([2, 64], [64, 4], [3, 4], [2, 32], [2, 32], "qzeros rows must be K/group_size"),
    ([2, 64], [64, 4], [2, 8], [2, 32], [2, 32], "qzeros packed N must be N/8"),
    ([2, 64], [64, 4], [2, 4], [1, 32], [2, 32], "scales rows must be K/group_size"),
    ([2, 64], [64, 4], [2, 4], [2, 64], [2, 32], "scales N must match shape.n"),
])
def test_awq_gemm_linear_host_asserts(inp, qw, qz, sc, out, msg):
    shape = cawq.ShapeConfig.new(2, 32, 64, 32, 32, 32)
    st = _gemm_linear_host(inp, qw, qz, sc, out, shape)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    with pytest.raises(ShapeError, match=msg):
        check(st)


def test_awq_gemm_linear_uses_decode_rules_for_small_m():
    # launch_m <= 8 validates with the decode rules (awq_kernel_gemm.rs:691-696)
    shape = cawq.ShapeConfig.new(2, 32, 64, 7, 32, 32)  # tile_m 7: fine for decode
    st = _gemm_linear_host([2, 64], [64, 4], [2, 4], [2, 32], [2, 32], shape)
    assert st == _lib.CAWQ_ERR_NULL_POINTER  # every shape rule passed; no buffers given
    shape = cawq.ShapeConfig.new(12, 32, 64, 7, 32, 32)
    st = _gemm_linear_host([12, 64], [64, 4], [2, 4], [2, 32], [12, 32], shape)
    with pytest.raises(ShapeError, match="m_tile_size must be divisible by ROWS_PER_THREAD"):
        check(st)


def test_awq_gemm_linear_rejects_non_32bit_packed():
    shape = cawq.ShapeConfig.new(2, 32, 64, 32, 32, 32)
    st = _gemm_linear_host([2, 64], [64, 4], [2, 4], [2, 32], [2, 32], shape, qw_elem=2)
    with pytest.raises(DTypeError, match="qweight must have i32/u32 dtype"):
        check(st)


def _dq_host(qw_elem=4, qz_elem=4, out_width=32, height=32, g=32):
    lib = _lib.lib()
    return lib.cawq_dequantize_native(
        ctypes.byref(_desc([height, out_width // 8], qw_elem)),
        ctypes.byref(_desc([height // g, out_width // 8], qz_elem)),
        ctypes.byref(_desc([height // g, out_width], 4)),
        ctypes.byref(_desc([height, out_width], 4)), g, _lib.CAWQ_F32, _lib.CAWQ_ORDER_NATURAL, None)


@pytest.mark.parametrize("elem", [2, 8])
def test_dequantize_rejects_non_32bit_q_weight(elem):
    # tests/awq_test.rs:223-377
    with pytest.raises(DTypeError, match="AWQ packed q_weight must use 32-bit elements"):
        check(_dq_host(qw_elem=elem))


@pytest.mark.parametrize("elem", [2, 8])
def test_dequantize_rejects_non_32bit_q_zeros(elem):
    with pytest.raises(DTypeError, match="AWQ packed q_zeros must use 32-bit elements"):
        check(_dq_host(qz_elem=elem))


def test_dequantize_rejects_out_width_not_multiple_of_32():
    # awq_dequantize.rs:302-336
    with pytest.raises(ShapeError, match="out_width % 32 == 0"):
        check(_dq_host(out_width=16, height=64, g=4))


def test_compute_on_cpu_tensors_fails_loudly():
    layer = cawq.AWQGEMMLinearConfig(64, 32, 64).build(device="cpu")
    with pytest.raises(CubeAwqError, match="no CPU fallback"):
        layer.forward(torch.zeros(1, 64))
