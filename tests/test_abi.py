"""The C ABI library loads without a GPU and exports what the header declares."""

import ctypes
import os
import re

import pytest

import cube_awq_b200 as cawq
from cube_awq_b200 import _lib
from conftest import REPO


def _declared():
    with open(os.path.join(REPO, "include", "cube_awq.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cawq_[a-z0-9_]+)\s*\(", text)))


def test_header_declarations_are_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/cube_awq.h but not exported"
    assert sorted(_lib.EXPORTED) == declared


def test_only_c_abi_symbols_are_exported():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    syms = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert syms and all(s.startswith("cawq_") for s in syms), syms


def test_version_and_no_device_on_cpu_box():
    assert cawq.version().startswith("cube_awq")
    import torch
    if not torch.cuda.is_available():
        assert _lib.lib().cawq_device_supported(0) == 0


def test_gpu_entry_points_refuse_without_sm100():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    lib = _lib.lib()
    st = lib.cawq_dequantize(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                             ctypes.c_void_p(16), 32, 32, 32, _lib.CAWQ_F32, _lib.CAWQ_ORDER_NATURAL,
                             None)
    assert st in (_lib.CAWQ_ERR_CUDA, _lib.CAWQ_ERR_UNSUPPORTED)
    assert _lib.last_error()


@pytest.mark.parametrize("n,world", [(57344, 8), (12288, 4), (4096, 2), (64, 2)])
def test_column_shards_tile_n(n, world):
    lib = _lib.lib()
    spans = []
    for r in range(world):
        b, l = ctypes.c_size_t(), ctypes.c_size_t()
        assert lib.cawq_tp_column_shard(n, world, r, ctypes.byref(b), ctypes.byref(l)) == 0
        spans.append((b.value, l.value))
    assert spans[0][0] == 0 and sum(l for _, l in spans) == n
    assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def test_row_shards_follow_group_boundaries():
    lib = _lib.lib()
    b, l = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.cawq_tp_row_shard(28672, 128, 8, 3, ctypes.byref(b), ctypes.byref(l)) == 0
    assert (b.value, l.value) == (3 * 3584, 3584) and b.value % 128 == 0
    assert lib.cawq_tp_row_shard(4096, 128, 3, 0, ctypes.byref(b), ctypes.byref(l)) == \
        _lib.CAWQ_ERR_INVALID_SHAPE
    assert "world" in _lib.last_error()
    assert lib.cawq_tp_column_shard(4096, 3, 0, ctypes.byref(b), ctypes.byref(l)) == \
        _lib.CAWQ_ERR_INVALID_SHAPE


def test_silu_mul_entry_checks_arguments_before_the_device():
    # dtype and the 256-column rule are checked before any device call, so the
    # errors are the same on a CPU box
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    st = lib.cawq_gemm_silu_mul(p, p, p, p, None, p, 1, 128, 512, 128, _lib.CAWQ_F32, 0, None)
    assert st == _lib.CAWQ_ERR_DTYPE and "F16" in _lib.last_error()
    st = lib.cawq_gemm_silu_mul(p, p, p, p, None, p, 1, 128, 384, 128, _lib.CAWQ_F16, 0, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE and "256" in _lib.last_error()
    st = lib.cawq_interleave_gate_up(p, p, 4, 96, 64, 2, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    st = lib.cawq_interleave_gate_up(p, p, 4, 128, 64, 8, None)
    assert st == _lib.CAWQ_ERR_INVALID_ARGUMENT
    assert lib.cawq_interleave_gate_up(p, p, 0, 128, 64, 2, None) == 0  # nothing to move


def test_qkv_entry_checks_split_before_the_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)
    args = lambda nq, nkv, ldk: (p, p, p, p, None, p, p, p, 1, 128, nq, nkv, 128, _lib.CAWQ_F16,
                                 _lib.CAWQ_F16, 0, ldk, 0, None)
    assert lib.cawq_gemm_qkv(*args(496, 136, 0)) == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "multiples of 32" in _lib.last_error()
    assert lib.cawq_gemm_qkv(*args(512, 128, 64)) == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "ld_k" in _lib.last_error()
    a = list(args(512, 128, 0))
    a[8] = 0  # no rows: nothing to do, no device needed
    assert lib.cawq_gemm_qkv(*a) == 0


def test_p2p_entries_check_the_peer_table_before_the_device():
    lib = _lib.lib()
    p = ctypes.c_void_p(16)

    def table(world=2, rank=0, bases=(256, 512), nbytes=1 << 20):
        t = _lib.PeersC()
        t.world, t.rank, t.bytes, t.timeout_ms = world, rank, nbytes, 0
        for j, b in enumerate(bases):
            t.base[j] = b
        return t

    def call(t, epoch=1, rows=1, n=1024, dtype=_lib.CAWQ_F16, fn="cawq_gemm_colpar_p2p"):
        return getattr(lib, fn)(ctypes.byref(t), epoch, p, p, p, p, None, p, rows, 512, n, 128,
                                dtype, None)

    assert call(table(), dtype=_lib.CAWQ_F32) == _lib.CAWQ_ERR_DTYPE
    assert call(table(world=9, bases=[256] * 8)) == _lib.CAWQ_ERR_INVALID_ARGUMENT
    assert call(table(bases=(256, 0))) == _lib.CAWQ_ERR_ALIGNMENT
    assert call(table(bases=(256, 300))) == _lib.CAWQ_ERR_ALIGNMENT  # not 256-byte aligned
    assert call(table(), epoch=0) == _lib.CAWQ_ERR_INVALID_ARGUMENT
    assert call(table(nbytes=4096), rows=8) == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "per slot" in _lib.last_error()
    # row-parallel needs world planes of fp32 partial sums per slot
    # (4 KB slots: enough for one f16 row of the gather, not for 2 fp32 planes)
    assert call(table(nbytes=256 + 2 * 4096), rows=1,
                fn="cawq_gemm_rowpar_p2p") == _lib.CAWQ_ERR_INVALID_SHAPE
    assert call(table(), n=1000) == _lib.CAWQ_ERR_INVALID_SHAPE  # not whole 32-column shards
    assert call(table(), rows=0) == 0  # nothing to do, no device needed


def test_p2p_layers_need_a_peer_table():
    import torch
    from cube_awq_b200 import tp
    qw = torch.zeros(128, 8, dtype=torch.int32)
    qz = torch.zeros(1, 8, dtype=torch.int32)
    s = torch.ones(1, 64, dtype=torch.float16)
    with pytest.raises(ValueError):
        tp.ColumnParallelAWQLinear(qw, qz, s, backend="p2p")
    with pytest.raises(ValueError):
        tp.RowParallelAWQLinear(qw, qz, s, backend="p2p")
