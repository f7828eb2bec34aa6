"""cawq_gemm_rowpar_noalloc: the row-parallel GEMM for callers that cannot
allocate a workspace -- hosts whose device memory already belongs to their own
pool, or C-ABI hosts with no allocator for an fp32 buffer -- so its partial
sums go to a 4 MiB scratch array compiled into the library instead.

The file name makes pytest collect it last. The GPU test runs the entry point
twice in a row (the second call finds the first call's sums in the scratch)
and compares both results with cawq_gemm_rowpar given a workspace of its own,
on a one-rank NCCL communicator, then with the fp64 oracle: a small f16 case,
a bf16 case with bias, and one whose rows * n fills the scratch exactly. The
CPU tests check that requests larger than the scratch are refused (one row
past the limit, and sizes whose rows * n would wrap around).
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from cube_awq_b200 import _lib, tp
from helpers import GEMM_TOL, max_rel_err, random_awq, to_torch


CODE = {"f16": _lib.CAWQ_F16, "bf16": _lib.CAWQ_BF16}
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}


def _call(fn, comm, x, qw, qz, s, b, out, rows, k, n, g, dtype="f16", extra=()):
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    return fn(comm, p(x), p(qw), p(qz), p(s), p(b), p(out), *[p(e) for e in extra], rows, k, n,
              g, CODE[dtype], stream)


def test_oversize_request_is_refused_without_a_gpu():
    L = _lib.lib()
    rows, n = 1024, 2048  # 2 Mi partial sums > 1 Mi floats of scratch
    st = L.cawq_gemm_rowpar_noalloc(None, None, None, None, None, None, None, rows, 4096, n, 128,
                                    _lib.CAWQ_F16, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "CAWQ_ROWPAR_SCRATCH_FLOATS" in _lib.last_error()
    assert rows * n > _lib.CAWQ_ROWPAR_SCRATCH_FLOATS


def test_one_row_past_the_limit_is_refused_without_a_gpu():
    L = _lib.lib()
    n = 4096
    rows = _lib.CAWQ_ROWPAR_SCRATCH_FLOATS // n + 1
    st = L.cawq_gemm_rowpar_noalloc(None, None, None, None, None, None, None, rows, 2048, n, 128,
                                    _lib.CAWQ_F16, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "CAWQ_ROWPAR_SCRATCH_FLOATS" in _lib.last_error()


def test_wrapping_request_is_refused_without_a_gpu():
    L = _lib.lib()
    rows, n = 1 << 62, 8  # rows * n wraps to 0 in 64 bits
    st = L.cawq_gemm_rowpar_noalloc(None, None, None, None, None, None, None, rows, 4096, n, 128,
                                    _lib.CAWQ_F16, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "CAWQ_ROWPAR_SCRATCH_FLOATS" in _lib.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n,dtype,bias", [
    (6, 4096, "f16", True),
    (5, 2048, "bf16", True),
    (256, 4096, "f16", False),   # rows * n == CAWQ_ROWPAR_SCRATCH_FLOATS: the whole array
])
def test_noalloc_matches_the_workspace_entry_point(cuda_device, rows, n, dtype, bias):
    L = _lib.lib()
    comm = tp.TPComm(timeout_ms=60000)  # one rank: the all-reduce is a copy
    try:
        k, g = 2048, 128
        assert rows * n <= _lib.CAWQ_ROWPAR_SCRATCH_FLOATS
        x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed=61 + rows)
        t = lambda a, d: to_torch(a, d, cuda_device)
        xt, qwt, qzt, st_ = t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype)
        bt = t(b, dtype) if bias else None
        partial = torch.empty(rows * n, dtype=torch.float32, device=cuda_device)
        y_ws = torch.empty(rows, n, dtype=TDT[dtype], device=cuda_device)
        st = _call(L.cawq_gemm_rowpar, comm.handle, xt, qwt, qzt, st_, bt, y_ws, rows, k, n, g,
                   dtype, extra=(partial,))
        assert st == 0, _lib.last_error()
        outs = []
        for _ in range(2):  # the second call starts on the first call's sums
            y = torch.full((rows, n), float("nan"), dtype=TDT[dtype], device=cuda_device)
            st = _call(L.cawq_gemm_rowpar_noalloc, comm.handle, xt, qwt, qzt, st_, bt, y, rows, k,
                       n, g, dtype)
            assert st == 0, _lib.last_error()
            outs.append(y)
        torch.cuda.synchronize()
        for y in outs:
            assert torch.equal(y, y_ws)
        ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b if bias else None, dtype=dtype,
                              deq_round=False)
        got = y_ws.float().cpu().numpy().astype(np.float64)
        assert max_rel_err(got, ref) <= GEMM_TOL[dtype]
    finally:
        comm.close()
