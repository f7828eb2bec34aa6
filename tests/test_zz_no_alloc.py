"""cawq_gemm_rowpar_noalloc: the row-parallel GEMM for callers that cannot
allocate a workspace -- hosts whose device memory already belongs to their own
pool, or C-ABI hosts with no allocator for an fp32 buffer -- so its partial
sums go to a 4 MiB scratch array compiled into the library instead.

The file name makes pytest collect it last. The GPU test runs the entry point
twice in a row (the second call finds the first call's sums in the scratch)
and compares both results with cawq_gemm_rowpar given a workspace of its own,
on a one-rank NCCL communicator, then with the fp64 oracle. The CPU tests
check that requests larger than the scratch are refused, including sizes
whose rows * n would wrap around.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from cube_awq_b200 import _lib, tp
from helpers import GEMM_TOL, max_rel_err, random_awq, to_torch


def _call(fn, comm, x, qw, qz, s, b, out, rows, k, n, g, extra=()):
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    return fn(comm, p(x), p(qw), p(qz), p(s), p(b), p(out), *[p(e) for e in extra], rows, k, n,
              g, _lib.CAWQ_F16, stream)


def test_oversize_request_is_refused_without_a_gpu():
    L = _lib.lib()
    rows, n = 1024, 2048  # 2 Mi partial sums > 1 Mi floats of scratch
    st = L.cawq_gemm_rowpar_noalloc(None, None, None, None, None, None, None, rows, 4096, n, 128,
                                    _lib.CAWQ_F16, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "CAWQ_ROWPAR_SCRATCH_FLOATS" in _lib.last_error()
    assert rows * n > _lib.CAWQ_ROWPAR_SCRATCH_FLOATS


def test_wrapping_request_is_refused_without_a_gpu():
    L = _lib.lib()
    rows, n = 1 << 62, 8  # rows * n wraps to 0 in 64 bits
    st = L.cawq_gemm_rowpar_noalloc(None, None, None, None, None, None, None, rows, 4096, n, 128,
                                    _lib.CAWQ_F16, None)
    assert st == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "CAWQ_ROWPAR_SCRATCH_FLOATS" in _lib.last_error()


@pytest.mark.gpu
def test_noalloc_matches_the_workspace_entry_point(cuda_device):
    L = _lib.lib()
    comm = tp.TPComm(timeout_ms=60000)  # one rank: the all-reduce is a copy
    try:
        rows, k, n, g = 6, 2048, 4096, 128
        x, qw, qz, s, b = random_awq(k, n, g, "f16", rows, seed=61)
        t = lambda a, d: to_torch(a, d, cuda_device)
        xt, qwt, qzt, st_, bt = t(x, "f16"), t(qw, "u32"), t(qz, "u32"), t(s, "f16"), t(b, "f16")
        partial = torch.empty(rows * n, dtype=torch.float32, device=cuda_device)
        y_ws = torch.empty(rows, n, dtype=torch.float16, device=cuda_device)
        st = _call(L.cawq_gemm_rowpar, comm.handle, xt, qwt, qzt, st_, bt, y_ws, rows, k, n, g,
                   extra=(partial,))
        assert st == 0, _lib.last_error()
        outs = []
        for _ in range(2):  # the second call starts on the first call's sums
            y = torch.full((rows, n), float("nan"), dtype=torch.float16, device=cuda_device)
            st = _call(L.cawq_gemm_rowpar_noalloc, comm.handle, xt, qwt, qzt, st_, bt, y, rows, k,
                       n, g)
            assert st == 0, _lib.last_error()
            outs.append(y)
        torch.cuda.synchronize()
        for y in outs:
            assert torch.equal(y, y_ws)
        ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b, dtype="f16", deq_round=False)
        assert max_rel_err(y_ws.float().cpu().numpy().astype(np.float64), ref) <= GEMM_TOL["f16"]
    finally:
        comm.close()
