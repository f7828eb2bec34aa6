"""Rank bodies of the tensor-parallel tests (run in spawned processes).

On the CPU the local GEMM is the oracle (injected through the layers' `gemm`
argument), so gloo ranks check the sharding and collective plumbing. On GPUs
the layers run the library's kernels over NCCL (torch.distributed or the
library's own communicator).
"""

from __future__ import annotations

import os
import sys
import traceback
from datetime import timedelta

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def oracle_gemm(x, qweight, qzeros, scales, group_size, bias=None, out=None, out_dtype=None,
                order="awq"):
    """CPU stand-in for cube_awq_b200.gemm (exact accumulation, f32 output)."""
    import torch

    import oracle
    y = oracle.gemm_f64(x.numpy(), qweight.numpy().view(np.uint32),
                        qzeros.numpy().view(np.uint32), scales.numpy(), group_size,
                        bias=None if bias is None else bias.numpy(), dtype="f32", order=order)
    return torch.from_numpy(y).to(out_dtype or x.dtype)


def problem(k, n, g, rows, seed):
    """Full-layer tensors, identical on every rank (seeded)."""
    import torch
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    t = torch.from_numpy
    return t(x), t(qw.view(np.int32)), t(qz.view(np.int32)), t(s), t(b)


def cpu_rank(rank, world, port, case, q):
    import torch
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60))
        from cube_awq_b200 import tp
        k, n, g, rows = case
        x, qw, qz, s, b = problem(k, n, g, rows, seed=k + n)
        full = oracle_gemm(x, qw, qz, s, g, bias=b)
        # column-parallel with the gather: every rank holds the full output
        col = tp.ColumnParallelAWQLinear(qw, qz, s, b, gemm=oracle_gemm)
        y = col.forward(x.reshape(1, rows, k))
        assert tuple(y.shape) == (1, rows, n), y.shape
        assert torch.equal(y.reshape(rows, n), full), "column-parallel differs"
        # row-parallel from the full input: fp32 partials + all-reduce + bias
        row = tp.RowParallelAWQLinear(qw, qz, s, b, input_is_parallel=False, gemm=oracle_gemm)
        y2 = row.forward(x)
        err = (y2 - full).abs().max().item() / full.abs().max().item()
        assert err < 1e-5, f"row-parallel error {err}"
        # an MLP pair: column-parallel without gather feeds row-parallel
        n2 = 64 * world
        _, qw2, qz2, s2, b2 = problem(n, n2, g, rows, seed=7)
        col2 = tp.ColumnParallelAWQLinear(qw, qz, s, b, gather_output=False, gemm=oracle_gemm)
        row2 = tp.RowParallelAWQLinear(qw2, qz2, s2, b2, gemm=oracle_gemm)
        h = col2.forward(x)
        assert h.shape[-1] == n // world
        y3 = row2.forward(h)
        ref3 = oracle_gemm(full, qw2, qz2, s2, g, bias=b2)
        err3 = (y3 - ref3).abs().max().item() / ref3.abs().max().item()
        assert err3 < 1e-5, f"MLP pair error {err3}"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:
        q.put((rank, traceback.format_exc()))


def gpu_rank(rank, world, port, cases, backend, q):
    import torch
    import torch.distributed as dist
    comm = peers = None
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        import oracle
        from cube_awq_b200 import tp
        if backend in ("native", "p2p"):
            comm = tp.TPComm(timeout_ms=60000)
        if backend == "p2p":
            peers = tp.TPPeers(comm, 256 << 20, timeout_ms=5000)
        msgs = []
        for (k, n, g, rows) in cases:
            x, qw, qz, s, b = problem(k, n, g, rows, seed=k + n + rows)
            xh, sh, bh = x.half(), s.half(), b.half()
            ref = oracle.gemm_f64(xh.numpy(), qw.numpy().view(np.uint32),
                                  qz.numpy().view(np.uint32), sh.numpy(), g, bias=bh.numpy(),
                                  dtype="f16", deq_round=False)
            d = lambda t: t.to(dev)
            col = tp.ColumnParallelAWQLinear(d(qw), d(qz), d(sh), d(bh), backend=backend,
                                             comm=comm, peers=peers)
            y = col.forward(d(xh))
            row = tp.RowParallelAWQLinear(d(qw), d(qz), d(sh), d(bh), input_is_parallel=False,
                                          backend=backend, comm=comm, peers=peers)
            y2 = row.forward(d(xh))
            if backend == "p2p":
                # again (the other slot), then bit for bit against the NCCL path:
                # the same local GEMM, and with two ranks the same fp32 sum
                y_again, y2_again = col.forward(d(xh)), row.forward(d(xh))
                ncol = tp.ColumnParallelAWQLinear(d(qw), d(qz), d(sh), d(bh), backend="native",
                                                  comm=comm)
                nrow = tp.RowParallelAWQLinear(d(qw), d(qz), d(sh), d(bh),
                                               input_is_parallel=False, backend="native",
                                               comm=comm)
                yn, y2n = ncol.forward(d(xh)), nrow.forward(d(xh))
                torch.cuda.synchronize()
                for name, a_, b_ in (("colpar", y, yn), ("colpar again", y_again, yn),
                                     ("rowpar", y2, y2n), ("rowpar again", y2_again, y2n)):
                    if not torch.equal(a_, b_):
                        msgs.append(f"p2p {name} k={k} n={n} rows={rows} differs from NCCL")
            torch.cuda.synchronize()
            for name, got in (("colpar", y), ("rowpar", y2)):
                g64 = got.float().cpu().numpy().astype(np.float64)
                err = np.abs(g64 - ref).max() / np.abs(ref).max()
                if not err <= 5e-3:
                    msgs.append(f"{name} k={k} n={n} rows={rows}: rel err {err:.3e}")
        from cube_awq_b200 import device_error
        if device_error() != 0:
            msgs.append("device error word set")
        if peers is not None:
            torch.cuda.synchronize()
            dist.barrier()  # every rank's last fused call has completed
            peers.close()
            peers = None
        if comm is not None:
            comm.close()
            comm = None
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if not msgs else "; ".join(msgs)))
    except Exception:
        q.put((rank, traceback.format_exc()))
