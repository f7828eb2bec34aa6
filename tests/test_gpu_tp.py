"""Tensor-parallel layers on 2 GPUs over NCCL (skipped with fewer GPUs).

Each rank builds the column- and row-parallel layers from the same full
tensors and checks the full output against the fp64 oracle of the
unsharded layer, with torch.distributed's NCCL and with the library's own
communicator (cawq_gemm_colpar / cawq_gemm_rowpar), and with the collective
fused into the GEMM's epilogue (cawq_gemm_colpar_p2p / _rowpar_p2p, also
compared bit for bit with the NCCL path). Rows 1 and 8 run the decode kernel
(rows = 1 gathers in place), 300, 600 and 2100 the tensor-core kernel; from
600 rows the fused row-parallel layer reduce-scatters and all-gathers
(reading the peers' buffers) instead of pushing whole partials, and at 2100
rows the fused column-parallel layer reads the peer's shard instead of
pushing its own.
"""

import multiprocessing as mp
import socket

import pytest
import torch

import tp_worker

pytestmark = pytest.mark.gpu

# the last two cases exchange more than 4 MiB per rank, so the fused
# row-parallel layer takes its reduce-scatter + all-gather path; the last one
# has more than 8 MiB of peer shards, so the column-parallel layer pulls
CASES = [(1024, 2048, 128, 1), (1024, 2048, 128, 8), (2048, 1024, 64, 300),
         (2048, 2048, 128, 600), (1024, 4096, 128, 2100)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("backend", ["torch", "native", "p2p"])
def test_two_gpu_tensor_parallel(backend):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_worker.gpu_rank, args=(r, world, port, CASES, backend, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, msg = q.get(timeout=300)
            results[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        assert results.get(rank) == "ok", f"rank {rank}: {results.get(rank)}"
