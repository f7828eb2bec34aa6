"""Tensor-parallel layers with world_size-2 gloo ranks on the CPU.

The local GEMM is the oracle (no GPU here); what is checked is the layers'
shard arithmetic and collectives: a column-parallel layer with its
all-gather, a row-parallel layer with its fp32 all-reduce and bias, and the
column -> row pair of an MLP, each against the unsharded layer.
"""

import multiprocessing as mp
import socket

import pytest

from cube_awq_b200 import ShapeError, tp

import tp_worker


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_worker.cpu_rank, args=(r, world, port, case, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, msg = q.get(timeout=180)
            results[rank] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        assert results.get(rank) == "ok", f"rank {rank}: {results.get(rank)}"


@pytest.mark.parametrize("case", [(256, 128, 64, 3), (512, 256, 128, 1)])
def test_two_gloo_ranks(case):
    _run(2, case)


def test_shards_cover_and_tile():
    assert tp.column_shard(57344, 8, 3) == (3 * 7168, 7168)
    assert tp.row_shard(28672, 128, 8, 7) == (7 * 3584, 3584)
    with pytest.raises(ShapeError):
        tp.column_shard(4096 + 32, 2, 0)      # N / world not a multiple of 32
    with pytest.raises(ShapeError):
        tp.row_shard(128 * 3, 128, 2, 0)      # 3 groups over 2 ranks
