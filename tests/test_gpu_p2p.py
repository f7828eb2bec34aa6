"""The fused tensor-parallel layers (cawq_gemm_colpar_p2p / _rowpar_p2p) on
one GPU: the one-rank case against cawq_gemm, and the bounded wait for a
peer that never signals. The two-rank exchange over NVLink is in
test_gpu_tp.py (skipped with fewer than two GPUs).

The timeout case is the failure-detection test of these layers: the wait
runs out on a flag nothing sets, the kernel records bit 1 of the device
error word and returns without writing the output, and the context stays
usable. It needs no second process and no fault.
"""

import pytest
import torch

import cube_awq_b200 as cawq
from cube_awq_b200 import _lib, tp
from helpers import random_awq, to_torch

pytestmark = pytest.mark.gpu

K, N, G = 1024, 768, 128


def _layer(dev, rows, dtype, seed):
    x, qw, qz, s, b = random_awq(K, N, G, dtype, rows, seed)
    t = lambda a, d: to_torch(a, d, dev)
    return t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), t(b, dtype)


def _buffer(dev, nbytes):
    return torch.zeros(nbytes, dtype=torch.uint8, device=dev)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 7, 200])
def test_one_rank_matches_gemm(cuda_device, dtype, rows):
    nbytes = 256 + 2 * (rows * N * 4 + 4096)
    buf = _buffer(cuda_device, nbytes)
    peers = tp.TPPeers.from_pointers(1, 0, [buf.data_ptr()], nbytes)
    x, qw, qz, s, b = _layer(cuda_device, rows, dtype, seed=rows)
    col = tp.ColumnParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers)
    row = tp.RowParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers)
    for _ in range(3):  # epochs 1..6: both slots, twice
        y = col(x)
        y2 = row(x)
    ref = cawq.gemm(x, qw, qz, s, G, bias=b)
    part = cawq.gemm(x, qw, qz, s, G, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert peers.epoch == 6
    assert torch.equal(y, ref)
    assert torch.equal(y2, (part + b.float()).to(x.dtype))
    assert cawq.device_error() == 0


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 7, 200])
def test_pushed_copies_equal_the_local_result(cuda_device, dtype, rows):
    # Rank 0 of a two-rank table whose "peer" buffer is a second local buffer,
    # with its own flag word for rank 1 preset far ahead, so the wait passes
    # at once: the decode / prefill epilogue's replicated stores are checked
    # bit for bit against the local GEMM, without a second process.
    nbytes = 256 + 2 * (2 * rows * N * 4 + 4096)
    own, other = _buffer(cuda_device, nbytes), _buffer(cuda_device, nbytes)
    own.view(torch.int32)[1] = 1 << 20
    peers = tp.TPPeers.from_pointers(2, 0, [own.data_ptr(), other.data_ptr()], nbytes)
    x, qw, qz, s, b = _layer(cuda_device, rows, dtype, seed=rows + 10)
    slot = peers.slot_bytes
    col = tp.ColumnParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers)
    y = col(x)                                   # epoch 1: slot 1
    row = tp.RowParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers,
                                  input_is_parallel=False)
    y2 = row(x)                                  # epoch 2: slot 0
    torch.cuda.synchronize()
    half = N // 2
    mine = cawq.gemm(x, col.qweight, col.qzeros, col.scales, G, bias=col.bias)
    view = lambda t, off, dt, shape: t[off:off + shape[0] * shape[1] * (4 if dt == torch.float32
                                                                         else 2)] \
        .view(dt).view(*shape)
    tdt = x.dtype
    assert torch.equal(y[:, :half], mine)
    assert torch.equal(view(other, 256 + slot, tdt, (rows, N))[:, :half], mine)
    part = cawq.gemm(x[:, :K // 2].contiguous(), row.qweight, row.qzeros, row.scales, G,
                     out_dtype=torch.float32)
    assert torch.equal(view(other, 256, torch.float32, (rows, N)), part)
    assert torch.equal(y2, (part + b.float()).to(tdt))  # plane 1 is still zero
    assert cawq.device_error() == 0


def test_missing_peer_times_out_without_writing(cuda_device):
    # a two-rank table whose "peer" buffer is a second local buffer: nothing
    # ever publishes rank 1's flag, so the wait gives up after 100 ms
    nbytes = 256 + 2 * 65536
    own, other = _buffer(cuda_device, nbytes), _buffer(cuda_device, nbytes)
    peers = tp.TPPeers.from_pointers(2, 0, [own.data_ptr(), other.data_ptr()], nbytes,
                                     timeout_ms=100)
    x, qw, qz, s, b = _layer(cuda_device, 1, "f16", seed=3)
    out = torch.full((1, N), 7.0, dtype=torch.float16, device=cuda_device)
    cawq.device_error(reset=True)
    st = _lib.lib().cawq_gemm_colpar_p2p(
        peers.table, peers.next_epoch(), x.data_ptr(), qw[:, :N // 16].contiguous().data_ptr(),
        qz[:, :N // 16].contiguous().data_ptr(), s[:, :N // 2].contiguous().data_ptr(), None,
        out.data_ptr(), 1, K, N, G, _lib.CAWQ_F16, None)
    assert st == 0  # the launch succeeds; the failure shows on the device
    word = cawq.device_error(reset=True)
    assert word & 2
    assert (out == 7).all()  # nothing written after the wait gave up
    # the pushed half landed in the stand-in peer's slot 1 (epoch 1)
    assert other[256:].view(torch.float16).abs().sum() > 0
    # the context is still usable
    y = cawq.gemm(x, qw, qz, s, G)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all() and cawq.device_error() == 0


def test_rejects_small_buffers_and_epoch_zero(cuda_device):
    buf = _buffer(cuda_device, 4096)
    peers = tp.TPPeers.from_pointers(1, 0, [buf.data_ptr()], 4096)
    x, qw, qz, s, b = _layer(cuda_device, 8, "f16", seed=1)
    out = torch.empty(8, N, dtype=torch.float16, device=cuda_device)
    args = (x.data_ptr(), qw.data_ptr(), qz.data_ptr(), s.data_ptr(), None, out.data_ptr(), 8, K,
            N, G, _lib.CAWQ_F16, None)
    assert _lib.lib().cawq_gemm_colpar_p2p(peers.table, 1, *args) == _lib.CAWQ_ERR_INVALID_SHAPE
    assert "per slot" in _lib.last_error()
    assert _lib.lib().cawq_gemm_rowpar_p2p(peers.table, 0, *args) == \
        _lib.CAWQ_ERR_INVALID_ARGUMENT


def _two_rank_stand_in(dev, nbytes, sets=(1,)):
    # rank 0 of a two-rank table whose "peer" buffer is a second local buffer;
    # rank 1's flag word of every set used is preset far ahead, so the waits
    # pass at once
    own, other = _buffer(dev, nbytes), _buffer(dev, nbytes)
    for w in sets:
        own.view(torch.int32)[w] = 1 << 20
    return own, other, tp.TPPeers.from_pointers(2, 0, [own.data_ptr(), other.data_ptr()], nbytes)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_colpar_large_output_push_on_one_gpu(cuda_device, dtype):
    # Above 8 MiB of peer shards the column-parallel GEMM writes only its own
    # slot and the output; a kernel after it pushes the shard into the peer's
    # slot, and after the flag exchange the peer's shard is copied from this
    # rank's own slot, where the peer pushed it (preset here with known data).
    rows, k, n, g = 2100, 512, 4096, 128
    es = 2
    slot_need = rows * n * es
    own, other, peers = _two_rank_stand_in(cuda_device, 256 + 2 * (slot_need + 4096))
    x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed=41)
    t = lambda a, d: to_torch(a, d, cuda_device)
    x, qw, qz, s, b = t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), t(b, dtype)
    off = 256 + peers.slot_bytes                   # epoch 1: slot 1
    tdt = x.dtype
    half = n // 2
    own_slot = own[off:off + slot_need].view(tdt).view(rows, n)
    own_slot[:, half:].copy_(torch.randn(rows, half, device=cuda_device).to(tdt))  # the peer's
    pushed = own_slot[:, half:].clone()
    col = tp.ColumnParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers)
    y = col(x)
    torch.cuda.synchronize()
    assert cawq.device_error() == 0
    mine = cawq.gemm(x, col.qweight, col.qzeros, col.scales, g, bias=col.bias)
    assert torch.equal(y[:, :half], mine)
    assert torch.equal(y[:, half:], pushed)
    assert torch.equal(own_slot[:, :half], mine)
    peer_slot = other[off:off + slot_need].view(tdt).view(rows, n)
    assert torch.equal(peer_slot[:, :half], mine)  # pushed to the peer


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_rowpar_reduce_scatter_on_one_gpu(cuda_device, dtype):
    # rows * n * 4 bytes above 4 MiB take the reduce-scatter: the GEMM writes
    # this rank's fp32 partial into its own slot; a kernel copies the peer's
    # column chunk of it into the peer's receive region; after flag set A this
    # rank sums its own chunk over its partial and its receive region (rank
    # order), adds the bias, writes the output and the peer's gather region;
    # after flag set B it copies the other chunk from its own gather region.
    # The stand-in peer's data in this rank's buffer (receive region, gather
    # region) is preset with known values.
    rows, k, n, g = 600, 1024, 2048, 128
    plane = rows * n * 4
    pl = (plane + 255) // 256 * 256
    es = 2
    slot = 2 * pl + rows * n * es
    own, other, peers = _two_rank_stand_in(cuda_device, 256 + 2 * (slot + 4096), sets=(1, 9))
    x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed=31)
    t = lambda a, d: to_torch(a, d, cuda_device)
    x, qw, qz, s, b = t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), t(b, dtype)
    tdt = x.dtype
    cw = n // 2
    off = 256 + peers.slot_bytes                   # epoch 1: slot 1
    recv_in = own[off + pl:off + pl + 2 * rows * cw * 4].view(torch.float32).view(2, rows, cw)
    recv_in[1].copy_(torch.randn(rows, cw, device=cuda_device))      # from rank 1
    gath_in = own[off + 2 * pl:off + 2 * pl + rows * n * es].view(tdt).view(rows, n)
    gath_in.copy_(torch.randn(rows, n, device=cuda_device).to(tdt))  # rank 1's chunk
    row = tp.RowParallelAWQLinear(qw, qz, s, b, backend="p2p", peers=peers,
                                  input_is_parallel=False)
    y = row(x)
    torch.cuda.synchronize()
    assert cawq.device_error() == 0
    part = cawq.gemm(x[:, :k // 2].contiguous(), row.qweight, row.qzeros, row.scales, g,
                     out_dtype=torch.float32)
    want0 = ((part[:, :cw] + recv_in[1]) + b[:cw].float()).to(tdt)
    assert torch.equal(y[:, :cw], want0)
    assert torch.equal(y[:, cw:], gath_in[:, cw:])
    assert torch.equal(own[off:off + plane].view(torch.float32).view(rows, n), part)
    peer_recv = other[off + pl:off + pl + rows * cw * 4].view(torch.float32).view(rows, cw)
    assert torch.equal(peer_recv, part[:, cw:])    # recv[0] of the peer
    peer_gath = other[off + 2 * pl:off + 2 * pl + rows * n * es].view(tdt).view(rows, n)
    assert torch.equal(peer_gath[:, :cw], want0)
