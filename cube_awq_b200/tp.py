"""Tensor-parallel AWQ layers: one process per GPU, NCCL over NVLink.

BASELINE configs[4] shards a Llama-3-70B MLP over 1-8 B200s:

* column-parallel (gate_up, qkv): rank r owns output columns
  [r N/P, (r+1) N/P) — the matching columns of qweight / qzeros (N/8P packed
  words), scales and bias. x is replicated; the local GEMM gives [M, N/P];
  an all-gather rebuilds [M, N] when the caller needs the full output.
* row-parallel (down, o): rank r owns K rows [r K/P, (r+1) K/P), cut on
  quantization-group boundaries (its qzeros / scales rows follow). x arrives
  column-sharded [M, K/P] (the un-gathered output of a column-parallel
  layer); each rank computes an fp32 partial [M, N] and an fp32 all-reduce
  sums them; the bias is added once, after the sum.

The reference is single-device; these layers have no counterpart there. The
shard arithmetic is the C ABI's (cawq_tp_column_shard / cawq_tp_row_shard).

Two collective back ends:

* ``backend="torch"``: torch.distributed (NCCL between GPUs; any backend the
  group uses, e.g. gloo for host-side tests) around the fused GEMM.
* ``backend="native"``: the library's own NCCL communicator (``TPComm``); one
  C call (cawq_gemm_colpar / cawq_gemm_rowpar) runs the GEMM, the collective
  and the epilogue on the caller's stream — the path a non-Python host uses.
* ``backend="p2p"``: the collective fused into the GEMM (``TPPeers``; C calls
  cawq_gemm_colpar_p2p / cawq_gemm_rowpar_p2p): the GEMM's epilogue stores
  its output into every rank's peer buffer over NVLink, and a small kernel
  exchanges flags (bounded wait) and finishes the gather or the sum.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .errors import CubeAwqError, DTypeError, ShapeError, check
from .kernel import cawq_dtype, current_stream_handle, gemm as fused_gemm


# ------------------------------------------------------------ shard math
def column_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first column, columns) of rank's slice of N (cawq_tp_column_shard)."""
    b, l = ctypes.c_size_t(), ctypes.c_size_t()
    check(_lib.lib().cawq_tp_column_shard(n, world, rank, ctypes.byref(b), ctypes.byref(l)))
    return b.value, l.value


def row_shard(k: int, group_size: int, world: int, rank: int) -> tuple[int, int]:
    """(first K row, rows) of rank's slice of K on group boundaries (cawq_tp_row_shard)."""
    b, l = ctypes.c_size_t(), ctypes.c_size_t()
    check(_lib.lib().cawq_tp_row_shard(k, group_size, world, rank, ctypes.byref(b),
                                       ctypes.byref(l)))
    return b.value, l.value


def shard_columns(qweight, qzeros, scales, bias, world: int, rank: int):
    """Rank's column shard of full AutoAWQ tensors (contiguous copies)."""
    n = scales.shape[1]
    n0, nl = column_shard(n, world, rank)
    qw = qweight[:, n0 // 8:(n0 + nl) // 8].contiguous()
    qz = qzeros[:, n0 // 8:(n0 + nl) // 8].contiguous()
    s = scales[:, n0:n0 + nl].contiguous()
    b = bias[n0:n0 + nl].contiguous() if bias is not None else None
    return qw, qz, s, b


def shard_rows(qweight, qzeros, scales, group_size: int, world: int, rank: int):
    """Rank's K-row shard of full AutoAWQ tensors (contiguous copies)."""
    k = qweight.shape[0]
    k0, kl = row_shard(k, group_size, world, rank)
    g0, gl = k0 // group_size, kl // group_size
    return (qweight[k0:k0 + kl].contiguous(), qzeros[g0:g0 + gl].contiguous(),
            scales[g0:g0 + gl].contiguous())


def _world_rank(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


# ------------------------------------------------------- native comm
class TPComm:
    """The library's NCCL communicator over the ranks of ``group``.

    Rank 0 of the group creates the NCCL id and broadcasts it over the group
    (any torch.distributed backend); every rank then joins on its current
    CUDA device. ``timeout_ms`` bounds the join.
    """

    def __init__(self, group=None, timeout_ms: int = 60000):
        self.world, self.rank = _world_rank(group)
        raw = ctypes.create_string_buffer(_lib.CAWQ_TP_ID_BYTES)
        if self.rank == 0:
            check(_lib.lib().cawq_tp_unique_id(raw))
        box = [bytes(raw.raw)]
        if self.world > 1:
            src = dist.get_global_rank(group, 0) if group is not None else 0
            dist.broadcast_object_list(box, src=src, group=group)
        ident = ctypes.create_string_buffer(box[0], _lib.CAWQ_TP_ID_BYTES)
        h = ctypes.c_void_p()
        check(_lib.lib().cawq_tp_init(self.world, self.rank, ident, timeout_ms, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            check(_lib.lib().cawq_tp_destroy(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TPPeers:
    """Peer buffers of the fused tensor-parallel layers (cawq_tp_p2p_create):
    one buffer of ``nbytes`` per rank, mapped into every rank's process over
    CUDA IPC, set up collectively over ``comm``. Every fused call takes the
    next epoch of this object, so all ranks must make the same calls in the
    same order. ``timeout_ms`` bounds each wait for the peers' flags."""

    def __init__(self, comm: Optional["TPComm"], nbytes: int, timeout_ms: int = 2000,
                 _table=None):
        self.epoch = 0
        self._owned = _table is None
        if _table is None:
            p = ctypes.POINTER(_lib.PeersC)()
            check(_lib.lib().cawq_tp_p2p_create(comm.handle, nbytes, timeout_ms, ctypes.byref(p)))
            self.table = p
        else:
            self.table = _table
        self.world = self.table.contents.world
        self.rank = self.table.contents.rank
        self.slot_bytes = ((nbytes - _lib.CAWQ_TP_P2P_HEADER) // 2) // 256 * 256

    @classmethod
    def from_pointers(cls, world: int, rank: int, bases, nbytes: int,
                      timeout_ms: int = 2000) -> "TPPeers":
        """A table over buffers the caller has mapped itself (any symmetric
        memory allocator); they must be zero before the first call."""
        t = _lib.PeersC()
        t.world, t.rank, t.bytes, t.timeout_ms = world, rank, nbytes, timeout_ms
        for j, b in enumerate(bases):
            t.base[j] = b
        obj = cls(None, nbytes, timeout_ms, _table=ctypes.pointer(t))
        obj._keep = t
        return obj

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def close(self) -> None:
        if self._owned and getattr(self, "table", None):
            check(_lib.lib().cawq_tp_p2p_destroy(self.table))
        self.table = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


GemmFn = Callable[..., torch.Tensor]


def _stream_ptr(t: torch.Tensor) -> int:
    return current_stream_handle(t.get_device())


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return t.data_ptr() if t is not None else None


def _check_native_input(x2: torch.Tensor, scales: torch.Tensor, k: int) -> None:
    """The C calls take raw pointers: before one, the input must be a device
    tensor on the weights' GPU, in the scales' dtype (the kernels read x and
    scales with one element size) and with the shard's K columns."""
    if x2.dtype != scales.dtype:
        raise DTypeError(f"input dtype {x2.dtype} must equal the scales dtype {scales.dtype}",
                         _lib.CAWQ_ERR_DTYPE)
    if x2.shape[-1] != k:
        raise ShapeError(f"input last dim ({x2.shape[-1]}) must be {k}",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    if not x2.is_cuda or not scales.is_cuda or x2.get_device() != scales.get_device():
        raise CubeAwqError(f"the input must be on the weights' GPU ({scales.device}), "
                           f"got {x2.device}", _lib.CAWQ_ERR_INVALID_ARGUMENT)


# ------------------------------------------------------------- layers
class ColumnParallelAWQLinear:
    """Column-parallel AWQGEMMLinear: this rank's N/P output columns.

    Built from the FULL layer tensors (every rank passes the same ones) and
    keeps only its shard. ``forward`` returns the full [..., N] output when
    ``gather_output`` is true, else this rank's [..., N/P] slice (what a
    following row-parallel layer takes).
    """

    def __init__(self, qweight, qzeros, scales, bias=None, *, group=None,
                 gather_output: bool = True, backend: str = "torch",
                 comm: Optional[TPComm] = None, gemm: Optional[GemmFn] = None,
                 peers: Optional[TPPeers] = None):
        self.group = group
        # the fused layers' ranks are the peer table's
        self.world, self.rank = ((peers.world, peers.rank) if backend == "p2p" and peers
                                 else _world_rank(group))
        self.n = scales.shape[1]
        self.k = qweight.shape[0]
        self.group_size = self.k // scales.shape[0]
        self.qweight, self.qzeros, self.scales, self.bias = shard_columns(
            qweight, qzeros, scales, bias, self.world, self.rank)
        self.gather_output = gather_output
        if backend not in ("torch", "native", "p2p"):
            raise ValueError("backend must be 'torch', 'native' or 'p2p'")
        if backend == "native" and comm is None:
            raise ValueError("backend='native' needs a TPComm")
        if backend == "p2p" and peers is None:
            raise ValueError("backend='p2p' needs TPPeers")
        self.backend, self.comm, self.peers = backend, comm, peers
        self.gemm = gemm or fused_gemm
        self._gather_ws = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        m = x2.shape[0]
        if self.backend in ("p2p", "native") and self.gather_output:
            _check_native_input(x2, self.scales, self.k)
        if self.backend == "p2p" and self.gather_output:
            out = torch.empty(m, self.n, dtype=x2.dtype, device=x2.device)
            check(_lib.lib().cawq_gemm_colpar_p2p(
                self.peers.table, self.peers.next_epoch(), _ptr(x2), _ptr(self.qweight),
                _ptr(self.qzeros), _ptr(self.scales), _ptr(self.bias), _ptr(out), m, self.k,
                self.n, self.group_size, cawq_dtype(x2.dtype), _stream_ptr(x2)))
            return out.reshape(*lead, self.n)
        if self.backend == "native" and self.gather_output:
            out = torch.empty(m, self.n, dtype=x2.dtype, device=x2.device)
            ws = None
            if m > 1:
                if self._gather_ws is None or self._gather_ws.numel() < m * self.n or \
                        self._gather_ws.dtype != x2.dtype:
                    self._gather_ws = torch.empty(m * self.n, dtype=x2.dtype, device=x2.device)
                ws = self._gather_ws
            check(_lib.lib().cawq_gemm_colpar(
                self.comm.handle, _ptr(x2), _ptr(self.qweight), _ptr(self.qzeros),
                _ptr(self.scales), _ptr(self.bias), _ptr(out), _ptr(ws), m, self.k, self.n,
                self.group_size, cawq_dtype(x2.dtype), _stream_ptr(x2)))
            return out.reshape(*lead, self.n)
        local = self.gemm(x2, self.qweight, self.qzeros, self.scales, self.group_size,
                          bias=self.bias)
        if not self.gather_output or self.world == 1:
            return local.reshape(*lead, local.shape[-1])
        parts = [torch.empty_like(local) for _ in range(self.world)]
        dist.all_gather(parts, local, group=self.group)
        return torch.cat(parts, dim=-1).reshape(*lead, self.n)

    __call__ = forward


class RowParallelAWQLinear:
    """Row-parallel AWQGEMMLinear: this rank's K/P input rows.

    Built from the FULL layer tensors. ``forward`` takes this rank's
    [..., K/P] columns of the input when ``input_is_parallel`` (else the full
    [..., K] input, of which it uses its own columns) and returns the full
    [..., N] output on every rank: fp32 partials, an fp32 all-reduce, then
    the bias, cast to the input dtype.
    """

    def __init__(self, qweight, qzeros, scales, bias=None, *, group=None,
                 input_is_parallel: bool = True, backend: str = "torch",
                 comm: Optional[TPComm] = None, gemm: Optional[GemmFn] = None,
                 peers: Optional[TPPeers] = None):
        self.group = group
        # the fused layers' ranks are the peer table's
        self.world, self.rank = ((peers.world, peers.rank) if backend == "p2p" and peers
                                 else _world_rank(group))
        self.k = qweight.shape[0]
        self.n = scales.shape[1]
        self.group_size = self.k // scales.shape[0]
        self.k0, self.kl = row_shard(self.k, self.group_size, self.world, self.rank)
        self.qweight, self.qzeros, self.scales = shard_rows(qweight, qzeros, scales,
                                                            self.group_size, self.world, self.rank)
        self.bias = bias
        self.input_is_parallel = input_is_parallel
        if backend not in ("torch", "native", "p2p"):
            raise ValueError("backend must be 'torch', 'native' or 'p2p'")
        if backend == "native" and comm is None:
            raise ValueError("backend='native' needs a TPComm")
        if backend == "p2p" and peers is None:
            raise ValueError("backend='p2p' needs TPPeers")
        self.backend, self.comm, self.peers = backend, comm, peers
        self.gemm = gemm or fused_gemm
        self._partial = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not self.input_is_parallel:
            x2 = x2[:, self.k0:self.k0 + self.kl]
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        m = x2.shape[0]
        if self.backend in ("p2p", "native"):
            _check_native_input(x2, self.scales, self.kl)
        if self.backend == "p2p":
            out = torch.empty(m, self.n, dtype=x2.dtype, device=x2.device)
            check(_lib.lib().cawq_gemm_rowpar_p2p(
                self.peers.table, self.peers.next_epoch(), _ptr(x2), _ptr(self.qweight),
                _ptr(self.qzeros), _ptr(self.scales), _ptr(self.bias), _ptr(out), m, self.k,
                self.n, self.group_size, cawq_dtype(x2.dtype), _stream_ptr(x2)))
            return out.reshape(*lead, self.n)
        if self.backend == "native":
            if self._partial is None or self._partial.numel() < m * self.n:
                self._partial = torch.empty(m * self.n, dtype=torch.float32, device=x2.device)
            out = torch.empty(m, self.n, dtype=x2.dtype, device=x2.device)
            check(_lib.lib().cawq_gemm_rowpar(
                self.comm.handle, _ptr(x2), _ptr(self.qweight), _ptr(self.qzeros),
                _ptr(self.scales), _ptr(self.bias), _ptr(out), _ptr(self._partial), m, self.k,
                self.n, self.group_size, cawq_dtype(x2.dtype), _stream_ptr(x2)))
            return out.reshape(*lead, self.n)
        partial = self.gemm(x2, self.qweight, self.qzeros, self.scales, self.group_size,
                            out_dtype=torch.float32)
        if self.world > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        if self.bias is not None:
            partial = partial + self.bias.to(torch.float32)
        return partial.to(x2.dtype).reshape(*lead, self.n)

    __call__ = forward
