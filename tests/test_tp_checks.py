"""Argument checks of the tensor-parallel layers' C-call back ends, on the CPU.

The 'native' and 'p2p' forwards hand raw pointers to the library. Before the
call they must refuse an input whose dtype differs from the scales' (the
kernels read x and scales with one element size), one with the wrong K, and
one that is not on the weights' GPU (here: a CPU tensor). None of these
reach the library, so they run without a GPU.
"""

import types

import numpy as np
import pytest
import torch

from cube_awq_b200 import CubeAwqError, DTypeError, ShapeError, tp


def _full(k=256, n=128, g=64, dtype=torch.float16):
    rng = np.random.default_rng(3)
    qw = torch.from_numpy(rng.integers(0, 2**31, (k, n // 8), dtype=np.int64).astype(np.int32))
    qz = torch.from_numpy(rng.integers(0, 2**31, (k // g, n // 8), dtype=np.int64).astype(np.int32))
    s = torch.from_numpy(rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)).to(dtype)
    return qw, qz, s


def _fake_peers():
    return types.SimpleNamespace(world=1, rank=0, table=None, next_epoch=lambda: 1)


def _layers(backend):
    qw, qz, s = _full()
    kw = {"comm": object()} if backend == "native" else {"peers": _fake_peers()}
    col = tp.ColumnParallelAWQLinear(qw, qz, s, backend=backend, **kw)
    row = tp.RowParallelAWQLinear(qw, qz, s, backend=backend, **kw)
    return col, row


@pytest.mark.parametrize("backend", ["native", "p2p"])
def test_refuses_dtype_mismatch(backend):
    col, row = _layers(backend)
    x = torch.zeros(2, 256, dtype=torch.float32)  # f32 input, f16 scales
    with pytest.raises(DTypeError):
        col.forward(x)
    with pytest.raises(DTypeError):
        row.forward(x)


@pytest.mark.parametrize("backend", ["native", "p2p"])
def test_refuses_wrong_k(backend):
    col, row = _layers(backend)
    x = torch.zeros(2, 192, dtype=torch.float16)
    with pytest.raises(ShapeError):
        col.forward(x)
    with pytest.raises(ShapeError):
        row.forward(x)


@pytest.mark.parametrize("backend", ["native", "p2p"])
def test_refuses_host_input(backend):
    col, row = _layers(backend)
    x = torch.zeros(2, 256, dtype=torch.float16)  # right dtype and K, but on the host
    with pytest.raises(CubeAwqError):
        col.forward(x)
    with pytest.raises(CubeAwqError):
        row.forward(x)
