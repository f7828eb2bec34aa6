"""CPU oracle for the AWQ hot path — TEST INFRASTRUCTURE ONLY.

ctypes binding of ``liboracle_awq.so`` (``awq_oracle.c``), a plain-C
restatement of the reference's arithmetic (joshuawm/cube-awq):

* ``dequant``   — ``src/kernel/awq_kernel.rs:38-60`` ((q - z) * s in F)
* ``gemm_ref``  — ``src/kernel/awq_kernel_gemm.rs:346-399, 555-605`` and the
  golden ``cpu_ref`` of ``:793-829`` (F arithmetic, k ascending, bias after:
  ``src/modules/awq_gemm.rs:225-228``)
* ``gemm_f64``  — the same sum accumulated exactly in double

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module. The product
package never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_awq.so")
_lib = None

DTYPES = {"f32": 0, "f16": 1, "bf16": 2}
ORDERS = {"awq": 0, "natural": 1}
# numpy storage of each dtype code (bf16 is carried as raw uint16 bits)
_NP_STORAGE = {0: np.float32, 1: np.float16, 2: np.uint16}

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)          # awq_gemm.rs:248 (packing)
AWQ_REVERSE_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)  # awq_gemm.rs:249 (unpacking)


def build(force: bool = False) -> str:
    """Compile liboracle_awq.so with the Makefile beside this file."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(os.path.join(_HERE, f)) for f in ("awq_oracle.c", "awq_oracle.h")
    ):
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
        L.awqo_nibble.argtypes = [ctypes.c_uint32, i, i]
        L.awqo_nibble.restype = ctypes.c_uint32
        L.awqo_dequant.argtypes = [vp, vp, vp, vp, sz, sz, sz, i, i]
        L.awqo_dequant.restype = None
        L.awqo_gemm_ref.argtypes = [vp, vp, vp, vp, vp, vp, sz, sz, sz, sz, i, i, i]
        L.awqo_gemm_ref.restype = None
        L.awqo_gemm_f64.argtypes = [vp, vp, vp, vp, vp, vp, sz, sz, sz, sz, i, i, i, i]
        L.awqo_gemm_f64.restype = None
        L.awqo_max_threads.argtypes = []
        L.awqo_max_threads.restype = i
        L.awqo_f32_to_bf16.argtypes = [ctypes.c_float]
        L.awqo_f32_to_bf16.restype = ctypes.c_uint16
        L.awqo_f64_to_f16.argtypes = [ctypes.c_double]
        L.awqo_f64_to_f16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _u32(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype == np.int32:
        a = a.view(np.uint32)
    assert a.dtype == np.uint32, a.dtype
    return a


def _float_buf(a, dt: int) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=_NP_STORAGE[dt])


def max_threads() -> int:
    return int(lib().awqo_max_threads())


def nibble(packed: int, col: int, order: str = "awq") -> int:
    return int(lib().awqo_nibble(ctypes.c_uint32(packed & 0xFFFFFFFF), col, ORDERS[order]))


def dequant(qweight, qzeros, scales, group_size: int, dtype: str = "f32", order: str = "natural"):
    """out[K, N] = (q - z) * s rounded once to dtype (awq_kernel.rs:59)."""
    dt = DTYPES[dtype]
    qw, qz = _u32(qweight), _u32(qzeros)
    sc = _float_buf(scales, dt)
    K, N = qw.shape[0], qw.shape[1] * 8
    out = np.empty((K, N), dtype=_NP_STORAGE[dt])
    lib().awqo_dequant(_ptr(qw), _ptr(qz), _ptr(sc), _ptr(out), K, N, group_size, dt, ORDERS[order])
    return out


def gemm_ref(x, qweight, qzeros, scales, group_size: int, bias=None, dtype: str = "f32",
             order: str = "awq", threads: int = 0):
    """The reference's numerics (every op rounded in F, k ascending)."""
    dt = DTYPES[dtype]
    qw, qz = _u32(qweight), _u32(qzeros)
    x2 = _float_buf(x, dt).reshape(-1, qw.shape[0])
    sc = _float_buf(scales, dt)
    b = None if bias is None else _float_buf(bias, dt)
    M, K, N = x2.shape[0], qw.shape[0], qw.shape[1] * 8
    out = np.empty((M, N), dtype=_NP_STORAGE[dt])
    lib().awqo_gemm_ref(_ptr(x2), _ptr(qw), _ptr(qz), _ptr(sc), _ptr(b), _ptr(out),
                        M, K, N, group_size, dt, ORDERS[order], threads)
    return out


def gemm_f64(x, qweight, qzeros, scales, group_size: int, bias=None, dtype: str = "f32",
             order: str = "awq", deq_round: bool = True, threads: int = 0):
    """Exact (double) accumulation of x · w; w rounded to F if deq_round."""
    dt = DTYPES[dtype]
    qw, qz = _u32(qweight), _u32(qzeros)
    x2 = _float_buf(x, dt).reshape(-1, qw.shape[0])
    sc = _float_buf(scales, dt)
    b = None if bias is None else _float_buf(bias, dt)
    M, K, N = x2.shape[0], qw.shape[0], qw.shape[1] * 8
    out = np.empty((M, N), dtype=np.float64)
    lib().awqo_gemm_f64(_ptr(x2), _ptr(qw), _ptr(qz), _ptr(sc), _ptr(b), _ptr(out),
                        M, K, N, group_size, dt, ORDERS[order], int(deq_round), threads)
    return out


def bf16_bits(x) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest even); returns uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_to_f32(bits) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
