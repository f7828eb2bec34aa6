"""ctypes binding of libcube_awq.so (the C ABI declared in include/cube_awq.h).

The shared library is built in-tree by ``cube_awq_b200.build``. Loading it
needs no GPU; the GPU entry points return CAWQ_ERR_UNSUPPORTED or
CAWQ_ERR_CUDA when no sm_100 device is present. There is no CPU fallback:
every call that computes goes through this library.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libcube_awq.so")

# cawq_status
CAWQ_OK = 0
CAWQ_ERR_INVALID_SHAPE = 1
CAWQ_ERR_DTYPE = 2
CAWQ_ERR_ALIGNMENT = 3
CAWQ_ERR_CUDA = 4
CAWQ_ERR_NCCL = 5
CAWQ_ERR_TIMEOUT = 6
CAWQ_ERR_UNSUPPORTED = 7
CAWQ_ERR_NULL_POINTER = 8
CAWQ_ERR_INVALID_ARGUMENT = 9

# cawq_dtype / cawq_order / cawq_path
CAWQ_F32, CAWQ_F16, CAWQ_BF16 = 0, 1, 2
CAWQ_ORDER_AWQ, CAWQ_ORDER_NATURAL = 0, 1
CAWQ_PATH_AUTO, CAWQ_PATH_DECODE, CAWQ_PATH_PREFILL, CAWQ_PATH_GENERIC = 0, 1, 2, 3

MAX_RANK = 8

# Every function include/cube_awq.h declares (checked by the CPU tests).
EXPORTED = (
    "cawq_last_error", "cawq_version", "cawq_device_supported", "cawq_device_error",
    "cawq_shape_config_new", "cawq_shape_config_new_with_valid_m",
    "cawq_validate_launch_params", "cawq_validate_decode_launch_params",
    "cawq_select_tile_m", "cawq_select_tile_n",
    "cawq_awq_gemm_linear", "cawq_gemm", "cawq_gemm_with_plan",
    "cawq_gemm_silu_mul", "cawq_gemm_silu_mul_with_plan", "cawq_interleave_gate_up",
    "cawq_gemm_qkv",
    "cawq_plan_get", "cawq_plan_set", "cawq_plan_cache_clear", "cawq_autotune",
    "cawq_dequantize_native", "cawq_dequantize",
    "cawq_tp_column_shard", "cawq_tp_row_shard", "cawq_tp_interleave_columns",
    "cawq_tp_unique_id", "cawq_tp_init", "cawq_tp_destroy", "cawq_tp_info",
    "cawq_gemm_colpar", "cawq_gemm_rowpar", "cawq_gemm_rowpar_noalloc",
    "cawq_tp_p2p_create", "cawq_tp_p2p_destroy", "cawq_gemm_colpar_p2p", "cawq_gemm_rowpar_p2p",
)

CAWQ_ROWPAR_SCRATCH_FLOATS = 1 << 20

CAWQ_TP_ID_BYTES = 128
CAWQ_TP_MAX_PEERS = 8
CAWQ_TP_P2P_HEADER = 256


class PeersC(ctypes.Structure):
    """cawq_tp_peers: every rank's peer buffer as mapped in this process."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int),
                ("base", ctypes.c_void_p * CAWQ_TP_MAX_PEERS), ("bytes", ctypes.c_size_t),
                ("timeout_ms", ctypes.c_int)]


class ShapeConfigC(ctypes.Structure):
    _fields_ = [("m", ctypes.c_size_t), ("k", ctypes.c_size_t), ("n", ctypes.c_size_t),
                ("tile_m", ctypes.c_size_t), ("tile_n", ctypes.c_size_t),
                ("inner_k", ctypes.c_size_t), ("line_size", ctypes.c_size_t),
                ("m_valid", ctypes.c_size_t)]


class TensorDescC(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("rank", ctypes.c_int),
                ("shape", ctypes.c_size_t * MAX_RANK), ("elem_size", ctypes.c_size_t)]


class GemmArgsC(ctypes.Structure):
    _fields_ = [("input", TensorDescC), ("qweight", TensorDescC), ("qzeros", TensorDescC),
                ("scales", TensorDescC), ("bias", TensorDescC), ("output", TensorDescC),
                ("dtype", ctypes.c_int), ("group_size", ctypes.c_size_t)]


class PlanC(ctypes.Structure):
    _fields_ = [("path", ctypes.c_int), ("split", ctypes.c_int), ("warps", ctypes.c_int),
                ("tile_n", ctypes.c_int), ("stages", ctypes.c_int),
                ("reserved", ctypes.c_int * 3)]

    def as_dict(self) -> dict:
        return {"path": self.path, "split": self.split, "warps": self.warps,
                "tile_n": self.tile_n, "stages": self.stages, "pdl": self.reserved[0] == 0,
                "l2_prefetch": self.reserved[1], "mma": "i8" if self.reserved[2] else "f16"}


_lib = None
_lock = threading.Lock()


def _declare(L) -> None:
    sz, vp, i, u32p = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
    st = ctypes.c_int
    L.cawq_last_error.argtypes = []
    L.cawq_last_error.restype = ctypes.c_char_p
    L.cawq_version.argtypes = []
    L.cawq_version.restype = ctypes.c_char_p
    L.cawq_device_supported.argtypes = [i]
    L.cawq_device_supported.restype = i
    L.cawq_device_error.argtypes = [i, ctypes.POINTER(ctypes.c_uint32)]
    L.cawq_device_error.restype = st
    L.cawq_shape_config_new.argtypes = [sz] * 6 + [ctypes.POINTER(ShapeConfigC)]
    L.cawq_shape_config_new.restype = st
    L.cawq_shape_config_new_with_valid_m.argtypes = [sz] * 7 + [ctypes.POINTER(ShapeConfigC)]
    L.cawq_shape_config_new_with_valid_m.restype = st
    L.cawq_validate_launch_params.argtypes = [ctypes.POINTER(ShapeConfigC), sz]
    L.cawq_validate_launch_params.restype = st
    L.cawq_validate_decode_launch_params.argtypes = [ctypes.POINTER(ShapeConfigC), sz]
    L.cawq_validate_decode_launch_params.restype = st
    L.cawq_select_tile_m.argtypes = [sz]
    L.cawq_select_tile_m.restype = sz
    L.cawq_select_tile_n.argtypes = [sz]
    L.cawq_select_tile_n.restype = sz
    L.cawq_awq_gemm_linear.argtypes = [ctypes.POINTER(GemmArgsC), ctypes.POINTER(ShapeConfigC), vp]
    L.cawq_awq_gemm_linear.restype = st
    gemm_args = [vp, u32p, u32p, vp, vp, vp, sz, sz, sz, sz, i, i, i, sz]
    L.cawq_gemm.argtypes = gemm_args + [vp]
    L.cawq_gemm.restype = st
    L.cawq_gemm_with_plan.argtypes = gemm_args + [ctypes.POINTER(PlanC), vp]
    L.cawq_gemm_with_plan.restype = st
    silu_args = [vp, u32p, u32p, vp, vp, vp, sz, sz, sz, sz, i, sz]
    L.cawq_gemm_silu_mul.argtypes = silu_args + [vp]
    L.cawq_gemm_silu_mul.restype = st
    L.cawq_gemm_silu_mul_with_plan.argtypes = silu_args + [ctypes.POINTER(PlanC), vp]
    L.cawq_gemm_silu_mul_with_plan.restype = st
    L.cawq_interleave_gate_up.argtypes = [vp, vp, sz, sz, sz, sz, vp]
    L.cawq_interleave_gate_up.restype = st
    L.cawq_gemm_qkv.argtypes = [vp, u32p, u32p, vp, vp, vp, vp, vp, sz, sz, sz, sz, sz, i, i,
                                sz, sz, sz, vp]
    L.cawq_gemm_qkv.restype = st
    L.cawq_plan_get.argtypes = [sz, sz, sz, sz, i, ctypes.POINTER(PlanC)]
    L.cawq_plan_get.restype = st
    L.cawq_plan_set.argtypes = [sz, sz, sz, sz, i, ctypes.POINTER(PlanC)]
    L.cawq_plan_set.restype = st
    L.cawq_plan_cache_clear.argtypes = []
    L.cawq_plan_cache_clear.restype = None
    L.cawq_autotune.argtypes = [vp, u32p, u32p, vp, vp, sz, sz, sz, sz, i,
                                ctypes.POINTER(PlanC), vp]
    L.cawq_autotune.restype = st
    desc = ctypes.POINTER(TensorDescC)
    L.cawq_dequantize_native.argtypes = [desc, desc, desc, desc, sz, i, i, vp]
    L.cawq_dequantize_native.restype = st
    L.cawq_dequantize.argtypes = [u32p, u32p, vp, vp, sz, sz, sz, i, i, vp]
    L.cawq_dequantize.restype = st
    L.cawq_tp_column_shard.argtypes = [sz, i, i, ctypes.POINTER(sz), ctypes.POINTER(sz)]
    L.cawq_tp_column_shard.restype = st
    L.cawq_tp_row_shard.argtypes = [sz, sz, i, i, ctypes.POINTER(sz), ctypes.POINTER(sz)]
    L.cawq_tp_row_shard.restype = st
    L.cawq_tp_interleave_columns.argtypes = [vp, vp, sz, sz, i, i, vp]
    L.cawq_tp_interleave_columns.restype = st
    L.cawq_tp_unique_id.argtypes = [ctypes.c_char_p]
    L.cawq_tp_unique_id.restype = st
    L.cawq_tp_init.argtypes = [i, i, ctypes.c_char_p, i, ctypes.POINTER(vp)]
    L.cawq_tp_init.restype = st
    L.cawq_tp_destroy.argtypes = [vp]
    L.cawq_tp_destroy.restype = st
    L.cawq_tp_info.argtypes = [vp, ctypes.POINTER(i), ctypes.POINTER(i)]
    L.cawq_tp_info.restype = st
    tp_args = [vp, vp, u32p, u32p, vp, vp, vp, vp, sz, sz, sz, sz, i, vp]
    L.cawq_gemm_colpar.argtypes = tp_args
    L.cawq_gemm_colpar.restype = st
    L.cawq_gemm_rowpar.argtypes = tp_args
    L.cawq_gemm_rowpar.restype = st
    L.cawq_gemm_rowpar_noalloc.argtypes = tp_args[:7] + tp_args[8:]
    L.cawq_gemm_rowpar_noalloc.restype = st
    peers_p = ctypes.POINTER(PeersC)
    L.cawq_tp_p2p_create.argtypes = [vp, sz, i, ctypes.POINTER(peers_p)]
    L.cawq_tp_p2p_create.restype = st
    L.cawq_tp_p2p_destroy.argtypes = [peers_p]
    L.cawq_tp_p2p_destroy.restype = st
    p2p_args = [peers_p, ctypes.c_uint32, vp, vp, vp, vp, vp, vp, sz, sz, sz, sz, i, vp]
    L.cawq_gemm_colpar_p2p.argtypes = p2p_args
    L.cawq_gemm_colpar_p2p.restype = st
    L.cawq_gemm_rowpar_p2p.argtypes = p2p_args
    L.cawq_gemm_rowpar_p2p.restype = st


def lib():
    """The loaded library; raises if libcube_awq.so has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m cube_awq_b200.build` "
                        "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                _declare(L)
                _lib = L
    return _lib


def last_error() -> str:
    return lib().cawq_last_error().decode("utf-8", "replace")
