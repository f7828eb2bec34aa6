"""cube_awq_b200 — B200 (sm_100a) implementation of the AWQ INT4 hot path of
joshuawm/cube-awq: the fused dequant-GEMM (decode and prefill kernels) and the
standalone dequantize kernel, behind the reference's module API.

    from cube_awq_b200 import AWQGEMMLinearConfig
    layer = AWQGEMMLinearConfig(4096, 4096, 128).with_bias(False).build("cuda:0", torch.float16)
    layer.qweight.copy_(qweight); layer.qzeros.copy_(qzeros); layer.scales.copy_(scales)
    y = layer.forward(x)          # x [..., 4096] -> y [..., 4096]

All compute runs in the CUDA library ``libcube_awq.so`` (C ABI:
``include/cube_awq.h``); importing this package loads it, and without it
every compute call raises ImportError (there is no CPU fallback). Build it
with ``python -m cube_awq_b200.build``.
"""

from . import _lib
from .errors import (CubeAwqError, DeviceTimeoutError, DTypeError, ShapeError,
                     UnsupportedDeviceError)
from .kernel import (DECODE_M_THRESHOLD, DECODE_TILE_M, ShapeConfig, autotune, awq_gemm_linear,
                     dequantize_awq, dequantize_native, device_error, gemm, gemm_qkv,
                     gemm_silu_mul, interleave_gate_up, plan_cache_clear, plan_get, plan_set,
                     select_tile_m, select_tile_n, validate_decode_launch_params,
                     validate_launch_params, version)
from .modules import (AWQGateUpSiluMul, AWQGEMMLinear, AWQGEMMLinearConfig, AWQLinear,
                      AWQLinearConfig, AWQQKVLinear)
from .tp import ColumnParallelAWQLinear, RowParallelAWQLinear, TPComm, TPPeers
from .loader import fuse_decoder_layers, load_awq_linears

import os as _os

if _os.path.exists(_lib.LIB_PATH):
    try:
        _lib.lib()  # load now; without the library every compute call raises (no CPU fallback)
    except (OSError, AttributeError):
        # a library from an older build: `python -m cube_awq_b200.build` must
        # still be able to run; every compute call raises until it is rebuilt
        pass

__all__ = [
    "AWQGateUpSiluMul", "AWQGEMMLinear", "AWQGEMMLinearConfig", "AWQLinear", "AWQLinearConfig",
    "AWQQKVLinear",
    "ColumnParallelAWQLinear", "RowParallelAWQLinear", "TPComm", "TPPeers", "load_awq_linears",
    "fuse_decoder_layers",
    "CubeAwqError", "DeviceTimeoutError", "DTypeError", "ShapeError", "UnsupportedDeviceError",
    "DECODE_M_THRESHOLD", "DECODE_TILE_M", "ShapeConfig", "autotune", "awq_gemm_linear",
    "dequantize_awq", "dequantize_native", "device_error", "gemm", "gemm_qkv", "gemm_silu_mul",
    "interleave_gate_up", "plan_cache_clear",
    "plan_get", "plan_set", "select_tile_m", "select_tile_n", "validate_decode_launch_params",
    "validate_launch_params", "version",
]
