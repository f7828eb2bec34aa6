"""Kernel-level API: the counterpart of the reference's ``src/kernel`` module.

=========================================  ==========================================
reference (joshuawm/cube-awq)              here
=========================================  ==========================================
``ShapeConfig`` (awq_kernel_gemm.rs:35-79)  :class:`ShapeConfig`
``validate_launch_params`` (:160)           :func:`validate_launch_params`
``validate_decode_launch_params`` (:164)    :func:`validate_decode_launch_params`
``awq_gemm_linear`` (:626-771)              :func:`awq_gemm_linear`
``dequantize_native`` (awq_kernel.rs:63)    :func:`dequantize_native`
``dequantize_awq`` (kernel/mod.rs:9-51)     :func:`dequantize_awq`
=========================================  ==========================================

Buffers are torch tensors on an sm_100 GPU (torch supplies device memory and
the current stream); all arithmetic runs in libcube_awq.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .errors import CubeAwqError, DTypeError, ShapeError, check

DECODE_M_THRESHOLD = 8  # awq_kernel_gemm.rs:81
DECODE_TILE_M = 8       # awq_kernel_gemm.rs:82

_DTYPES = {torch.float32: _lib.CAWQ_F32, torch.float16: _lib.CAWQ_F16,
           torch.bfloat16: _lib.CAWQ_BF16}
_PACKED = (torch.int32, getattr(torch, "uint32", torch.int32))


def cawq_dtype(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise DTypeError(f"unsupported float dtype {dtype}; use float32, float16 or bfloat16",
                         _lib.CAWQ_ERR_DTYPE) from None


# The current stream of a device as a cudaStream_t, without building a
# torch.cuda.Stream object (about 2 us per call otherwise).
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream_handle(device_index: int) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream


def stream_handle(t: torch.Tensor) -> Optional[int]:
    return current_stream_handle(t.get_device()) if t.is_cuda else None


def _desc(t: Optional[torch.Tensor]) -> _lib.TensorDescC:
    d = _lib.TensorDescC()
    if t is None:
        d.data = None
        d.rank = 0
        d.elem_size = 0
        return d
    if t.dim() > _lib.MAX_RANK:
        raise ShapeError(f"tensor rank {t.dim()} exceeds {_lib.MAX_RANK}", _lib.CAWQ_ERR_INVALID_SHAPE)
    d.data = t.data_ptr() if t.numel() > 0 else None
    d.rank = t.dim()
    for i, s in enumerate(t.shape):
        d.shape[i] = s
    d.elem_size = t.element_size()
    return d


def _require_cuda(*tensors: Optional[torch.Tensor]) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise CubeAwqError("cube_awq_b200 computes on an sm_100 GPU only; got a CPU tensor "
                               "(there is no CPU fallback)", _lib.CAWQ_ERR_UNSUPPORTED)


@dataclass
class ShapeConfig:
    """Mirror of the reference ShapeConfig (awq_kernel_gemm.rs:35-79)."""

    m: int
    k: int
    n: int
    tile_m: int
    tile_n: int
    inner_k: int
    line_size: int = 4
    m_valid: int = -1

    def __post_init__(self):
        if self.m_valid < 0:
            self.m_valid = self.m

    @classmethod
    def new(cls, m: int, n: int, k: int, m_tile_size: int, n_tile_size: int,
            inner_k_size: int) -> "ShapeConfig":
        """ShapeConfig::new — note the (m, n, k) argument order of the reference."""
        return cls(m=m, k=k, n=n, tile_m=m_tile_size, tile_n=n_tile_size, inner_k=inner_k_size)

    @classmethod
    def new_with_valid_m(cls, m: int, n: int, k: int, m_tile_size: int, n_tile_size: int,
                         inner_k_size: int, m_valid: int) -> "ShapeConfig":
        return cls(m=m, k=k, n=n, tile_m=m_tile_size, tile_n=n_tile_size,
                   inner_k=inner_k_size, m_valid=m_valid)

    def to_c(self) -> _lib.ShapeConfigC:
        return _lib.ShapeConfigC(self.m, self.k, self.n, self.tile_m, self.tile_n, self.inner_k,
                                 self.line_size, self.m_valid)


def validate_launch_params(shape: ShapeConfig, group_size: int) -> None:
    """Prefill-kernel rules (awq_kernel_gemm.rs:89-162); raises ShapeError."""
    c = shape.to_c()
    check(_lib.lib().cawq_validate_launch_params(ctypes.byref(c), group_size))


def validate_decode_launch_params(shape: ShapeConfig, group_size: int) -> None:
    """Decode-kernel rules (awq_kernel_gemm.rs:164-171); raises ShapeError."""
    c = shape.to_c()
    check(_lib.lib().cawq_validate_decode_launch_params(ctypes.byref(c), group_size))


def select_tile_m(m: int) -> int:
    """awq_gemm.rs:30-42, including the AWQ_GEMM_FORCE_TILE_M override."""
    return int(_lib.lib().cawq_select_tile_m(m))


def select_tile_n(n: int) -> int:
    """awq_gemm.rs:44-52."""
    return int(_lib.lib().cawq_select_tile_n(n))


def awq_gemm_linear(input: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                    scales: torch.Tensor, output: torch.Tensor, shape: Optional[ShapeConfig],
                    group_size: int, bias: Optional[torch.Tensor] = None) -> None:
    """awq_gemm_linear (awq_kernel_gemm.rs:626-771): output = input · deq(W) (+ bias).

    Same shape asserts and messages, m_valid resolution and decode/prefill rule
    check as the reference; one fused launch on the current stream. Rows at
    or beyond the resolved m_valid are left untouched, as in the reference.
    """
    _require_cuda(input, qweight, qzeros, scales, output, bias)
    for name, t in (("input", input), ("qweight", qweight), ("qzeros", qzeros),
                    ("scales", scales), ("output", output), ("bias", bias)):
        if t is not None and not t.is_contiguous():
            raise ShapeError(f"{name} must be contiguous (row-major)", _lib.CAWQ_ERR_INVALID_SHAPE)
    args = _lib.GemmArgsC()
    args.input = _desc(input)
    args.qweight = _desc(qweight)
    args.qzeros = _desc(qzeros)
    args.scales = _desc(scales)
    args.bias = _desc(bias)
    args.output = _desc(output)
    args.dtype = cawq_dtype(input.dtype)
    args.group_size = group_size
    c = shape.to_c() if shape is not None else None
    check(_lib.lib().cawq_awq_gemm_linear(ctypes.byref(args),
                                          ctypes.byref(c) if c is not None else None,
                                          stream_handle(input)))


def dequantize_native(q_weight: torch.Tensor, q_zeros: torch.Tensor, q_scales: torch.Tensor,
                      output: torch.Tensor, group_size: int, order: str = "natural") -> None:
    """dequantize_native (awq_kernel.rs:63-111): output[K, N] = (q - z) * s in F.

    Natural nibble order as the reference kernel reads it; ``order="awq"`` is
    an extension that reads the GEMM's AutoAWQ order instead.
    """
    _require_cuda(q_weight, q_zeros, q_scales, output)
    lib = _lib.lib()
    st = lib.cawq_dequantize_native(
        ctypes.byref(_desc(q_weight)), ctypes.byref(_desc(q_zeros)), ctypes.byref(_desc(q_scales)),
        ctypes.byref(_desc(output)), group_size, cawq_dtype(output.dtype), _order(order),
        stream_handle(output))
    check(st)


def dequantize_awq(weight: torch.Tensor, zeros: torch.Tensor, scales: torch.Tensor,
                   group_size: int, order: str = "natural") -> torch.Tensor:
    """dequantize_awq (kernel/mod.rs:9-51): allocates and returns out[K, N]."""
    if weight.dtype not in _PACKED:
        raise DTypeError("assertion failed: matches!(w_primitive.dtype(), DType::I32 | DType::U32)",
                         _lib.CAWQ_ERR_DTYPE)
    if zeros.dtype not in _PACKED:
        raise DTypeError("assertion failed: matches!(z_primitive.dtype(), DType::I32 | DType::U32)",
                         _lib.CAWQ_ERR_DTYPE)
    h = weight.shape[0]
    w = scales.shape[-1]
    out = torch.empty((h, w), dtype=scales.dtype, device=scales.device)
    dequantize_native(weight, zeros, scales, out, group_size, order=order)
    return out


def _order(order: str) -> int:
    if order == "awq":
        return _lib.CAWQ_ORDER_AWQ
    if order == "natural":
        return _lib.CAWQ_ORDER_NATURAL
    raise ValueError(f"order must be 'awq' or 'natural', got {order!r}")


def gemm(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
         group_size: int, bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         out_dtype: Optional[torch.dtype] = None, order: str = "awq",
         plan: Optional[dict] = None) -> torch.Tensor:
    """Hot-path fused GEMM (cawq_gemm): out[rows, N] = x[rows, K] · deq(W) (+ bias).

    ``x`` is [rows, K] (contiguous); ``out`` may be a [rows, >= N] view with a
    unit column stride (its row stride becomes ``ld_out``). ``out_dtype`` is
    x.dtype or float32 (fp32 partial sums). ``plan`` pins a kernel (see
    :func:`plan_get`).
    """
    _require_cuda(x, qweight, qzeros, scales, bias, out)
    if x.dim() != 2 or not x.is_contiguous():
        raise ShapeError("x must be a contiguous [rows, K] tensor", _lib.CAWQ_ERR_INVALID_SHAPE)
    rows, k = x.shape
    n = qweight.shape[1] * 8
    odt = out_dtype or x.dtype
    if out is None:
        out = torch.empty((rows, n), dtype=odt, device=x.device)
    if out.dtype != odt or out.dim() != 2 or out.shape[0] != rows or out.shape[1] < n or \
            (rows > 0 and out.stride(1) != 1):
        raise ShapeError("out must be a [rows, >= N] tensor with unit column stride",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    for name, t in (("qweight", qweight), ("qzeros", qzeros), ("scales", scales), ("bias", bias)):
        if t is not None and not t.is_contiguous():
            raise ShapeError(f"{name} must be contiguous", _lib.CAWQ_ERR_INVALID_SHAPE)
    if qweight.dtype not in _PACKED:
        raise DTypeError("qweight must have i32/u32 dtype", _lib.CAWQ_ERR_DTYPE)
    if qzeros.dtype not in _PACKED:
        raise DTypeError("qzeros must have i32/u32 dtype", _lib.CAWQ_ERR_DTYPE)
    if scales.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype):
        raise DTypeError("scales and bias must have the input's float dtype (F)", _lib.CAWQ_ERR_DTYPE)
    if qweight.shape[0] != k:
        raise ShapeError("input last dim (K) must match qweight rows", _lib.CAWQ_ERR_INVALID_SHAPE)
    groups = scales.shape[0]
    if groups == 0 or k % groups != 0 or qzeros.shape[0] != groups or scales.shape[1] != n or \
            qzeros.shape[1] * 8 != n:
        raise ShapeError("qzeros must be [K/g, N/8] and scales [K/g, N]", _lib.CAWQ_ERR_INVALID_SHAPE)
    if group_size * groups != k:
        raise ShapeError("group_size must equal K / scales rows", _lib.CAWQ_ERR_INVALID_SHAPE)
    lib = _lib.lib()
    ld_out = out.stride(0) if rows > 0 else n
    args = (x.data_ptr(), qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
            bias.data_ptr() if bias is not None else None, out.data_ptr(), rows, k, n, group_size,
            cawq_dtype(x.dtype), cawq_dtype(odt), _order(order), ld_out)
    if plan is None:
        check(lib.cawq_gemm(*args, stream_handle(x)))
    else:
        p = _plan_c(plan)
        check(lib.cawq_gemm_with_plan(*args, ctypes.byref(p), stream_handle(x)))
    return out


def gemm_qkv(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
             group_size: int, n_q: int, n_kv: int, bias: Optional[torch.Tensor] = None,
             out: Optional[tuple] = None, out_dtype: Optional[torch.dtype] = None) -> tuple:
    """Fused qkv projection with a split epilogue (cawq_gemm_qkv): one GEMM
    over the concatenated [q | k | v] weights (AutoAWQ layout, N = n_q +
    2 n_kv) that writes q [rows, n_q], k and v [rows, n_kv] to three outputs.
    ``out`` = (q, k, v) may be views with a unit column stride (for example
    rows of a key / value cache); each output element equals the one
    :func:`gemm` writes for that column. Returns (q, k, v)."""
    _require_cuda(x, qweight, qzeros, scales, bias)
    if x.dim() != 2 or not x.is_contiguous():
        raise ShapeError("x must be a contiguous [rows, K] tensor", _lib.CAWQ_ERR_INVALID_SHAPE)
    rows, k = x.shape
    n = qweight.shape[1] * 8
    if n_q <= 0 or n_kv <= 0 or n_q + 2 * n_kv != n:
        raise ShapeError(f"n_q + 2 n_kv must equal the weight's {n} columns",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    odt = out_dtype or x.dtype
    if out is None:
        out = tuple(torch.empty((rows, w), dtype=odt, device=x.device) for w in (n_q, n_kv, n_kv))
    if len(out) != 3:
        raise ShapeError("out must be a (q, k, v) triple", _lib.CAWQ_ERR_INVALID_SHAPE)
    _require_cuda(*out)
    for t, w in zip(out, (n_q, n_kv, n_kv)):
        if t.dtype != odt or t.dim() != 2 or t.shape[0] != rows or t.shape[1] < w or \
                (rows > 0 and t.stride(1) != 1):
            raise ShapeError("each output must be a [rows, >= width] tensor with unit column "
                             "stride", _lib.CAWQ_ERR_INVALID_SHAPE)
    for name, t in (("qweight", qweight), ("qzeros", qzeros), ("scales", scales), ("bias", bias)):
        if t is not None and not t.is_contiguous():
            raise ShapeError(f"{name} must be contiguous", _lib.CAWQ_ERR_INVALID_SHAPE)
    if qweight.dtype not in _PACKED or qzeros.dtype not in _PACKED:
        raise DTypeError("qweight and qzeros must have i32/u32 dtype", _lib.CAWQ_ERR_DTYPE)
    if scales.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype):
        raise DTypeError("scales and bias must have the input's float dtype (F)", _lib.CAWQ_ERR_DTYPE)
    groups = scales.shape[0]
    if qweight.shape[0] != k or groups == 0 or qzeros.shape[0] != groups or \
            scales.shape[1] != n or qzeros.shape[1] * 8 != n or group_size * groups != k:
        raise ShapeError("qweight [K, N/8], qzeros [K/g, N/8], scales [K/g, N] expected",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    q, kk, v = out
    lds = [t.stride(0) if rows > 0 else w for t, w in zip(out, (n_q, n_kv, n_kv))]
    check(_lib.lib().cawq_gemm_qkv(
        x.data_ptr(), qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
        bias.data_ptr() if bias is not None else None, q.data_ptr(), kk.data_ptr(), v.data_ptr(),
        rows, k, n_q, n_kv, group_size, cawq_dtype(x.dtype), cawq_dtype(odt), *lds,
        stream_handle(x)))
    return q, kk, v


def interleave_gate_up(t: torch.Tensor) -> torch.Tensor:
    """[..rows.., gate | up] columns -> the block-interleaved order of
    :func:`gemm_silu_mul` (cawq_interleave_gate_up): blocks of 128 columns
    alternate gate, up, gate, ... For packed tensors (qweight / qzeros, 8
    columns per int32 word) the blocks are 16 words; for scales / bias, 128
    elements. Returns a new contiguous tensor on the same device."""
    _require_cuda(t)
    t = t.contiguous()
    packed = t.dtype in _PACKED
    block = 16 if packed else 128
    cols = t.shape[-1]
    if cols % (2 * block) != 0:
        raise ShapeError(f"the last dim ({cols}) must be two halves of whole {block}-element blocks",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    if t.element_size() not in (2, 4):
        raise DTypeError("elements must be 2 or 4 bytes", _lib.CAWQ_ERR_DTYPE)
    rows = t.numel() // cols
    out = torch.empty_like(t)
    check(_lib.lib().cawq_interleave_gate_up(t.data_ptr(), out.data_ptr(), rows, cols // 2, block,
                                              t.element_size(), stream_handle(t)))
    return out


def gemm_silu_mul(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor,
                  scales: torch.Tensor, group_size: int, bias: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, plan: Optional[dict] = None) -> torch.Tensor:
    """gate_up GEMM with the SiLU gate in its epilogue (cawq_gemm_silu_mul):
    out[rows, N/2] = silu(x · W_gate + b_gate) * (x · W_up + b_up), with the
    weights (and bias) in the block-interleaved column order of
    :func:`interleave_gate_up`. f16 / bf16."""
    _require_cuda(x, qweight, qzeros, scales, bias, out)
    if x.dim() != 2 or not x.is_contiguous():
        raise ShapeError("x must be a contiguous [rows, K] tensor", _lib.CAWQ_ERR_INVALID_SHAPE)
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise DTypeError("the SiLU-gated GEMM takes f16 or bf16 input", _lib.CAWQ_ERR_DTYPE)
    rows, k = x.shape
    n = qweight.shape[1] * 8
    if out is None:
        out = torch.empty((rows, n // 2), dtype=x.dtype, device=x.device)
    if out.dtype != x.dtype or out.dim() != 2 or out.shape[0] != rows or out.shape[1] < n // 2 or \
            (rows > 0 and out.stride(1) != 1):
        raise ShapeError("out must be a [rows, >= N/2] tensor with unit column stride",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    for name, t in (("qweight", qweight), ("qzeros", qzeros), ("scales", scales), ("bias", bias)):
        if t is not None and not t.is_contiguous():
            raise ShapeError(f"{name} must be contiguous", _lib.CAWQ_ERR_INVALID_SHAPE)
    if scales.dtype != x.dtype or (bias is not None and bias.dtype != x.dtype):
        raise DTypeError("scales and bias must have the input's float dtype (F)", _lib.CAWQ_ERR_DTYPE)
    groups = scales.shape[0]
    if qweight.shape[0] != k or groups == 0 or qzeros.shape[0] != groups or \
            scales.shape[1] != n or qzeros.shape[1] * 8 != n or group_size * groups != k:
        raise ShapeError("qweight [K, N/8], qzeros [K/g, N/8], scales [K/g, N] expected",
                         _lib.CAWQ_ERR_INVALID_SHAPE)
    lib = _lib.lib()
    ld_out = out.stride(0) if rows > 0 else n // 2
    args = (x.data_ptr(), qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
            bias.data_ptr() if bias is not None else None, out.data_ptr(), rows, k, n, group_size,
            cawq_dtype(x.dtype), ld_out)
    if plan is None:
        check(lib.cawq_gemm_silu_mul(*args, stream_handle(x)))
    else:
        p = _plan_c(plan)
        check(lib.cawq_gemm_silu_mul_with_plan(*args, ctypes.byref(p), stream_handle(x)))
    return out


class PreparedWeights:
    """Validated weights of one layer and the constant part of its cawq_gemm
    call, so a forward pass only checks the input and makes one C call. It
    holds the tensors it was made from (``matches`` compares identity)."""

    __slots__ = ("qweight", "qzeros", "scales", "bias", "k", "n", "group_size", "dtype",
                 "code", "order", "ptrs", "device", "dev_index", "tail", "call", "fast")

    def __init__(self, qweight, qzeros, scales, group_size, bias=None, order="awq"):
        _require_cuda(qweight, qzeros, scales, bias)
        for name, t in (("qweight", qweight), ("qzeros", qzeros), ("scales", scales),
                        ("bias", bias)):
            if t is not None and not t.is_contiguous():
                raise ShapeError(f"{name} must be contiguous", _lib.CAWQ_ERR_INVALID_SHAPE)
        if qweight.dtype not in _PACKED:
            raise DTypeError("qweight must have i32/u32 dtype", _lib.CAWQ_ERR_DTYPE)
        if qzeros.dtype not in _PACKED:
            raise DTypeError("qzeros must have i32/u32 dtype", _lib.CAWQ_ERR_DTYPE)
        if bias is not None and bias.dtype != scales.dtype:
            raise DTypeError("scales and bias must have the input's float dtype (F)",
                             _lib.CAWQ_ERR_DTYPE)
        k, n = qweight.shape[0], qweight.shape[1] * 8
        groups = scales.shape[0]
        if groups == 0 or k % groups != 0 or qzeros.shape[0] != groups or \
                scales.shape[1] != n or qzeros.shape[1] * 8 != n:
            raise ShapeError("qzeros must be [K/g, N/8] and scales [K/g, N]",
                             _lib.CAWQ_ERR_INVALID_SHAPE)
        if group_size * groups != k:
            raise ShapeError("group_size must equal K / scales rows", _lib.CAWQ_ERR_INVALID_SHAPE)
        self.qweight, self.qzeros, self.scales, self.bias = qweight, qzeros, scales, bias
        self.k, self.n, self.group_size = k, n, group_size
        self.dtype, self.code, self.order = scales.dtype, cawq_dtype(scales.dtype), _order(order)
        self.ptrs = (qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
                     bias.data_ptr() if bias is not None else None)
        self.device = scales.device
        self.dev_index = scales.get_device()
        # cawq_gemm's arguments after `rows`, and the bound C function
        self.tail = (k, n, group_size, self.code, self.code, self.order, n)
        self.call = _lib.lib().cawq_gemm
        # the compiled forward (checks, allocation and C call in C++), if built
        ext = _torch_ext()
        self.fast = ext.Layer(qweight, qzeros, scales, bias, group_size,
                              self.order) if ext is not None else None

    def matches(self, qweight, qzeros, scales, bias) -> bool:
        return (self.qweight is qweight and self.qzeros is qzeros and self.scales is scales and
                self.bias is bias)


_EXT = False  # not looked up yet


def _torch_ext():
    """_cawq_torch (csrc/cawq_torch.cpp), the compiled host path of the
    module forward over libcube_awq.so, or None if it was not built."""
    global _EXT
    if _EXT is False:
        try:
            from . import _cawq_torch as ext
        except ImportError:
            ext = None
        _EXT = ext
    return _EXT


def gemm_prepared(w: PreparedWeights, x: torch.Tensor) -> torch.Tensor:
    """cawq_gemm with prepared weights: x [rows, K] (contiguous, F) -> [rows, N]."""
    # the per-call host work is kept to the checks, one allocation and one C
    # call: at decode sizes it is of the order of the kernel's own time
    if x.dtype != w.dtype:
        raise DTypeError("scales and bias must have the input's float dtype (F)",
                         _lib.CAWQ_ERR_DTYPE)
    if x.get_device() != w.dev_index:
        _require_cuda(x)
        raise CubeAwqError(f"x is on {x.device}, the weights on {w.device}",
                           _lib.CAWQ_ERR_INVALID_ARGUMENT)
    rows, k = x.shape
    if k != w.k:
        raise ShapeError("input last dim (K) must match qweight rows", _lib.CAWQ_ERR_INVALID_SHAPE)
    out = x.new_empty((rows, w.n))
    st = w.call(x.data_ptr(), *w.ptrs, out.data_ptr(), rows, *w.tail,
                current_stream_handle(w.dev_index))
    if st:
        check(st)
    return out


def _plan_c(plan: dict) -> _lib.PlanC:
    p = _lib.PlanC()
    p.path = int(plan.get("path", 0))
    p.split = int(plan.get("split", 0))
    p.warps = int(plan.get("warps", 0))
    p.tile_n = int(plan.get("tile_n", 0))
    p.stages = int(plan.get("stages", 0))
    p.reserved[0] = 0 if plan.get("pdl", True) else 1
    p.reserved[1] = int(plan.get("l2_prefetch", 0))
    mma = plan.get("mma", "f16")
    if mma not in ("f16", "i8"):
        raise ValueError("plan['mma'] must be 'f16' or 'i8'")
    p.reserved[2] = 1 if mma == "i8" else 0
    return p


PATHS = {"auto": _lib.CAWQ_PATH_AUTO, "decode": _lib.CAWQ_PATH_DECODE,
         "prefill": _lib.CAWQ_PATH_PREFILL, "generic": _lib.CAWQ_PATH_GENERIC}


def plan_get(rows: int, k: int, n: int, group_size: int, dtype: torch.dtype) -> dict:
    """The kernel choice cawq_gemm would make for this problem (needs a GPU)."""
    p = _lib.PlanC()
    check(_lib.lib().cawq_plan_get(rows, k, n, group_size, cawq_dtype(dtype), ctypes.byref(p)))
    return p.as_dict()


def plan_set(rows: int, k: int, n: int, group_size: int, dtype: torch.dtype, plan: dict) -> None:
    p = _plan_c(plan)
    check(_lib.lib().cawq_plan_set(rows, k, n, group_size, cawq_dtype(dtype), ctypes.byref(p)))


def plan_cache_clear() -> None:
    _lib.lib().cawq_plan_cache_clear()


def autotune(x: torch.Tensor, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
             group_size: int, out: Optional[torch.Tensor] = None) -> dict:
    """Times every candidate kernel on these buffers and caches the fastest."""
    _require_cuda(x, qweight, qzeros, scales, out)
    rows, k = x.shape
    n = qweight.shape[1] * 8
    if out is None:
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    p = _lib.PlanC()
    check(_lib.lib().cawq_autotune(x.data_ptr(), qweight.data_ptr(), qzeros.data_ptr(),
                                   scales.data_ptr(), out.data_ptr(), rows, k, n, group_size,
                                   cawq_dtype(x.dtype), ctypes.byref(p), stream_handle(x)))
    return p.as_dict()


def device_error(reset: bool = True) -> int:
    """Device-side error word (bit 0: a bounded wait timed out; bit 1: a fused
    tensor-parallel call gave up waiting for a peer). Synchronises."""
    w = ctypes.c_uint32(0)
    check(_lib.lib().cawq_device_error(1 if reset else 0, ctypes.byref(w)))
    return int(w.value)


def version() -> str:
    return _lib.lib().cawq_version().decode()
