"""Module API: the counterpart of the reference's ``src/modules``.

``AWQGEMMLinearConfig(d_in, d_out, g).with_bias(b).build(device)`` and
``AWQLinearConfig(d_in, d_out, g).build(device)`` keep the reference's names,
argument meaning, parameter shapes and assert messages
(src/modules/awq_gemm.rs:54-233, src/modules/awq_dequantize.rs:9-109).
Parameters are plain torch tensors (the reference's Burn ``Param`` wrapper and
state loading are not part of this path); assign real AWQ tensors to
``qweight``, ``qzeros``, ``scales`` and ``bias`` after ``build``.
"""

from __future__ import annotations

import copy
from typing import Optional

import torch

from . import _lib
from .errors import CubeAwqError, DTypeError, ShapeError
from .errors import check
from .kernel import (PreparedWeights, cawq_dtype, current_stream_handle, dequantize_awq, gemm,
                     gemm_prepared, gemm_qkv, gemm_silu_mul, interleave_gate_up)

AWQ_PACK_FACTOR = 8  # awq_gemm.rs:12
TILE_N_BASE = 32     # awq_gemm.rs:13
INNER_K = 64         # awq_gemm.rs:16


def _shape_assert(cond: bool, msg: str) -> None:
    if not cond:
        raise ShapeError(msg, _lib.CAWQ_ERR_INVALID_SHAPE)


class AWQGEMMLinearConfig:
    """awq_gemm.rs:54-125."""

    def __init__(self, d_input: int, d_output: int, group_size: int):
        self.d_input = d_input
        self.d_output = d_output
        self.group_size = group_size
        self.bias = False

    def with_bias(self, bias: bool) -> "AWQGEMMLinearConfig":
        c = copy.copy(self)
        c.bias = bool(bias)
        return c

    def build(self, device="cuda", dtype: torch.dtype = torch.float32) -> "AWQGEMMLinear":
        """awq_gemm.rs:77-124: asserts, then [K, N/8] / [K/g, N/8] / [K/g, N] / [N] params."""
        _shape_assert(self.group_size > 0, "group_size must be > 0")
        _shape_assert(self.d_output % AWQ_PACK_FACTOR == 0,
                      f"d_output must be divisible by {AWQ_PACK_FACTOR}")
        _shape_assert(self.d_output % TILE_N_BASE == 0,
                      f"d_output must be divisible by TILE_N ({TILE_N_BASE})")
        _shape_assert(self.d_input % INNER_K == 0, f"d_input must be divisible by INNER_K ({INNER_K})")
        _shape_assert(self.d_input % self.group_size == 0, "d_input must be divisible by group_size")
        d_out_packed = self.d_output // AWQ_PACK_FACTOR
        num_groups = self.d_input // self.group_size
        qweight = torch.empty((self.d_input, d_out_packed), dtype=torch.int32, device=device)
        qzeros = torch.empty((num_groups, d_out_packed), dtype=torch.int32, device=device)
        scales = torch.empty((num_groups, self.d_output), dtype=dtype, device=device)
        bias = torch.zeros((self.d_output,), dtype=dtype, device=device) if self.bias else None
        return AWQGEMMLinear(qweight, qzeros, scales, bias)


class AWQGEMMLinear:
    """awq_gemm.rs:127-233: fused dequant-GEMM layer (AutoAWQ order)."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                 bias: Optional[torch.Tensor] = None):
        self.qweight = qweight
        self.qzeros = qzeros
        self.scales = scales
        self.bias = bias
        self._prep = None  # validated call arguments (re-made when a tensor is replaced)

    def group_size(self) -> int:
        """awq_gemm.rs:136-140: K / scale rows."""
        return self.qweight.shape[0] // self.scales.shape[0]

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        """awq_gemm.rs:146-232: [..., K] -> [..., N]; bias fused after the K sum."""
        w = self._prep
        if w is not None and w.matches(self.qweight, self.qzeros, self.scales, self.bias):
            # the common decode / prefill call: checks, allocation and the C
            # call in compiled code; an input it does not take goes on below
            if w.fast is not None:
                r = w.fast.forward(input)
                if r.__class__ is torch.Tensor:
                    return r
                if r is not None:
                    check(r)
            elif input.dim() == 2 and input.shape[1] == w.k and input.is_contiguous():
                return gemm_prepared(w, input)
        _shape_assert(input.dim() >= 2, "input tensor must have at least 2 dims: [..., K]")
        k = input.shape[-1]
        _shape_assert(k > 0, "input last dim (K) must be > 0")
        _shape_assert(input.numel() % k == 0, "input elements must be divisible by K")
        m = input.numel() // k
        x = input.reshape(m, k)
        if not x.is_contiguous():
            x = x.contiguous()
        _shape_assert(k == self.qweight.shape[0], "input last dim (K) must match qweight rows")
        w = self._prep
        if w is None or not w.matches(self.qweight, self.qzeros, self.scales, self.bias):
            w = self._prep = PreparedWeights(self.qweight, self.qzeros, self.scales,
                                             self.group_size(), bias=self.bias, order="awq")
        out = gemm_prepared(w, x)
        return out.reshape(*input.shape[:-1], out.shape[-1])

    __call__ = forward


class AWQLinearConfig:
    """awq_dequantize.rs:9-42."""

    def __init__(self, d_input: int, d_output: int, group_size: int):
        self.d_input = d_input
        self.d_output = d_output
        self.group_size = group_size

    def build(self, device="cuda", dtype: torch.dtype = torch.float32) -> "AWQLinear":
        # awq_dequantize.rs:26-28: bare assert! (message = the condition)
        _shape_assert(self.d_output % 8 == 0, "assertion failed: self.d_output % 8 == 0")
        if self.group_size == 0:
            raise ShapeError("attempt to calculate the remainder with a divisor of zero",
                             _lib.CAWQ_ERR_INVALID_SHAPE)
        _shape_assert(self.d_input % self.group_size == 0,
                      "assertion failed: self.d_input % self.group_size == 0")
        _shape_assert(self.d_output % 32 == 0, "assertion failed: self.d_output % 32 == 0")
        d_out = self.d_output // 8
        g_input = self.d_input // self.group_size
        return AWQLinear(
            torch.empty((self.d_input, d_out), dtype=torch.int32, device=device),
            torch.empty((g_input, d_out), dtype=torch.int32, device=device),
            torch.empty((g_input, self.d_output), dtype=dtype, device=device))


class AWQLinear:
    """awq_dequantize.rs:44-109: dequantize (natural nibble order) / forward."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor):
        self.qweight = qweight
        self.qzeros = qzeros
        self.scales = scales
        self._prep = None  # validated call arguments (re-made when a tensor is replaced)

    def group_size(self) -> int:
        """awq_dequantize.rs:52-56: K / scale rows."""
        return self.qweight.shape[0] // self.scales.shape[0]

    def dequantize(self) -> torch.Tensor:
        """awq_dequantize.rs:62-72: the full-precision [K, N] weight in F."""
        return dequantize_awq(self.qweight, self.qzeros, self.scales, self.group_size())

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        """awq_dequantize.rs:74-108: input[M, K] · dequantize() -> [M, N].

        The reference dequantizes into a [K, N] tensor and runs a separate
        matmul; here the same natural-order weights are dequantized inside the
        fused GEMM, with fp32 accumulation. Rank-2 input only, as in the
        reference (a rank-3 input fails with RankMismatch there, :283-300).
        """
        if input.dim() != 2:
            raise CubeAwqError(
                f"RankMismatch: AWQLinear.forward takes a rank-2 [M, K] input, got rank {input.dim()}",
                _lib.CAWQ_ERR_INVALID_SHAPE)
        x = input if input.is_contiguous() else input.contiguous()
        w = self._prep
        if w is None or not w.matches(self.qweight, self.qzeros, self.scales, None):
            w = self._prep = PreparedWeights(self.qweight, self.qzeros, self.scales,
                                             self.group_size(), order="natural")
        if w.fast is not None:
            r = w.fast.forward(x)
            if r.__class__ is torch.Tensor:
                return r
            if r is not None:
                check(r)
        return gemm_prepared(w, x)

    __call__ = forward


class AWQGateUpSiluMul:
    """The gate and up projections of a gated MLP in one fused GEMM with the
    SiLU gate in its epilogue: forward(x) = silu(x·W_gate + b_gate) *
    (x·W_up + b_up), [..., K] -> [..., I]. The reference runs gate_proj and
    up_proj as two AWQGEMMLinear calls (awq_gemm.rs:146-232) and leaves the
    activation to its caller; this layer reads each weight once, never writes
    the [.., 2I] pre-activation and makes one launch.

    The two layers' AutoAWQ tensors are packed once, at construction, into
    the block-interleaved column order of the fused kernel (128 gate columns,
    128 up columns, ...); I must be a multiple of 128 and F f16 or bf16.
    """

    def __init__(self, gate: "AWQGEMMLinear", up: "AWQGEMMLinear"):
        _shape_assert(gate.qweight.shape == up.qweight.shape and
                      gate.scales.shape == up.scales.shape and
                      gate.qzeros.shape == up.qzeros.shape,
                      "gate and up projections must have the same shapes")
        _shape_assert((gate.bias is None) == (up.bias is None),
                      "gate and up projections must both have a bias or both have none")
        if gate.scales.dtype not in (torch.float16, torch.bfloat16) or \
                up.scales.dtype != gate.scales.dtype:
            raise DTypeError("the SiLU-gated GEMM takes f16 or bf16 scales", _lib.CAWQ_ERR_DTYPE)
        inter = gate.scales.shape[1]
        _shape_assert(inter % 128 == 0,
                      f"the intermediate size ({inter}) must be a multiple of 128")
        self.d_input = gate.qweight.shape[0]
        self.d_output = inter
        self._group_size = gate.group_size()
        _shape_assert(self._group_size == up.group_size(), "gate and up group sizes differ")
        cat = lambda a, b: interleave_gate_up(torch.cat([a, b], dim=-1))
        self.qweight = cat(gate.qweight, up.qweight)
        self.qzeros = cat(gate.qzeros, up.qzeros)
        self.scales = cat(gate.scales, up.scales)
        self.bias = cat(gate.bias, up.bias) if gate.bias is not None else None
        self._inter = inter
        self._call = _lib.lib().cawq_gemm_silu_mul
        self._prepare()

    def _prepare(self) -> None:
        """The constant part of the C call for the 2-D fast path of forward,
        made from the tensors held now; forward re-makes it when one of them
        has been replaced (identity check), so it never reads freed memory."""
        self._held = (self.qweight, self.qzeros, self.scales, self.bias)
        self._dev = self.scales.get_device()
        self._ptrs = (self.qweight.data_ptr(), self.qzeros.data_ptr(), self.scales.data_ptr(),
                      self.bias.data_ptr() if self.bias is not None else None)
        self._tail = (self.d_input, 2 * self._inter, self._group_size,
                      cawq_dtype(self.scales.dtype), self._inter)

    def _current(self) -> bool:
        h = self._held
        return (self.qweight is h[0] and self.qzeros is h[1] and self.scales is h[2] and
                self.bias is h[3])

    def group_size(self) -> int:
        return self._group_size

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if not self._current():
            self._prepare()
        if (input.dim() == 2 and input.shape[1] == self.d_input and
                input.dtype == self.scales.dtype and input.get_device() == self._dev and
                input.is_contiguous()):
            # the common call: checks, one allocation, one C call
            rows = input.shape[0]
            out = input.new_empty((rows, self.d_output))
            st = self._call(input.data_ptr(), *self._ptrs, out.data_ptr(), rows, *self._tail,
                            current_stream_handle(self._dev))
            if st:
                check(st)
            return out
        _shape_assert(input.dim() >= 2, "input tensor must have at least 2 dims: [..., K]")
        k = input.shape[-1]
        _shape_assert(k == self.d_input, "input last dim (K) must match qweight rows")
        x = input.reshape(-1, k)
        if not x.is_contiguous():
            x = x.contiguous()
        out = gemm_silu_mul(x, self.qweight, self.qzeros, self.scales, self._group_size,
                            bias=self.bias)
        return out.reshape(*input.shape[:-1], self.d_output)

    __call__ = forward


class AWQQKVLinear:
    """The q, k and v projections of an attention block in one fused GEMM
    with a split epilogue: forward(x) -> (q [..., n_q], k [..., n_kv],
    v [..., n_kv]). The reference runs them as three AWQGEMMLinear forwards
    (awq_gemm.rs:146-232), each reading x and paying a launch; here the three
    layers' AutoAWQ tensors are concatenated once along the output columns
    and one launch writes the three outputs, optionally into caller-given
    views (``out=``, e.g. rows of a key / value cache). Every element equals
    the one the single-layer forward of the concatenated layer writes.
    n_q and n_kv: multiples of 32.
    """

    def __init__(self, q: "AWQGEMMLinear", k: "AWQGEMMLinear", v: "AWQGEMMLinear"):
        layers = (q, k, v)
        _shape_assert(q.qweight.shape[0] == k.qweight.shape[0] == v.qweight.shape[0],
                      "q, k and v projections must have the same input size")
        _shape_assert(k.scales.shape == v.scales.shape,
                      "k and v projections must have the same shapes")
        _shape_assert(len({l.group_size() for l in layers}) == 1,
                      "q, k and v projections must have the same group size")
        _shape_assert(len({l.bias is None for l in layers}) == 1,
                      "q, k and v projections must all have a bias or all have none")
        _shape_assert(len({l.scales.dtype for l in layers}) == 1,
                      "q, k and v projections must have the same float dtype")
        self.n_q = q.scales.shape[1]
        self.n_kv = k.scales.shape[1]
        _shape_assert(self.n_q % 32 == 0 and self.n_kv % 32 == 0,
                      "q and k/v output sizes must be multiples of 32")
        self.d_input = q.qweight.shape[0]
        self._group_size = q.group_size()
        cat = lambda name: torch.cat([getattr(l, name) for l in layers], dim=-1).contiguous()
        self.qweight = cat("qweight")
        self.qzeros = cat("qzeros")
        self.scales = cat("scales")
        self.bias = cat("bias") if q.bias is not None else None
        self._call = _lib.lib().cawq_gemm_qkv
        self._prepare()

    def _prepare(self) -> None:
        """The constant part of the C call for the fast path of forward, made
        from the tensors held now; forward re-makes it when one of them has
        been replaced (identity check), so it never reads freed memory."""
        self._held = (self.qweight, self.qzeros, self.scales, self.bias)
        self._dev = self.scales.get_device()
        self._ptrs = (self.qweight.data_ptr(), self.qzeros.data_ptr(), self.scales.data_ptr(),
                      self.bias.data_ptr() if self.bias is not None else None)
        code = cawq_dtype(self.scales.dtype) if self._dev >= 0 else 0
        self._tail = (self.d_input, self.n_q, self.n_kv, self._group_size, code, code)

    def _current(self) -> bool:
        h = self._held
        return (self.qweight is h[0] and self.qzeros is h[1] and self.scales is h[2] and
                self.bias is h[3])

    def group_size(self) -> int:
        return self._group_size

    def forward(self, input: torch.Tensor, out: Optional[tuple] = None) -> tuple:
        if not self._current():
            self._prepare()
        _shape_assert(input.dim() >= 2, "input tensor must have at least 2 dims: [..., K]")
        k = input.shape[-1]
        _shape_assert(k == self.d_input, "input last dim (K) must match qweight rows")
        x = input.reshape(-1, k)
        if not x.is_contiguous():
            x = x.contiguous()
        if (out is None and x.dtype == self.scales.dtype and x.get_device() == self._dev and
                self._dev >= 0):
            # the common call: checks, three allocations, one C call
            rows = x.shape[0]
            q, kk, v = (x.new_empty((rows, self.n_q)), x.new_empty((rows, self.n_kv)),
                        x.new_empty((rows, self.n_kv)))
            st = self._call(x.data_ptr(), *self._ptrs, q.data_ptr(), kk.data_ptr(), v.data_ptr(),
                            rows, *self._tail, self.n_q, self.n_kv, self.n_kv,
                            current_stream_handle(self._dev))
            if st:
                check(st)
            lead = input.shape[:-1]
            return (q.reshape(*lead, self.n_q), kk.reshape(*lead, self.n_kv),
                    v.reshape(*lead, self.n_kv))
        q, kk, v = gemm_qkv(x, self.qweight, self.qzeros, self.scales, self._group_size,
                            self.n_q, self.n_kv, bias=self.bias, out=out)
        if out is not None:
            return q, kk, v
        lead = input.shape[:-1]
        return q.reshape(*lead, self.n_q), kk.reshape(*lead, self.n_kv), v.reshape(*lead, self.n_kv)

    __call__ = forward
