"""AutoAWQ checkpoint loader: safetensors shards -> AWQGEMMLinear layers.

AutoAWQ stores each quantized linear ``<prefix>`` as ``<prefix>.qweight``
(int32 [K, N/8]), ``<prefix>.qzeros`` (int32 [K/g, N/8]) and
``<prefix>.scales`` (f16 [K/g, N]), optionally ``<prefix>.bias`` ([N]), with
the GEMM nibble order the reference unpacks (README "AWQ Weight Format";
src/kernel/awq_kernel_gemm.rs:10-30). The tensors are used as stored: the
fused kernels read this layout directly, nothing is repacked. The group size
is K / scales rows, as AWQGEMMLinear::group_size computes it
(src/modules/awq_gemm.rs:136-140).
"""

from __future__ import annotations

import glob
import os
from typing import Dict, Iterable, List, Optional, Union

import torch

from .errors import ShapeError
from .modules import AWQGEMMLinear
from . import _lib

_SUFFIXES = ("qweight", "qzeros", "scales", "bias")


def _files(path: Union[str, Iterable[str]]) -> List[str]:
    if isinstance(path, str):
        if os.path.isdir(path):
            found = sorted(glob.glob(os.path.join(path, "*.safetensors")))
            if not found:
                raise FileNotFoundError(f"no *.safetensors files in {path}")
            return found
        return [path]
    return list(path)


def check_layer(prefix: str, qweight: torch.Tensor, qzeros: torch.Tensor,
                scales: torch.Tensor, bias: Optional[torch.Tensor] = None) -> int:
    """Validates one AutoAWQ layer; returns its group size."""
    bad = lambda m: ShapeError(f"{prefix}: {m}", _lib.CAWQ_ERR_INVALID_SHAPE)
    if qweight.dim() != 2 or qzeros.dim() != 2 or scales.dim() != 2:
        raise bad("qweight, qzeros and scales must be 2-D")
    if qweight.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
        raise bad(f"qweight must be int32, got {qweight.dtype}")
    if qzeros.dtype != qweight.dtype:
        raise bad(f"qzeros must be {qweight.dtype}, got {qzeros.dtype}")
    if scales.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise bad(f"scales must be f16 / bf16 / f32, got {scales.dtype}")
    k, n = qweight.shape[0], qweight.shape[1] * 8
    groups = scales.shape[0]
    if scales.shape[1] != n:
        raise bad(f"scales must be [K/g, {n}], got {list(scales.shape)}")
    if qzeros.shape != (groups, qweight.shape[1]):
        raise bad(f"qzeros must be [{groups}, {qweight.shape[1]}], got {list(qzeros.shape)}")
    if groups == 0 or k % groups != 0:
        raise bad(f"K = {k} is not a multiple of the {groups} scale rows")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != n):
        raise bad(f"bias must be [{n}], got {list(bias.shape)}")
    return k // groups


def load_awq_linears(path: Union[str, Iterable[str]], device: Union[str, torch.device] = "cuda",
                     dtype: Optional[torch.dtype] = None,
                     prefixes: Optional[Iterable[str]] = None) -> Dict[str, AWQGEMMLinear]:
    """Every quantized linear of an AutoAWQ checkpoint as an AWQGEMMLinear.

    ``path`` is a safetensors file, a directory of shards or a list of files.
    ``dtype`` optionally converts scales / bias (the activations' F); the
    packed tensors keep their bits. ``prefixes`` restricts the layers loaded.
    """
    from safetensors import safe_open

    wanted = set(prefixes) if prefixes is not None else None
    where: Dict[str, Dict[str, str]] = {}
    for f in _files(path):
        with safe_open(f, framework="pt", device="cpu") as h:
            for key in h.keys():
                prefix, _, suffix = key.rpartition(".")
                if suffix in _SUFFIXES and prefix:
                    where.setdefault(prefix, {})[suffix] = f
    layers: Dict[str, AWQGEMMLinear] = {}
    handles = {}
    try:
        for prefix in sorted(where):
            parts = where[prefix]
            if "qweight" not in parts:
                continue  # a dense layer's bias, not a quantized linear
            if wanted is not None and prefix not in wanted:
                continue
            missing = [s for s in ("qzeros", "scales") if s not in parts]
            if missing:
                raise ShapeError(f"{prefix}: missing {', '.join(missing)}",
                                 _lib.CAWQ_ERR_INVALID_SHAPE)
            t = {}
            for suffix, f in parts.items():
                if f not in handles:
                    handles[f] = safe_open(f, framework="pt", device="cpu").__enter__()
                t[suffix] = handles[f].get_tensor(f"{prefix}.{suffix}")
            check_layer(prefix, t["qweight"], t["qzeros"], t["scales"], t.get("bias"))
            scales, bias = t["scales"], t.get("bias")
            if dtype is not None:
                scales = scales.to(dtype)
                bias = bias.to(dtype) if bias is not None else None
            elif bias is not None:
                bias = bias.to(scales.dtype)
            layers[prefix] = AWQGEMMLinear(
                t["qweight"].to(device).contiguous(), t["qzeros"].to(device).contiguous(),
                scales.to(device).contiguous(),
                bias.to(device).contiguous() if bias is not None else None)
    finally:
        for h in handles.values():
            h.__exit__(None, None, None)
    if wanted is not None and wanted - set(layers):
        raise KeyError(f"layers not in the checkpoint: {sorted(wanted - set(layers))}")
    return layers


# ----------------------------------------------------- fused neighbours
_GATE_UP = ("gate_proj", "up_proj")
_QKV = ("q_proj", "k_proj", "v_proj")


def plan_fusions(names: Iterable[str]) -> Dict[str, tuple]:
    """Groups of sibling layers that the fused modules can replace, by the
    usual decoder-layer names: ``<p>.gate_proj`` + ``<p>.up_proj`` ->
    ``<p>.gate_up_proj`` ("gate_up"), ``<p>.q_proj`` + ``<p>.k_proj`` +
    ``<p>.v_proj`` -> ``<p>.qkv_proj`` ("qkv"). Returns {fused name: (kind,
    member names in order)}; host-only, no tensors involved."""
    names = set(names)
    out: Dict[str, tuple] = {}
    for name in sorted(names):
        parent, _, leaf = name.rpartition(".")
        base = parent + "." if parent else ""
        if leaf == _GATE_UP[0] and base + _GATE_UP[1] in names:
            out[base + "gate_up_proj"] = ("gate_up", tuple(base + m for m in _GATE_UP))
        elif leaf == _QKV[0] and all(base + m in names for m in _QKV[1:]):
            out[base + "qkv_proj"] = ("qkv", tuple(base + m for m in _QKV))
    return out


def fuse_decoder_layers(layers: Dict[str, AWQGEMMLinear]) -> Dict[str, object]:
    """The loaded layers with each gate / up pair replaced by one
    ``AWQGateUpSiluMul`` (``<p>.gate_up_proj``: forward gives silu(gate) *
    up) and each q / k / v triple by one ``AWQQKVLinear`` (``<p>.qkv_proj``:
    forward gives (q, k, v)). Groups the fused kernels cannot take (an
    intermediate size that is not a multiple of 128, f32 scales, q / k / v
    sizes that are not multiples of 32, mismatched shapes) stay as they are.
    The fused modules hold their own copies of the weights (interleaved or
    concatenated); the members are dropped from the returned dict."""
    from .errors import CubeAwqError
    from .modules import AWQGateUpSiluMul, AWQQKVLinear
    out: Dict[str, object] = dict(layers)
    for fused, (kind, members) in plan_fusions(layers).items():
        parts = [layers[m] for m in members]
        try:
            mod = AWQGateUpSiluMul(*parts) if kind == "gate_up" else AWQQKVLinear(*parts)
        except CubeAwqError:
            continue
        for m in members:
            del out[m]
        out[fused] = mod
    return out
