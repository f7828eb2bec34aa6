"""Test helpers: fixture loading, packing, tolerance checks."""

from __future__ import annotations

import json
import os

import numpy as np

from conftest import GOLDEN

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # awq_gemm.rs:248


def load_npz(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def load_json(name: str):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def uniform_word(nib: int) -> int:
    v = 0
    for i in range(8):
        v |= (nib & 0xF) << (4 * i)
    return v


def uniform_kat_tensors(kat: dict):
    """Inputs of a closed-form KAT (awq_kernel_gemm.rs:1119-1391) as numpy arrays."""
    b, m, k, n, gs = kat["b"], kat["m"], kat["k"], kat["n"], kat["group_size"]
    rows = b * m
    if kat["input"] == "mod7x0.1":
        x = ((np.arange(rows * k) % 7).astype(np.float32) * np.float32(0.1)).astype(np.float32)
    elif isinstance(kat["input"], list):
        x = np.concatenate([np.full(m * k, v, dtype=np.float32) for v in kat["input"]])
    else:
        x = np.full(rows * k, kat["input"], dtype=np.float32)
    x = x.reshape(rows, k)
    qw = np.full((k, n // 8), uniform_word(kat["w_nibble"]), dtype=np.uint32)
    qz = np.full((k // gs, n // 8), uniform_word(kat["z_nibble"]), dtype=np.uint32)
    if isinstance(kat["scales"], list):
        sc = np.concatenate([np.full(n, v, dtype=np.float32) for v in kat["scales"]]).reshape(k // gs, n)
    else:
        sc = np.full((k // gs, n), kat["scales"], dtype=np.float32)
    return x, qw, qz, sc


def kat_expected(kat: dict, x: np.ndarray) -> np.ndarray:
    b, m, n = kat["b"], kat["m"], kat["n"]
    if kat["expected"] == "rowsum":
        return np.repeat(x.astype(np.float64).sum(axis=1, keepdims=True), n, axis=1)
    if isinstance(kat["expected"], list):
        return np.concatenate([np.full((m, n), v) for v in kat["expected"]])
    return np.full((b * m, n), float(kat["expected"]))


def max_rel_err(actual, ref) -> float:
    """max |actual - ref| / ||ref||_inf (the north-star GEMM tolerance measure)."""
    actual = np.asarray(actual, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(actual - ref).max() / scale)


def to_torch(a: np.ndarray, dtype: str, device):
    """numpy storage (f32 / f16 / bf16-as-uint16 / uint32) -> torch tensor on device."""
    import torch
    if dtype == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)
    if dtype == "u32":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(device)
    if dtype == "f16":
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(device)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def to_numpy(t, dtype: str) -> np.ndarray:
    import torch
    t = t.detach().cpu()
    if dtype == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f64(a: np.ndarray, dtype: str) -> np.ndarray:
    import oracle
    if dtype == "bf16":
        return oracle.bf16_to_f32(a).astype(np.float64)
    return a.astype(np.float64)


def random_awq(k: int, n: int, g: int, dtype: str, rows: int, seed: int = 0):
    """Seeded random problem in numpy storage of `dtype`: x ~ N(0,1), s ~ U(0.001, 0.02)."""
    import oracle
    rng = np.random.default_rng(seed)
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float32)
    x = rng.standard_normal((rows, k)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    if dtype == "f16":
        return x.astype(np.float16), qw, qz, s.astype(np.float16), b.astype(np.float16)
    if dtype == "bf16":
        return oracle.bf16_bits(x), qw, qz, oracle.bf16_bits(s), oracle.bf16_bits(b)
    return x, qw, qz, s, b


# max |y - y_ref| / ||y_ref||_inf allowed against the exact (fp64) oracle:
# f32 is the north-star bound; 16-bit outputs add one output rounding.
GEMM_TOL = {"f32": 1e-3, "f16": 5e-3, "bf16": 1e-2}
