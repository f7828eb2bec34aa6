"""Fused GEMM parity on the GPU against the oracle and the reference's tests.

* closed-form KATs of awq_kernel_gemm.rs:1119-1391 through awq_gemm_linear,
  with the reference harness's ShapeConfig (run_kernel, :870-960);
* module fixtures of awq_gemm.rs:408-604 through AWQGEMMLinear.forward;
* seeded random problems on every kernel path and plan, f32 / f16 / bf16,
  against the exact (fp64) oracle with max|y - y_ref| <= tol * ||y_ref||_inf
  (tol: f32 1e-3, f16 5e-3, bf16 1e-2; see helpers.GEMM_TOL).
"""

import numpy as np
import pytest
import torch

import cube_awq_b200 as cawq
import oracle
from helpers import (GEMM_TOL, as_f64, kat_expected, load_json, load_npz, max_rel_err,
                     random_awq, to_numpy, to_torch, uniform_kat_tensors)

pytestmark = pytest.mark.gpu

KATS = load_json("kat_gemm_uniform.json")
PATH_DECODE, PATH_PREFILL, PATH_GENERIC = 1, 2, 3


def _harness_shape(kat):
    # run_kernel (awq_kernel_gemm.rs:881-899): tile_m 32, inner_k 64 or 32
    k, n, gs = kat["k"], kat["n"], kat["group_size"]
    inner_k = 64 if (k >= 64 and k % 64 == 0 and gs >= 64 and gs % 64 == 0) else 32
    tile_n = 128 if (n >= 128 and n % 128 == 0) else 64 if (n >= 64 and n % 64 == 0) else 32
    return cawq.ShapeConfig.new(kat["b"] * kat["m"], n, k, 32, tile_n, inner_k)


@pytest.mark.parametrize("kat", KATS, ids=[k["name"] for k in KATS])
def test_kernel_kats(cuda_device, kat):
    x, qw, qz, sc = uniform_kat_tensors(kat)
    out = torch.full((x.shape[0], kat["n"]), float("nan"), device=cuda_device)
    cawq.awq_gemm_linear(to_torch(x, "f32", cuda_device), to_torch(qw, "u32", cuda_device),
                         to_torch(qz, "u32", cuda_device), to_torch(sc, "f32", cuda_device), out,
                         _harness_shape(kat), kat["group_size"])
    got = out.cpu().numpy()
    assert np.abs(got - kat_expected(kat, x)).max() <= kat["tol"]


MODULE_FIXTURES = [
    "module_forward_b2_m32_k64_n32_g32.npz",
    "module_forward_bias_b2_m32_k64_n32_g32.npz",
    "module_forward_decode_b2_m1_k64_n32_g64.npz",
    "module_forward_4d_1x16x14_k64_n32_g32.npz",
]


@pytest.mark.parametrize("name", MODULE_FIXTURES)
def test_module_forward_fixtures(cuda_device, name):
    f = load_npz(name)
    bias = f.get("bias")
    layer = cawq.AWQGEMMLinear(to_torch(f["qweight"], "u32", cuda_device),
                               to_torch(f["qzeros"], "u32", cuda_device),
                               to_torch(f["scales"], "f32", cuda_device),
                               None if bias is None else to_torch(bias, "f32", cuda_device))
    y = layer.forward(to_torch(f["x"], "f32", cuda_device))
    assert list(y.shape) == list(f["expected"].shape)
    got = y.cpu().numpy()
    assert np.abs(got - f["expected"]).max() <= float(f["tol"])
    assert max_rel_err(got, f["expected"]) <= 1e-3


def test_module_handles_non_divisible_m(cuda_device):
    # awq_gemm.rs:505-515
    f = load_npz("module_forward_b2_m32_k64_n32_g32.npz")
    layer = cawq.AWQGEMMLinear(to_torch(f["qweight"], "u32", cuda_device),
                               to_torch(f["qzeros"], "u32", cuda_device),
                               to_torch(f["scales"], "f32", cuda_device))
    y = layer.forward(torch.zeros(1, 14, 64, device=cuda_device))
    assert list(y.shape) == [1, 14, 32]
    assert float(y.abs().max()) == 0.0


def _run(cuda_device, dtype, rows, k, n, g, plan=None, bias=False, order="awq", out_dtype=None,
         seed=0):
    x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed)
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dtype]
    y = cawq.gemm(to_torch(x, dtype, cuda_device), to_torch(qw, "u32", cuda_device),
                  to_torch(qz, "u32", cuda_device), to_torch(s, dtype, cuda_device), g,
                  bias=to_torch(b, dtype, cuda_device) if bias else None, order=order,
                  plan=plan, out_dtype=out_dtype)
    torch.cuda.synchronize()
    got = as_f64(to_numpy(y, dtype if y.dtype == tdt else "f32"), dtype if y.dtype == tdt else "f32")
    ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b if bias else None, dtype=dtype, order=order,
                          deq_round=False)
    return got, ref, (x, qw, qz, s, b)


DECODE_SHAPES = [(128, 256, 32), (512, 384, 64), (1024, 4096, 128), (4096, 4160, 128),
                 (11008, 512, 128), (3584, 4608, 64), (1024, 256, 16), (960, 384, 48),
                 (1280, 512, 80)]


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 2, 5, 8, 9, 16])
@pytest.mark.parametrize("k,n,g", DECODE_SHAPES)
def test_decode_default_plan_parity(cuda_device, dtype, rows, k, n, g):
    got, ref, _ = _run(cuda_device, dtype, rows, k, n, g)
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]


@pytest.mark.parametrize("split", [1, 2, 3, 4, 5, 6, 8, 12, 16])
@pytest.mark.parametrize("warps", [2, 4, 6, 8])
@pytest.mark.parametrize("stages", [1, 2, 3, 4])
@pytest.mark.parametrize("rows,dtype,mma", [(3, "f32", "f16"), (3, "f16", "f16"),
                                            (3, "f16", "i8"), (4, "bf16", "i8"),
                                            (11, "f16", "f16")])
def test_decode_every_plan(cuda_device, split, warps, stages, rows, dtype, mma):
    # warps = 128-column strips per CTA (two consumer warps each), split = CTAs
    # of a cluster along K (any size: the band's 8-column words are dealt out
    # in rounded-up slices, so 12 CTAs over 2 strips leave the last one none);
    # N = 1184 leaves the last band of every strip count partly out of range.
    # mma "i8" selects the integer tensor path (rows <= 4 with 16-bit X, here
    # g = 128); "f16" is the f16 / bf16 MMA path.
    if rows > 8 and 2 * warps > 8:
        pytest.skip("more warps than a 16-row tile allows")
    plan = {"path": PATH_DECODE, "split": split, "warps": warps, "stages": stages, "mma": mma}
    got, ref, _ = _run(cuda_device, dtype, rows, 2048, 1184, 128, plan=plan)
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 2, 4])
@pytest.mark.parametrize("g", [64, 128, 256])
def test_decode_integer_path_with_activation_outliers(cuda_device, dtype, rows, g):
    # The integer path scales each 64-k slice of an X row by a power of two of
    # its own maximum: a few activations 300x larger than the rest cost the
    # other values of their slice some bits, which the tolerance still covers;
    # the result also stays close to the f16 / bf16 MMA path's.
    k, n = 4096, 1024
    _, qw, qz, s, _ = random_awq(k, n, g, dtype, rows, seed=77)
    rng = np.random.default_rng(78)
    x32 = rng.standard_normal((rows, k)).astype(np.float32)
    x32[:, rng.choice(k, size=12, replace=False)] *= 300.0
    x = x32.astype(np.float16) if dtype == "f16" else oracle.bf16_bits(x32)
    t = lambda a, d: to_torch(a, d, cuda_device)
    args = (t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), g)
    plan = {"path": PATH_DECODE, "split": 4, "warps": 2, "stages": 4}
    y_i8 = as_f64(to_numpy(cawq.gemm(*args, plan=dict(plan, mma="i8")), dtype), dtype)
    y_f16 = as_f64(to_numpy(cawq.gemm(*args, plan=plan), dtype), dtype)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype=dtype, deq_round=False)
    assert max_rel_err(y_i8, ref) <= GEMM_TOL[dtype]
    assert max_rel_err(y_i8, y_f16) <= GEMM_TOL[dtype]


@pytest.mark.parametrize("pdl", [True, False])
@pytest.mark.parametrize("rows", [1, 12])
def test_decode_chain_with_and_without_programmatic_launch(cuda_device, pdl, rows):
    # Two dependent GEMMs back to back on one stream: the second reads the
    # first one's output as X (programmatic dependent launch must wait for it).
    k, n, g = 2048, 2048, 128
    x, qw, qz, s, _ = random_awq(k, n, g, "f16", rows, seed=21)
    _, qw2, qz2, s2, _ = random_awq(n, k, g, "f16", rows, seed=22)
    plan = {"path": PATH_DECODE, "split": 4, "warps": 4, "stages": 2, "pdl": pdl}
    t = lambda a, d: to_torch(a, d, cuda_device)
    y1 = torch.empty(rows, n, dtype=torch.float16, device=cuda_device)
    y2 = torch.empty(rows, k, dtype=torch.float16, device=cuda_device)
    for _ in range(3):
        cawq.gemm(t(x, "f16"), t(qw, "u32"), t(qz, "u32"), t(s, "f16"), g, out=y1, plan=plan)
        cawq.gemm(y1, t(qw2, "u32"), t(qz2, "u32"), t(s2, "f16"), g, out=y2, plan=plan)
    torch.cuda.synchronize()
    y1n = y1.cpu().numpy()
    ref1 = oracle.gemm_f64(x, qw, qz, s, g, dtype="f16", deq_round=False)
    assert max_rel_err(y1n.astype(np.float64), ref1) <= GEMM_TOL["f16"]
    ref2 = oracle.gemm_f64(y1n, qw2, qz2, s2, g, dtype="f16", deq_round=False)
    assert max_rel_err(y2.float().cpu().numpy(), ref2) <= GEMM_TOL["f16"]


@pytest.mark.parametrize("pdl", [True, False])
@pytest.mark.parametrize("rows,halves,split", [(64, 1, 4), (200, 2, 1), (300, 1, 2)])
def test_prefill_chain_with_and_without_programmatic_launch(cuda_device, pdl, rows, halves,
                                                             split):
    # Three dependent prefill GEMMs back to back, each reading the previous
    # output as X and writing a buffer the one before it read: the kernel's
    # X loads must wait for the previous grid, and so must its stores.
    k, g = 1024, 128
    x, qw, qz, s, _ = random_awq(k, k, g, "f16", rows, seed=31)
    _, qw2, qz2, s2, _ = random_awq(k, k, g, "f16", rows, seed=32)
    plan = {"path": PATH_PREFILL, "warps": halves, "split": split, "pdl": pdl}
    t = lambda a, d: to_torch(a, d, cuda_device)
    w1 = (t(qw, "u32"), t(qz, "u32"), t(s, "f16"))
    w2 = (t(qw2, "u32"), t(qz2, "u32"), t(s2, "f16"))
    a = t(x, "f16")
    b = torch.empty_like(a)
    for _ in range(2):
        a = t(x, "f16")
        cawq.gemm(a, *w1, g, out=b, plan=plan)   # b = x W1
        cawq.gemm(b, *w2, g, out=a, plan=plan)   # a = b W2 (a was read by the first)
        cawq.gemm(a, *w1, g, out=b, plan=plan)   # b = a W1 (b was read by the second)
    torch.cuda.synchronize()
    h1 = oracle.gemm_f64(x, qw, qz, s, g, dtype="f16", deq_round=True).astype(np.float16)
    h2 = oracle.gemm_f64(h1, qw2, qz2, s2, g, dtype="f16", deq_round=True)
    assert max_rel_err(a.float().cpu().numpy(), h2) <= 2 * GEMM_TOL["f16"]
    h3 = oracle.gemm_f64(a.cpu().numpy(), qw, qz, s, g, dtype="f16", deq_round=True)
    assert max_rel_err(b.float().cpu().numpy(), h3) <= GEMM_TOL["f16"]


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rows,k,n,g", [(1, 64, 32, 32), (7, 256, 96, 32), (33, 512, 256, 64),
                                        (130, 256, 4096, 128)])
def test_generic_path_parity(cuda_device, dtype, rows, k, n, g):
    got, ref, _ = _run(cuda_device, dtype, rows, k, n, g, plan={"path": PATH_GENERIC})
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]


@pytest.mark.parametrize("path", [PATH_DECODE, PATH_GENERIC])
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_bias_natural_order_and_fp32_out(cuda_device, path, dtype):
    plan = {"path": path, "split": 4, "warps": 8, "stages": 2} if path == PATH_DECODE else {"path": path}
    got, ref, _ = _run(cuda_device, dtype, 4, 1024, 512, 64, plan=plan, bias=True, order="natural",
                       out_dtype=torch.float32)
    assert max_rel_err(got, ref) <= (GEMM_TOL["f32"] if dtype == "f32" else 2e-3)


def test_column_slice_output_ld(cuda_device):
    # a column shard writing into its slice of a wider output (ld_out = 1024)
    x, qw, qz, s, _ = random_awq(512, 256, 128, "f16", 2, seed=4)
    full = torch.zeros(2, 1024, dtype=torch.float16, device=cuda_device)
    cawq.gemm(to_torch(x, "f16", cuda_device), to_torch(qw, "u32", cuda_device),
              to_torch(qz, "u32", cuda_device), to_torch(s, "f16", cuda_device), 128,
              out=full[:, 256:512])
    ref = oracle.gemm_f64(x, qw, qz, s, 128, dtype="f16", deq_round=False)
    got = full.float().cpu().numpy()
    assert max_rel_err(got[:, 256:512], ref) <= GEMM_TOL["f16"]
    assert float(full[:, :256].abs().max()) == 0.0 and float(full[:, 512:].abs().max()) == 0.0


def test_cfg1_decode_full_size_f32(cuda_device):
    # M=1, K=N=4096, g=128, f32, against the reference numerics
    got, ref, (x, qw, qz, s, _) = _run(cuda_device, "f32", 1, 4096, 4096, 128, seed=0x5EED)
    assert max_rel_err(got, ref) <= 1e-3
    ref_numerics = oracle.gemm_ref(x, qw, qz, s, 128, dtype="f32").astype(np.float64)
    assert max_rel_err(got, ref_numerics) <= 1e-3
    assert cawq.device_error() == 0


def test_f16_distance_to_reference_numerics_is_reported(cuda_device):
    # The reference accumulates in f16; this build in fp32. Both are compared
    # with the exact sum: the fused kernel must be at least as close.
    got, ref, (x, qw, qz, s, _) = _run(cuda_device, "f16", 1, 4096, 1024, 128, seed=3)
    ref16 = oracle.gemm_ref(x, qw, qz, s, 128, dtype="f16").astype(np.float64)
    assert max_rel_err(got, ref) <= max_rel_err(ref16, ref) + 1e-3


PREFILL_SHAPES = [(17, 128, 256, 64), (128, 512, 512, 128), (200, 512, 768, 128),
                  (37, 1024, 4160, 64), (513, 2048, 1024, 128), (1000, 1024, 800, 128),
                  (256, 4096, 4096, 128)]


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows,k,n,g", PREFILL_SHAPES)
def test_prefill_tcgen05_parity(cuda_device, dtype, rows, k, n, g):
    # The tensor-core path dequantizes in F exactly as the reference does, so
    # it is compared with the oracle that rounds the weights to F.
    x, qw, qz, s, _ = random_awq(k, n, g, dtype, rows, seed=rows + n)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[dtype]
    y = cawq.gemm(to_torch(x, dtype, cuda_device), to_torch(qw, "u32", cuda_device),
                  to_torch(qz, "u32", cuda_device), to_torch(s, dtype, cuda_device), g,
                  plan={"path": PATH_PREFILL})
    torch.cuda.synchronize()
    got = as_f64(to_numpy(y, dtype), dtype)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype=dtype, deq_round=True)
    assert max_rel_err(got, ref) <= GEMM_TOL[dtype]


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_prefill_bias_natural_order_fp32_out_and_ld(cuda_device, dtype):
    rows, k, n, g = 300, 1024, 512, 128
    x, qw, qz, s, b = random_awq(k, n, g, dtype, rows, seed=9)
    full = torch.zeros(rows, 2 * n, dtype=torch.float32, device=cuda_device)
    cawq.gemm(to_torch(x, dtype, cuda_device), to_torch(qw, "u32", cuda_device),
              to_torch(qz, "u32", cuda_device), to_torch(s, dtype, cuda_device), g,
              bias=to_torch(b, dtype, cuda_device), out=full[:, n:], out_dtype=torch.float32,
              order="natural", plan={"path": PATH_PREFILL})
    torch.cuda.synchronize()
    ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b, dtype=dtype, order="natural", deq_round=True)
    got = full.cpu().numpy()
    assert max_rel_err(got[:, n:], ref) <= 2e-3
    assert float(np.abs(got[:, :n]).max()) == 0.0


def test_planner_picks_prefill_for_large_m(cuda_device):
    assert cawq.plan_get(2048, 4096, 4096, 128, torch.float16)["path"] == PATH_PREFILL
    assert cawq.plan_get(1, 4096, 4096, 128, torch.float16)["path"] == PATH_DECODE
    # f32 activations: the tcgen05 kernel with x split into bf16 hi + lo
    assert cawq.plan_get(2048, 4096, 4096, 128, torch.float32)["path"] == PATH_PREFILL
    # 128 x 256 tiles once they fill the GPU, else 128 x 128
    assert cawq.plan_get(2048, 4096, 4096, 128, torch.float32)["tile_n"] == 256
    assert cawq.plan_get(512, 4096, 4096, 128, torch.float32)["tile_n"] == 128
    # ... which needs whole 64-row groups; the CUDA-core kernel takes the rest
    assert cawq.plan_get(2048, 4096, 4096, 32, torch.float32)["path"] == PATH_GENERIC


PREFILL_F32_SHAPES = [(17, 128, 256, 64), (128, 512, 512, 128), (200, 512, 800, 128),
                      (37, 1024, 4160, 64), (513, 2048, 1024, 256), (129, 4096, 4096, 128)]


@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("rows,k,n,g", PREFILL_F32_SHAPES)
def test_prefill_f32_tcgen05_parity(cuda_device, rows, k, n, g, tile_n):
    # f32 x and scales on the tensor cores: exact (q - z) weights, x as bf16
    # hi + lo, each group's sum scaled in fp32; N = 800 / 4160 end in a
    # partial column tile (of 128 or 256). The north star's bound against the
    # exact sum, and against the reference's own f32 numerics.
    x, qw, qz, s, _ = random_awq(k, n, g, "f32", rows, seed=rows + n + 1)
    t = lambda a, d: to_torch(a, d, cuda_device)
    y = cawq.gemm(t(x, "f32"), t(qw, "u32"), t(qz, "u32"), t(s, "f32"), g,
                  plan={"path": PATH_PREFILL, "tile_n": tile_n})
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = oracle.gemm_f64(x, qw, qz, s, g, dtype="f32", deq_round=False)
    assert max_rel_err(got, ref) <= 1e-4
    ref_numerics = oracle.gemm_ref(x, qw, qz, s, g, dtype="f32").astype(np.float64)
    assert max_rel_err(got, ref_numerics) <= GEMM_TOL["f32"]


@pytest.mark.parametrize("tile_n", [128, 256])
def test_prefill_f32_bias_natural_order_ld_and_determinism(cuda_device, tile_n):
    rows, k, n, g = 300, 1024, 512, 128
    x, qw, qz, s, b = random_awq(k, n, g, "f32", rows, seed=19)
    t = lambda a, d: to_torch(a, d, cuda_device)
    full = torch.zeros(rows, 2 * n, dtype=torch.float32, device=cuda_device)
    args = (t(x, "f32"), t(qw, "u32"), t(qz, "u32"), t(s, "f32"), g)
    plan = {"path": PATH_PREFILL, "tile_n": tile_n}
    cawq.gemm(*args, bias=t(b, "f32"), out=full[:, n:], order="natural", plan=plan)
    y2 = cawq.gemm(*args, bias=t(b, "f32"), order="natural", plan=plan)
    torch.cuda.synchronize()
    ref = oracle.gemm_f64(x, qw, qz, s, g, bias=b, dtype="f32", order="natural",
                          deq_round=False)
    got = full.cpu().numpy()
    assert max_rel_err(got[:, n:], ref) <= 1e-4
    assert float(np.abs(got[:, :n]).max()) == 0.0
    assert torch.equal(full[:, n:], y2)


def test_prefill_f32_full_size_sampled_rows(cuda_device):
    # configs[2] with f32 activations: M = 2048 on the 4096 x 4096 layer
    from cube_awq_b200 import synth
    k, n, g, m = 4096, 4096, 128, 2048
    w = synth.make_weights(k, n, g, torch.float32, cuda_device, seed=87)
    xt = synth.make_input(m, k, torch.float32, cuda_device, seed=88)
    y = cawq.gemm(xt, w.qweight, w.qzeros, w.scales, g)
    y2 = cawq.gemm(xt, w.qweight, w.qzeros, w.scales, g)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    rows = np.arange(0, m, 32)
    x = xt.cpu().numpy()[rows]
    ref = oracle.gemm_f64(x, w.qweight.cpu().numpy(), w.qzeros.cpu().numpy(),
                          w.scales.cpu().numpy(), g, dtype="f32", deq_round=False)
    assert max_rel_err(y.cpu().numpy()[rows].astype(np.float64), ref) <= 1e-4
    assert cawq.device_error() == 0


def test_prefill_full_size_sampled_rows(cuda_device):
    # M = 2048 on the 4096 x 4096 layer; 64 sampled rows checked
    from cube_awq_b200 import synth
    k, n, g, m = 4096, 4096, 128, 2048
    w = synth.make_weights(k, n, g, torch.float16, cuda_device, seed=77)
    xt = synth.make_input(m, k, torch.float16, cuda_device, seed=78)
    y = cawq.gemm(xt, w.qweight, w.qzeros, w.scales, g)
    torch.cuda.synchronize()
    rows = np.arange(0, m, 32)
    x = xt.cpu().numpy()[rows]
    ref = oracle.gemm_f64(x, w.qweight.cpu().numpy(), w.qzeros.cpu().numpy(),
                          w.scales.cpu().numpy(), g, dtype="f16", deq_round=True)
    assert max_rel_err(y.float().cpu().numpy()[rows], ref) <= GEMM_TOL["f16"]
    assert cawq.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_is_deterministic_at_full_size(cuda_device, dtype):
    # The tensor-core path has no atomics: repeated launches on the same
    # inputs must agree bit for bit (a pipeline race would show up here).
    from cube_awq_b200 import synth
    k, n, g, m = 4096, 4096, 128, 2048
    w = synth.make_weights(k, n, g, dtype, cuda_device, seed=81)
    x = synth.make_input(m, k, dtype, cuda_device, seed=82)
    plan = {"path": PATH_PREFILL}
    y0 = cawq.gemm(x, w.qweight, w.qzeros, w.scales, g, plan=plan)
    for _ in range(8):
        y = cawq.gemm(x, w.qweight, w.qzeros, w.scales, g, plan=plan)
        assert torch.equal(y, y0)
    yg = cawq.gemm(x, w.qweight, w.qzeros, w.scales, g, plan={"path": PATH_GENERIC})
    torch.cuda.synchronize()
    rel = (y0.float() - yg.float()).abs().max() / yg.float().abs().max()
    assert float(rel) <= GEMM_TOL["f16" if dtype == torch.float16 else "bf16"]


def test_module_sees_replaced_weights(cuda_device):
    # AWQGEMMLinear keeps its validated call arguments between forwards; a
    # tensor assigned to the layer afterwards must be used by the next call.
    t = lambda a, d: to_torch(a, d, cuda_device)
    x, qw, qz, s, b = random_awq(512, 256, 128, "f16", 3, seed=51)
    _, qw2, qz2, s2, _ = random_awq(512, 256, 128, "f16", 3, seed=52)
    layer = cawq.AWQGEMMLinear(t(qw, "u32"), t(qz, "u32"), t(s, "f16"))
    xt = t(x, "f16")
    y1 = layer.forward(xt)
    layer.qweight, layer.qzeros, layer.scales = t(qw2, "u32"), t(qz2, "u32"), t(s2, "f16")
    y2 = layer.forward(xt)
    layer.bias = t(b, "f16")
    y3 = layer.forward(xt)
    torch.cuda.synchronize()
    for got, (w_, z_, s_, b_) in ((y1, (qw, qz, s, None)), (y2, (qw2, qz2, s2, None)),
                                  (y3, (qw2, qz2, s2, b))):
        ref = oracle.gemm_f64(x, w_, z_, s_, 128, bias=b_, dtype="f16", deq_round=False)
        assert max_rel_err(got.float().cpu().numpy(), ref) <= GEMM_TOL["f16"]


@pytest.mark.parametrize("halves", [1, 2])
@pytest.mark.parametrize("split", [1, 2, 4, 8])
@pytest.mark.parametrize("rows", [20, 64, 128, 200])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_prefill_every_plan(cuda_device, halves, split, rows, dtype):
    # 128- or 256-row tiles, K split over 1..8 CTAs of a cluster (the partial
    # sums meet in the owner CTAs); N = 768 is three 256-column tiles
    plan = {"path": PATH_PREFILL, "warps": halves, "split": split}
    if halves == 2 and split > 4:
        with pytest.raises(Exception):
            _run(cuda_device, dtype, rows, 1024, 768, 128, plan=plan)
        return
    x, qw, qz, s, b = random_awq(1024, 768, 128, dtype, rows, seed=rows + split)
    t = lambda a, d: to_torch(a, d, cuda_device)
    y = cawq.gemm(t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), 128, bias=t(b, dtype),
                  plan=plan)
    y2 = cawq.gemm(t(x, dtype), t(qw, "u32"), t(qz, "u32"), t(s, dtype), 128, bias=t(b, dtype),
                   plan=plan)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # partial sums are added in rank order
    ref = oracle.gemm_f64(x, qw, qz, s, 128, bias=b, dtype=dtype, deq_round=True)
    assert max_rel_err(as_f64(to_numpy(y, dtype), dtype), ref) <= GEMM_TOL[dtype]


def test_planner_splits_k_for_mid_m(cuda_device):
    # Qwen2 o_proj at M = 64: 14 output tiles -> clusters of 8 CTAs along K;
    # qkv: 18 tiles, of which only 16 clusters of 8 (one CTA per SM) are
    # resident at once on a B200, so the planner halves the split instead of
    # leaving two clusters for a second wave
    p = cawq.plan_get(64, 3584, 3584, 64, torch.float16)
    assert p["path"] == PATH_PREFILL and p["warps"] == 1 and p["split"] == 8
    p = cawq.plan_get(64, 3584, 4608, 64, torch.float16)
    assert p["path"] == PATH_PREFILL and p["warps"] == 1 and p["split"] == 4
    p = cawq.plan_get(2048, 4096, 4096, 128, torch.float16)
    assert p["path"] == PATH_PREFILL and p["warps"] == 2 and p["split"] == 1


def test_planner_cost_model_for_rows_above_128(cuda_device):
    # 128-row tiles with split K where 256-row tiles would leave most SMs
    # idle (Qwen2 o_proj / down at M = 256: 14 column tiles), 256-row tiles
    # where the columns alone fill the GPU (Qwen2 gate_up: 148 column tiles)
    for n, k in ((3584, 3584), (3584, 18944)):
        p = cawq.plan_get(256, k, n, 64, torch.float16)
        assert p["path"] == PATH_PREFILL and p["warps"] == 1 and p["split"] >= 2, p
    p = cawq.plan_get(256, 3584, 37888, 64, torch.float16)
    assert p["path"] == PATH_PREFILL and p["warps"] == 2 and p["split"] == 1, p
    for m in (1024, 2048, 4096):
        p = cawq.plan_get(m, 4096, 22016, 128, torch.float16)
        assert p["warps"] == 2, (m, p)
