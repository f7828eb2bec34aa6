"""AutoAWQ safetensors loader: finds every quantized linear, checks the
layout, keeps the packed bits, and (on a GPU) runs the loaded layers."""

import numpy as np
import pytest
import torch

import oracle
from cube_awq_b200 import ShapeError
from cube_awq_b200.loader import load_awq_linears
from helpers import GEMM_TOL, max_rel_err


def _layer(rng, k, n, g, bias=False):
    qw = rng.integers(0, 2**32, (k, n // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    qz = rng.integers(0, 2**32, (k // g, n // 8), dtype=np.uint64).astype(np.uint32).view(np.int32)
    s = rng.uniform(0.001, 0.02, (k // g, n)).astype(np.float16)
    out = {"qweight": torch.from_numpy(qw), "qzeros": torch.from_numpy(qz),
           "scales": torch.from_numpy(s)}
    if bias:
        out["bias"] = torch.from_numpy(rng.uniform(-0.5, 0.5, n).astype(np.float16))
    return out


@pytest.fixture
def checkpoint(tmp_path):
    from safetensors.torch import save_file
    rng = np.random.default_rng(3)
    shards = [
        {"model.layers.0.self_attn.q_proj": _layer(rng, 256, 128, 64),
         "model.layers.0.mlp.down_proj": _layer(rng, 512, 256, 128, bias=True)},
        {"model.layers.1.self_attn.q_proj": _layer(rng, 256, 128, 64),
         "model.norm": None},
    ]
    paths = []
    for i, shard in enumerate(shards):
        flat = {}
        for prefix, tensors in shard.items():
            if tensors is None:
                flat[f"{prefix}.weight"] = torch.ones(256, dtype=torch.float16)
                continue
            for name, t in tensors.items():
                flat[f"{prefix}.{name}"] = t
        p = tmp_path / f"model-{i:05d}.safetensors"
        save_file(flat, str(p))
        paths.append(p)
    return tmp_path, shards


def test_loads_every_quantized_linear_of_all_shards(checkpoint):
    root, shards = checkpoint
    layers = load_awq_linears(str(root), device="cpu")
    assert sorted(layers) == ["model.layers.0.mlp.down_proj", "model.layers.0.self_attn.q_proj",
                              "model.layers.1.self_attn.q_proj"]
    down = layers["model.layers.0.mlp.down_proj"]
    src = shards[0]["model.layers.0.mlp.down_proj"]
    assert down.group_size() == 128
    assert torch.equal(down.qweight, src["qweight"]) and torch.equal(down.qzeros, src["qzeros"])
    assert torch.equal(down.scales, src["scales"]) and torch.equal(down.bias, src["bias"])
    assert layers["model.layers.0.self_attn.q_proj"].group_size() == 64
    assert layers["model.layers.0.self_attn.q_proj"].bias is None


def test_prefix_filter_and_dtype(checkpoint):
    root, _ = checkpoint
    layers = load_awq_linears(str(root), device="cpu", dtype=torch.bfloat16,
                              prefixes=["model.layers.1.self_attn.q_proj"])
    assert list(layers) == ["model.layers.1.self_attn.q_proj"]
    assert layers["model.layers.1.self_attn.q_proj"].scales.dtype == torch.bfloat16
    with pytest.raises(KeyError):
        load_awq_linears(str(root), device="cpu", prefixes=["model.layers.9.mlp.up_proj"])


def test_rejects_inconsistent_layers(tmp_path):
    from safetensors.torch import save_file
    rng = np.random.default_rng(4)
    t = _layer(rng, 256, 128, 64)
    t["scales"] = t["scales"][:, :64].contiguous()  # wrong N
    save_file({f"a.{k}": v for k, v in t.items()}, str(tmp_path / "x.safetensors"))
    with pytest.raises(ShapeError, match="scales must be"):
        load_awq_linears(str(tmp_path), device="cpu")
    save_file({"b.qweight": t["qweight"]}, str(tmp_path / "x.safetensors"))
    with pytest.raises(ShapeError, match="missing qzeros, scales"):
        load_awq_linears(str(tmp_path), device="cpu")


@pytest.mark.gpu
def test_loaded_layers_run_on_the_gpu(checkpoint, cuda_device):
    root, shards = checkpoint
    layers = load_awq_linears(str(root), device=cuda_device)
    down = layers["model.layers.0.mlp.down_proj"]
    src = shards[0]["model.layers.0.mlp.down_proj"]
    x = np.random.default_rng(5).standard_normal((3, 512)).astype(np.float16)
    y = down.forward(torch.from_numpy(x).to(cuda_device))
    ref = oracle.gemm_f64(x, src["qweight"].numpy().view(np.uint32),
                          src["qzeros"].numpy().view(np.uint32), src["scales"].numpy(), 128,
                          bias=src["bias"].numpy(), dtype="f16", deq_round=False)
    assert max_rel_err(y.float().cpu().numpy().astype(np.float64), ref) <= GEMM_TOL["f16"]


def test_plan_fusions_groups_decoder_siblings():
    from cube_awq_b200.loader import plan_fusions
    names = ["model.layers.0.mlp.gate_proj", "model.layers.0.mlp.up_proj",
             "model.layers.0.mlp.down_proj", "model.layers.0.self_attn.q_proj",
             "model.layers.0.self_attn.k_proj", "model.layers.0.self_attn.v_proj",
             "model.layers.0.self_attn.o_proj", "model.layers.1.mlp.gate_proj",  # no up: alone
             "model.layers.1.self_attn.q_proj", "model.layers.1.self_attn.k_proj"]  # no v
    got = plan_fusions(names)
    assert got == {
        "model.layers.0.mlp.gate_up_proj": ("gate_up", ("model.layers.0.mlp.gate_proj",
                                                        "model.layers.0.mlp.up_proj")),
        "model.layers.0.self_attn.qkv_proj": ("qkv", ("model.layers.0.self_attn.q_proj",
                                                      "model.layers.0.self_attn.k_proj",
                                                      "model.layers.0.self_attn.v_proj")),
    }


@pytest.mark.gpu
def test_fused_decoder_layers_match_the_separate_ones(tmp_path, cuda_device):
    from safetensors.torch import save_file
    from cube_awq_b200 import fuse_decoder_layers
    rng = np.random.default_rng(11)
    k = 256
    src = {"m.0.mlp.gate_proj": _layer(rng, k, 256, 64), "m.0.mlp.up_proj": _layer(rng, k, 256, 64),
           "m.0.attn.q_proj": _layer(rng, k, 256, 64, bias=True),
           "m.0.attn.k_proj": _layer(rng, k, 64, 64, bias=True),
           "m.0.attn.v_proj": _layer(rng, k, 64, 64, bias=True),
           # an intermediate size of 192 is not whole 128-column blocks: stays unfused
           "m.1.mlp.gate_proj": _layer(rng, k, 192, 64), "m.1.mlp.up_proj": _layer(rng, k, 192, 64)}
    save_file({f"{p}.{n}": t for p, ts in src.items() for n, t in ts.items()},
              str(tmp_path / "m.safetensors"))
    layers = load_awq_linears(str(tmp_path), device=cuda_device)
    fused = fuse_decoder_layers(layers)
    assert set(fused) == {"m.0.mlp.gate_up_proj", "m.0.attn.qkv_proj", "m.1.mlp.gate_proj",
                          "m.1.mlp.up_proj"}
    x = torch.from_numpy(rng.standard_normal((5, k)).astype(np.float16)).to(cuda_device)
    h = fused["m.0.mlp.gate_up_proj"](x)
    g, u = layers["m.0.mlp.gate_proj"](x).float(), layers["m.0.mlp.up_proj"](x).float()
    ref = torch.nn.functional.silu(g) * u
    bound = 2.1 * GEMM_TOL["f16"] * g.abs().max() * u.abs().max()
    assert (h.float() - ref).abs().max() <= bound + 2 ** -11 * ref.abs().max()
    q, kk, v = fused["m.0.attn.qkv_proj"](x)
    for got, name in ((q, "q_proj"), (kk, "k_proj"), (v, "v_proj")):
        want = layers[f"m.0.attn.{name}"](x).float()
        assert (got.float() - want).abs().max() <= 2 * GEMM_TOL["f16"] * want.abs().max()
