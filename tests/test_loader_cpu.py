"""load_w4a4_model on a small synthetic checkpoint (CPU): the manifest contract,
per-layer shard hashes, q/k/v and gate/up concatenation along N, and the
tensor-parallel slicing of every projection kind."""
import hashlib
import json
import os
import sys

import pytest
import torch
from torch import nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-int4_b200"))

from safetensors.torch import save_file  # noqa: E402

from nanovllm.layers.linear_w4a4 import (W4A4MergedColumnParallelLinear, W4A4QKVParallelLinear,  # noqa: E402
                                         W4A4RowParallelLinear)
from nanovllm.utils import loader_w4a4  # noqa: E402

HIDDEN, HEAD, HEADS, KV_HEADS, INTER, LAYERS = 256, 64, 4, 2, 256, 2


def _sha(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


class _Layer(nn.Module):
    def __init__(self, rank, size):
        super().__init__()
        kw = dict(layout="block128", tp_rank=rank, tp_size=size)
        self.self_attn = nn.Module()
        self.self_attn.qkv_proj = W4A4QKVParallelLinear(HIDDEN, HEAD, HEADS, KV_HEADS, **kw)
        self.self_attn.o_proj = W4A4RowParallelLinear(HEADS * HEAD, HIDDEN, **kw)
        self.mlp = nn.Module()
        self.mlp.gate_up_proj = W4A4MergedColumnParallelLinear(HIDDEN, [INTER, INTER], **kw)
        self.mlp.down_proj = W4A4RowParallelLinear(INTER, HIDDEN, **kw)


class _Model(nn.Module):
    def __init__(self, rank=0, size=1):
        super().__init__()
        self.model = nn.Module()
        self.model.embed = nn.Parameter(torch.zeros(8, HIDDEN, dtype=torch.bfloat16))
        self.model.layers = nn.ModuleList(_Layer(rank, size) for _ in range(LAYERS))


def _sources():
    q, kv = HEADS * HEAD, KV_HEADS * HEAD
    return {"self_attn": {"q_proj": (q, HIDDEN), "k_proj": (kv, HIDDEN), "v_proj": (kv, HIDDEN),
                          "o_proj": (HIDDEN, HEADS * HEAD)},
            "mlp": {"gate_proj": (INTER, HIDDEN), "up_proj": (INTER, HIDDEN), "down_proj": (HIDDEN, INTER)}}


@pytest.fixture()
def checkpoint(tmp_path):
    base, ckpt = tmp_path / "base", tmp_path / "ckpt"
    base.mkdir()
    ckpt.mkdir()
    (base / "config.json").write_text(json.dumps({"hidden_size": HIDDEN}))
    save_file({"model.embed": torch.randn(8, HIDDEN).bfloat16()}, str(base / "model.safetensors"))
    g = torch.Generator().manual_seed(0)
    tensors, layers = {}, {}
    for i in range(LAYERS):
        t = {}
        for parent, projs in _sources().items():
            for name, (n, k) in projs.items():
                t[f"{parent}.{name}.packed"] = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
                t[f"{parent}.{name}.scale"] = (torch.rand(n, k // 128, generator=g) * 0.01 + 1e-3).bfloat16()
        for sign_name, k in (("qkv", HIDDEN), ("o", HEADS * HEAD), ("gate_up", HIDDEN), ("down", INTER)):
            t[f"signs.{sign_name}"] = torch.randint(0, 2, (k,), generator=g, dtype=torch.int8) * 2 - 1
        path = ckpt / f"layer_{i}.safetensors"
        save_file(t, str(path))
        layers[str(i)] = {"file": path.name, "sha256": _sha(path)}
        tensors[i] = t
    manifest = {"format": loader_w4a4.FORMAT, "complete": True, "layers": layers,
                "config": {"group_size": 128, "static_groups": True, "runtime_column_permutation": False,
                           "evaluation_activation_group_size": 128, "evaluation_activation_clipping": 0.9,
                           "layout_version": loader_w4a4.LAYOUT, "model_config_sha256": _sha(base / "config.json")}}
    (ckpt / "manifest.json").write_text(json.dumps(manifest))
    return base, ckpt, tensors


def _full(t, parent, names):
    return (torch.cat([t[f"{parent}.{n}.packed"] for n in names]), torch.cat([t[f"{parent}.{n}.scale"] for n in names]))


def test_load_unsharded(checkpoint):
    base, ckpt, tensors = checkpoint
    model = _Model()
    info = loader_w4a4.load_w4a4_model(model, str(base), str(ckpt))
    assert info["projections"] == 7 * LAYERS and info["native_linear_modules"] == 4 * LAYERS
    for i, layer in enumerate(model.model.layers):
        t = tensors[i]
        packed, scale = _full(t, "self_attn", ("q_proj", "k_proj", "v_proj"))
        assert torch.equal(layer.self_attn.qkv_proj.packed_weight, packed)
        assert torch.equal(layer.self_attn.qkv_proj.weight_scale, scale)
        assert torch.equal(layer.self_attn.qkv_proj.signs, t["signs.qkv"])
        packed, scale = _full(t, "mlp", ("gate_proj", "up_proj"))
        assert torch.equal(layer.mlp.gate_up_proj.packed_weight, packed)
        assert torch.equal(layer.mlp.down_proj.packed_weight, t["mlp.down_proj.packed"])
        assert torch.equal(layer.self_attn.o_proj.weight_scale, t["self_attn.o_proj.scale"])


def test_load_tensor_parallel_slices(checkpoint):
    base, ckpt, tensors = checkpoint
    for rank in range(2):
        model = _Model(rank, 2)
        loader_w4a4.load_w4a4_model(model, str(base), str(ckpt))
        layer, t = model.model.layers[1], tensors[1]
        # qkv: this rank's heads of q, then of k, then of v
        parts = [t[f"self_attn.{n}.packed"].chunk(2, 0)[rank] for n in ("q_proj", "k_proj", "v_proj")]
        assert torch.equal(layer.self_attn.qkv_proj.packed_weight, torch.cat(parts))
        # gate/up: this rank's half of gate, then of up
        parts = [t[f"mlp.{n}.scale"].chunk(2, 0)[rank] for n in ("gate_proj", "up_proj")]
        assert torch.equal(layer.mlp.gate_up_proj.weight_scale, torch.cat(parts))
        # row parallel: this rank's 128-group columns, and its slice of the signs
        k = INTER // 2
        assert torch.equal(layer.mlp.down_proj.packed_weight, t["mlp.down_proj.packed"][:, rank * k // 2:(rank + 1) * k // 2])
        assert torch.equal(layer.mlp.down_proj.weight_scale, t["mlp.down_proj.scale"][:, rank * k // 128:(rank + 1) * k // 128])
        assert torch.equal(layer.mlp.down_proj.signs, t["signs.down"][rank * k:(rank + 1) * k])


@pytest.mark.parametrize("key,value", [("complete", False), ("format", "other")])
def test_manifest_contract_rejected(checkpoint, key, value):
    base, ckpt, _ = checkpoint
    manifest = json.loads((ckpt / "manifest.json").read_text())
    manifest[key] = value
    (ckpt / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="Incomplete or unsupported"):
        loader_w4a4.load_w4a4_model(_Model(), str(base), str(ckpt))


def test_quantization_contract_rejected(checkpoint):
    base, ckpt, _ = checkpoint
    manifest = json.loads((ckpt / "manifest.json").read_text())
    manifest["config"]["evaluation_activation_clipping"] = 1.0
    (ckpt / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="contract"):
        loader_w4a4.load_w4a4_model(_Model(), str(base), str(ckpt))


def test_tampered_shard_rejected(checkpoint):
    base, ckpt, _ = checkpoint
    with open(ckpt / "layer_1.safetensors", "r+b") as f:
        f.seek(-1, 2)
        last = f.read(1)
        f.seek(-1, 2)
        f.write(bytes([last[0] ^ 1]))
    with pytest.raises(ValueError, match="Invalid checkpoint shard"):
        loader_w4a4.load_w4a4_model(_Model(), str(base), str(ckpt))


def test_base_config_mismatch_rejected(checkpoint):
    base, ckpt, _ = checkpoint
    (base / "config.json").write_text(json.dumps({"hidden_size": HIDDEN + 1}))
    with pytest.raises(ValueError, match="Base model config"):
        loader_w4a4.load_w4a4_model(_Model(), str(base), str(ckpt))


@pytest.mark.parametrize("what", ["scale", "signs"])
def test_invalid_values_rejected(checkpoint, what):
    base, ckpt, tensors = checkpoint
    t = dict(tensors[0])
    if what == "scale":
        t["mlp.up_proj.scale"] = t["mlp.up_proj.scale"].clone()
        t["mlp.up_proj.scale"][3, 0] = 0
    else:
        t["signs.o"] = t["signs.o"].clone()
        t["signs.o"][5] = 2
    path = ckpt / "layer_0.safetensors"
    save_file(t, str(path))
    manifest = json.loads((ckpt / "manifest.json").read_text())
    manifest["layers"]["0"]["sha256"] = _sha(path)
    (ckpt / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="Invalid weight/scale" if what == "scale" else "Invalid RHT signs"):
        loader_w4a4.load_w4a4_model(_Model(), str(base), str(ckpt))
