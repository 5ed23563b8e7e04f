"""Checkpoint loading for the W4A4 model, planned per tensor-parallel rank.

Drop-in entry point: ``load_w4a4_model(model, model_path, checkpoint_path)``
(the reference's ``nanovllm/utils/loader_w4a4.py:31-96``).  What is kept from
the reference is the *format contract* -- the manifest fields and values a
checkpoint must declare (format ``rht_gptq_static_group128_bf16_scale_i4_v1``,
complete, group size 128, static groups, no runtime column permutation,
activation groups of 128 with clip 0.9, layout
``row_DH_paley12_kron_sylvester_v1``, the base ``config.json`` SHA-256, one
shard file per decoder layer with its SHA-256) and the tensor names inside a
shard (``signs.{qkv,o,gate_up,down}`` int8 [K]; ``{self_attn|mlp}.<proj>.packed``
int8 [N, K/2] and ``.scale`` bf16 [N, K/128]), together with the exception
types and messages callers match on.

How it loads is this file's own design:

1. ``ShardPlan.for_module`` turns each W4A4 projection module into a plan:
   which rows (column-parallel: this rank's slice of *each* source matrix,
   e.g. its q, k and v heads) or which K columns (row-parallel: its
   128-group-aligned K shard, and the matching slice of the signs) it keeps.
   The plan is derived from the module's partition attributes alone.
2. ``LayerShard`` opens one layer's file after checking its SHA-256 and reads
   only the planned slices (``safe_open(...).get_slice``), validating dtype
   and shape from the header before any payload is read, and the values
   (signs in {-1, +1}, finite positive scales) on what this rank keeps.
3. The planned pieces are concatenated in source order and copied into the
   module's buffers once.

So a rank of a TP group reads about 1/tp of every projection payload instead
of the whole checkpoint.  BF16 base parameters (embeddings, norms, LM head)
come from the base model directory and are handed to each parameter's
``weight_loader`` when it has one.
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path

import torch

FORMAT = "rht_gptq_static_group128_bf16_scale_i4_v1"
LAYOUT = "row_DH_paley12_kron_sylvester_v1"
GROUP = 128

# Manifest fields of the format contract and the values a checkpoint must declare.
CONTRACT = {
    "group_size": GROUP,
    "static_groups": True,
    "runtime_column_permutation": False,
    "evaluation_activation_group_size": GROUP,
    "evaluation_activation_clipping": 0.9,
    "layout_version": LAYOUT,
}

# Fused projection -> (module parent, module attribute, checkpoint sources in N order, sign key).
PROJECTIONS = {
    "qkv": ("self_attn", "qkv_proj", ("q_proj", "k_proj", "v_proj")),
    "o": ("self_attn", "o_proj", ("o_proj",)),
    "gate_up": ("mlp", "gate_up_proj", ("gate_proj", "up_proj")),
    "down": ("mlp", "down_proj", ("down_proj",)),
}


def file_sha256(path: Path) -> str:
    with open(path, "rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def validate_manifest(manifest: dict) -> dict:
    """The checkpoint's declared contract; raises ValueError when it is not the
    one the kernels implement."""
    if manifest.get("format") != FORMAT or manifest.get("complete") is not True:
        raise ValueError("Incomplete or unsupported W4A4 checkpoint")
    declared = manifest.get("config") or {}
    for field, required in CONTRACT.items():
        value = declared.get(field)
        same = value is required if isinstance(required, bool) else value == required
        if not same:
            raise ValueError(f"Checkpoint quantization contract differs from the native kernel ({field})")
    return declared


def checkpoint_activation_contract(checkpoint_path) -> tuple[str, int]:
    """(activation layout, lowest code) the checkpoint's modules must be built
    with: the format fixes the full-width row_DH transform and codes in [-7, 7]
    (nanovllm/layers/linear_w4a4.py:23-36 of the reference)."""
    manifest = json.loads((Path(checkpoint_path) / "manifest.json").read_text())
    validate_manifest(manifest)
    return LAYOUT, -7


@dataclass(frozen=True)
class ShardPlan:
    """What one rank keeps of a fused projection: per source matrix a row range
    (column-parallel) or one K-column range shared by all sources
    (row-parallel), and the slice of the sign vector."""
    rows: tuple          # per source: (start, stop) of the rows kept, or None for all
    k_cols: tuple | None  # (start, stop) of the K columns kept, or None for all
    full_k: int
    local_n: int

    @staticmethod
    def for_module(module, source_rows: list[int]) -> "ShardPlan":
        tp_size = getattr(module, "tp_size", 1)
        tp_rank = getattr(module, "tp_rank", 0)
        full_k = getattr(module, "full_input_size", module.in_features)
        if tp_size == 1:
            return ShardPlan(tuple(None for _ in source_rows), None, full_k, sum(source_rows))
        if hasattr(module, "full_input_size"):  # K shard on 128-group boundaries
            k = module.in_features
            return ShardPlan(tuple(None for _ in source_rows), (tp_rank * k, (tp_rank + 1) * k), full_k,
                             sum(source_rows))
        rows = []
        for n in source_rows:  # every source matrix is split evenly across the ranks
            if n % tp_size:
                raise ValueError(f"{n} rows do not split over {tp_size} ranks")
            share = n // tp_size
            rows.append((tp_rank * share, (tp_rank + 1) * share))
        return ShardPlan(tuple(rows), None, full_k, sum(b - a for a, b in rows))

    def sign_range(self, module):
        if self.k_cols is None or getattr(module, "gather_input", False):
            return 0, self.full_k
        return self.k_cols


class LayerShard:
    """One decoder layer's checkpoint file, hash-checked, read slice by slice."""

    def __init__(self, root: Path, entry: dict, index: int):
        from safetensors import safe_open
        path = (root / entry["file"]).resolve()
        if not path.is_relative_to(root) or not path.is_file() or file_sha256(path) != entry["sha256"]:
            raise ValueError(f"Invalid checkpoint shard: layer {index}")
        self.index = index
        self._handle = safe_open(str(path), framework="pt", device="cpu")

    def rows_of(self, name: str) -> int:
        return self._handle.get_slice(name).get_shape()[0]

    def read(self, name: str, rows, cols, dtype, width: int) -> torch.Tensor:
        view = self._handle.get_slice(name)
        shape = view.get_shape()
        if view.get_dtype() != {torch.int8: "I8", torch.bfloat16: "BF16"}[dtype] or len(shape) != 2 \
                or shape[1] != width:
            raise ValueError(f"Invalid weight/scale at layer {self.index}/{name}")
        r0, r1 = rows if rows is not None else (0, shape[0])
        c0, c1 = cols if cols is not None else (0, shape[1])
        return view[r0:r1, c0:c1]

    def signs(self, key: str, full_k: int, start: int, stop: int) -> torch.Tensor:
        view = self._handle.get_slice(f"signs.{key}")
        if view.get_dtype() != "I8" or view.get_shape() != [full_k]:
            raise ValueError(f"Invalid RHT signs at layer {self.index}/{key}")
        s = view[start:stop]
        if not bool(((s == 1) | (s == -1)).all()):
            raise ValueError(f"Invalid RHT signs at layer {self.index}/{key}")
        return s


def _load_projection(shard: LayerShard, module, key: str, parent: str, sources) -> int:
    names = [f"{parent}.{src}" for src in sources]
    plan = ShardPlan.for_module(module, [shard.rows_of(f"{n}.packed") for n in names])
    full_n = getattr(module, "full_output_size", module.out_features)
    if sum(shard.rows_of(f"{n}.packed") for n in names) != full_n:
        raise ValueError(f"Invalid weight/scale at layer {shard.index}/{key}")
    cols_p = None if plan.k_cols is None else (plan.k_cols[0] // 2, plan.k_cols[1] // 2)
    cols_s = None if plan.k_cols is None else (plan.k_cols[0] // GROUP, plan.k_cols[1] // GROUP)
    packed, scale = [], []
    for name, rows in zip(names, plan.rows):
        p = shard.read(f"{name}.packed", rows, cols_p, torch.int8, plan.full_k // 2)
        s = shard.read(f"{name}.scale", rows, cols_s, torch.bfloat16, plan.full_k // GROUP)
        if p.shape[0] != s.shape[0] or not bool(torch.isfinite(s).all()) or not bool((s > 0).all()):
            raise ValueError(f"Invalid weight/scale at layer {shard.index}/{name}")
        packed.append(p)
        scale.append(s)
    lo, hi = plan.sign_range(module)
    signs = shard.signs(key, plan.full_k, lo, hi)
    packed, scale = torch.cat(packed), torch.cat(scale)
    if packed.shape != module.packed_weight.shape or scale.shape != module.weight_scale.shape \
            or signs.shape != module.signs.shape:
        raise ValueError(f"Invalid weight/scale at layer {shard.index}/{key}")
    with torch.no_grad():
        module.packed_weight.copy_(packed)
        module.weight_scale.copy_(scale)
        module.signs.copy_(signs)
    return len(sources)


def _load_base_parameters(model, base: Path) -> None:
    from safetensors import safe_open
    wanted = dict(model.named_parameters())
    for path in sorted(base.glob("*.safetensors")):
        with safe_open(str(path), framework="pt", device="cpu") as handle:
            for name in set(handle.keys()) & wanted.keys():
                param = wanted.pop(name)
                value = handle.get_tensor(name)
                if value.dtype != torch.bfloat16 or param.dtype != torch.bfloat16:
                    raise ValueError(f"Expected BF16 base parameter: {name}")
                loader = getattr(param, "weight_loader", None)
                with torch.no_grad():
                    loader(param, value) if loader is not None else param.data.copy_(value)
    if wanted:
        raise ValueError(f"Missing base parameters: {sorted(wanted)}")


def _base_dir(model_path) -> Path:
    base = Path(model_path)
    if base.is_dir():
        return base
    from huggingface_hub import snapshot_download
    return Path(snapshot_download(repo_id=str(model_path), local_files_only=True))


@torch.no_grad()
def load_w4a4_model(model, model_path, checkpoint_path):
    """Load the base BF16 parameters and every W4A4 projection (this rank's
    slices) of ``model`` from the checkpoint; returns a summary dict."""
    from nanovllm.layers.linear_w4a4 import W4A4Linear
    base = _base_dir(model_path)
    root = Path(checkpoint_path).resolve()
    manifest = json.loads((root / "manifest.json").read_text())
    declared = validate_manifest(manifest)
    if file_sha256(base / "config.json") != declared.get("model_config_sha256"):
        raise ValueError("Base model config does not match the calibrated checkpoint")
    layers = model.model.layers
    if set(manifest.get("layers", {})) != {str(i) for i in range(len(layers))}:
        raise ValueError("Checkpoint layer set does not match the model")

    _load_base_parameters(model, base)
    projections = 0
    for index, layer in enumerate(layers):
        shard = LayerShard(root, manifest["layers"][str(index)], index)
        for key, (parent, attr, sources) in PROJECTIONS.items():
            module = getattr(getattr(layer, parent), attr)
            if not isinstance(module, W4A4Linear):
                raise TypeError(f"Expected W4A4Linear at layer {index}/{attr}")
            projections += _load_projection(shard, module, key, parent, sources)
    return {"format": FORMAT, "projections": projections, "native_linear_modules": len(layers) * len(PROJECTIONS),
            "checkpoint_manifest_sha256": file_sha256(root / "manifest.json"),
            "weight_group_size": GROUP, "activation_group_size": CONTRACT["evaluation_activation_group_size"],
            "activation_clipping": CONTRACT["evaluation_activation_clipping"], "scale_dtype": "bfloat16",
            "split_k": False}
