"""BF16 / GPTQ checkpoint loading for the engine's Qwen3 model (the role of
the reference's ``nanovllm/utils/loader.py``): every safetensors tensor of
the model directory is copied into the parameter of the same name; q/k/v and
gate/up tensors go into their fused projection (``packed_modules_mapping``),
and each tensor-parallel layer keeps its shard (column-parallel blocks by
rows, row-parallel by input columns, vocabulary tables by rows)."""
from __future__ import annotations

from pathlib import Path

import torch

from nanovllm.layers.common import DenseColumnParallel, DenseRowParallel, VocabParallelEmbedding


def _copy_shard(module, param_name: str, param, value: torch.Tensor, shard=None) -> None:
    if isinstance(module, DenseColumnParallel):
        sizes = module.output_sizes
        index = {"q": 0, "k": 1, "v": 2}.get(shard, shard)
        local = [n // module.tp_size for n in sizes]
        offset = sum(local[:index])
        piece = value.chunk(module.tp_size, 0)[module.tp_rank]
        param.data.narrow(0, offset, local[index]).copy_(piece)
    elif isinstance(module, DenseRowParallel):
        param.data.copy_(value.chunk(module.tp_size, 1)[module.tp_rank])
    elif isinstance(module, VocabParallelEmbedding):
        param.data.copy_(value.narrow(0, module.start, module.per_rank))
    else:
        param.data.copy_(value)


@torch.no_grad()
def load_model(model: torch.nn.Module, path: str) -> None:
    from safetensors import safe_open
    mapping = getattr(model, "packed_modules_mapping", {})
    modules = dict(model.named_modules())
    params = dict(model.named_parameters())
    files = sorted(Path(path).glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors files in {path}")
    for file in files:
        with safe_open(str(file), framework="pt", device="cpu") as f:
            for name in f.keys():
                if name.endswith(".g_idx"):
                    continue
                target, shard = name, None
                if name not in params:
                    for src, (dst, sid) in mapping.items():
                        if src in name and name.replace(src, dst) in params:
                            target, shard = name.replace(src, dst), sid
                            break
                if target not in params:
                    raise KeyError(f"checkpoint tensor {name} has no parameter in the model")
                module = modules[target.rsplit(".", 1)[0]]
                _copy_shard(module, target, params[target], f.get_tensor(name), shard)
