"""Seeded random weights for ``load_format="dummy"`` (no checkpoint offline).

Every rank draws the same full tensors on its device (one generator seeded per
tensor) and keeps its tensor-parallel shard, so a model has the same weights at
every TP size.  Distributions: BF16 matrices N(0, 0.02); RMSNorm weights 1;
W4A4 projections as the benchmark's config 0 (INT4 codes uniform in [-8, 7],
per-(n, 128-group) BF16 scales |N(0, 0.02)| / 7, RHT signs +-1); W4A16 as
config 3 (uniform uint4 codes and zero points, FP16 scales |N(0, 0.02)|).
"""
from __future__ import annotations

import zlib

import torch

from nanovllm.layers.common import DenseColumnParallel, DenseRowParallel, RMSNorm, VocabParallelEmbedding
from nanovllm.layers.linear_w4a16 import W4A16Linear
from nanovllm.layers.linear_w4a4 import W4A4Linear


def _gen(device, seed: int, name: str) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed * 1000003 + zlib.crc32(name.encode()))


@torch.no_grad()
def init_random_weights(model: torch.nn.Module, seed: int = 0) -> None:
    for name, mod in model.named_modules():
        if isinstance(mod, W4A4Linear):
            dev = mod.packed_weight.device
            g = _gen(dev, seed, name)
            n = getattr(mod, "full_output_size", mod.out_features)
            k = getattr(mod, "full_input_size", mod.in_features)
            packed = torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=dev, generator=g)
            scale = (torch.randn(n, k // 128, device=dev, generator=g).abs() * (0.02 / 7)).bfloat16()
            signs = torch.randint(0, 2, (k,), dtype=torch.int8, device=dev, generator=g) * 2 - 1
            mod.load_full(packed, scale, signs)
        elif isinstance(mod, W4A16Linear):
            dev = mod.qweight.device
            g = _gen(dev, seed, name)
            for p in (mod.qweight, mod.qzeros):
                p.copy_(torch.randint(-2 ** 31, 2 ** 31 - 1, p.shape, dtype=torch.int64, device=dev,
                                      generator=g).to(torch.int32))
            mod.scales.copy_((torch.randn(mod.scales.shape, device=dev, generator=g).abs() * 0.02).half())
        elif isinstance(mod, DenseColumnParallel):
            dev = mod.weight.device
            g = _gen(dev, seed, name)
            parts = []
            for n in mod.output_sizes:
                full = torch.randn(n, mod.weight.shape[1], device=dev, generator=g) * 0.02
                size = n // mod.tp_size
                parts.append(full.narrow(0, mod.tp_rank * size, size))
            mod.weight.copy_(torch.cat(parts).to(mod.weight.dtype))
        elif isinstance(mod, DenseRowParallel):
            dev = mod.weight.device
            g = _gen(dev, seed, name)
            k = mod.weight.shape[1] * mod.tp_size
            full = torch.randn(mod.weight.shape[0], k, device=dev, generator=g) * 0.02
            mod.weight.copy_(full.narrow(1, mod.tp_rank * mod.weight.shape[1], mod.weight.shape[1]).to(mod.weight.dtype))
        elif isinstance(mod, VocabParallelEmbedding):
            dev = mod.weight.device
            g = _gen(dev, seed, name)
            rows = mod.per_rank * mod.tp_size
            for r0 in range(0, rows, 16384):  # full table in row blocks (bounded temporary)
                n = min(16384, rows - r0)
                blk = torch.randn(n, mod.weight.shape[1], device=dev, generator=g) * 0.02
                lo, hi = max(r0, mod.start), min(r0 + n, mod.start + mod.per_rank)
                if lo < hi:
                    mod.weight[lo - mod.start:hi - mod.start].copy_(blk[lo - r0:hi - r0].to(mod.weight.dtype))
        elif isinstance(mod, RMSNorm):
            mod.weight.fill_(1.0)
