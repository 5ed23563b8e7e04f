"""Small layers of the end-to-end model: RMSNorm, the rotary cos/sin table,
SiluAndMul, vocab-parallel embedding and LM head, BF16 tensor-parallel
linears, and the sampler.

Numerics follow the reference's compiled torch code:
* RMSNorm (``nanovllm/layers/layernorm.py:17-40``): FP32 math, the normalised
  value rounded to BF16, then a BF16 product with the weight; with a residual
  the sum x + residual is taken in FP32 and the new residual is its BF16;
* rotary table (``rotary_embedding.py:27-35``): inv_freq = 1 / base^(2i/D) and
  t * inv_freq in FP32, cos | sin concatenated;
* SiluAndMul (``activation.py:8-11``): silu(gate) * up in FP32, one rounding;
* sampler (``sampler.py:7-12``): softmax(logits / T) divided by Exp(1) noise,
  argmax; temperature 0 is plain argmax (greedy).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        xf = x.float()
        if residual is not None:
            xf = xf + residual.float()
            residual = xf.to(x.dtype)
        y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight
        return y if residual is None else (y, residual)


def rotary_cos_sin(head_dim: int, max_position: int, base: float) -> torch.Tensor:
    """float32 [max_position, head_dim]: cos of the D/2 frequencies, then sin."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).contiguous()


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    g, u = x.float().chunk(2, -1)
    return (F.silu(g) * u).to(x.dtype)


def _tp(tp_rank=None, tp_size=None):
    """(rank, size) of the tensor-parallel group: the given values, else the
    default process group's, else a single rank."""
    if tp_size is None:
        tp_size = dist.get_world_size() if dist.is_initialized() else 1
    if tp_rank is None:
        tp_rank = dist.get_rank() if dist.is_initialized() else 0
    return tp_rank, tp_size


class VocabParallelEmbedding(nn.Module):
    """Embedding rows sharded over the TP ranks (nanovllm/layers/embed_head.py:9-42)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, tp_rank=None, tp_size=None):
        super().__init__()
        self.tp_rank, self.tp_size = _tp(tp_rank, tp_size)
        if num_embeddings % self.tp_size:
            raise ValueError("vocabulary not divisible by the TP size")
        self.per_rank = num_embeddings // self.tp_size
        self.start = self.per_rank * self.tp_rank
        self.weight = nn.Parameter(torch.empty(self.per_rank, embedding_dim))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        if self.tp_size == 1:
            return F.embedding(ids, self.weight)
        local = ids - self.start
        mask = (local >= 0) & (local < self.per_rank)
        y = F.embedding(local.clamp(0, self.per_rank - 1), self.weight) * mask.unsqueeze(-1).to(self.weight.dtype)
        dist.all_reduce(y)
        return y


class ParallelLMHead(VocabParallelEmbedding):
    """Logits of this rank's vocabulary shard, gathered on every rank (every
    rank then samples the same token; the reference gathers to rank 0 only)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        logits = F.linear(x, self.weight)
        if self.tp_size == 1:
            return logits
        parts = [torch.empty_like(logits) for _ in range(self.tp_size)]
        dist.all_gather(parts, logits)
        return torch.cat(parts, -1)


class DenseColumnParallel(nn.Module):
    """BF16 linear sharded along N (nanovllm/layers/linear.py:54-128); the
    output blocks (q | k | v or gate | up) are sharded separately."""

    def __init__(self, input_size: int, output_sizes: list[int], tp_rank=None, tp_size=None):
        super().__init__()
        self.tp_rank, self.tp_size = _tp(tp_rank, tp_size)
        for n in output_sizes:
            if n % self.tp_size:
                raise ValueError("output block not divisible by the TP size")
        self.output_sizes = list(output_sizes)
        self.weight = nn.Parameter(torch.empty(sum(output_sizes) // self.tp_size, input_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight)


class DenseRowParallel(nn.Module):
    """BF16 linear sharded along K with an all-reduce of the partial outputs
    (nanovllm/layers/linear.py:131-155)."""

    def __init__(self, input_size: int, output_size: int, tp_rank=None, tp_size=None):
        super().__init__()
        self.tp_rank, self.tp_size = _tp(tp_rank, tp_size)
        if input_size % self.tp_size:
            raise ValueError("input not divisible by the TP size")
        self.weight = nn.Parameter(torch.empty(output_size, input_size // self.tp_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x, self.weight)
        if self.tp_size > 1:
            dist.all_reduce(y)
        return y


class Sampler(nn.Module):
    def forward(self, logits: torch.Tensor, temperatures: torch.Tensor, generator=None) -> torch.Tensor:
        logits = logits.float()
        greedy = logits.argmax(-1)
        if bool((temperatures == 0).all()):
            return greedy
        t = torch.where(temperatures > 0, temperatures, torch.ones_like(temperatures))
        probs = torch.softmax(logits / t.unsqueeze(-1), dim=-1)
        noise = torch.empty_like(probs).exponential_(1, generator=generator).clamp_min_(1e-10)
        sampled = (probs / noise).argmax(-1)
        return torch.where(temperatures > 0, sampled, greedy)
