"""Attention of the end-to-end model over a paged BF16 KV cache.

Replaces ``nanovllm/layers/attention.py`` of the reference (flash-attn plus a
Triton store kernel) and the q/k norm + rotary steps of
``nanovllm/models/qwen3.py:87-92``:

* ``nv4_qk_norm_rope_store`` (one launch): per-head RMSNorm of q and k, rotary
  embedding, K/V written to the cache rows of the step's tokens;
* decode: ``nv4_paged_decode_attention`` (paged, grouped-query, split per KV
  page, then a merge kernel);
* prefill: ``torch.nn.functional.scaled_dot_product_attention`` per request on
  the step's own K/V (causal; prefix reuse is off, so a prompt never attends to
  tokens of an earlier step).

The step's metadata lives in a module-level ``StepContext`` that the model
runner sets before each forward (and that CUDA-graph capture binds to static
buffers).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from nanovllm import _native


@dataclass
class StepContext:
    is_prefill: bool = False
    slot_mapping: torch.Tensor | None = None   # int32 [T]
    seq_lens: list[int] | None = None          # prefill: tokens of each request, in order
    context_lens: torch.Tensor | None = None   # decode: int32 [B]
    block_tables: torch.Tensor | None = None   # decode: int32 [B, max_pages]
    workspace: torch.Tensor | None = None      # decode attention partials


_CTX = StepContext()


def set_context(ctx: StepContext) -> None:
    global _CTX
    _CTX = ctx


def get_context() -> StepContext:
    return _CTX


class PagedAttention(nn.Module):
    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, scale: float, eps: float):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.scale, self.eps = scale, eps
        self.k_cache = self.v_cache = None   # [pages, 256, Hkv, D], bound by the model runner

    def forward(self, qkv: torch.Tensor, positions: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                cos_sin: torch.Tensor) -> torch.Tensor:
        ctx = get_context()
        t = qkv.shape[0]
        q = torch.empty((t, self.num_heads, self.head_dim), dtype=qkv.dtype, device=qkv.device)
        k = torch.empty((t, self.num_kv_heads, self.head_dim), dtype=qkv.dtype, device=qkv.device) \
            if ctx.is_prefill else None
        store = self.k_cache is not None and ctx.slot_mapping is not None
        _native.qk_norm_rope_store(qkv, q_weight, k_weight, cos_sin, positions,
                                   ctx.slot_mapping if store else None, q, k,
                                   self.k_cache if store else None, self.v_cache if store else None,
                                   self.num_heads, self.num_kv_heads, self.eps)
        if ctx.is_prefill:
            q_end = self.num_heads * self.head_dim
            v = qkv[:, q_end + self.num_kv_heads * self.head_dim:].view(t, self.num_kv_heads, self.head_dim)
            out = torch.empty_like(q)
            start = 0
            for n in ctx.seq_lens:
                sl = slice(start, start + n)
                o = F.scaled_dot_product_attention(q[sl].transpose(0, 1).unsqueeze(0),
                                                   k[sl].transpose(0, 1).unsqueeze(0),
                                                   v[sl].transpose(0, 1).unsqueeze(0),
                                                   is_causal=True, scale=self.scale, enable_gqa=True)
                out[sl] = o[0].transpose(0, 1)
                start += n
            return out.view(t, -1)
        out = torch.empty_like(q)
        _native.paged_decode_attention(q, self.k_cache, self.v_cache, ctx.block_tables, ctx.context_lens, out,
                                       ctx.workspace, self.scale)
        return out.view(t, -1)
