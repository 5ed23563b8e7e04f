"""Qwen3 causal LM for the engine (the reference's ``nanovllm/models/qwen3.py``
and ``qwen3_w4a16.py``), in three linear flavours:

* ``"w4a4"``: the projections are the W4A4 tensor-parallel linears
  (``W4A4QKVParallelLinear`` / ``W4A4MergedColumnParallelLinear`` /
  ``W4A4RowParallelLinear``) with their producers fused into the activation
  prep: the residual add + input / post-attention RMSNorm into the QKV and
  gate/up preps, SiluAndMul into the down prep;
* ``"bf16"``: BF16 tensor-parallel linears on cuBLAS (the same-box
  comparator of the benchmark);
* ``"w4a16"``: GPTQ ``W4A16Linear`` for q, k, v, o, gate, up and down
  (one GPU, as the reference's ``qwen3_w4a16.py``).

Parameter and buffer names match the reference's, so the checkpoint loaders
find them: ``model.layers.N.self_attn.qkv_proj.packed_weight`` and so on.
"""
from __future__ import annotations

import torch
from torch import nn

from nanovllm.layers.attention import PagedAttention
from nanovllm.layers.common import (DenseColumnParallel, DenseRowParallel, ParallelLMHead, RMSNorm,
                                    VocabParallelEmbedding, rotary_cos_sin, silu_and_mul)
from nanovllm.layers.linear_w4a16 import W4A16Linear
from nanovllm.layers.linear_w4a4 import (W4A4MergedColumnParallelLinear, W4A4QKVParallelLinear,
                                         W4A4RowParallelLinear)

MODES = ("bf16", "w4a4", "w4a16")


class Qwen3Attention(nn.Module):
    def __init__(self, cfg, mode: str, tp_rank: int, tp_size: int, w4a4_kw: dict):
        super().__init__()
        self.mode = mode
        heads, kv_heads = cfg.num_attention_heads, cfg.num_key_value_heads
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // heads
        if heads % tp_size or kv_heads % tp_size:
            raise ValueError("attention heads not divisible by the TP size")
        self.num_heads, self.num_kv_heads, self.head_dim = heads // tp_size, kv_heads // tp_size, head_dim
        hidden = cfg.hidden_size
        if mode == "w4a4":
            self.qkv_proj = W4A4QKVParallelLinear(hidden, head_dim, heads, kv_heads, tp_rank=tp_rank, tp_size=tp_size,
                                                  **w4a4_kw)
            self.o_proj = W4A4RowParallelLinear(heads * head_dim, hidden, tp_rank=tp_rank, tp_size=tp_size,
                                                **w4a4_kw)
        elif mode == "w4a16":
            self.q_proj = W4A16Linear(hidden, heads * head_dim)
            self.k_proj = W4A16Linear(hidden, kv_heads * head_dim)
            self.v_proj = W4A16Linear(hidden, kv_heads * head_dim)
            self.o_proj = W4A16Linear(heads * head_dim, hidden)
        else:
            self.qkv_proj = DenseColumnParallel(hidden, [heads * head_dim, kv_heads * head_dim, kv_heads * head_dim],
                                                tp_rank, tp_size)
            self.o_proj = DenseRowParallel(heads * head_dim, hidden, tp_rank, tp_size)
        eps = cfg.rms_norm_eps
        self.q_norm = RMSNorm(head_dim, eps)
        self.k_norm = RMSNorm(head_dim, eps)
        self.attn = PagedAttention(self.num_heads, self.num_kv_heads, head_dim, head_dim ** -0.5, eps)

    def qkv(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "w4a16":
            return torch.cat((self.q_proj(x), self.k_proj(x), self.v_proj(x)), -1)
        return self.qkv_proj(x)

    def attend(self, qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
        o = self.attn(qkv, positions, self.q_norm.weight, self.k_norm.weight, cos_sin)
        return self.o_proj(o)


class Qwen3MLP(nn.Module):
    def __init__(self, cfg, mode: str, tp_rank: int, tp_size: int, w4a4_kw: dict):
        super().__init__()
        self.mode = mode
        hidden, inter = cfg.hidden_size, cfg.intermediate_size
        if cfg.hidden_act != "silu":
            raise ValueError("Qwen3 MLP uses silu")
        if mode == "w4a4":
            self.gate_up_proj = W4A4MergedColumnParallelLinear(hidden, [inter, inter], tp_rank=tp_rank,
                                                               tp_size=tp_size, **w4a4_kw)
            self.down_proj = W4A4RowParallelLinear(inter, hidden, tp_rank=tp_rank, tp_size=tp_size, **w4a4_kw)
        elif mode == "w4a16":
            self.gate_proj = W4A16Linear(hidden, inter)
            self.up_proj = W4A16Linear(hidden, inter)
            self.down_proj = W4A16Linear(inter, hidden)
        else:
            self.gate_up_proj = DenseColumnParallel(hidden, [inter, inter], tp_rank, tp_size)
            self.down_proj = DenseRowParallel(inter, hidden, tp_rank, tp_size)

    def gate_up(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "w4a16":
            return torch.cat((self.gate_proj(x), self.up_proj(x)), -1)
        return self.gate_up_proj(x)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, cfg, mode: str, tp_rank: int, tp_size: int, w4a4_kw: dict):
        super().__init__()
        self.mode = mode
        self.self_attn = Qwen3Attention(cfg, mode, tp_rank, tp_size, w4a4_kw)
        self.mlp = Qwen3MLP(cfg, mode, tp_rank, tp_size, w4a4_kw)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)

    def forward(self, positions, h, residual, cos_sin):
        attn, mlp = self.self_attn, self.mlp
        if self.mode == "w4a4":
            # residual add + RMSNorm fused into the QKV prep (residual None: rms of h, residual = h)
            qkv, residual = attn.qkv_proj.forward_add_rmsnorm(h, residual, self.input_layernorm.weight,
                                                             self.input_layernorm.eps)
            h = attn.attend(qkv, positions, cos_sin)
            gu, residual = mlp.gate_up_proj.forward_add_rmsnorm(h, residual, self.post_attention_layernorm.weight,
                                                                self.post_attention_layernorm.eps)
            return mlp.down_proj.forward_silu_mul(gu), residual
        if residual is None:
            x, residual = self.input_layernorm(h), h
        else:
            x, residual = self.input_layernorm(h, residual)
        h = attn.attend(attn.qkv(x), positions, cos_sin)
        x, residual = self.post_attention_layernorm(h, residual)
        return mlp.down_proj(silu_and_mul(mlp.gate_up(x))), residual


class Qwen3Model(nn.Module):
    def __init__(self, cfg, mode: str, tp_rank: int, tp_size: int, w4a4_kw: dict, max_position: int):
        super().__init__()
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, tp_rank, tp_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(cfg, mode, tp_rank, tp_size, w4a4_kw)
                                     for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        theta = getattr(cfg, "rope_theta", None)
        if theta is None:
            theta = (getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 1000000.0)
        self.register_buffer("cos_sin", rotary_cos_sin(head_dim, max_position, float(theta)), persistent=False)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        h, residual = self.embed_tokens(input_ids), None
        for layer in self.layers:
            h, residual = layer(positions, h, residual, self.cos_sin)
        h, _ = self.norm(h, residual)
        return h


class Qwen3ForCausalLM(nn.Module):
    packed_modules_mapping = {"q_proj": ("qkv_proj", "q"), "k_proj": ("qkv_proj", "k"), "v_proj": ("qkv_proj", "v"),
                              "gate_proj": ("gate_up_proj", 0), "up_proj": ("gate_up_proj", 1)}

    def __init__(self, cfg, mode: str = "bf16", tp_rank: int = 0, tp_size: int = 1, w4a4_layout: str = "block128",
                 w4a4_clamp_lo: int = -8, max_position: int | None = None):
        super().__init__()
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        if mode == "w4a16" and tp_size != 1:
            raise ValueError("the W4A16 model runs on one GPU (as the reference's)")
        kw = {"layout": w4a4_layout, "clamp_lo": w4a4_clamp_lo}
        self.mode = mode
        self.model = Qwen3Model(cfg, mode, tp_rank, tp_size, kw, max_position or cfg.max_position_embeddings)
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size, tp_rank, tp_size)
        if getattr(cfg, "tie_word_embeddings", False):
            self.lm_head.weight = self.model.embed_tokens.weight

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids, positions)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(hidden)
