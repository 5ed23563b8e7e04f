"""Seeded synthetic inputs for the quantized-linear path (CPU generation).

No checkpoint, model weights or dataset are available, so every test and the
benchmark draw inputs here, on the CPU with ``torch.Generator`` (deterministic
across machines), and copy them to the device afterwards.  The distributions
follow the benchmark configurations:

* activations: N(0,1) BF16 with 0.5% of the channels (fixed seeded indices)
  scaled by 20 as outliers;
* RHT signs: ``make_signs`` as in ``benchmarks/rht_reference.py:57-59``;
* W4A4 weights: signed INT4 codes uniform in [-8, 7], packed two per byte with
  the even K index in the low nibble, per-(n, 128-group) BF16 scales
  |N(0, 0.02)| / 7;
* W4A16 weights: GPTQ uint4 codes uniform in [0, 15] packed 8 per int32 along K,
  zero points uniform in [0, 15] packed 8 per int32 along N, per-(group, n)
  scales |N(0, 0.02)| stored as FP16 (the module parameter dtype).

``make_input`` restates the reference harness input with its deterministic
edge rows (``benchmarks/rht_a4_bench_common.py:361-377``).
"""
from __future__ import annotations

import torch

GROUP = 128
QWEN3_8B_SHAPES = {          # name: (N, K) of the fused projections
    "qkv": (6144, 4096),
    "o": (4096, 4096),
    "gate_up": (24576, 4096),
    "down": (4096, 12288),
}


def make_signs(k: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randint(0, 2, (k,), generator=g, dtype=torch.int8) * 2 - 1).contiguous()


def outlier_channels(k: int, seed: int) -> torch.Tensor:
    count = max(1, (k * 5) // 1000)
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randperm(k, generator=g)[:count]


def activations(m: int, k: int, seed: int) -> torch.Tensor:
    """BF16 [m, k]: N(0,1) with 0.5% of channels x20."""
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    x = torch.randn(m, k, generator=g, dtype=torch.float32)
    x[:, outlier_channels(k, seed)] *= 20
    return x.bfloat16().contiguous()


def make_input(m: int, k: int, seed: int = 20261108) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed + m * 17 + k)
    x = torch.randn(m, k, dtype=torch.bfloat16, generator=g)
    x[0].zero_()
    if m > 1:
        x[1].zero_()
        x[1, k // 12 if k == 12288 else 5] = 1000
    if m > 2:
        x[2].fill_(1)
    if m > 3:
        x[3, ::2] = 1
        x[3, 1::2] = -1
    if m > 4:
        x[4].mul_(1e-9)
    if m > 5:
        x[5].mul_(1e4)
    return x.contiguous()


def exponent_extremes(m: int, k: int, seed: int = 20261108) -> torch.Tensor:
    """Rows scaled by 2^e, e cycling over BF16 exponent extremes; last row zero
    (the sweep of benchmarks/verify_rht_a4_extremes.py, generated on the CPU)."""
    exponents = [-130, -126, -120, -80, -30, 0, 30, 80, 100]
    g = torch.Generator(device="cpu").manual_seed(seed + m + k)
    x = torch.randn(m, k, dtype=torch.bfloat16, generator=g).float()
    e = torch.tensor([exponents[i % len(exponents)] for i in range(m)], dtype=torch.int32)
    x = torch.ldexp(x, e[:, None].float()).bfloat16().contiguous()
    x[-1].zero_()
    return x


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """int8 codes [..., K] -> int8 packed [..., K/2], even K in the low nibble."""
    c = codes.to(torch.int8)
    return ((c[..., ::2] & 15) | ((c[..., 1::2] & 15) << 4)).to(torch.int8).contiguous()


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.int16) & 255
    lo, hi = p & 15, (p >> 4) & 15
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack((lo, hi), dim=-1).flatten(-2).to(torch.int8)


def w4a4_weights(n: int, k: int, seed: int):
    """(codes int8 [n,k], packed int8 [n,k/2], scale bf16 [n,k/128])."""
    g = torch.Generator(device="cpu").manual_seed(seed + 2)
    codes = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    scale = (torch.randn(n, k // GROUP, generator=g).abs() * 0.02 / 7).bfloat16()
    return codes, pack_int4(codes), scale.contiguous()


def config0(seed: int = 0, m: int = 16, k: int = 4096, n: int = 4096):
    """Config 0 of the benchmark: X [16,4096], signs, W [4096,4096] packed + scales."""
    x = activations(m, k, seed)
    signs = make_signs(k, seed)
    codes, packed, scale = w4a4_weights(n, k, seed)
    return x, signs, codes, packed, scale


def w4a16_weights(n: int, k: int, seed: int, group: int = GROUP):
    """GPTQ tensors: qweight int32 [k/8, n], qzeros int32 [k/group, n/8], scales fp16 [k/group, n]."""
    g = torch.Generator(device="cpu").manual_seed(seed + 3)
    w = torch.randint(0, 16, (k, n), generator=g, dtype=torch.int64)
    z = torch.randint(0, 16, (k // group, n), generator=g, dtype=torch.int64)
    scales = (torch.randn(k // group, n, generator=g).abs() * 0.02).half()
    shifts = 4 * torch.arange(8, dtype=torch.int64)
    qweight = (w.reshape(k // 8, 8, n) << shifts[None, :, None]).sum(1)
    qzeros = (z.reshape(k // group, n // 8, 8) << shifts[None, None, :]).sum(2)
    to_i32 = lambda t: torch.where(t >= 2 ** 31, t - 2 ** 32, t).to(torch.int32).contiguous()
    return to_i32(qweight), to_i32(qzeros), scales.contiguous()


# Qwen3-8B architecture (the benchmark's end-to-end configuration): no weights
# exist offline, so the engine runs it with load_format="dummy".
QWEN3_8B_CONFIG = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 4096,
    "intermediate_size": 12288, "num_hidden_layers": 36, "num_attention_heads": 32, "num_key_value_heads": 8,
    "head_dim": 128, "hidden_act": "silu", "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
    "max_position_embeddings": 40960, "vocab_size": 151936, "tie_word_embeddings": False,
    "attention_bias": False, "torch_dtype": "bfloat16", "bos_token_id": 151643, "eos_token_id": 151645,
}


def write_qwen3_config(directory: str, **overrides) -> str:
    """Write a Hugging Face config.json for a Qwen3 model (Qwen3-8B unless
    overridden, e.g. fewer layers for tests) into `directory`; returns it."""
    import json
    import os
    os.makedirs(directory, exist_ok=True)
    cfg = dict(QWEN3_8B_CONFIG, **overrides)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return directory
