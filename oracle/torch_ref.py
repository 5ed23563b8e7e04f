"""The reference's own PyTorch CPU path, restated in torch.  TEST INFRASTRUCTURE ONLY.

Only ``bench.py`` (its ``cpu_baseline`` leg and the ``--impl reference`` arm)
and ``tests/`` may import this module; the product path never does.

``oracle/nv4_oracle.py`` is the bit-exact checker (numpy, exact FP32-FMA
emulation, slow).  This file is the *timed* CPU baseline: the same torch
operations, in the same order and on the same CPU tensors, that the
reference's PyTorch path runs for one W4A4 linear --

  1. ``x.float() * signs`` then the normalized Sylvester FWHT of each 128-wide
     K group (``benchmarks/rht_reference.py:26-39`` ``fwht`` on
     ``[M, K/128, 128]``; the sign multiply first as ``rht`` at ``:62-67``);
  2. per-group absmax quantisation, scale = bf16(max(absmax*0.9/7, tiny)),
     1.0 for an all-zero group, codes = round(x/scale) clamped to
     [clamp_lo, 7] (``benchmarks/a4_group_quant.py:60-70`` ``quantize_rotated``,
     with the clamp floor as a parameter: -7 there, -8 in the benchmark
     configurations);
  3. nibble packing (``benchmarks/rht_reference.py:80-83`` ``pack_int4``);
  4. the grouped GEMM reference that emulates the FP32 FMA chain in FP64
     (``benchmarks/verify_w4a4_aw_grouped.py:13-29`` ``reference``), then
     ``.bfloat16()``;

plus the decoder layer's producers in FP32 torch ops (``nanovllm/layers/
layernorm.py:29-40`` add + RMSNorm, ``nanovllm/layers/activation.py:8-11``
SiluAndMul) so that one decoder layer of the benchmark chain can be timed.
The unpacked codes are what the reference GEMM consumes, so step 3's packed
bytes are produced (as the path does) and the codes are passed on.

``tests/test_torch_ref_cpu.py`` checks this restatement against the numpy
oracle bit for bit on small cases.
"""
from __future__ import annotations

import math

import torch

GROUP = 128
_SQRT_GROUP = math.sqrt(GROUP)


def fwht_groups(x: torch.Tensor) -> torch.Tensor:
    """Normalized Sylvester transform of the last dimension (power of two):
    butterflies with step 1, 2, 4, ... then a division by sqrt(n)."""
    n = x.shape[-1]
    shape = x.shape
    y = x
    step = 1
    while step < n:
        z = y.reshape(*shape[:-1], n // (2 * step), 2, step)
        lo, hi = z[..., 0, :], z[..., 1, :]
        y = torch.stack((lo + hi, lo - hi), dim=-2).reshape(shape)
        step *= 2
    return y / math.sqrt(n)


def rotate_block128(x: torch.Tensor, signs: torch.Tensor) -> torch.Tensor:
    m, k = x.shape
    signed = x.float() * signs.to(torch.float32)
    return fwht_groups(signed.reshape(m, k // GROUP, GROUP)).reshape(m, k)


def quantize_rotated(x: torch.Tensor, clamp_lo: int = -8, clip: float = 0.9):
    m, k = x.shape
    grouped = x.float().reshape(m, k // GROUP, GROUP)
    maximum = grouped.abs().amax(-1)
    scale = torch.where(maximum == 0, 1.0,
                        (maximum * clip / 7).clamp_min(torch.finfo(torch.bfloat16).tiny)).bfloat16()
    codes = (grouped / scale.float().unsqueeze(-1)).round().clamp(clamp_lo, 7)
    return codes.reshape(m, k).to(torch.int8), scale


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    return ((codes[..., ::2] & 15) | ((codes[..., 1::2] & 15) << 4)).contiguous()


def grouped_gemm(qa: torch.Tensor, qw: torch.Tensor, sa: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """FP32 INT4 group dots, FP64 product and sum rounded to FP32 per group."""
    m, k = qa.shape
    total = torch.zeros((m, qw.shape[0]), dtype=torch.float32, device=qa.device)
    qaf, qwf = qa.float(), qw.float()
    for g in range(k // GROUP):
        sl = slice(g * GROUP, (g + 1) * GROUP)
        dot = qaf[:, sl] @ qwf[:, sl].T
        scale = sa[:, g].float()[:, None] * sw[:, g].float()[None, :]
        total = (dot.double() * scale.double() + total.double()).float()
    return total


def w4a4_linear(x: torch.Tensor, signs: torch.Tensor, w_codes: torch.Tensor, w_scale: torch.Tensor,
                clamp_lo: int = -8) -> torch.Tensor:
    """One W4A4 linear (block128 layout): x bf16 [M, K] -> bf16 [M, N]."""
    codes, scale = quantize_rotated(rotate_block128(x, signs), clamp_lo)
    pack_int4(codes)
    return grouped_gemm(codes, w_codes.to(x.device), scale, w_scale.to(x.device)).bfloat16()


def add_rmsnorm(x: torch.Tensor, residual, weight: torch.Tensor, eps: float):
    """(bf16(bf16(xf * rsqrt(mean(xf^2) + eps)) * weight), bf16(xf)), xf = x (+ residual) in FP32."""
    xf = x.float() if residual is None else x.float() + residual.float()
    new_residual = xf.bfloat16()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    h = (xf * torch.rsqrt(var + eps)).bfloat16() * weight
    return h, new_residual


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    gate, up = gate_up.float().chunk(2, -1)
    return (torch.nn.functional.silu(gate) * up).bfloat16()
