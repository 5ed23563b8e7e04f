"""Grouped INT4 x INT4 GEMM with BF16 group scales on both operands.

Drop-in for ``nanovllm/kernels/w4a4_grouped_kernel.py`` of the reference: same
names, argument meaning, validation errors and results.  Per group g of 128
along K (in increasing g) the exact INT32 dot product is accumulated as
``total = fma(f32(dot), f32(sa)*f32(sw), total)``, and the BF16 output is the
round-to-nearest-even of ``total`` (w4a4_grouped_kernel.py:64-90).  With a
per-channel ``w_scale`` [N] the product uses ``sa`` alone and ``sw`` multiplies
the final sum.  The implementation is libnv4's sm_100a CUDA kernel; there is no
split-K, so outputs are bit-identical to the reference's sequential FMA chain.
"""
from dataclasses import dataclass
from functools import lru_cache

import torch

from nanovllm import _native

GROUP_SIZE = 128


@dataclass(frozen=True)
class GroupedConfig:
    """Kept for API compatibility (w4a4_grouped_kernel.py:21-28); the CUDA
    kernels choose their own tiles, these fields are validated only."""
    bm: int = 32
    bn: int = 64
    stages: int = 2
    threads: int = 128
    cache_scales: bool = False
    cache_weight_scales: bool = False


def _check(M, N, K, cfg):
    if min(M, N, K, cfg.bm, cfg.bn, cfg.threads) < 1 or cfg.stages < 0 or K % GROUP_SIZE or N % 8 \
            or cfg.threads % 32:
        raise ValueError("Require positive dimensions, K divisible by 128, N divisible by 8, and whole warps")


@lru_cache(None)
def compile_grouped_gemm(M, N, K, cfg=GroupedConfig(), output_fp32=False, weight_grouped=False):
    """Returns ``fn(A_packed, W_packed, Sa, Sw, C)`` writing C (BF16, or FP32 with
    ``output_fp32``) -- the reference's compiled-kernel call signature."""
    _check(M, N, K, cfg)
    flags = (_native.GEMM_W_SCALE_GROUPED if weight_grouped else 0) | (_native.GEMM_OUT_FP32 if output_fp32 else 0)
    out_dtype = torch.float32 if output_fp32 else torch.bfloat16

    def launch(a_packed, w_packed, a_scale, w_scale, out):
        if a_packed.shape != (M, K // 2) or w_packed.shape != (N, K // 2) or out.shape != (M, N) \
                or out.dtype != out_dtype:
            raise ValueError("Arguments do not match the compiled shape")
        expected_w = (N, K // GROUP_SIZE) if weight_grouped else (N,)
        if a_scale.shape != (M, K // GROUP_SIZE) or w_scale.shape != expected_w:
            raise ValueError("Require Sa[M,K/128] and Sw[N] or Sw[N,K/128]")
        tensors = (a_packed, w_packed, a_scale, w_scale, out)
        if any(not t.is_cuda or not t.is_contiguous() or t.device != a_packed.device for t in tensors):
            raise ValueError("All inputs must be contiguous CUDA tensors on one device")
        _native.w4a4_grouped_gemm(a_packed, w_packed, a_scale, w_scale, out, flags)
        return out
    return launch


@lru_cache(None)
def best_grouped_config(M, N, K, weight_grouped=False):
    return GroupedConfig() if M <= 32 else GroupedConfig(64, 128, 2, 128)


def _validate(a_packed, w_packed, a_scale, w_scale):
    if a_packed.ndim != 2 or w_packed.ndim != 2 or a_packed.shape[1] != w_packed.shape[1]:
        raise ValueError("Packed inputs must have compatible [M,K/2] and [N,K/2] shapes")
    M, K = a_packed.shape[0], a_packed.shape[1] * 2
    N = w_packed.shape[0]
    if a_packed.dtype != torch.int8 or w_packed.dtype != torch.int8:
        raise TypeError("Packed inputs must use int8 storage")
    if K % GROUP_SIZE or N % 8 or min(M, N, K) < 1:
        raise ValueError("Require positive dimensions, K divisible by 128, N divisible by 8")
    weight_grouped = w_scale.ndim == 2
    expected_w_scale = (N, K // GROUP_SIZE) if weight_grouped else (N,)
    if a_scale.shape != (M, K // GROUP_SIZE) or w_scale.shape != expected_w_scale:
        raise ValueError("Require Sa[M,K/128] and Sw[N] or Sw[N,K/128]")
    if a_scale.dtype != torch.bfloat16 or w_scale.dtype != torch.bfloat16:
        raise TypeError("Both scale tensors must be BF16")
    tensors = (a_packed, w_packed, a_scale, w_scale)
    if any(not value.is_cuda or not value.is_contiguous() or value.device != a_packed.device for value in tensors):
        raise ValueError("All inputs must be contiguous CUDA tensors on one device")
    return M, N, K, weight_grouped


def w4a4_grouped_gemm(a_packed, w_packed, a_scale, w_scale, out=None, config=None, *, out_fp32=False):
    """Packed INT4; BF16 Sa[M,K/128], Sw[N] or Sw[N,K/128], output[M,N].

    ``out_fp32=True`` (keyword-only extension) writes the FP32 total before the
    BF16 rounding, like the reference's ``output_fp32`` diagnostic kernel.
    """
    M, N, K, weight_grouped = _validate(a_packed, w_packed, a_scale, w_scale)
    dtype = torch.float32 if out_fp32 else torch.bfloat16
    if out is None:
        out = torch.empty((M, N), device=a_packed.device, dtype=dtype)
    if out.shape != (M, N) or out.dtype != dtype or out.device != a_packed.device or not out.is_contiguous():
        raise ValueError("Output must be contiguous BF16 [M,N] on the input device")
    if config is not None:
        _check(M, N, K, config)
    flags = (_native.GEMM_W_SCALE_GROUPED if weight_grouped else 0) | (_native.GEMM_OUT_FP32 if out_fp32 else 0)
    _native.w4a4_grouped_gemm(a_packed, w_packed, a_scale, w_scale, out, flags)
    return out


def w4a4_grouped_gemm_i8(a_codes, w_packed, a_scale, w_scale, out=None, *, out_fp32=False, force_stream=False):
    """``w4a4_grouped_gemm`` with activations as the INT8 [M, K] codes written by
    ``rht_quant_i8`` (same results; used by the linear layers).  More than 64
    tokens run on the tcgen05 kernel, fewer on the mma.sync weight-streaming
    kernel; ``force_stream=True`` selects the latter for any size."""
    if a_codes.ndim != 2 or w_packed.ndim != 2 or a_codes.shape[1] != w_packed.shape[1] * 2:
        raise ValueError("Require INT8 codes [M,K] and packed weights [N,K/2]")
    if a_codes.dtype != torch.int8 or w_packed.dtype != torch.int8:
        raise TypeError("Codes and packed weights must use int8 storage")
    M, K, N = a_codes.shape[0], a_codes.shape[1], w_packed.shape[0]
    if K % GROUP_SIZE or N % 8 or min(M, N, K) < 1:
        raise ValueError("Require positive dimensions, K divisible by 128, N divisible by 8")
    weight_grouped = w_scale.ndim == 2
    expected_w_scale = (N, K // GROUP_SIZE) if weight_grouped else (N,)
    if a_scale.shape != (M, K // GROUP_SIZE) or w_scale.shape != expected_w_scale:
        raise ValueError("Require Sa[M,K/128] and Sw[N] or Sw[N,K/128]")
    if a_scale.dtype != torch.bfloat16 or w_scale.dtype != torch.bfloat16:
        raise TypeError("Both scale tensors must be BF16")
    tensors = (a_codes, w_packed, a_scale, w_scale)
    if any(not t.is_cuda or not t.is_contiguous() or t.device != a_codes.device for t in tensors):
        raise ValueError("All inputs must be contiguous CUDA tensors on one device")
    dtype = torch.float32 if out_fp32 else torch.bfloat16
    if out is None:
        out = torch.empty((M, N), device=a_codes.device, dtype=dtype)
    if out.shape != (M, N) or out.dtype != dtype or out.device != a_codes.device or not out.is_contiguous():
        raise ValueError("Output must be contiguous [M,N] on the input device")
    flags = (_native.GEMM_W_SCALE_GROUPED if weight_grouped else 0) | (_native.GEMM_OUT_FP32 if out_fp32 else 0)
    if force_stream:
        flags |= _native.GEMM_FORCE_STREAM
    _native.w4a4_gemm_i8(a_codes, w_packed, a_scale, w_scale, out, flags)
    return out


def w4a4_group_dots(a_packed, w_packed):
    """Exact per-group INT32 dot products [K/128, M, N] (diagnostic)."""
    if a_packed.ndim != 2 or w_packed.ndim != 2 or a_packed.shape[1] != w_packed.shape[1]:
        raise ValueError("Packed inputs must have compatible [M,K/2] and [N,K/2] shapes")
    if a_packed.dtype != torch.int8 or w_packed.dtype != torch.int8:
        raise TypeError("Packed inputs must use int8 storage")
    M, K, N = a_packed.shape[0], a_packed.shape[1] * 2, w_packed.shape[0]
    if K % GROUP_SIZE:
        raise ValueError("K must be a multiple of 128")
    dots = torch.empty((K // GROUP_SIZE, M, N), device=a_packed.device, dtype=torch.int32)
    _native.w4a4_group_dots(a_packed.contiguous(), w_packed.contiguous(), dots)
    return dots
