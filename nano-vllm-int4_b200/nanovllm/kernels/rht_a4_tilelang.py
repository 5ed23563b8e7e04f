"""Activation prep for W4A4: RHT + per-128-group INT4 quantisation + packing.

Drop-in for ``nanovllm/kernels/rht_a4_tilelang.py`` of the reference (the
module name is kept so that callers and the reference's plugin harness
``bench_rht_a4.py --impl nanovllm.kernels.rht_a4_tilelang:rht_quant_pack`` need
no change); the implementation is the sm_100a CUDA kernel in libnv4.

``rht_quant_pack(x, signs, *, out_packed, out_scale)`` keeps the reference
contract (``benchmarks/rht_a4_bench_common.py:276-293``): layout
``row_DH_paley12_kron_sylvester_v1``, clip 0.9, BF16 scale rounded before the
codes, codes in [-7, 7], outputs written in place and returned, current CUDA
stream, no host synchronisation, CUDA-graph safe.  Two keyword-only extensions
select the other layout and code range used by the benchmark configurations:
``layout="block128"`` (normalized 128-point WHT per K group, any K % 128 == 0)
and ``clamp_lo=-8``.
"""
from dataclasses import dataclass
from functools import lru_cache

import torch

from nanovllm import _native

LAYOUT_VERSION = "row_DH_paley12_kron_sylvester_v1"


@dataclass(frozen=True)
class Config:
    """Kept for API compatibility (rht_a4_tilelang.py:13-16).  The CUDA kernel
    chooses its own geometry; these fields are validated and otherwise unused."""
    threads_per_row: int = 128
    rows_per_block: int = 1


def _check_config(cfg: Config) -> None:
    if cfg.threads_per_row not in (32, 64, 128, 256, 512) or cfg.rows_per_block < 1 \
            or cfg.threads_per_row * cfg.rows_per_block > 1024:
        raise ValueError("Unsupported RHT configuration")


@lru_cache(None)
def compile_kernel(K, cfg=Config()):
    """Returns a launcher ``fn(x, signs, packed, scale)`` for the reference layout
    (rht_a4_tilelang.py:19-136 compiled a TileLang kernel here)."""
    if K not in (4096, 12288):
        raise ValueError("Unsupported RHT configuration")
    _check_config(cfg)

    def launch(x, signs, packed, scale):
        _native.rht_quant_pack(x, signs, packed, scale, _native.LAYOUT_ROW_DH, -7)
    return launch


@lru_cache(None)
def best_config(M, K):
    return Config()


def _layout_id(layout) -> int:
    if isinstance(layout, int):
        if layout not in (_native.LAYOUT_BLOCK128, _native.LAYOUT_ROW_DH):
            raise ValueError(f"unknown layout {layout}")
        return layout
    try:
        return _native.LAYOUTS[layout]
    except KeyError:
        raise ValueError(f"unknown layout {layout!r}") from None


def rht_quant_pack(x, signs, *, out_packed, out_scale, config=None, layout=LAYOUT_VERSION, clamp_lo=-7):
    lid = _layout_id(layout)
    if x.ndim != 2 or x.dtype != torch.bfloat16 or x.shape[0] < 1:
        raise ValueError('Expected BF16 X[M,K], M>0, K=4096/12288')
    m, k = x.shape
    if lid == _native.LAYOUT_ROW_DH and k not in (4096, 12288):
        raise ValueError('Expected BF16 X[M,K], M>0, K=4096/12288')
    if lid == _native.LAYOUT_BLOCK128 and (k < 128 or k % 128):
        raise ValueError('Expected BF16 X[M,K], M>0, K a multiple of 128 for the block128 layout')
    if signs.shape != (k,) or signs.dtype != torch.int8:
        raise ValueError('Expected INT8 signs[K]')
    if out_packed.shape != (m, k // 2) or out_packed.dtype != torch.int8:
        raise ValueError('Expected INT8 output[M,K/2]')
    if out_scale.shape != (m, k // 128) or out_scale.dtype != torch.bfloat16:
        raise ValueError('Expected BF16 scales[M,K/128]')
    if any(not t.is_cuda or not t.is_contiguous() or t.device != x.device for t in [x, signs, out_packed, out_scale]):
        raise ValueError('All tensors must be contiguous on one CUDA device')
    if clamp_lo not in (-7, -8):
        raise ValueError('clamp_lo must be -7 or -8')
    if config is not None:
        _check_config(config)
    _native.rht_quant_pack(x, signs, out_packed, out_scale, lid, clamp_lo)
    return out_packed, out_scale


def rht_quant_i8(x, signs, *, out_codes, out_scale, layout=LAYOUT_VERSION, clamp_lo=-7):
    """Same transform and quantisation as ``rht_quant_pack``, with the codes
    written as GEMM-ready INT8 ``out_codes`` [M, K] (each 32-wide K chunk holds
    its 16 even-k codes, then its 16 odd-k codes) for ``w4a4_grouped_gemm_i8``."""
    lid = _layout_id(layout)
    if x.ndim != 2 or x.dtype != torch.bfloat16 or x.shape[0] < 1:
        raise ValueError('Expected BF16 X[M,K], M>0')
    m, k = x.shape
    if (lid == _native.LAYOUT_ROW_DH and k not in (4096, 12288)) or k % 128 or k < 128:
        raise ValueError('Unsupported K for this layout')
    if signs.shape != (k,) or signs.dtype != torch.int8:
        raise ValueError('Expected INT8 signs[K]')
    if out_codes.shape != (m, k) or out_codes.dtype != torch.int8:
        raise ValueError('Expected INT8 codes[M,K]')
    if out_scale.shape != (m, k // 128) or out_scale.dtype != torch.bfloat16:
        raise ValueError('Expected BF16 scales[M,K/128]')
    if any(not t.is_cuda or not t.is_contiguous() or t.device != x.device for t in [x, signs, out_codes, out_scale]):
        raise ValueError('All tensors must be contiguous on one CUDA device')
    if clamp_lo not in (-7, -8):
        raise ValueError('clamp_lo must be -7 or -8')
    _native.rht_quant_i8(x, signs, out_codes, out_scale, lid, clamp_lo)
    return out_codes, out_scale


def silu_mul_rht_quant_i8(gate_up, signs, *, out_codes, out_scale, layout=LAYOUT_VERSION, clamp_lo=-7):
    """``rht_quant_i8`` of ``SiluAndMul(gate_up)`` in one kernel (the down
    projection's prep fused with its producer, nanovllm/layers/activation.py:8-11):
    ``gate_up`` is BF16 [M, 2K] (gate, then up); the prep input
    bf16(silu(gate) * up) is computed in FP32 with one rounding, as the
    reference's compiled SiluAndMul, and never written to memory."""
    lid = _layout_id(layout)
    if gate_up.ndim != 2 or gate_up.dtype != torch.bfloat16 or gate_up.shape[0] < 1 or gate_up.shape[1] % 2:
        raise ValueError('Expected BF16 gate_up[M,2K], M>0')
    m, k = gate_up.shape[0], gate_up.shape[1] // 2
    if (lid == _native.LAYOUT_ROW_DH and k not in (4096, 12288)) or k % 128 or k < 128:
        raise ValueError('Unsupported K for this layout')
    if signs.shape != (k,) or signs.dtype != torch.int8:
        raise ValueError('Expected INT8 signs[K]')
    if out_codes.shape != (m, k) or out_codes.dtype != torch.int8:
        raise ValueError('Expected INT8 codes[M,K]')
    if out_scale.shape != (m, k // 128) or out_scale.dtype != torch.bfloat16:
        raise ValueError('Expected BF16 scales[M,K/128]')
    if any(not t.is_cuda or not t.is_contiguous() or t.device != gate_up.device
           for t in [gate_up, signs, out_codes, out_scale]):
        raise ValueError('All tensors must be contiguous on one CUDA device')
    if clamp_lo not in (-7, -8):
        raise ValueError('clamp_lo must be -7 or -8')
    _native.silu_mul_rht_quant_i8(gate_up, signs, out_codes, out_scale, lid, clamp_lo)
    return out_codes, out_scale


def add_rmsnorm_rht_quant_i8(x, residual, weight, eps, signs, *, out_codes, out_scale, out_residual=None,
                             out_normed=None, layout=LAYOUT_VERSION, clamp_lo=-7):
    """``rht_quant_i8`` of ``RMSNorm(x + residual)`` in one kernel (the QKV /
    gate-up prep fused with the decoder layer's add + RMSNorm,
    nanovllm/layers/layernorm.py:33-45; ``residual=None`` is rms_forward).
    Writes the new residual bf16(x + residual) to ``out_residual`` (required
    with a residual) and, if given, the normalized BF16 activation to
    ``out_normed``.  Returns ``(out_codes, out_scale)``."""
    lid = _layout_id(layout)
    if x.ndim != 2 or x.dtype != torch.bfloat16 or x.shape[0] < 1:
        raise ValueError('Expected BF16 X[M,K], M>0')
    m, k = x.shape
    if (lid == _native.LAYOUT_ROW_DH and k != 4096) or (lid == _native.LAYOUT_BLOCK128 and (k % 512 or k > 16384)):
        raise ValueError('Unsupported K for this layout')
    for name, t in (('residual', residual), ('out_residual', out_residual), ('out_normed', out_normed)):
        if t is not None and (t.shape != (m, k) or t.dtype != torch.bfloat16):
            raise ValueError(f'Expected BF16 {name}[M,K]')
    if residual is not None and out_residual is None:
        raise ValueError('out_residual is required with a residual')
    if weight.shape != (k,) or weight.dtype != torch.bfloat16:
        raise ValueError('Expected BF16 weight[K]')
    if signs.shape != (k,) or signs.dtype != torch.int8:
        raise ValueError('Expected INT8 signs[K]')
    if out_codes.shape != (m, k) or out_codes.dtype != torch.int8:
        raise ValueError('Expected INT8 codes[M,K]')
    if out_scale.shape != (m, k // 128) or out_scale.dtype != torch.bfloat16:
        raise ValueError('Expected BF16 scales[M,K/128]')
    ts = [t for t in (x, residual, weight, signs, out_codes, out_scale, out_residual, out_normed) if t is not None]
    if any(not t.is_cuda or not t.is_contiguous() or t.device != x.device for t in ts):
        raise ValueError('All tensors must be contiguous on one CUDA device')
    if clamp_lo not in (-7, -8):
        raise ValueError('clamp_lo must be -7 or -8')
    _native.add_rmsnorm_rht_quant_i8(x, residual, weight, eps, signs, out_codes, out_scale, out_residual, out_normed,
                                     lid, clamp_lo)
    return out_codes, out_scale


def i8_to_codes(codes_i8: torch.Tensor) -> torch.Tensor:
    """Undo the GEMM-ready K order of ``rht_quant_i8`` (for checks): [M, K] codes in k order."""
    m, k = codes_i8.shape
    c = codes_i8.reshape(m, k // 32, 2, 16)          # [chunk][even/odd][i]
    return c.permute(0, 1, 3, 2).reshape(m, k)        # k = 2i + parity
