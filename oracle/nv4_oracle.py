"""CPU oracle for the quantized-linear hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it.  The product path
(``nanovllm.kernels.*``, ``nanovllm.layers.*``) runs the sm_100a CUDA library
and raises when that library is missing; it never falls back to this file.

It restates the reference algorithms in numpy, op for op, so that every FP32
rounding the reference performs happens here in the same order:

* ``rotate_block128`` -- sign multiply then a normalized Sylvester FWHT of each
  128-wide K group, evaluated as the reference's PyTorch path on CPU does it
  (``benchmarks/rht_reference.py:26-39`` ``fwht``; sign first as in
  ``benchmarks/rht_reference.py:62-67`` ``rht``).  The 1/sqrt(128) step is an
  IEEE division by fl32(sqrt(128)) -- torch on CPU divides, it does not
  multiply by a reciprocal.
* ``rotate_row_dh`` -- the checkpoint layout ``row_DH_paley12_kron_sylvester_v1``
  as the production kernel computes it (``nanovllm/kernels/rht_a4_tilelang.py``
  :58-100): full-width FWHT, exact power-of-two normalisation, and for K=12288
  the Paley H12 mix summed source 0..11 in FP32 then multiplied by
  fl32(1/sqrt(12)).
* ``quantize_block128`` -- ``benchmarks/a4_group_quant.py:206-216``
  (``quantize_rotated``) on CPU: scale = bf16(max(fl(fl(absmax*0.9)/7), tiny)),
  1.0 for an all-zero group, codes = round-half-even(x / scale) clamped to
  [clamp_lo, 7] (the reference clamps to -7; BASELINE configs use -8).
* ``quantize_row_dh`` -- ``rht_a4_tilelang.py:123-131``: the scale uses
  ``__fmul_rn(__fmul_rn(absmax, 0.9f), fl32(1/7))``.
* ``pack_int4`` / ``unpack_int4`` -- ``benchmarks/rht_reference.py:80-90``.
* ``grouped_gemm`` -- ``nanovllm/kernels/w4a4_grouped_kernel.py:64-90`` and its
  oracle ``benchmarks/verify_w4a4_aw_grouped.py:117-133``: exact INT32 group
  dots, then ``total = fma(f32(dot), f32(sa)*f32(sw), total)`` for g = 0..G-1,
  one FP32 rounding per group, BF16 output.  The FMA is emulated exactly
  (TwoSum in float64 plus a midpoint fix-up), which the reference's
  float64-then-float32 emulation approximates.
* ``silu_mul_bf16_bits`` -- ``nanovllm/layers/activation.py:8-11``
  (SiluAndMul under torch.compile): bf16(silu(g) * u) with silu and the
  product in FP32, one rounding at the end; silu(g) = g / (1 + exp(-g)).
  numpy's exp and CUDA's expf may differ by an ulp, so this restatement of a
  transcendental is compared with a tolerance (the GPU path is checked
  exactly against torch's FP32 arithmetic on the same device).
* ``add_rmsnorm_bf16_bits`` -- ``nanovllm/layers/layernorm.py:33-45``
  (add_rms_forward; rms_forward without a residual): FP32 sum, BF16 residual,
  var = mean(xf^2), bf16(bf16(xf * rsqrt(var + eps)) * weight).  The order of
  the FP32 reduction is numpy's, so this restatement is compared with a
  tolerance.
* ``w4a16_dequant`` / ``w4a16_gemm`` -- ``nanovllm/layers/linear_w4a16.py:45-59``:
  ``bf16(0x4300 | (w+15-z)) - 144`` times the BF16-rounded FP16 scale, rounded
  to BF16, then an FP32-accumulated GEMM.  The reference has no W4A16 test, so
  this restatement is *parity unpinned* and is compared with a tolerance.
"""
from __future__ import annotations

import math

import numpy as np

GROUP = 128
BF16_TINY = np.float32(2.0 ** -126)           # torch.finfo(torch.bfloat16).tiny
CLIP = np.float32(0.9)
SQRT128 = np.float32(math.sqrt(128.0))        # fl32(sqrt(128)), the CPU divisor
INV_SQRT12 = np.float32(1.0 / math.sqrt(12.0))  # T.float32(1/sqrt(12)) in the TileLang kernel
INV7 = np.float32(1.0 / 7.0)                  # T.float32(1/7) in the TileLang kernel
SEVEN = np.float32(7.0)
LAYOUT_BLOCK128 = 0
LAYOUT_ROW_DH = 1


# ---------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 BF16 bit patterns -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 BF16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def f16_to_bf16_f32(x: np.ndarray) -> np.ndarray:
    """FP16 values -> BF16 (round to nearest even) -> float32."""
    return round_to_bf16(np.asarray(x, dtype=np.float16).astype(np.float32))


# ---------------------------------------------------------------- transforms
def fwht_lastdim(y: np.ndarray) -> np.ndarray:
    """Unnormalized Sylvester butterflies, lowest index bit first.

    Same stage order and pairing as ``rht_reference.fwht`` (``:33-38``): at each
    step the low element a and high element b become (a + b, a - b), in FP32.
    """
    y = np.ascontiguousarray(y, dtype=np.float32)
    n = y.shape[-1]
    if n < 1 or n & (n - 1):
        raise ValueError("FWHT requires a power-of-two last dimension")
    shape = y.shape
    step = 1
    while step < n:
        z = y.reshape(*shape[:-1], n // (2 * step), 2, step)
        a, b = z[..., 0, :], z[..., 1, :]
        y = np.stack((a + b, a - b), axis=-2).reshape(shape)
        step *= 2
    return y


def _signed(x_f32: np.ndarray, signs: np.ndarray) -> np.ndarray:
    signs = np.asarray(signs)
    if signs.shape != (x_f32.shape[-1],):
        raise ValueError("one sign per input channel is required")
    return np.asarray(x_f32, dtype=np.float32) * signs.astype(np.float32)


def rotate_block128(x_f32: np.ndarray, signs: np.ndarray) -> np.ndarray:
    """Block-diagonal normalized 128-point WHT per K group (CPU torch semantics)."""
    v = _signed(x_f32, signs)
    m, k = v.shape
    if k % GROUP:
        raise ValueError("K must be a multiple of 128")
    y = fwht_lastdim(v.reshape(m, k // GROUP, GROUP))
    return (y / SQRT128).astype(np.float32).reshape(m, k)


def _h12_positive(source: int, destination: int) -> bool:
    """Sign of H12[source, destination] of the Paley matrix (rht_reference.py:15-23)."""
    if source == 0 or destination == 0:
        return True
    return ((destination - source) % 11) in (1, 3, 4, 5, 9)


def rotate_row_dh(x_f32: np.ndarray, signs: np.ndarray) -> np.ndarray:
    """Checkpoint layout: X D H with H = H4096, or H12 (x) H1024 for K = 12288."""
    v = _signed(x_f32, signs)
    m, k = v.shape
    if k == 4096:
        return (fwht_lastdim(v) * np.float32(1.0 / 64.0)).astype(np.float32)
    if k != 12288:
        raise ValueError("row_DH layout supports K = 4096 or 12288")
    z = fwht_lastdim(v.reshape(m, 12, 1024)) * np.float32(1.0 / 32.0)
    out = np.empty_like(z)
    for d in range(12):
        acc = np.zeros((m, 1024), dtype=np.float32)
        for s in range(12):
            acc = acc + z[:, s, :] if _h12_positive(s, d) else acc - z[:, s, :]
        out[:, d, :] = acc * INV_SQRT12
    return out.reshape(m, k)


def h12_matrix() -> np.ndarray:
    return np.array([[1.0 if _h12_positive(s, d) else -1.0 for d in range(12)]
                     for s in range(12)], dtype=np.float64)


# ---------------------------------------------------------------- quantizers
def _group_max(r: np.ndarray) -> np.ndarray:
    m, k = r.shape
    return np.abs(r.reshape(m, k // GROUP, GROUP)).max(axis=-1).astype(np.float32)


def scales_block128(r: np.ndarray) -> np.ndarray:
    mx = _group_max(r)
    t = (mx * CLIP).astype(np.float32)
    t = (t / SEVEN).astype(np.float32)
    t = np.maximum(t, BF16_TINY)
    return round_to_bf16(np.where(mx == 0, np.float32(1.0), t).astype(np.float32))


def scales_row_dh(r: np.ndarray) -> np.ndarray:
    mx = _group_max(r)
    t = (mx * CLIP).astype(np.float32)
    t = (t * INV7).astype(np.float32)
    t = np.maximum(t, BF16_TINY)
    return round_to_bf16(np.where(mx == 0, np.float32(1.0), t).astype(np.float32))


def quotients(r: np.ndarray, scale_f32: np.ndarray) -> np.ndarray:
    """Pre-rounding FP32 quotients x / scale (IEEE division)."""
    m, k = r.shape
    q = r.reshape(m, k // GROUP, GROUP) / scale_f32[..., None]
    return q.astype(np.float32).reshape(m, k)


def codes_from_quotients(q: np.ndarray, clamp_lo: int = -8) -> np.ndarray:
    return np.clip(np.rint(q), clamp_lo, 7).astype(np.int8)   # rint = half to even


def quantize(r: np.ndarray, layout: int, clamp_lo: int = -8):
    """Returns (codes int8 [M,K], scales float32 (bf16-valued) [M,K/128], quotients)."""
    if clamp_lo not in (-7, -8):
        raise ValueError("clamp_lo must be -7 or -8")
    s = scales_block128(r) if layout == LAYOUT_BLOCK128 else scales_row_dh(r)
    q = quotients(r, s)
    return codes_from_quotients(q, clamp_lo), s, q


def rotate(x_f32, signs, layout):
    return rotate_block128(x_f32, signs) if layout == LAYOUT_BLOCK128 else rotate_row_dh(x_f32, signs)


def prepare(x_bf16_bits: np.ndarray, signs: np.ndarray, layout: int = LAYOUT_BLOCK128,
            clamp_lo: int = -8):
    """Full activation prep: returns (packed uint8 [M,K/2], scale bf16 bits [M,K/128],
    codes, quotients, rotated)."""
    x = bf16_bits_to_f32(x_bf16_bits)
    r = rotate(x, signs, layout)
    codes, s, q = quantize(r, layout, clamp_lo)
    return pack_int4(codes), f32_to_bf16_bits(s), codes, q, r


def silu_mul_bf16_bits(gate_up_bits: np.ndarray) -> np.ndarray:
    """SiluAndMul of a gate/up BF16 row block [M, 2K] -> BF16 bits [M, K]
    (activation.py:8-11 as compiled: FP32 silu and product, one rounding)."""
    gu = bf16_bits_to_f32(gate_up_bits)
    k = gu.shape[-1] // 2
    g, u = gu[..., :k], gu[..., k:]
    with np.errstate(over="ignore"):
        s = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    return f32_to_bf16_bits((s * u).astype(np.float32))


def add_rmsnorm_bf16_bits(x_bits: np.ndarray, residual_bits, weight_bits: np.ndarray, eps: float = 1e-6):
    """RMSNorm(x + residual) of BF16 rows (layernorm.py:33-45) -> (normed bits,
    new residual bits); residual None is rms_forward (the residual is x)."""
    xf = bf16_bits_to_f32(x_bits)
    if residual_bits is not None:
        xf = (xf + bf16_bits_to_f32(residual_bits)).astype(np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    r = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = round_to_bf16((xf * r).astype(np.float32))
    h = f32_to_bf16_bits((y * bf16_bits_to_f32(weight_bits)).astype(np.float32))
    return h, f32_to_bf16_bits(xf)


def boundary_mask(q: np.ndarray, ulps: int = 1) -> np.ndarray:
    """True where q is within `ulps` FP32 ulps of a round-half-even boundary k+0.5."""
    q = np.asarray(q, dtype=np.float32)
    h = np.floor(q) + np.float32(0.5)
    lo = q.copy()
    hi = q.copy()
    for _ in range(ulps):
        lo = np.nextafter(lo, np.float32(-np.inf))
        hi = np.nextafter(hi, np.float32(np.inf))
    near_up = (lo <= h) & (h <= hi)
    h2 = h - np.float32(1.0)
    near_dn = (lo <= h2) & (h2 <= hi)
    return near_up | near_dn


# ---------------------------------------------------------------- packing
def pack_int4(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.int8)
    if c.shape[-1] % 2:
        raise ValueError("even K required")
    lo = c[..., ::2].astype(np.uint8) & 15
    hi = c[..., 1::2].astype(np.uint8) & 15
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed).view(np.uint8) if np.asarray(packed).dtype == np.int8 else np.asarray(packed, np.uint8)
    lo = (p & 15).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack((lo, hi), axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2).astype(np.int8)


# ---------------------------------------------------------------- exact FP32 FMA
def fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 fma(a, b, c) for float32 a, b, c whose exact
    product a*b fits in a float64 (true for INT14 dots times BF16-product scales).
    """
    p = np.asarray(a, np.float64) * np.asarray(b, np.float64)
    c64 = np.asarray(c, np.float64)
    s = p + c64
    r = s.astype(np.float32)
    # Double rounding can only bite when s = fl64(p + c) lies exactly on a float32
    # midpoint: for float32-normal magnitudes that is the bit pattern ...1000...0
    # in the 29 mantissa bits float64 has beyond float32.  Subnormal-range sums
    # take the general test.  Both are rare; only those elements are fixed up.
    bits = s.view(np.uint64)
    cand = ((bits & np.uint64(0x1FFFFFFF)) == np.uint64(0x10000000)) | (np.abs(s) < 2.0 ** -125)
    cand &= np.isfinite(s)
    if cand.any():
        idx = np.nonzero(cand)
        ps, cs, ss = p[idx], c64[idx] if c64.shape == s.shape else np.broadcast_to(c64, s.shape)[idx], s[idx]
        bb = ss - ps
        err = (ps - (ss - bb)) + (cs - bb)        # TwoSum: p + c == s + err exactly
        rr = r[idx]
        r64 = rr.astype(np.float64)
        diff = ss - r64
        toward = np.where(diff > 0, np.float32(np.inf), np.float32(-np.inf)).astype(np.float32)
        other = np.nextafter(rr, toward)
        half = np.abs(other.astype(np.float64) - r64) * 0.5
        tie = (diff != 0) & (np.abs(diff) == half)
        # s sits on a float32 midpoint; the exact sum lies beyond it when err pushes
        # toward `other`.
        fix = tie & (err != 0) & (np.sign(err) == np.sign(diff))
        r[idx] = np.where(fix, other, rr)
    return r.astype(np.float32)


def group_dots(qa: np.ndarray, qw: np.ndarray) -> np.ndarray:
    """Exact per-group INT32 dot products, [G, M, N].

    Evaluated with a float32 matmul, which is exact here in any summation order:
    every product is an integer of magnitude <= 64 and every partial sum of a
    128-term group is an integer of magnitude <= 8192 < 2^24.
    """
    m, k = qa.shape
    n = qw.shape[0]
    g = k // GROUP
    a = np.ascontiguousarray(qa.astype(np.float32).reshape(m, g, GROUP).transpose(1, 0, 2))
    w = np.ascontiguousarray(qw.astype(np.float32).reshape(n, g, GROUP).transpose(1, 2, 0))
    return np.matmul(a, w).astype(np.int32)


def grouped_gemm_f32(qa: np.ndarray, qw: np.ndarray, sa_f32: np.ndarray, sw_f32: np.ndarray,
                     dots: np.ndarray | None = None) -> np.ndarray:
    """FP32 result of the grouped INT4 GEMM (w4a4_grouped_kernel.py:64-90).

    sw_f32 is [N, G] (weight-grouped) or [N] (per-channel, applied after the sum).
    """
    m, k = qa.shape
    n = qw.shape[0]
    g_count = k // GROUP
    total = np.zeros((m, n), dtype=np.float32)
    sa = np.asarray(sa_f32, np.float32)
    sw = np.asarray(sw_f32, np.float32)
    for g in range(g_count):
        if dots is not None:
            d = dots[g].astype(np.float32)
        else:   # exact: integer partial sums below 2^24 (see group_dots)
            a_g = qa[:, g * GROUP:(g + 1) * GROUP].astype(np.float32)
            w_g = qw[:, g * GROUP:(g + 1) * GROUP].astype(np.float32)
            d = a_g @ w_g.T
        if sw.ndim == 2:
            scale = (sa[:, g][:, None] * sw[:, g][None, :]).astype(np.float32)
        else:
            scale = np.broadcast_to(sa[:, g][:, None], (m, n)).astype(np.float32)
        total = fma_f32(d, scale, total)
    if sw.ndim == 1:
        total = (total * sw[None, :]).astype(np.float32)
    return total


def grouped_gemm_bf16_bits(qa, qw, sa_f32, sw_f32) -> np.ndarray:
    return f32_to_bf16_bits(grouped_gemm_f32(qa, qw, sa_f32, sw_f32))


def w4a4_linear(x_bf16_bits, signs, w_packed, w_scale_bits, layout=LAYOUT_BLOCK128, clamp_lo=-8,
                w_codes=None):
    """Whole W4A4Linear forward (linear_w4a4.py:27-36): prep + grouped GEMM, BF16 bits out.

    ``w_codes`` (the unpacked weight codes) may be passed to skip unpacking.
    """
    packed, sbits, codes, _, _ = prepare(x_bf16_bits, signs, layout, clamp_lo)
    qw = unpack_int4(w_packed) if w_codes is None else w_codes
    return grouped_gemm_bf16_bits(codes, qw, bf16_bits_to_f32(sbits), bf16_bits_to_f32(w_scale_bits))


# ---------------------------------------------------------------- W4A16
def w4a16_unpack(qweight: np.ndarray, qzeros: np.ndarray):
    """GPTQ layouts (linear_w4a16.py:44-50): qweight int32 [K/8, N] packs k%8 at
    bits 4*(k%8); qzeros int32 [K/128, N/8] packs n%8 at bits 4*(n%8)."""
    qw = np.asarray(qweight).view(np.uint32)
    k8, n = qw.shape
    shifts = (4 * np.arange(8, dtype=np.uint32))[None, :, None]
    w = ((qw[:, None, :] >> shifts) & 15).reshape(k8 * 8, n).astype(np.int32)
    qz = np.asarray(qzeros).view(np.uint32)
    g, n8 = qz.shape
    z = ((qz[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))[None, None, :]) & 15).reshape(g, n8 * 8)
    return w, z.astype(np.int32)


def w4a16_dequant(qweight, qzeros, scales_f16, group_size: int = 128) -> np.ndarray:
    """Dequantized BF16 weights [K, N] as float32 values (linear_w4a16.py:45-55)."""
    w, z = w4a16_unpack(qweight, qzeros)
    k, n = w.shape
    zz = np.repeat(z, group_size, axis=0)
    code = (w + 15 - zz).astype(np.uint16) | np.uint16(0x4300)
    val = bf16_bits_to_f32(code) - np.float32(144.0)       # exact: w - z - 1
    s = np.repeat(f16_to_bf16_f32(scales_f16), group_size, axis=0)
    return round_to_bf16((val * s).astype(np.float32))


def w4a16_gemm_f64(x_bf16_bits, qweight, qzeros, scales_f16) -> np.ndarray:
    """float64 product of BF16 X and the exactly dequantized BF16 weights."""
    x = bf16_bits_to_f32(x_bf16_bits).astype(np.float64)
    w = w4a16_dequant(qweight, qzeros, scales_f16).astype(np.float64)
    return x @ w
