"""The arithmetic shortcuts of the activation-prep kernel (csrc/rht_quant.cu),
checked on the host against exactly rounded results -- no GPU needed.

* div_sqrt128: x / fl32(sqrt(128)) as q0 = RN(x * r), q1 = RN(q0 + RN(x - q0*d) * r)
  with r = RN(1/d) and fused multiply-adds.  It must equal the IEEE quotient for
  every float32 significand (checked exhaustively) at every exponent the kernel
  uses it for (|x| >= 2^-100; smaller values take the IEEE division).
* quant_code: round-half-even(RN(v / s)) from q = RN(v * RN(1/s)) when q is at
  least 2^-17 away from a half-integer, for |v / s| < 7.82 (what the group
  scale guarantees); the kernel takes the IEEE quotient inside that margin.

Every float32 operation is emulated exactly in float64 (products of two
float32 values are exact there); sums that float64 could round, and ties, are
settled with rational arithmetic.
"""
from fractions import Fraction

import numpy as np

D = np.float32(float.fromhex("0x1.6a09e6p+3"))    # fl32(sqrt(128))
R = np.float32(float.fromhex("0x1.6a09e6p-4"))    # RN(1 / D)
MID = 1 << 28                                     # float64 low bits of an exact float32 midpoint
LOW = (1 << 29) - 1


def rn32_of_exact(values):
    """Round exact rationals (Fractions) to float32, ties to even."""
    out = np.empty(len(values), dtype=np.float32)
    for i, ex in enumerate(values):
        near = np.float32(float(ex))
        cands = [np.nextafter(near, np.float32(-np.inf)), near, np.nextafter(near, np.float32(np.inf))]
        out[i] = min(cands, key=lambda t: (abs(Fraction(float(t)) - ex), int(np.float32(t).view(np.int32)) & 1))
    return out


def rn32_sum(a, b):
    """RN32(a + b) for exact float64 arrays a, b (TwoSum; rationals at float32 midpoints)."""
    s = a + b
    bb = s - a
    err = (a - (s - bb)) + (b - bb)
    c = s.astype(np.float32)
    fix = np.nonzero(((s.view(np.int64) & LOW) == MID) & (err != 0))[0]
    if len(fix):
        c[fix] = rn32_of_exact([Fraction(float(a[i])) + Fraction(float(b[i])) for i in fix])
    return c


def rn32_quotient(x, d):
    """RN32(x / d) exactly for float32 arrays."""
    y = x.astype(np.float64) / np.float64(d)
    q = y.astype(np.float32)
    near = np.nonzero(np.abs((y.view(np.int64) & LOW) - MID) < 8)[0]
    if len(near):
        q[near] = rn32_of_exact([Fraction(float(x[i])) / Fraction(float(d if np.ndim(d) == 0 else d[i])) for i in near])
    return q


def div_sqrt128_emulated(x):
    x64 = x.astype(np.float64)
    q0 = (x64 * np.float64(R)).astype(np.float32)
    e = (x64 - q0.astype(np.float64) * np.float64(D)).astype(np.float32)   # exact residual, one rounding
    return rn32_sum(q0.astype(np.float64), e.astype(np.float64) * np.float64(R))


def test_reciprocal_constant_is_nearest():
    exact = Fraction(1) / Fraction(float(D))
    neighbours = [np.nextafter(R, np.float32(0)), np.nextafter(R, np.float32(1))]
    assert all(abs(Fraction(float(R)) - exact) < abs(Fraction(float(t)) - exact) for t in neighbours)


def test_div_sqrt128_every_significand():
    mant = np.arange(1 << 23, dtype=np.int64)
    x = ((np.int64(127) << 23) | mant).astype(np.int32).view(np.float32)   # all of [1, 2)
    got = div_sqrt128_emulated(x)
    ref = rn32_quotient(x, D)
    assert np.array_equal(got.view(np.int32), ref.view(np.int32))


def test_div_sqrt128_across_exponents():
    rng = np.random.default_rng(0)
    for e2 in range(-100, 128):
        m = rng.integers(0, 1 << 23, 4000)
        x = (((e2 + 127) << 23) | m).astype(np.int32).view(np.float32)
        x = np.concatenate([x, -x])
        got = div_sqrt128_emulated(x)
        assert np.array_equal(got.view(np.int32), rn32_quotient(x, D).view(np.int32)), e2


def quant_fast(v, s):
    """Emulation of quant_code's fast path: (code, needs_ieee_fallback)."""
    rs = rn32_of_exact([Fraction(1) / Fraction(float(t)) for t in np.unique(s)])
    table = dict(zip(np.unique(s).tolist(), rs.tolist()))
    r = np.array([table[t] for t in s.tolist()], dtype=np.float32)
    q = (v.astype(np.float64) * r.astype(np.float64)).astype(np.float32)
    k = np.rint(q)
    near = np.abs(np.abs(q - k) - np.float32(0.5)) < np.float32(2.0 ** -17)
    return k, near


def test_quant_code_shortcut_matches_rounded_quotient():
    rng = np.random.default_rng(1)
    n = 200000
    # BF16 scales over a wide exponent range and values with |v / s| < 7.82
    s = (rng.uniform(1, 2, n) * 2.0 ** rng.integers(-60, 60, n)).astype(np.float32)
    s = (s.view(np.uint32) & 0xFFFF0000).view(np.float32)
    ratio = rng.uniform(-7.82, 7.82, n)
    # adversarial quarter: quotients within a few float32 ulps of a half-integer
    half = rng.integers(-8, 8, n // 4) + 0.5
    ratio[: n // 4] = half * (1 + rng.integers(-64, 65, n // 4) * 2.0 ** -24)
    v = (ratio * s.astype(np.float64)).astype(np.float32)
    keep = np.abs(v.astype(np.float64) / s) < 7.82
    v, s = v[keep], s[keep]
    k, near = quant_fast(v, s)
    ref = np.rint(rn32_quotient(v, s))
    assert np.array_equal(k[~near], ref[~near])
    assert near.sum() > 0        # the adversarial cases reach the IEEE fallback


def test_silu_mul_oracle_cpu():
    """The oracle's SiluAndMul restatement (FP32 silu and product, one BF16
    rounding) against torch's FP32 arithmetic on the CPU: equal within one BF16
    ulp (numpy's exp and torch's may differ in the last FP32 bit), with the
    exact special cases g = 0 -> 0 and a saturated silu(g) = g for large g."""
    import torch
    from oracle import nv4_oracle as o
    g = torch.Generator().manual_seed(0)
    gu = (torch.randn(16, 2 * 512, generator=g) * 3.0).bfloat16()
    gu[0, :4] = torch.tensor([0.0, 40.0, -40.0, -100.0]).bfloat16()
    gu[0, 512:516] = torch.tensor([3.0, 2.0, 5.0, 1.0]).bfloat16()
    bits = gu.view(torch.int16).numpy().view(np.uint16)
    got = o.silu_mul_bf16_bits(bits)
    gf, uf = gu[:, :512].float(), gu[:, 512:].float()
    want = ((gf / (1.0 + torch.exp(-gf))) * uf).bfloat16().view(torch.int16).numpy().view(np.uint16)
    diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.995
    vals = o.bf16_bits_to_f32(got[0, :4])
    assert vals[0] == 0.0 and vals[1] == 80.0 and vals[2] <= 0.0 and abs(vals[3]) == 0.0
