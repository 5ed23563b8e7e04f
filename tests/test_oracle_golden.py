"""Pin the CPU oracle to the reference: known-answer tests and golden fixtures.

The fixtures in tests/golden were produced by the reference's own PyTorch
code (tests/golden/make_golden.py); here the oracle must reproduce every one
of them, so that the GPU parity tests, which compare against the oracle, are
anchored to the reference.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

import cases
from oracle import nv4_oracle as o

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def test_kat_impulses_match_reference():
    kat = np.load(os.path.join(GOLDEN, "kat.npz"))
    # K=4096: (-1)^popcount(j & 5) / 64 (bench_rht_a4.py:27-29)
    x = np.zeros((1, 4096), np.float32)
    x[0, 5] = 1
    got = o.rotate_row_dh(x, np.ones(4096, np.int8))[0]
    expected = np.array([(-1) ** bin(j & 5).count("1") / 64 for j in range(4096)])
    np.testing.assert_array_equal(got, expected.astype(np.float32))
    np.testing.assert_allclose(got, kat["impulse_k4096_i5"], rtol=0, atol=1e-12)
    # K=12288, impulse at 1024: Paley row 1 repeated per 1024 block (bench_rht_a4.py:31-34)
    x = np.zeros((1, 12288), np.float32)
    x[0, 1024] = 1
    got = o.rotate_row_dh(x, np.ones(12288, np.int8))[0]
    residues = {i * i % 11 for i in range(1, 11)}
    row = [1] + [(-1 if j == 0 else 1 if j in residues else -1) for j in range(11)]
    expected = np.repeat(np.array(row, np.float64), 1024) / math.sqrt(12288)
    np.testing.assert_allclose(got, expected, rtol=2e-7, atol=0)
    np.testing.assert_allclose(got, kat["impulse_k12288_i1024"], rtol=2e-7, atol=0)


@pytest.mark.parametrize("layout", [o.LAYOUT_BLOCK128, o.LAYOUT_ROW_DH])
def test_kat_quantizer(layout):
    kat = np.load(os.path.join(GOLDEN, "kat.npz"))
    for name in ("ties", "bf16first", "zero", "tiny"):
        values = kat[f"{name}_values"].astype(np.float32)
        codes, scale, _ = o.quantize(values, layout, clamp_lo=-7)
        np.testing.assert_array_equal(codes, kat[f"{name}_codes"].astype(np.int8).reshape(codes.shape),
                                      err_msg=name)
        np.testing.assert_array_equal(scale, kat[f"{name}_scale"].astype(np.float32).reshape(scale.shape),
                                      err_msg=name)
    # the tie row rounds half to even and clamps: -7.5 -> -7 only with clamp -7
    codes, _, _ = o.quantize(kat["ties_values"].astype(np.float32), layout, clamp_lo=-8)
    assert codes[0, :10].tolist() == [-8, -6, -4, -2, 0, 0, 2, 4, 6, 8 - 1]


def test_kat_packed_bytes():
    kat = np.load(os.path.join(GOLDEN, "kat.npz"))
    packed = o.pack_int4(kat["pack_codes"].astype(np.int8))
    assert packed.flatten().tolist() == [0x98, 0xBA, 0xDC, 0xFE, 0x10, 0x32, 0x54, 0x76]
    np.testing.assert_array_equal(packed, kat["pack_bytes"])
    np.testing.assert_array_equal(o.unpack_int4(packed), kat["pack_codes"])


def _prep_cases():
    out = []
    for kind, k, m in cases.ROWDH_CASES:
        out.append(("rowdh", kind, k, m, -7))
    for kind, k, m in cases.BLOCK128_CASES:
        for lo in (-8, -7):
            out.append((f"block128c{-lo}", kind, k, m, lo))
    return out


@pytest.mark.parametrize("lname,kind,k,m,lo", _prep_cases())
def test_prep_fixtures(lname, kind, k, m, lo, manifest):
    data = np.load(os.path.join(GOLDEN, "prep.npz"))
    key = cases.case_key(lname, kind, k, m)
    x, signs = cases.prep_case(kind, k, m)
    assert cases.sha(x, signs) == manifest["hashes"][key], "regenerated inputs differ from the fixture's"
    layout = o.LAYOUT_ROW_DH if lname == "rowdh" else o.LAYOUT_BLOCK128
    packed, sbits, codes, _, _ = o.prepare(u16(x), signs.numpy(), layout, lo)
    ref_codes = o.unpack_int4(data[key + "_packed"])
    near = np.unpackbits(data[key + "_near"])[: m * k].reshape(m, k).astype(bool)
    mismatch = codes != ref_codes
    assert not (mismatch & ~near).any(), "code differs away from a rounding boundary"
    assert mismatch.mean() <= 1e-4
    np.testing.assert_array_equal(sbits, data[key + "_scale"])


@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("m,n,k", cases.GEMM_SHAPES)
def test_gemm_fixtures(m, n, k, grouped, manifest):
    data = np.load(os.path.join(GOLDEN, "gemm.npz"))
    key = cases.gemm_key(m, n, k, grouped)
    qa, qw, sa, sw = cases.gemm_case(m, n, k, grouped)
    assert cases.sha(qa, qw, sa, sw) == manifest["hashes"][key]
    out = o.grouped_gemm_f32(qa.numpy(), qw.numpy(), sa.float().numpy(), sw.float().numpy())
    np.testing.assert_array_equal(out, data[key + "_f32"])
    np.testing.assert_array_equal(o.f32_to_bf16_bits(out), data[key + "_bf16"])
    precise = data[key + "_f64"]
    rrmse = np.sqrt(np.mean((out.astype(np.float64) - precise) ** 2)) / max(np.sqrt(np.mean(precise ** 2)), 1e-20)
    assert rrmse < 2e-6


def test_config0_chain(manifest):
    data = np.load(os.path.join(GOLDEN, "config0.npz"))
    x, signs, codes_w, packed_w, sw = cases.synthetic.config0(seed=0)
    assert cases.sha(x, signs, packed_w, sw) == manifest["hashes"]["config0"]
    packed, sbits, codes, _, _ = o.prepare(u16(x), signs.numpy(), o.LAYOUT_BLOCK128, -8)
    np.testing.assert_array_equal(packed, data["packed"])
    np.testing.assert_array_equal(sbits, data["scale"])
    out = o.w4a4_linear(u16(x), signs.numpy(), packed_w.numpy().view(np.uint8), u16(sw), o.LAYOUT_BLOCK128, -8)
    np.testing.assert_array_equal(out, data["out_bf16"])


def test_negative_control_detects_corrupt_code():
    """A corrupted code must be caught by the comparison (bench_rht_a4.py:142-152),
    planted in the oracle's output on the CPU."""
    data = np.load(os.path.join(GOLDEN, "prep.npz"))
    key = cases.case_key("block128c8", "input", 4096, 7)
    x, signs = cases.prep_case("input", 4096, 7)
    packed, _, _, _, _ = o.prepare(u16(x), signs.numpy(), o.LAYOUT_BLOCK128, -8)
    packed = packed.copy()
    packed[0, 0] ^= 1
    assert (o.unpack_int4(packed) != o.unpack_int4(data[key + "_packed"])).sum() == 1


def test_fma_emulation_is_exact():
    rng = np.random.default_rng(0)
    a = rng.integers(-8192, 8193, 200000).astype(np.float32)
    b = (rng.random(200000) * 1e-3).astype(np.float32)
    c = (rng.standard_normal(200000) * 10).astype(np.float32)
    got = o.fma_f32(a, b, c)
    from fractions import Fraction
    for i in range(0, 200000, 997):
        exact = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        r = np.float32(float(exact))       # double rounding possible: check neighbours
        cands = [np.nextafter(r, np.float32(-np.inf)), r, np.nextafter(r, np.float32(np.inf))]
        best = min(cands, key=lambda v: (abs(Fraction(float(v)) - exact), int(np.float32(v).view(np.uint32)) & 1))
        assert got[i] == best


def test_boundary_mask():
    q = np.array([2.5, np.nextafter(np.float32(2.5), np.float32(0)), 2.25, -3.5, 7.0], np.float32)
    assert o.boundary_mask(q, 1).tolist() == [True, True, False, True, False]


def test_w4a16_dequant_bit_trick():
    """bf16(0x4300 | (w+15-z)) - 144 == w - z - 1 for every nibble pair (linear_w4a16.py:52-53)."""
    w = np.repeat(np.arange(16), 16)
    z = np.tile(np.arange(16), 16)
    code = (w + 15 - z).astype(np.uint16) | np.uint16(0x4300)
    val = o.bf16_bits_to_f32(code) - np.float32(144)
    np.testing.assert_array_equal(val, (w - z - 1).astype(np.float32))


def test_w4a16_unpack_layout():
    from nanovllm.utils import synthetic
    qweight, qzeros, scales = synthetic.w4a16_weights(64, 256, seed=5)
    w, z = o.w4a16_unpack(qweight.numpy(), qzeros.numpy())
    g = torch.Generator().manual_seed(5 + 3)
    w_ref = torch.randint(0, 16, (256, 64), generator=g, dtype=torch.int64).numpy()
    z_ref = torch.randint(0, 16, (2, 64), generator=g, dtype=torch.int64).numpy()
    np.testing.assert_array_equal(w, w_ref)
    np.testing.assert_array_equal(z, z_ref)
