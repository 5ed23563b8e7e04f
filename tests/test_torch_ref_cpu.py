"""The timed CPU baseline (oracle/torch_ref.py, the reference's PyTorch path
restated in torch) computes what the bit-exact numpy oracle computes."""
import numpy as np
import torch

from nanovllm.utils import synthetic
from oracle import nv4_oracle as o
from oracle import torch_ref


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_w4a4_linear_matches_oracle():
    x, signs, codes, packed, scale = synthetic.config0(seed=5, m=8, k=1024, n=256)
    got = torch_ref.w4a4_linear(x, signs, codes, scale, clamp_lo=-8)
    want = o.w4a4_linear(_bits(x), signs.numpy(), packed.numpy().view(np.uint8), _bits(scale),
                         o.LAYOUT_BLOCK128, -8, w_codes=codes.numpy())
    assert np.array_equal(_bits(got), want)


def test_prep_matches_oracle_codes_and_scales():
    x = synthetic.make_input(33, 1024)
    signs = synthetic.make_signs(1024, 7)
    codes, scale = torch_ref.quantize_rotated(torch_ref.rotate_block128(x, signs), -8)
    want_packed, want_scale, want_codes = o.prepare(_bits(x), signs.numpy(), o.LAYOUT_BLOCK128, -8)[:3]
    assert np.array_equal(codes.numpy(), want_codes)
    assert np.array_equal(_bits(scale), want_scale)
    packed = torch_ref.pack_int4(codes)
    assert np.array_equal(packed.numpy().view(np.uint8), want_packed)


def test_producers_close_to_oracle():
    g = torch.Generator().manual_seed(3)
    gu = torch.randn(4, 512, generator=g).bfloat16()
    got = torch_ref.silu_mul(gu).float().numpy()
    want = o.bf16_bits_to_f32(o.silu_mul_bf16_bits(_bits(gu)))
    assert np.allclose(got, want, rtol=1e-2, atol=1e-6)
    x = torch.randn(4, 256, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(256, generator=g)).bfloat16()
    h, res = torch_ref.add_rmsnorm(x, x, w, 1e-6)
    want_h, want_res = o.add_rmsnorm_bf16_bits(_bits(x), _bits(x), _bits(w), 1e-6)
    assert np.array_equal(_bits(res), want_res)
    assert np.allclose(h.float().numpy(), o.bf16_bits_to_f32(want_h), rtol=2e-2, atol=1e-6)
