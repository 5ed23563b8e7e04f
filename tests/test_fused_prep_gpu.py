"""GPU parity of the preps fused with their producers.

SiluAndMul (nanovllm/layers/activation.py:8-11) into the down projection's prep: ``silu_mul_rht_quant_i8(gate_up)`` must
equal ``rht_quant_i8`` of the BF16 activation bf16(silu(g) * u) computed in
FP32 by torch on the same device (g / (1 + exp(-g)), IEEE division, one product
rounding) -- codes and scales bit for bit -- for both layouts, decode and
prefill row counts, in place, with nothing written outside the outputs and the
input unchanged, and under CUDA-graph replay.  The CPU oracle's restatement of
the activation agrees within one BF16 ulp (numpy's exp is not CUDA's expf).

Residual add + RMSNorm (nanovllm/layers/layernorm.py:33-45) into the QKV /
gate-up prep: the new residual equals bf16(x + residual) bit for bit; the codes
and scales equal the unfused prep of the kernel's own normalized activation
bit for bit; that activation equals torch's FP32 RMSNorm within two BF16 ulps (the sum
of squares is reduced in a different order, and two roundings follow) and
exactly in almost every element; the layer method equals the plain layer on that activation."""
import numpy as np
import pytest
import torch

from gpu_helpers import Guarded, u16
from nanovllm import _native
from nanovllm.kernels.rht_a4_tilelang import add_rmsnorm_rht_quant_i8, rht_quant_i8, silu_mul_rht_quant_i8
from nanovllm.layers.linear_w4a4 import W4A4Linear
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o

pytestmark = pytest.mark.gpu


def gate_up_input(m, k, seed):
    """BF16 [m, 2k]: N(0, 1.5) with some large magnitudes, so silu's tails
    (exp overflow for g << 0, silu(g) ~ g for g >> 0) are exercised."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, 2 * k, generator=g) * 1.5
    idx = torch.randint(0, 2 * k, (m, 8), generator=g)
    x.scatter_(1, idx, torch.randn(m, 8, generator=g) * 60.0)
    return x.bfloat16()


def torch_silu_mul(gate_up):
    k = gate_up.shape[1] // 2
    g, u = gate_up[:, :k].float(), gate_up[:, k:].float()
    return ((g / (1.0 + torch.exp(-g))) * u).bfloat16()


def fused(gate_up, signs, layout, lo):
    m, k = gate_up.shape[0], gate_up.shape[1] // 2
    codes = Guarded((m, k), torch.int8, gate_up.device, -69, 85)
    scale = Guarded((m, k // 128), torch.bfloat16, gate_up.device, -17.0, float("nan"))
    before = gate_up.clone()
    ret = silu_mul_rht_quant_i8(gate_up, signs, out_codes=codes.view, out_scale=scale.view, layout=layout,
                                clamp_lo=lo)
    torch.cuda.synchronize()
    assert ret[0].data_ptr() == codes.view.data_ptr() and ret[1].data_ptr() == scale.view.data_ptr()
    assert codes.intact() and scale.intact(), "kernel wrote outside its outputs"
    assert torch.equal(gate_up, before), "kernel modified its input"
    assert _native.device_error() == 0
    return codes.view, scale.view


def unfused(h, signs, layout, lo):
    m, k = h.shape
    codes = torch.empty(m, k, dtype=torch.int8, device=h.device)
    scale = torch.empty(m, k // 128, dtype=torch.bfloat16, device=h.device)
    rht_quant_i8(h, signs, out_codes=codes, out_scale=scale, layout=layout, clamp_lo=lo)
    return codes, scale


@pytest.mark.parametrize("layout,lo", [("block128", -8), ("row_DH_paley12_kron_sylvester_v1", -7)])
@pytest.mark.parametrize("k", [4096, 12288])
@pytest.mark.parametrize("m", [1, 7, 32, 33, 300])
def test_fused_equals_unfused(cuda_device, layout, lo, k, m):
    gu = gate_up_input(m, k, seed=m * 7 + k).to(cuda_device)
    signs = synthetic.make_signs(k, 20261108 + k).to(cuda_device)
    codes, scale = fused(gu, signs, layout, lo)
    ref_codes, ref_scale = unfused(torch_silu_mul(gu), signs, layout, lo)
    assert torch.equal(codes, ref_codes), f"{int((codes != ref_codes).sum())} codes differ"
    assert torch.equal(scale.view(torch.int16), ref_scale.view(torch.int16))


def test_activation_matches_cpu_oracle(cuda_device):
    gu = gate_up_input(64, 4096, seed=3)
    h_gpu = u16(torch_silu_mul(gu.to(cuda_device)))
    h_cpu = o.silu_mul_bf16_bits(u16(gu))
    diff = np.abs(h_gpu.astype(np.int32) - h_cpu.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.999


def test_layer_forward_silu_mul(cuda_device):
    k, n, m = 12288, 4096, 32
    lin = W4A4Linear(k, n, layout="block128", clamp_lo=-8).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    lin.load_full(torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=cuda_device, generator=g),
                  (torch.rand(n, k // 128, device=cuda_device, generator=g) * 0.003 + 1e-4).bfloat16(),
                  synthetic.make_signs(k, 9).to(cuda_device))
    gu = gate_up_input(m, k, seed=11).to(cuda_device)
    assert torch.equal(lin.forward_silu_mul(gu), lin(torch_silu_mul(gu)))
    # graph replay reads the updated input
    out = lin.forward_silu_mul(gu)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = lin.forward_silu_mul(gu)
    for seed in (12, 13):
        gu.copy_(gate_up_input(m, k, seed=seed).to(cuda_device))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, lin(torch_silu_mul(gu))), seed
    del graph
    assert _native.device_error() == 0


def test_argument_errors(cuda_device):
    gu = gate_up_input(4, 4096, seed=1).to(cuda_device)
    signs = synthetic.make_signs(4096, 1).to(cuda_device)
    codes = torch.empty(4, 4096, dtype=torch.int8, device=cuda_device)
    scale = torch.empty(4, 32, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        silu_mul_rht_quant_i8(gu[:, :-1], signs, out_codes=codes, out_scale=scale)
    with pytest.raises(ValueError):
        silu_mul_rht_quant_i8(gu.float(), signs, out_codes=codes, out_scale=scale)
    with pytest.raises(ValueError):
        silu_mul_rht_quant_i8(gu, signs[:-1], out_codes=codes, out_scale=scale)
    with pytest.raises(ValueError):
        silu_mul_rht_quant_i8(gu, signs, out_codes=codes[:, :-1], out_scale=scale)


def torch_rmsnorm(x, residual, weight, eps):
    xf = x.float() if residual is None else x.float() + residual.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    return ((xf * torch.rsqrt(var + eps)).bfloat16().float() * weight.float()).bfloat16(), xf.bfloat16()


def norm_inputs(m, k, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 0.7).bfloat16().to(dev)
    res = (torch.randn(m, k, generator=g) * 3.0).bfloat16().to(dev)
    w = (1.0 + 0.2 * torch.randn(k, generator=g)).bfloat16().to(dev)
    return x, res, w


@pytest.mark.parametrize("layout,lo,k", [("block128", -8, 4096), ("block128", -8, 12288),
                                         ("row_DH_paley12_kron_sylvester_v1", -7, 4096)])
@pytest.mark.parametrize("m", [1, 7, 32, 33, 300])
@pytest.mark.parametrize("with_residual", [True, False])
def test_add_rmsnorm_fused(cuda_device, layout, lo, k, m, with_residual):
    x, res, w = norm_inputs(m, k, seed=m * 3 + k, dev=cuda_device)
    if not with_residual:
        res = None
    signs = synthetic.make_signs(k, 20261108 + k).to(cuda_device)
    codes = Guarded((m, k), torch.int8, cuda_device, -69, 85)
    scale = Guarded((m, k // 128), torch.bfloat16, cuda_device, -17.0, float("nan"))
    normed = Guarded((m, k), torch.bfloat16, cuda_device, -5.0, float("nan"))
    new_res = Guarded((m, k), torch.bfloat16, cuda_device, -7.0, float("nan")) if with_residual else None
    before = [t.clone() for t in (x, w) + ((res,) if with_residual else ())]
    add_rmsnorm_rht_quant_i8(x, res, w, 1e-6, signs, out_codes=codes.view, out_scale=scale.view,
                             out_residual=None if new_res is None else new_res.view, out_normed=normed.view,
                             layout=layout, clamp_lo=lo)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    for g in (codes, scale, normed) + ((new_res,) if with_residual else ()):
        assert g.intact(), "kernel wrote outside its outputs"
    after = [x, w] + ([res] if with_residual else [])
    assert all(torch.equal(a, b) for a, b in zip(before, after)), "kernel modified an input"
    want_h, want_res = torch_rmsnorm(x, res, w, 1e-6)
    if with_residual:
        assert torch.equal(new_res.view.view(torch.int16), want_res.view(torch.int16))
    hd = (normed.view.view(torch.int16).int() - want_h.view(torch.int16).int()).abs()
    # var reduced in another order can move bf16(xf * r) by one ulp, and the
    # second rounding (times the weight) can make that two
    assert int(hd.max()) <= 2 and float((hd == 0).float().mean()) > 0.99
    ref_codes, ref_scale = unfused(normed.view, signs, layout, lo)
    assert torch.equal(codes.view, ref_codes)
    assert torch.equal(scale.view.view(torch.int16), ref_scale.view(torch.int16))


def test_layer_forward_add_rmsnorm(cuda_device):
    k, n, m = 4096, 6144, 32
    lin = W4A4Linear(k, n, layout="block128", clamp_lo=-8).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    lin.load_full(torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=cuda_device, generator=g),
                  (torch.rand(n, k // 128, device=cuda_device, generator=g) * 0.003 + 1e-4).bfloat16(),
                  synthetic.make_signs(k, 9).to(cuda_device))
    x, res, w = norm_inputs(m, k, seed=21, dev=cuda_device)
    out, new_res = lin.forward_add_rmsnorm(x, res, w, 1e-6)
    normed = torch.empty_like(x)
    codes = torch.empty(m, k, dtype=torch.int8, device=cuda_device)
    scale = torch.empty(m, k // 128, dtype=torch.bfloat16, device=cuda_device)
    add_rmsnorm_rht_quant_i8(x, res, w, 1e-6, lin.signs, out_codes=codes, out_scale=scale,
                             out_residual=torch.empty_like(x), out_normed=normed, layout="block128", clamp_lo=-8)
    assert torch.equal(out, lin(normed))
    assert torch.equal(new_res, (x.float() + res.float()).bfloat16())
    out2, same = lin.forward_add_rmsnorm(x, None, w, 1e-6)
    assert same is x and out2.shape == (m, n)
    assert _native.device_error() == 0


def test_add_rmsnorm_argument_errors(cuda_device):
    x, res, w = norm_inputs(4, 4096, seed=1, dev=cuda_device)
    signs = synthetic.make_signs(4096, 1).to(cuda_device)
    codes = torch.empty(4, 4096, dtype=torch.int8, device=cuda_device)
    scale = torch.empty(4, 32, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):  # a residual without a place for the new residual
        add_rmsnorm_rht_quant_i8(x, res, w, 1e-6, signs, out_codes=codes, out_scale=scale)
    with pytest.raises(ValueError):
        add_rmsnorm_rht_quant_i8(x, None, w[:-1], 1e-6, signs, out_codes=codes, out_scale=scale)
    with pytest.raises(ValueError):  # row_DH takes K = 4096 only
        x2 = torch.zeros(4, 12288, dtype=torch.bfloat16, device=cuda_device)
        add_rmsnorm_rht_quant_i8(x2, None, torch.ones(12288, dtype=torch.bfloat16, device=cuda_device), 1e-6,
                                 synthetic.make_signs(12288, 1).to(cuda_device),
                                 out_codes=torch.empty(4, 12288, dtype=torch.int8, device=cuda_device),
                                 out_scale=torch.empty(4, 96, dtype=torch.bfloat16, device=cuda_device),
                                 layout="row_DH")
