"""GPU parity of the down projection's prep fused with its producer, SiluAndMul
(nanovllm/layers/activation.py:8-11): ``silu_mul_rht_quant_i8(gate_up)`` must
equal ``rht_quant_i8`` of the BF16 activation bf16(silu(g) * u) computed in
FP32 by torch on the same device (g / (1 + exp(-g)), IEEE division, one product
rounding) -- codes and scales bit for bit -- for both layouts, decode and
prefill row counts, in place, with nothing written outside the outputs and the
input unchanged, and under CUDA-graph replay.  The CPU oracle's restatement of
the activation agrees within one BF16 ulp (numpy's exp is not CUDA's expf)."""
import numpy as np
import pytest
import torch

from gpu_helpers import Guarded, u16
from nanovllm import _native
from nanovllm.kernels.rht_a4_tilelang import rht_quant_i8, silu_mul_rht_quant_i8
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
