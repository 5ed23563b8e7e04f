"""GPU parity of the grouped INT4 GEMM.

BF16 outputs must equal the reference's sequential-FMA result bit for bit
(benchmarks/verify_w4a4_aw_grouped.py:170-177), the FP32 diagnostic output
must equal the FP32 reference exactly, the per-group INT32 dots must equal the
exact integer dots, and a constant dyadic scale must reduce to the ungrouped
product (verify_w4a4_grouped.py:75-79, verify_w4a4_aw_grouped.py:188-194).
"""
import json
import os

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import Guarded, u16
from nanovllm import _native
from nanovllm.kernels import w4a4_grouped_kernel as wk
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def pack(q):
    return synthetic.pack_int4(q)


def run_gemm(ap, wp, sa, sw, fp32=False, repeats=1):
    m, n = ap.shape[0], wp.shape[0]
    out = Guarded((m, n), torch.float32 if fp32 else torch.bfloat16, ap.device, -1234.0, float("nan"))
    for _ in range(repeats):
        out.view.fill_(float("nan"))
        ret = wk.w4a4_grouped_gemm(ap, wp, sa, sw, out=out.view, out_fp32=fp32)
        assert ret.data_ptr() == out.view.data_ptr()
        torch.cuda.synchronize()
        assert out.intact(), "kernel wrote outside its output"
    assert _native.device_error() == 0
    return out.view.cpu()


def oracle_out(qa, qw, sa, sw):
    return o.grouped_gemm_f32(qa.numpy(), qw.numpy(), sa.float().numpy(), sw.float().numpy())


@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("m,n,k", cases.GEMM_SHAPES)
def test_reference_shapes(cuda_device, m, n, k, grouped):
    data = np.load(os.path.join(GOLDEN, "gemm.npz"))
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        hashes = json.load(f)["hashes"]
    key = cases.gemm_key(m, n, k, grouped)
    qa, qw, sa, sw = cases.gemm_case(m, n, k, grouped)
    assert cases.sha(qa, qw, sa, sw) == hashes[key]
    d = cuda_device
    ap, wp, sad, swd = pack(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d)
    got = run_gemm(ap, wp, sad, swd, repeats=3)
    np.testing.assert_array_equal(u16(got), data[key + "_bf16"])
    got32 = run_gemm(ap, wp, sad, swd, fp32=True)
    np.testing.assert_array_equal(got32.numpy(), data[key + "_f32"])
    precise = data[key + "_f64"]
    rrmse = np.sqrt(np.mean((got32.numpy().astype(np.float64) - precise) ** 2)) / \
        max(np.sqrt(np.mean(precise ** 2)), 1e-20)
    assert rrmse < 2e-6
    # a constant dyadic activation scale reduces to the ungrouped integer product
    sad.fill_(0.125)
    expected = ((qa.float() @ qw.float().T) * 0.125)
    expected = expected * (sw.float()[None, :] if sw.ndim == 1 else 1.0)
    if sw.ndim == 1:
        got = wk.w4a4_grouped_gemm(ap, wp, sad, swd).cpu()
        assert torch.equal(got, expected.bfloat16())
    else:
        channel = torch.full((n,), 0.125, dtype=torch.bfloat16, device=d)
        repeated = channel[:, None].expand(n, k // 128).contiguous()
        a_only = o.grouped_gemm_f32(qa.numpy(), qw.numpy(), sa.float().numpy(), channel.float().cpu().numpy())
        sad.copy_(sa.to(d))
        got_c = wk.w4a4_grouped_gemm(ap, wp, sad, channel).cpu()
        got_r = wk.w4a4_grouped_gemm(ap, wp, sad, repeated).cpu()
        np.testing.assert_array_equal(u16(got_c), o.f32_to_bf16_bits(a_only))
        np.testing.assert_array_equal(u16(got_r), o.f32_to_bf16_bits(a_only))


@pytest.mark.parametrize("name", ["qkv", "o", "gate_up", "down"])
@pytest.mark.parametrize("m", [1, 8, 32])
def test_decode_shapes_exact(cuda_device, name, m):
    n, k = synthetic.QWEN3_8B_SHAPES[name]
    g = torch.Generator().manual_seed(m * 1000 + n)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    sa = (torch.rand(m, k // 128, generator=g) * 2).bfloat16()
    codes, packed_w, sw = synthetic.w4a4_weights(n, k, seed=m + n)
    got = run_gemm(pack(qa).to(cuda_device), packed_w.to(cuda_device), sa.to(cuda_device), sw.to(cuda_device))
    np.testing.assert_array_equal(u16(got), o.f32_to_bf16_bits(oracle_out(qa, codes, sa, sw)))


@pytest.mark.parametrize("m,n,k", [(5, 136, 4096), (33, 200, 1024), (100, 64, 2048), (512, 256, 4096),
                                   (1, 8, 128), (3, 24, 384)])
def test_tails_exact(cuda_device, m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    sa = (torch.rand(m, k // 128, generator=g) * 2).bfloat16()
    sw = (torch.rand(n, k // 128, generator=g) * .03).bfloat16()
    d = cuda_device
    got = run_gemm(pack(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d))
    np.testing.assert_array_equal(u16(got), o.f32_to_bf16_bits(oracle_out(qa, qw, sa, sw)))
    got32 = run_gemm(pack(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d), fp32=True)
    np.testing.assert_array_equal(got32.numpy(), oracle_out(qa, qw, sa, sw))


@pytest.mark.parametrize("m,n,k", [(17, 96, 512), (32, 128, 12288)])
def test_group_dots_exact(cuda_device, m, n, k):
    qa, qw, _, _ = cases.gemm_case(m, n, k, True)
    dots = wk.w4a4_group_dots(pack(qa).to(cuda_device), pack(qw).to(cuda_device)).cpu().numpy()
    np.testing.assert_array_equal(dots, o.group_dots(qa.numpy(), qw.numpy()))


def test_extreme_scales(cuda_device):
    """Scales at the BF16 extremes used by the quantizer (tiny groups, huge
    activations) keep the reference's FP32 semantics."""
    m, n, k = 16, 64, 1024
    g = torch.Generator().manual_seed(5)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    exps = torch.tensor([-126, -100, -60, -20, 0, 20, 60, 90], dtype=torch.float32)
    sa = torch.ldexp(torch.rand(m, k // 128, generator=g) + 1, exps[torch.arange(m * (k // 128)) % 8].reshape(m, -1))
    sa = sa.bfloat16()
    sw = (torch.rand(n, k // 128, generator=g) * .03).bfloat16()
    d = cuda_device
    got32 = run_gemm(pack(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d), fp32=True)
    np.testing.assert_array_equal(got32.numpy(), oracle_out(qa, qw, sa, sw))


@pytest.mark.parametrize("path", ["default", "mma_sync"])
@pytest.mark.parametrize("grouped", [True, False])
@pytest.mark.parametrize("m,n,k", [(1, 6144, 4096), (8, 4096, 4096), (32, 24576, 4096), (32, 4096, 12288),
                                   (17, 96, 512), (33, 136, 4096), (100, 64, 2048), (5, 24, 384),
                                   (128, 256, 4096), (300, 512, 1024), (1024, 384, 12288),
                                   (16, 30720, 1024), (3, 38016, 256), (24, 1000, 640),
                                   # 5-8 slabs per SM: one warp per slab with split token tiles
                                   # above 8 tokens, 4-slab CTAs (more CTAs than SMs) up to 8
                                   (32, 12288, 4096), (1, 12288, 4096), (12, 12288, 4096), (16, 4096, 4096)])
def test_i8_activation_gemm_exact(cuda_device, m, n, k, grouped, path):
    """nv4_w4a4_gemm_i8 (the path W4A4Linear uses) equals the oracle bit for bit
    on every kernel: the default dispatch (tcgen05 above 64 tokens, mma.sync
    below) and the mma.sync kernel forced."""
    from gpu_helpers import codes_to_i8_layout
    g = torch.Generator().manual_seed(m * 7 + n + k)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    sa = (torch.rand(m, k // 128, generator=g) * 2).bfloat16()
    sw = ((torch.rand(n, k // 128, generator=g) if grouped else torch.rand(n, generator=g)) * .03).bfloat16()
    d = cuda_device
    a8 = codes_to_i8_layout(qa).to(d)
    for fp32 in (False, True):
        out = Guarded((m, n), torch.float32 if fp32 else torch.bfloat16, d, -1234.0, float("nan"))
        wk.w4a4_grouped_gemm_i8(a8, pack(qw).to(d), sa.to(d), sw.to(d), out=out.view, out_fp32=fp32,
                                force_stream=path == "mma_sync")
        torch.cuda.synchronize()
        assert out.intact()
        ref = oracle_out(qa, qw, sa, sw)
        if fp32:
            np.testing.assert_array_equal(out.view.cpu().numpy(), ref)
        else:
            np.testing.assert_array_equal(u16(out.view), o.f32_to_bf16_bits(ref))
    assert _native.device_error() == 0


def test_i8_gemm_extreme_scales_use_exact_path(cuda_device):
    """Scales outside the two-FMA fast range take the reference's three-step form."""
    from gpu_helpers import codes_to_i8_layout
    m, n, k = 16, 64, 1024
    g = torch.Generator().manual_seed(9)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    exps = torch.tensor([-126, -110, -60, -20, 0, 20, 60, 105], dtype=torch.float32)
    sa = torch.ldexp(torch.rand(m, k // 128, generator=g) + 1,
                     exps[torch.arange(m * (k // 128)) % 8].reshape(m, -1)).bfloat16()
    sw = (torch.rand(n, k // 128, generator=g) * .03).bfloat16()
    sw[3, 2] = 2.0 ** -120
    d = cuda_device
    got = wk.w4a4_grouped_gemm_i8(codes_to_i8_layout(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d),
                                  out_fp32=True).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_out(qa, qw, sa, sw))


@pytest.mark.parametrize("m", [512, 2048, 4096])
@pytest.mark.parametrize("n,k", [(6144, 4096), (4096, 4096), (24576, 4096), (4096, 12288)])
def test_prefill_config2_shapes_sampled(cuda_device, m, n, k):
    """BASELINE config 2 at its real shapes on the tcgen05 kernel (the default
    dispatch above 64 tokens): the full GEMM runs on the GPU, and a seeded
    sample of 16 token rows x 512 weight columns is checked bit for bit
    against the oracle (rows and columns of the GEMM are independent)."""
    from gpu_helpers import codes_to_i8_layout
    d = cuda_device
    g = torch.Generator(device=d).manual_seed(m + n + k)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8, device=d)
    wp = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8, device=d)
    sa = (torch.rand(m, k // 128, generator=g, device=d) * 2 + 0.01).bfloat16()
    sw = (torch.rand(n, k // 128, generator=g, device=d) * .03 + 1e-4).bfloat16()
    out = Guarded((m, n), torch.bfloat16, d, -1234.0, float("nan"))
    wk.w4a4_grouped_gemm_i8(codes_to_i8_layout(qa), wp, sa, sw, out=out.view)
    torch.cuda.synchronize()
    assert out.intact() and _native.device_error() == 0
    gs = torch.Generator().manual_seed(m * n)
    rows = torch.randperm(m, generator=gs)[:16].sort().values
    cols = torch.randperm(n, generator=gs)[:512].sort().values
    qw = synthetic.unpack_int4(wp[cols.to(d)].cpu())
    ref = oracle_out(qa[rows.to(d)].cpu(), qw, sa[rows.to(d)].cpu(), sw[cols.to(d)].cpu())
    got = out.view[rows.to(d)][:, cols.to(d)]
    np.testing.assert_array_equal(u16(got), o.f32_to_bf16_bits(ref))
    assert not torch.isnan(out.view.float()).any()  # every element written


@pytest.mark.parametrize("grouped", [True, False])
def test_tc_extreme_scales_take_exact_path(cuda_device, grouped):
    """Above 64 tokens (the tcgen05 kernel): scale blocks with a scale outside
    the two-FMA range use the reference's three-step form, others the fast one,
    in one launch."""
    from gpu_helpers import codes_to_i8_layout
    m, n, k = 200, 384, 2048
    g = torch.Generator().manual_seed(13)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    sa = (torch.rand(m, k // 128, generator=g) * 2).bfloat16()
    sa[7, 3] = 2.0 ** -110      # group 3: slow for the tile holding token 7
    sa[150, 12] = 2.0 ** 100    # group 12: slow for the tile holding token 150
    sw = ((torch.rand(n, k // 128, generator=g) if grouped else torch.rand(n, generator=g)) * .03).bfloat16()
    if grouped:
        sw[300, 9] = 2.0 ** -120
    d = cuda_device
    got = wk.w4a4_grouped_gemm_i8(codes_to_i8_layout(qa).to(d), pack(qw).to(d), sa.to(d), sw.to(d),
                                  out_fp32=True).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_out(qa, qw, sa, sw))
    assert _native.device_error() == 0
