"""GPU parity of the linear modules (W4A4Linear, its TP shards, W4A16Linear) and
their CUDA-graph capture at the decode batch sizes the model runner uses."""
import os

import numpy as np
import pytest
import torch

from gpu_helpers import u16
from nanovllm import _native
from nanovllm.layers.linear_w4a16 import W4A16Linear
from nanovllm.layers.linear_w4a4 import (W4A4ColumnParallelLinear, W4A4Linear, W4A4MergedColumnParallelLinear,
                                         W4A4QKVParallelLinear, W4A4RowParallelLinear)
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def make_linear(cls_kw, n, k, seed, device, layout, lo):
    codes, packed, scale = synthetic.w4a4_weights(n, k, seed)
    signs = synthetic.make_signs(k, seed)
    layer = W4A4Linear(k, n, layout=layout, clamp_lo=lo).to(device)
    layer.load_full(packed.to(device), scale.to(device), signs.to(device))
    return layer, packed, scale, signs


@pytest.mark.parametrize("layout,lo", [("block128", -8), ("row_DH", -7)])
@pytest.mark.parametrize("name", ["qkv", "o", "gate_up", "down"])
def test_w4a4_linear_matches_oracle(cuda_device, layout, lo, name):
    n, k = synthetic.QWEN3_8B_SHAPES[name]
    layer, packed, scale, signs = make_linear(None, n, k, 21, cuda_device, layout, lo)
    x = synthetic.activations(32, k, seed=5)
    got = layer(x.to(cuda_device).reshape(4, 8, k)).reshape(32, n)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    lid = o.LAYOUT_BLOCK128 if layout == "block128" else o.LAYOUT_ROW_DH
    expected = o.w4a4_linear(u16(x), signs.numpy(), packed.numpy().view(np.uint8), u16(scale), lid, lo)
    np.testing.assert_array_equal(u16(got), expected)


def test_config0_golden(cuda_device):
    data = np.load(os.path.join(GOLDEN, "config0.npz"))
    x, signs, _, packed, sw = synthetic.config0(seed=0)
    layer = W4A4Linear(4096, 4096, layout="block128", clamp_lo=-8).to(cuda_device)
    layer.load_full(packed.to(cuda_device), sw.to(cuda_device), signs.to(cuda_device))
    got = layer(x.to(cuda_device))
    np.testing.assert_array_equal(u16(got), data["out_bf16"])


def test_cuda_graph_decode_batches(cuda_device):
    """Capture the layer for bs 32..1 in one graph pool (model_runner.py:250-265)
    and replay with new inputs."""
    n, k = synthetic.QWEN3_8B_SHAPES["qkv"]
    layer, packed, scale, signs = make_linear(None, n, k, 4, cuda_device, "block128", -8)
    xs = torch.zeros(32, k, dtype=torch.bfloat16, device=cuda_device)
    outs = torch.zeros(32, n, dtype=torch.bfloat16, device=cuda_device)
    graphs, pool = {}, None
    for bs in (32, 16, 8, 4, 2, 1):
        outs[:bs] = layer(xs[:bs])
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool):
            outs[:bs] = layer(xs[:bs])
        pool = g.pool() if pool is None else pool
        graphs[bs] = g
    torch.cuda.synchronize()
    for bs in (1, 2, 4, 8, 16, 32):
        x = synthetic.activations(bs, k, seed=bs)
        xs[:bs].copy_(x.to(cuda_device))
        graphs[bs].replay()
        torch.cuda.synchronize()
        expected = o.w4a4_linear(u16(x), signs.numpy(), packed.numpy().view(np.uint8), u16(scale),
                                 o.LAYOUT_BLOCK128, -8)
        np.testing.assert_array_equal(u16(outs[:bs]), expected)
    del graphs


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_tp_shards_single_gpu(cuda_device, tp):
    """Column shards concatenate to the full output exactly; row shards' FP32
    partials sum to the full result within FP32 rounding (one GPU, ranks emulated)."""
    k, n = 4096, 6144
    x = synthetic.activations(32, k, seed=tp).to(cuda_device)
    full, packed, scale, signs = make_linear(None, n, k, 8, cuda_device, "block128", -8)
    ref = full(x)
    parts = []
    for r in range(tp):
        col = W4A4QKVParallelLinear(k, 128, 32, 8, tp_rank=r, tp_size=tp).to(cuda_device)
        col.load_full(packed.to(cuda_device), scale.to(cuda_device), signs.to(cuda_device))
        parts.append(col(x))
    q, kv = 4096, 1024
    qs = torch.cat([p[:, :q // tp] for p in parts], 1)
    ks = torch.cat([p[:, q // tp:q // tp + kv // tp] for p in parts], 1)
    vs = torch.cat([p[:, q // tp + kv // tp:] for p in parts], 1)
    assert torch.equal(torch.cat([qs, ks, vs], 1), ref)

    kr, nr = 12288, 4096
    xr = synthetic.activations(32, kr, seed=tp + 1).to(cuda_device)
    full_r, packed_r, scale_r, signs_r = make_linear(None, nr, kr, 9, cuda_device, "block128", -8)
    ref_r = full_r(xr).float()
    total = torch.zeros(32, nr, device=cuda_device)
    kl = kr // tp
    from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
    for r in range(tp):
        row = W4A4RowParallelLinear(kr, nr, tp_rank=r, tp_size=tp).to(cuda_device)
        row.load_full(packed_r.to(cuda_device), scale_r.to(cuda_device), signs_r.to(cuda_device))
        c, s = row.quantize_input(xr[:, r * kl:(r + 1) * kl].contiguous())
        total += w4a4_grouped_gemm_i8(c, row.packed_weight, s, row.weight_scale, out_fp32=True)
    got = total.bfloat16().float()
    rel = (got - ref_r).norm() / ref_r.norm()
    assert rel < 1e-3
    assert (got == ref_r).float().mean() > 0.95


@pytest.mark.parametrize("n,k", [(6144, 4096), (24576, 4096), (4096, 12288)])
@pytest.mark.parametrize("m", [1, 16, 17, 32, 128])
def test_w4a16_matches_oracle(cuda_device, n, k, m):
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=n + k)
    layer = W4A16Linear(k, n).to(cuda_device)
    with torch.no_grad():
        layer.qweight.copy_(qweight)
        layer.qzeros.copy_(qzeros)
        layer.scales.copy_(scales)
    x = synthetic.activations(m, k, seed=m)
    got = layer(x.to(cuda_device)).float().cpu().numpy().astype(np.float64)
    torch.cuda.synchronize()
    expected = o.w4a16_gemm_f64(u16(x), qweight.numpy(), qzeros.numpy(), scales.numpy())
    rel = np.linalg.norm(got - expected) / np.linalg.norm(expected)
    assert rel < 4e-3, rel          # BF16 output rounding dominates (~2^-9 relative)
    exp_bf16 = o.round_to_bf16(expected.astype(np.float32)).astype(np.float64)
    rel_b = np.linalg.norm(got - exp_bf16) / np.linalg.norm(expected)
    assert rel_b < 1e-3, rel_b      # same BF16 rounding as the exact product, up to FP32 sums


@pytest.mark.parametrize("m,n,k", [(33, 192, 512), (300, 320, 1024), (257, 4096, 12288), (2048, 24576, 4096),
                                   (128, 6144, 4096), (128, 4096, 12288)])
def test_w4a16_prefill_tiles(cuda_device, m, n, k):
    """The tcgen05 W4A16 kernel (more than 16 tokens): ragged token and column
    tiles (zero-filled TMA boxes past M and N, stores masked), K split into 2-8
    slices (uneven ones at 128 x 6144 x 4096) summed by the second kernel, and
    an unsplit full config-3 prefill shape, on a sample of rows against the
    float64 oracle."""
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=7 * n + k)
    layer = W4A16Linear(k, n).to(cuda_device)
    with torch.no_grad():
        layer.qweight.copy_(qweight)
        layer.qzeros.copy_(qzeros)
        layer.scales.copy_(scales)
    x = synthetic.activations(m, k, seed=m + 5)
    out = torch.full((m + 1, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    out[:m].copy_(layer(x.to(cuda_device)))
    got = out.float().cpu().numpy().astype(np.float64)
    assert np.isnan(got[m]).all()  # the guard row is untouched
    rows = np.unique(np.concatenate([np.arange(0, m, max(1, m // 24)), [m - 1]]))
    expected = o.w4a16_gemm_f64(u16(x[rows]), qweight.numpy(), qzeros.numpy(), scales.numpy())
    rel = np.linalg.norm(got[rows] - expected) / np.linalg.norm(expected)
    assert rel < 4e-3, rel
    exp_bf16 = o.round_to_bf16(expected.astype(np.float32)).astype(np.float64)
    assert np.linalg.norm(got[rows] - exp_bf16) / np.linalg.norm(expected) < 1e-3


@pytest.mark.parametrize("m,n,k", [(128, 4096, 12288), (64, 6144, 4096)])
def test_w4a16_split_k_without_workspace(cuda_device, m, n, k):
    """A shape whose plan splits K: with the queried workspace the slices' FP32
    partials are summed by the second kernel; without one the kernel runs
    unsplit.  Both agree with the oracle and with each other up to FP32
    summation order."""
    ws_bytes = _native.w4a16_workspace_bytes(m, n, k, cuda_device)
    assert ws_bytes >= 2 * m * n * 4  # the plan splits
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=3 * n + k)
    qw, qz, sc = qweight.to(cuda_device), qzeros.to(cuda_device), scales.to(cuda_device)
    x = synthetic.activations(m, k, seed=m + 11)
    xd = x.to(cuda_device)
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device=cuda_device)
    split = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
    whole = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
    _native.w4a16_gemm(xd, qw, qz, sc, split, 128, ws)
    _native.w4a16_gemm(xd, qw, qz, sc, whole, 128, None)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    rows = np.arange(0, m, 5)
    expected = o.w4a16_gemm_f64(u16(x[rows]), qweight.numpy(), qzeros.numpy(), scales.numpy())
    for got in (split, whole):
        g = got.float().cpu().numpy().astype(np.float64)[rows]
        assert np.linalg.norm(g - expected) / np.linalg.norm(expected) < 4e-3
    # one BF16 rounding step apart, or FP32-summation noise near cancellations
    diff = (split.float() - whole.float()).abs()
    rms = whole.float().pow(2).mean().sqrt()
    assert (diff <= whole.float().abs() * 2 ** -7 + 1e-3 * rms).all()


def test_w4a16_large_m_and_graph(cuda_device):
    n, k, m = 6144, 4096, 2048
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=1)
    layer = W4A16Linear(k, n).to(cuda_device)
    with torch.no_grad():
        layer.qweight.copy_(qweight)
        layer.qzeros.copy_(qzeros)
        layer.scales.copy_(scales)
    x = synthetic.activations(m, k, seed=2)
    got = layer(x.to(cuda_device)).float().cpu().numpy().astype(np.float64)
    rows = np.arange(0, m, 97)
    expected = o.w4a16_gemm_f64(u16(x[rows]), qweight.numpy(), qzeros.numpy(), scales.numpy())
    assert np.linalg.norm(got[rows] - expected) / np.linalg.norm(expected) < 4e-3
    # graph capture at decode size (split-K workspace comes from the graph pool)
    xs = synthetic.activations(4, k, seed=3).to(cuda_device)
    out = layer(xs)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = layer(xs)
    new = synthetic.activations(4, k, seed=4)
    xs.copy_(new.to(cuda_device))
    g.replay()
    torch.cuda.synchronize()
    expected = o.w4a16_gemm_f64(u16(new), qweight.numpy(), qzeros.numpy(), scales.numpy())
    got = out.float().cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - expected) / np.linalg.norm(expected) < 4e-3
