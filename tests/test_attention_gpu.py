"""The end-to-end model's attention kernels against torch FP32 references:
paged decode attention (nv4_paged_decode_attention, the counterpart of
flash_attn_with_kvcache in the reference's nanovllm/layers/attention.py:71-73)
and the fused q/k RMSNorm + rotary + KV store (nv4_qk_norm_rope_store, the
reference's qwen3.py:87-92 and attention.py:10-40)."""
import math

import pytest
import torch

from nanovllm import _native
from nanovllm.layers.common import rotary_cos_sin

pytestmark = pytest.mark.gpu
D, PAGE = 128, 256


def attention_reference(q, k_cache, v_cache, tables, lens, scale):
    """FP32 softmax(q k^T * scale) v over each sequence's cached tokens."""
    b, hq, _ = q.shape
    hkv = k_cache.shape[2]
    out = torch.zeros(b, hq, D, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = int(lens[i])
        if n == 0:
            continue
        pages = tables[i, : (n + PAGE - 1) // PAGE].long()
        k = k_cache[pages].reshape(-1, hkv, D)[:n].float()
        v = v_cache[pages].reshape(-1, hkv, D)[:n].float()
        g = hq // hkv
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
        s = torch.einsum("hd,thd->ht", q[i].float(), k) * scale
        out[i] = torch.einsum("ht,thd->hd", torch.softmax(s, -1), v)
    return out


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 2), (4, 4), (8, 1)])
def test_paged_decode_attention(cuda_device, hq, hkv):
    g = torch.Generator(device=cuda_device).manual_seed(hq * 10 + hkv)
    lens = [1, 255, 256, 257, 700, 1536, 0, 4352]
    b, max_pages = len(lens), 17
    pages = 64
    k_cache = torch.randn(pages, PAGE, hkv, D, device=cuda_device, generator=g).bfloat16()
    v_cache = torch.randn(pages, PAGE, hkv, D, device=cuda_device, generator=g).bfloat16()
    perm = torch.randperm(pages, device=cuda_device, generator=g)
    tables = torch.zeros(b, max_pages, dtype=torch.int32, device=cuda_device)
    used = 0
    for i, n in enumerate(lens):
        np_ = (n + PAGE - 1) // PAGE
        tables[i, :np_] = perm[used:used + np_].int() if used + np_ <= pages else perm[:np_].int()
        used = (used + np_) % pages
    # poison the rows past each sequence's end in its last page: they must not leak in
    for i, n in enumerate(lens):
        if n % PAGE:
            last = int(tables[i, n // PAGE])
            k_cache[last, n % PAGE:] = float("nan")
            v_cache[last, n % PAGE:] = float("nan")
    lens_t = torch.tensor(lens, dtype=torch.int32, device=cuda_device)
    q = torch.randn(b, hq, D, device=cuda_device, generator=g).bfloat16()
    scale = 1.0 / math.sqrt(D)
    ws = torch.empty(_native.paged_attention_workspace_bytes(b, hq, max_pages) // 4, dtype=torch.float32,
                     device=cuda_device)
    out = torch.full((b, hq, D), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    _native.paged_decode_attention(q, k_cache, v_cache, tables, lens_t, out, ws, scale)
    torch.cuda.synchronize()
    ref = attention_reference(q, k_cache.nan_to_num(0.0), v_cache.nan_to_num(0.0), tables, lens_t, scale)
    got = out.float()
    assert torch.isfinite(got).all()
    assert (got[lens.index(0)] == 0).all()
    err = (got - ref).norm() / ref.norm()
    assert err < 1e-2, err  # BF16 P and output, FP32 accumulation
    assert (got - ref).abs().max() < 3e-2


def test_paged_decode_attention_in_graph(cuda_device):
    """Captured once, replayed with new lengths and queries (the decode graph)."""
    g = torch.Generator(device=cuda_device).manual_seed(5)
    b, hq, hkv, max_pages, pages = 4, 8, 2, 4, 16
    k_cache = torch.randn(pages, PAGE, hkv, D, device=cuda_device, generator=g).bfloat16()
    v_cache = torch.randn(pages, PAGE, hkv, D, device=cuda_device, generator=g).bfloat16()
    tables = torch.arange(b * max_pages, dtype=torch.int32, device=cuda_device).view(b, max_pages) % pages
    lens = torch.tensor([3, 300, 600, 900], dtype=torch.int32, device=cuda_device)
    q = torch.randn(b, hq, D, device=cuda_device, generator=g).bfloat16()
    ws = torch.empty(_native.paged_attention_workspace_bytes(b, hq, max_pages) // 4, dtype=torch.float32,
                     device=cuda_device)
    out = torch.empty(b, hq, D, dtype=torch.bfloat16, device=cuda_device)
    _native.paged_decode_attention(q, k_cache, v_cache, tables, lens, out, ws, 0.1)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _native.paged_decode_attention(q, k_cache, v_cache, tables, lens, out, ws, 0.1)
    lens.copy_(torch.tensor([1000, 1, 257, 512], dtype=torch.int32))
    q.copy_(torch.randn(b, hq, D, device=cuda_device, generator=g).bfloat16())
    graph.replay()
    torch.cuda.synchronize()
    ref = attention_reference(q, k_cache, v_cache, tables, lens, 0.1)
    assert (out.float() - ref).norm() / ref.norm() < 1e-2


def norm_rope_reference(x, w, cos_sin, pos, eps):
    """RMSNorm then rotary, as the reference's torch code (layernorm.py:17-27,
    rotary_embedding.py:6-14, 46-51)."""
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).bfloat16() * w
    cos, sin = cos_sin[pos].chunk(2, -1)
    x1, x2 = y.float().chunk(2, -1)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).bfloat16()


@pytest.mark.parametrize("t,hq,hkv", [(1, 32, 8), (37, 16, 4), (300, 8, 1)])
def test_qk_norm_rope_store(cuda_device, t, hq, hkv):
    g = torch.Generator(device=cuda_device).manual_seed(t + hq)
    eps = 1e-6
    qkv = torch.randn(t, (hq + 2 * hkv) * D, device=cuda_device, generator=g).bfloat16()
    qw = (1 + 0.1 * torch.randn(D, device=cuda_device, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device=cuda_device, generator=g)).bfloat16()
    cos_sin = rotary_cos_sin(D, 4096, 1e6).to(cuda_device)
    pos = torch.randint(0, 4096, (t,), device=cuda_device, generator=g)
    pages = 8
    slots = torch.randperm(pages * PAGE, device=cuda_device, generator=g)[:t].int()
    slots[::5] = -1  # padding rows store nothing
    k_cache = torch.zeros(pages, PAGE, hkv, D, dtype=torch.bfloat16, device=cuda_device)
    v_cache = torch.zeros_like(k_cache)
    q_out = torch.empty(t, hq, D, dtype=torch.bfloat16, device=cuda_device)
    k_out = torch.empty(t, hkv, D, dtype=torch.bfloat16, device=cuda_device)
    _native.qk_norm_rope_store(qkv, qw, kw, cos_sin, pos, slots, q_out, k_out, k_cache, v_cache, hq, hkv, eps)
    torch.cuda.synchronize()
    q, k, v = qkv.view(t, -1, D).split([hq, hkv, hkv], dim=1)
    q_ref = norm_rope_reference(q, qw, cos_sin, pos, eps)
    k_ref = norm_rope_reference(k, kw, cos_sin, pos, eps)
    for got, ref in ((q_out, q_ref), (k_out, k_ref)):
        diff = (got.float() - ref.float()).abs()
        assert diff.max() <= 2 * 2 ** -7 * ref.float().abs().max()  # a BF16 rounding apart at most
        assert (got == ref).float().mean() > 0.97
    rows_k = k_cache.view(-1, hkv, D)
    rows_v = v_cache.view(-1, hkv, D)
    keep = slots >= 0
    assert torch.equal(rows_k[slots[keep].long()], k_out[keep])
    assert torch.equal(rows_v[slots[keep].long()], v[keep])
    written = torch.zeros(pages * PAGE, dtype=torch.bool, device=cuda_device)
    written[slots[keep].long()] = True
    assert (rows_k[~written] == 0).all() and (rows_v[~written] == 0).all()
