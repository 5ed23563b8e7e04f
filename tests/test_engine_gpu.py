"""The engine end to end on a small random-init Qwen3 (2 layers, hidden 1024):
``LLM(model, w4a4_checkpoint=..., use_w4a16=..., load_format="dummy")`` then
``generate``.

* Greedy tokens from the captured decode graphs equal those of an eager run.
* The W4A4 model's prefill logits match a reference forward written with the
  reference's own formulas (oracle/torch_ref.py: block128 RHT, quantisation,
  the FP64 grouped-GEMM emulation; RMSNorm, rotary, causal softmax attention in
  torch) on the same weights.
"""
import gc
import math

import pytest
import torch
import torch.nn.functional as F

from nanovllm.utils import synthetic

pytestmark = pytest.mark.gpu

TINY = dict(num_hidden_layers=2, hidden_size=1024, intermediate_size=3072, num_attention_heads=8,
            num_key_value_heads=2, vocab_size=4096, max_position_embeddings=4096)


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    return synthetic.write_qwen3_config(str(tmp_path_factory.mktemp("qwen3_tiny")), **TINY)


def make_llm(model_dir, **kw):
    from nanovllm import LLM
    args = dict(load_format="dummy", max_model_len=1024, max_num_batched_tokens=2048, max_num_seqs=8,
                num_kvcache_blocks=48, seed=3)
    args.update(kw)
    return LLM(model_dir, **args)


def prompts(n=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    lengths = [7, 100, 257, 600, 3][:n]
    return [torch.randint(0, TINY["vocab_size"], (k,), generator=g).tolist() for k in lengths]


def run(model_dir, max_tokens=24, **kw):
    from nanovllm import SamplingParams
    llm = make_llm(model_dir, **kw)
    try:
        out = llm.generate(prompts(), SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True))
        return [o["token_ids"] for o in out], llm.stats
    finally:
        llm.exit()
        del llm
        gc.collect()
        torch.cuda.empty_cache()


@pytest.mark.parametrize("flavour", [dict(w4a4_checkpoint="random"), dict(), dict(use_w4a16=True)],
                         ids=["w4a4", "bf16", "w4a16"])
def test_graph_decode_matches_eager(cuda_device, model_dir, flavour):
    graph_tokens, stats = run(model_dir, **flavour)
    eager_tokens, _ = run(model_dir, enforce_eager=True, **flavour)
    assert all(len(t) == 24 for t in graph_tokens)
    assert all(0 <= x < TINY["vocab_size"] for t in graph_tokens for x in t)
    assert graph_tokens == eager_tokens
    assert stats["decode_steps"] >= 23 and stats["prefill_tokens"] == sum(len(p) for p in prompts())
    from nanovllm import _native
    assert _native.device_error() == 0


def _reference_logits(model, ids):
    """Prefill logits of the last token, recomputed on the CPU with the
    reference's formulas from the W4A4 model's own parameters and buffers."""
    from oracle import torch_ref
    cpu = lambda t: t.detach().cpu()
    m = model.model
    n = len(ids)
    cfg_eps = m.norm.eps
    h = F.embedding(torch.tensor(ids), cpu(m.embed_tokens.weight))
    pos = torch.arange(n)
    cos_sin = cpu(m.cos_sin)
    res = None

    def lin(mod, x):
        codes = synthetic.unpack_int4(cpu(mod.packed_weight))
        return torch_ref.w4a4_linear(x, cpu(mod.signs), codes, cpu(mod.weight_scale), clamp_lo=-8)

    def norm_rope(x, w):
        xf = x.float()
        y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg_eps)).bfloat16() * w
        cos, sin = cos_sin[pos].chunk(2, -1)
        x1, x2 = y.float().chunk(2, -1)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).bfloat16()

    for layer in m.layers:
        a, p = layer.self_attn, layer.mlp
        x, res = torch_ref.add_rmsnorm(h, res, cpu(layer.input_layernorm.weight), cfg_eps)
        if res is None:
            res = h
        qkv = lin(a.qkv_proj, x)
        hq, hkv, d = a.num_heads, a.num_kv_heads, a.head_dim
        q, k, v = qkv.view(n, -1, d).split([hq, hkv, hkv], dim=1)
        q = norm_rope(q, cpu(a.q_norm.weight))
        k = norm_rope(k, cpu(a.k_norm.weight))
        g = hq // hkv
        s = torch.einsum("qhd,khd->hqk", q.float(), k.float().repeat_interleave(g, 1)) / math.sqrt(d)
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v.float().repeat_interleave(g, 1)).bfloat16()
        h = lin(a.o_proj, o.reshape(n, -1))
        x, res = torch_ref.add_rmsnorm(h, res, cpu(layer.post_attention_layernorm.weight), cfg_eps)
        h = lin(p.down_proj, torch_ref.silu_mul(lin(p.gate_up_proj, x)))
    hf = h.float() + res.float()
    h = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + cfg_eps)).bfloat16() * cpu(m.norm.weight)
    return (h[-1:].float() @ cpu(model.lm_head.weight).float().T)[0]


def test_w4a4_prefill_logits_match_reference_forward(cuda_device, model_dir):
    from nanovllm.layers.attention import StepContext, set_context
    llm = make_llm(model_dir, w4a4_checkpoint="random", enforce_eager=True)
    try:
        model = llm.runner.model
        for ids in prompts(3, seed=11):
            n = len(ids)
            set_context(StepContext(is_prefill=True, seq_lens=[n]))
            with torch.inference_mode():
                hidden = model(torch.tensor(ids, device=cuda_device), torch.arange(n, device=cuda_device))
                got = model.compute_logits(hidden[-1:]).float()[0].cpu()
            set_context(StepContext())
            ref = _reference_logits(model, ids)
            rel = (got - ref).norm() / ref.norm()
            assert rel < 2e-2, rel
            assert got.argmax() == ref.argmax() or ref[got.argmax()] >= ref.max() - 1e-2 * ref.abs().max()
    finally:
        llm.exit()
        del llm
        gc.collect()
        torch.cuda.empty_cache()
