"""Host-side logic of the engine (no GPU): scheduler and KV page pool, config
checks, sampler, decode graph batch sizes, random-init tensor-parallel
sharding, the BF16 checkpoint loader, and the rotary table."""
import os

import pytest
import torch

from nanovllm.config import Config
from nanovllm.engine.runner import graph_batch_sizes
from nanovllm.engine.scheduler import PagePool, Scheduler
from nanovllm.engine.sequence import PAGE_TOKENS, Sequence, Status
from nanovllm.layers.common import Sampler, rotary_cos_sin
from nanovllm.models.qwen3 import Qwen3ForCausalLM
from nanovllm.sampling_params import SamplingParams
from nanovllm.utils import synthetic
from nanovllm.utils.random_init import init_random_weights

TINY = dict(num_hidden_layers=2, hidden_size=1024, intermediate_size=3072, num_attention_heads=8,
            num_key_value_heads=2, vocab_size=4096, max_position_embeddings=4096)


@pytest.fixture
def model_dir(tmp_path):
    return synthetic.write_qwen3_config(str(tmp_path), **TINY)


def seq(n, max_tokens=4, **kw):
    return Sequence(list(range(n)), SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True, **kw))


def test_prefill_then_decode_and_page_accounting():
    sch = Scheduler(max_num_seqs=4, max_num_batched_tokens=1000, num_pages=10, eos=-1)
    a, b, c = seq(300), seq(256), seq(600)
    for s in (a, b, c):
        sch.add(s)
    batch, prefill = sch.schedule()
    assert prefill and batch == [a, b]            # c does not fit the token budget with them
    assert len(a.pages) == 2 and len(b.pages) == 1 and len(sch.pool.free) == 7
    sch.postprocess(batch, [1, 2])
    batch, prefill = sch.schedule()
    assert prefill and batch == [c] and len(c.pages) == 3
    sch.postprocess(batch, [3])
    batch, prefill = sch.schedule()
    assert not prefill and batch == [a, b, c]
    # b grew to 257 tokens: its new token needs a second page
    assert len(b.pages) == 2 and len(sch.pool.free) == 3
    assert b.slot(256) == b.pages[1] * PAGE_TOKENS
    for _ in range(3):
        done = sch.postprocess(batch, [0, 0, 0])
        if done:
            break
        batch, _ = sch.schedule()
    assert all(s.status == Status.FINISHED for s in (a, b, c))
    assert sch.is_finished() and len(sch.pool.free) == 10


def test_preemption_frees_pages_and_requeues():
    sch = Scheduler(max_num_seqs=4, max_num_batched_tokens=4096, num_pages=3, eos=-1)
    a, b = seq(256, max_tokens=8), seq(256, max_tokens=8)
    sch.add(a)
    sch.add(b)
    batch, _ = sch.schedule()
    assert batch == [a, b] and len(sch.pool.free) == 1
    sch.postprocess(batch, [1, 1])              # both at 257 tokens: each needs a new page
    batch, prefill = sch.schedule()
    assert not prefill and batch == [a] and b.status == Status.WAITING and b.pages == []
    assert list(sch.waiting) == [b]


def test_eos_finishes_unless_ignored():
    sch = Scheduler(max_num_seqs=2, max_num_batched_tokens=100, num_pages=4, eos=7)
    a = Sequence([1, 2], SamplingParams(temperature=0.0, max_tokens=10))
    b = Sequence([1, 2], SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))
    sch.add(a)
    sch.add(b)
    batch, _ = sch.schedule()
    done = sch.postprocess(batch, [7, 7])
    assert done == [a] and not b.is_finished


def test_page_pool_and_prompt_limits():
    pool = PagePool(2)
    assert pool.take(2) == [0, 1]
    with pytest.raises(RuntimeError):
        pool.take(1)
    sch = Scheduler(4, 4096, 1, -1)
    with pytest.raises(ValueError):
        sch.add(seq(257))
    with pytest.raises(ValueError):
        Sequence([])
    with pytest.raises(ValueError):
        SamplingParams(temperature=-1)


def test_config_checks(model_dir):
    c = Config(model_dir, load_format="dummy", w4a4_checkpoint="random", tensor_parallel_size=4, max_model_len=100000)
    assert c.max_model_len == TINY["max_position_embeddings"] and c.max_num_batched_tokens >= c.max_model_len
    with pytest.raises(ValueError):
        Config(model_dir, w4a4_checkpoint="random")                      # random weights need dummy loading
    with pytest.raises(ValueError):
        Config(model_dir, load_format="dummy", w4a4_checkpoint="random", use_w4a16=True)
    with pytest.raises(ValueError):
        Config(model_dir, w4a4_checkpoint=model_dir)                     # no manifest.json
    with pytest.raises(ValueError):
        Config(model_dir, kvcache_block_size=512)
    with pytest.raises(ValueError):
        Config(model_dir, tensor_parallel_size=9)


def test_graph_batch_sizes():
    assert graph_batch_sizes(32) == [1, 2, 4, 8, 16, 32]
    assert graph_batch_sizes(40) == [1, 2, 4, 8, 16, 32, 40]
    assert graph_batch_sizes(3) == [1, 2, 3]


def test_sampler_greedy_and_temperature():
    torch.manual_seed(0)
    logits = torch.randn(4, 50)
    s = Sampler()
    assert torch.equal(s(logits, torch.zeros(4)), logits.argmax(-1))
    temps = torch.tensor([0.0, 1.0, 0.0, 0.5])
    out = s(logits, temps, torch.Generator().manual_seed(1))
    assert out[0] == logits[0].argmax() and out[2] == logits[2].argmax()
    again = s(logits, temps, torch.Generator().manual_seed(1))
    assert torch.equal(out, again)


def test_rotary_table_is_the_reference_formula():
    cs = rotary_cos_sin(128, 64, 1e6)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float) / 128))
    f = torch.arange(64, dtype=torch.float)[:, None] * inv[None, :]
    assert torch.equal(cs, torch.cat((f.cos(), f.sin()), -1))


@pytest.mark.parametrize("mode", ["w4a4", "bf16"])
def test_random_init_shards_concatenate_to_the_full_model(model_dir, mode):
    """Every TP rank draws the same full tensors and keeps its shard."""
    cfg = Config(model_dir, load_format="dummy", w4a4_checkpoint="random" if mode == "w4a4" else None).hf_config
    full = Qwen3ForCausalLM(cfg, mode, 0, 1, max_position=64)
    init_random_weights(full, 5)
    shards = []
    for r in range(2):
        m = Qwen3ForCausalLM(cfg, mode, r, 2, max_position=64)
        init_random_weights(m, 5)
        shards.append(m)
    la = [s.model.layers[1] for s in shards]
    lf = full.model.layers[1]
    if mode == "w4a4":
        # q heads of rank r, then its k and v heads
        hq, hkv, d = 4, 1, 128
        for r, l in enumerate(la):
            w = l.self_attn.qkv_proj.packed_weight
            fw = lf.self_attn.qkv_proj.packed_weight
            assert torch.equal(w[:hq * d], fw[r * hq * d:(r + 1) * hq * d])
            assert torch.equal(w[hq * d:(hq + hkv) * d], fw[8 * d + r * d:8 * d + (r + 1) * d])
        down = torch.cat([l.mlp.down_proj.packed_weight for l in la], 1)
        assert torch.equal(down, lf.mlp.down_proj.packed_weight)
        assert torch.equal(torch.cat([l.mlp.down_proj.signs for l in la]), lf.mlp.down_proj.signs)
    else:
        o = torch.cat([l.self_attn.o_proj.weight for l in la], 1)
        assert torch.equal(o, lf.self_attn.o_proj.weight)
        g = [l.mlp.gate_up_proj.weight for l in la]
        assert torch.equal(torch.cat([x[:1536] for x in g]), lf.mlp.gate_up_proj.weight[:3072])
    emb = torch.cat([s.model.embed_tokens.weight for s in shards])
    assert torch.equal(emb, full.model.embed_tokens.weight)


def test_bf16_loader_fills_fused_and_sharded_parameters(model_dir, tmp_path):
    from safetensors.torch import save_file
    from nanovllm.utils.loader import load_model
    cfg = Config(model_dir).hf_config
    src = Qwen3ForCausalLM(cfg, "bf16", 0, 1, max_position=64)
    init_random_weights(src, 9)
    tensors = {}
    for name, p in src.named_parameters():
        if "qkv_proj" in name:
            q, k, v = p.detach().split([1024, 256, 256])
            for part, t in zip("qkv", (q, k, v)):
                tensors[name.replace("qkv_proj", f"{part}_proj")] = t.contiguous()
        elif "gate_up_proj" in name:
            g, u = p.detach().chunk(2)
            tensors[name.replace("gate_up_proj", "gate_proj")] = g.contiguous()
            tensors[name.replace("gate_up_proj", "up_proj")] = u.contiguous()
        else:
            tensors[name] = p.detach().contiguous()
    path = tmp_path / "w"
    path.mkdir()
    save_file(tensors, str(path / "model.safetensors"))
    dst = Qwen3ForCausalLM(cfg, "bf16", 1, 2, max_position=64)
    load_model(dst, str(path))
    assert torch.equal(dst.model.layers[0].self_attn.o_proj.weight, src.model.layers[0].self_attn.o_proj.weight[:, 512:])
    qkv = dst.model.layers[0].self_attn.qkv_proj.weight
    sq = src.model.layers[0].self_attn.qkv_proj.weight
    assert torch.equal(qkv[:512], sq[512:1024]) and torch.equal(qkv[512:640], sq[1024 + 128:1280])
    assert torch.equal(dst.model.embed_tokens.weight, src.model.embed_tokens.weight[2048:])
