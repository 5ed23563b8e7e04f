"""The engine end to end on a small random-init Qwen3 (2 layers, hidden 1024):
``LLM(model, w4a4_checkpoint=..., use_w4a16=..., load_format="dummy")`` then
``generate``.

* Greedy tokens from the captured decode graphs equal those of an eager run,
  for the W4A4, BF16 and W4A16 models.
* The W4A4 model's greedy tokens equal those of the same engine whose W4A4
  linears (activation prep + grouped GEMM) run the reference's own formulas in
  torch (oracle/torch_ref.py).  The producers fused into the prep stay the
  native ones in both runs: the add + RMSNorm output differs from torch's by
  up to 2 BF16 ulps (another reduction order; tested in
  test_fused_prep_gpu.py), and one such flip can change a greedy token.
  (A free-running comparison with a separately written attention would not
  work: with INT4 activations, a 1e-3 difference in attention flips codes and
  compounds over layers; the linears themselves are bit-exact.)
"""
import gc

import pytest
import torch

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


def _reference_w4a4_forwards(monkeypatch):
    """Swap the W4A4 modules' forwards for the reference's formulas in torch
    (oracle/torch_ref.py: block128 RHT, quantisation, the FP64 grouped-GEMM
    emulation; SiluAndMul) running on the same device."""
    from nanovllm.layers import linear_w4a4 as lw
    from oracle import torch_ref

    def codes_of(mod):
        cache = mod.__dict__.setdefault("_ref_codes", {})
        if "w" not in cache:
            cache["w"] = synthetic.unpack_int4(mod.packed_weight.cpu()).to(mod.packed_weight.device)
        return cache["w"]

    def lin(mod, x):
        flat = x.reshape(-1, mod.in_features)
        y = torch_ref.w4a4_linear(flat, mod.signs, codes_of(mod), mod.weight_scale, clamp_lo=mod.clamp_lo)
        return y.reshape(*x.shape[:-1], mod.out_features)

    def forward(self, x):
        return lin(self, x)

    def forward_add_rmsnorm(self, x, residual, weight, eps=1e-6):
        # the producer stays the native fused kernel's (its add + RMSNorm output h,
        # written to out_normed); the linear on h is the reference's
        from nanovllm import _native
        flat = x.reshape(-1, self.in_features).contiguous()
        m, k = flat.shape
        codes = torch.empty((m, k), dtype=torch.int8, device=x.device)
        scale = torch.empty((m, k // 128), dtype=torch.bfloat16, device=x.device)
        res = None if residual is None else residual.reshape(-1, k).contiguous()
        new_res = None if res is None else torch.empty_like(flat)
        h = torch.empty_like(flat)
        _native.add_rmsnorm_rht_quant_i8(flat, res, weight, eps, self.signs, codes, scale, new_res, h,
                                         self.layout_id, self.clamp_lo)
        return lin(self, h).reshape(*x.shape[:-1], self.out_features), \
            (x if residual is None else new_res.reshape(x.shape))

    def forward_silu_mul(self, gu):
        return lin(self, torch_ref.silu_mul(gu))

    for cls in (lw.W4A4Linear, lw.W4A4RowParallelLinear):
        monkeypatch.setattr(cls, "forward", forward)
        monkeypatch.setattr(cls, "forward_silu_mul", forward_silu_mul)
    monkeypatch.setattr(lw.W4A4Linear, "forward_add_rmsnorm", forward_add_rmsnorm)


def test_w4a4_tokens_match_reference_linear_forward(cuda_device, model_dir, monkeypatch):
    """Greedy tokens of the engine (native kernels, CUDA graphs) equal those of
    the same engine whose W4A4 linears run the reference's formulas in torch
    (eager): the linears are bit-exact, everything else is the same code."""
    fast, _ = run(model_dir, max_tokens=6, w4a4_checkpoint="random")
    with monkeypatch.context() as mp:
        _reference_w4a4_forwards(mp)
        ref, _ = run(model_dir, max_tokens=6, w4a4_checkpoint="random", enforce_eager=True)
    assert fast == ref
