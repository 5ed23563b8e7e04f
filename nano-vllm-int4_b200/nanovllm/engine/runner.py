"""Model runner: one per GPU (the role of the reference's
``nanovllm/engine/model_runner.py``).

Builds the Qwen3 model in the configured linear flavour, loads or draws its
weights, allocates the paged KV cache from the GPU memory left after a
full-size prefill warm-up, and captures one CUDA graph per decode batch size
(1, 2, 4, 8 and multiples of 16 up to ``max_num_seqs``, the reference's list,
``model_runner.py:250-253``) sharing one memory pool.  Prefill runs eagerly.

Tensor parallelism is SPMD: every rank runs the same engine on the same
requests; the LM head gathers the vocabulary shards on every rank, so all ranks
sample the same tokens and stay in step without a control channel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from nanovllm.config import RANDOM_W4A4, Config
from nanovllm.engine.sequence import PAGE_TOKENS, Sequence
from nanovllm.layers.attention import PagedAttention, StepContext, set_context
from nanovllm.layers.common import Sampler
from nanovllm.models.qwen3 import Qwen3ForCausalLM


def graph_batch_sizes(max_bs: int) -> list[int]:
    return sorted(set([b for b in (1, 2, 4, 8) if b <= max_bs] + list(range(16, max_bs + 1, 16)) + [max_bs]))


class ModelRunner:
    def __init__(self, config: Config, rank: int = 0, world: int = 1):
        self.config, self.rank, self.world = config, rank, world
        cfg = config.hf_config
        self.device = torch.device("cuda", torch.cuda.current_device())
        if config.w4a4_checkpoint is not None:
            mode = "w4a4"
        elif config.use_w4a16:
            mode = "w4a16"
        else:
            mode = "bf16"
        self.mode = mode
        layout, clamp_lo = "block128", -8
        if mode == "w4a4" and config.w4a4_checkpoint != RANDOM_W4A4:
            from nanovllm.utils.loader_w4a4 import checkpoint_activation_contract
            layout, clamp_lo = checkpoint_activation_contract(config.w4a4_checkpoint)
        self.max_pages = (config.max_model_len + PAGE_TOKENS - 1) // PAGE_TOKENS
        dtype = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(self.device):
                self.model = Qwen3ForCausalLM(cfg, mode, rank, world, layout, clamp_lo,
                                              max_position=max(config.max_model_len, 1) + 1)
        finally:
            torch.set_default_dtype(dtype)
        self._load_weights()
        self.model.eval()
        self.sampler = Sampler()
        self.attn_layers = [m for m in self.model.modules() if isinstance(m, PagedAttention)]
        self.generator = torch.Generator(device=self.device).manual_seed(config.seed)
        self._warmup()
        self._allocate_kv_cache()
        self.graphs, self.graph_pool = {}, None
        if not config.enforce_eager:
            self._capture_graphs()

    # ------------------------------------------------------------ set-up
    def _load_weights(self):
        c = self.config
        if c.load_format == "dummy":
            from nanovllm.utils.random_init import init_random_weights
            init_random_weights(self.model, c.seed)
        elif self.mode == "w4a4":
            from nanovllm.utils.loader_w4a4 import load_w4a4_model
            self.quantization_info = load_w4a4_model(self.model, c.model, c.w4a4_checkpoint)
        else:
            from nanovllm.utils.loader import load_model
            load_model(self.model, c.model)

    @torch.inference_mode()
    def _warmup(self):
        """A prefill of max_num_batched_tokens (in max_model_len requests), so the
        KV cache is sized with the activation peak already accounted for."""
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(self.device)
        c = self.config
        n = min(c.max_num_batched_tokens, c.max_model_len)
        reqs = max(1, min(c.max_num_batched_tokens // n, c.max_num_seqs))
        ids = torch.zeros(reqs * n, dtype=torch.int64, device=self.device)
        pos = torch.arange(n, dtype=torch.int64, device=self.device).repeat(reqs)
        set_context(StepContext(is_prefill=True, seq_lens=[n] * reqs))
        self.model(ids, pos)
        set_context(StepContext())
        torch.cuda.synchronize(self.device)

    def _allocate_kv_cache(self):
        c, cfg = self.config, self.config.hf_config
        attn0 = self.attn_layers[0]
        page_bytes = 2 * len(self.attn_layers) * PAGE_TOKENS * attn0.num_kv_heads * attn0.head_dim * 2
        free, total = torch.cuda.mem_get_info(self.device)
        stats = torch.cuda.memory_stats(self.device)
        peak, current = stats["allocated_bytes.all.peak"], stats["allocated_bytes.all.current"]
        budget = int(total * c.gpu_memory_utilization) - (total - free) - (peak - current)
        pages = budget // page_bytes
        if c.num_kvcache_blocks > 0:
            pages = min(pages, c.num_kvcache_blocks)
        if self.world > 1:  # every rank must agree on the pool size
            t = torch.tensor([pages], device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            pages = int(t.item())
        if pages < 1:
            raise RuntimeError("no GPU memory left for the KV cache")
        c.num_kvcache_blocks = pages
        self.kv_cache = torch.empty((2, len(self.attn_layers), pages, PAGE_TOKENS, attn0.num_kv_heads,
                                     attn0.head_dim), dtype=torch.bfloat16, device=self.device)
        for i, layer in enumerate(self.attn_layers):
            layer.k_cache, layer.v_cache = self.kv_cache[0, i], self.kv_cache[1, i]
        from nanovllm import _native
        max_bs = min(c.max_num_seqs, 512)
        ws = _native.paged_attention_workspace_bytes(max_bs, attn0.num_heads, self.max_pages)
        self.workspace = torch.empty(ws // 4, dtype=torch.float32, device=self.device)

    @torch.inference_mode()
    def _capture_graphs(self):
        c, cfg = self.config, self.config.hf_config
        max_bs = min(c.max_num_seqs, 512)
        dev = self.device
        self.g_ids = torch.zeros(max_bs, dtype=torch.int64, device=dev)
        self.g_pos = torch.zeros(max_bs, dtype=torch.int64, device=dev)
        self.g_slots = torch.full((max_bs,), -1, dtype=torch.int32, device=dev)
        self.g_lens = torch.zeros(max_bs, dtype=torch.int32, device=dev)
        self.g_tables = torch.zeros((max_bs, self.max_pages), dtype=torch.int32, device=dev)
        self.g_out = torch.zeros((max_bs, cfg.hidden_size), dtype=torch.bfloat16, device=dev)
        self.graph_bs = graph_batch_sizes(max_bs)
        for bs in reversed(self.graph_bs):
            set_context(StepContext(False, self.g_slots[:bs], None, self.g_lens[:bs], self.g_tables[:bs],
                                    self.workspace))
            self.g_out[:bs] = self.model(self.g_ids[:bs], self.g_pos[:bs])  # warm-up (peer buffers, attributes)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, self.graph_pool):
                self.g_out[:bs] = self.model(self.g_ids[:bs], self.g_pos[:bs])
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            torch.cuda.synchronize(dev)
        set_context(StepContext())

    # ------------------------------------------------------------ steps
    def _tensor(self, values, dtype):
        return torch.tensor(values, dtype=dtype, pin_memory=True).to(self.device, non_blocking=True)

    @torch.inference_mode()
    def run(self, seqs: list[Sequence], is_prefill: bool) -> list[int]:
        temps = self._tensor([s.temperature for s in seqs], torch.float32)
        if is_prefill:
            ids, pos, slots, lens = [], [], [], []
            for s in seqs:
                n = len(s)
                ids.extend(s.token_ids)
                pos.extend(range(n))
                slots.extend(s.slot(i) for i in range(n))
                lens.append(n)
            set_context(StepContext(True, self._tensor(slots, torch.int32), lens))
            hidden = self.model(self._tensor(ids, torch.int64), self._tensor(pos, torch.int64))
            last = torch.tensor([sum(lens[:i + 1]) - 1 for i in range(len(lens))], device=self.device)
            hidden = hidden[last]
        else:
            bs = len(seqs)
            ids = [s.last_token for s in seqs]
            pos = [len(s) - 1 for s in seqs]
            slots = [s.slot(len(s) - 1) for s in seqs]
            lens = [len(s) for s in seqs]
            tables = [s.pages + [0] * (self.max_pages - len(s.pages)) for s in seqs]
            if self.config.enforce_eager or bs not in self.graphs and bs > max(self.graph_bs, default=0):
                set_context(StepContext(False, self._tensor(slots, torch.int32), None,
                                        self._tensor(lens, torch.int32), self._tensor(tables, torch.int32),
                                        self.workspace))
                hidden = self.model(self._tensor(ids, torch.int64), self._tensor(pos, torch.int64))
            else:
                gbs = next(b for b in self.graph_bs if b >= bs)
                self.g_ids[:bs].copy_(self._tensor(ids, torch.int64))
                self.g_pos[:bs].copy_(self._tensor(pos, torch.int64))
                self.g_slots.fill_(-1)
                self.g_slots[:bs].copy_(self._tensor(slots, torch.int32))
                self.g_lens.zero_()
                self.g_lens[:bs].copy_(self._tensor(lens, torch.int32))
                self.g_tables[:bs].copy_(self._tensor(tables, torch.int32))
                self.graphs[gbs].replay()
                hidden = self.g_out[:bs]
        set_context(StepContext())
        logits = self.model.compute_logits(hidden)
        return self.sampler(logits, temps, self.generator).tolist()

    def close(self):
        self.graphs.clear()
        self.graph_pool = None
        if self.world > 1 and self.mode == "w4a4":
            from nanovllm.layers.linear_w4a4 import release_peer_buffers
            release_peer_buffers()
        torch.cuda.synchronize(self.device)
