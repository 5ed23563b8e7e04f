"""Engine configuration (the reference's ``nanovllm/config.py:8-35`` semantics).

Same fields, defaults and checks as the reference, with two differences:

* tensor parallelism is allowed for W4A4 (the reference refuses it,
  ``config.py:32-33``): the W4A4 linears shard along N / group-aligned K;
* ``load_format="dummy"`` builds the model with seeded random weights instead of
  reading a checkpoint (no weights are available offline; the benchmark's
  end-to-end configuration is a random-init Qwen3-8B).  With it,
  ``w4a4_checkpoint="random"`` selects random W4A4 weights (block128 layout,
  codes in [-8, 7]) without a manifest on disk.

``model`` is a directory with the Hugging Face ``config.json`` (and, unless
the load format is dummy, safetensors weights).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

from transformers import AutoConfig

RANDOM_W4A4 = "random"


@dataclass(slots=True)
class Config:
    model: str
    max_num_batched_tokens: int = 16384
    max_num_seqs: int = 512
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.9
    tensor_parallel_size: int = 1
    enforce_eager: bool = False
    hf_config: AutoConfig | None = None
    eos: int = -1
    kvcache_block_size: int = 256
    num_kvcache_blocks: int = -1

    use_w4a16: bool = False
    w4a4_checkpoint: str | None = None
    load_format: str = "auto"
    seed: int = 0

    def __post_init__(self):
        if self.kvcache_block_size != 256:
            raise ValueError("kvcache_block_size must be 256 (the decode attention kernel's page)")
        if not 1 <= self.tensor_parallel_size <= 8:
            raise ValueError("tensor_parallel_size must be in 1..8")
        if self.load_format not in ("auto", "dummy"):
            raise ValueError("load_format must be 'auto' or 'dummy'")
        self.hf_config = AutoConfig.from_pretrained(self.model)
        self.max_model_len = min(self.max_model_len, self.hf_config.max_position_embeddings)
        if self.max_num_batched_tokens < self.max_model_len:
            raise ValueError("max_num_batched_tokens must hold one whole prompt (no chunked prefill)")
        if self.w4a4_checkpoint is not None:
            if self.use_w4a16:
                raise ValueError("W4A16 and W4A4 cannot be enabled together")
            if self.w4a4_checkpoint == RANDOM_W4A4:
                if self.load_format != "dummy":
                    raise ValueError("random W4A4 weights need load_format='dummy'")
            elif not os.path.isfile(os.path.join(self.w4a4_checkpoint, "manifest.json")):
                raise ValueError("w4a4_checkpoint must contain manifest.json")
