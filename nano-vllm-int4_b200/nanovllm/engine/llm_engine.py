"""The engine behind ``LLM`` (the role of the reference's
``nanovllm/engine/llm_engine.py``): a scheduler and one model runner per
process.

Tensor parallelism runs one process per GPU, SPMD: start the program on every
rank (``torchrun --nproc-per-node N``) and construct ``LLM(...,
tensor_parallel_size=N)`` and call ``generate`` with the same arguments on
each; the process group comes from the launcher's environment (NCCL).  With
``tensor_parallel_size == 1`` no process group is needed.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import fields
from time import perf_counter

import torch
import torch.distributed as dist

from nanovllm.config import Config
from nanovllm.engine.runner import ModelRunner
from nanovllm.engine.scheduler import Scheduler
from nanovllm.engine.sequence import Sequence
from nanovllm.sampling_params import SamplingParams


class LLMEngine:
    def __init__(self, model: str, **kwargs):
        names = {f.name for f in fields(Config)}
        config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
        self.config = config
        tp = config.tensor_parallel_size
        if tp > 1:
            if not dist.is_initialized():
                if int(os.environ.get("WORLD_SIZE", "1")) != tp:
                    raise RuntimeError("tensor_parallel_size > 1 needs one process per GPU: launch with "
                                       f"torchrun --nproc-per-node {tp}")
                torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                        device_id=torch.device("cuda", torch.cuda.current_device()))
            if dist.get_world_size() != tp:
                raise RuntimeError("the process group size differs from tensor_parallel_size")
            rank = dist.get_rank()
        else:
            rank = 0
        self.rank = rank
        self.runner = ModelRunner(config, rank, tp)
        self.tokenizer = None
        try:
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(model, use_fast=True)
        except Exception:  # a model directory with only config.json: token-id prompts
            self.tokenizer = None
        eos = getattr(self.tokenizer, "eos_token_id", None)
        if eos is None:
            eos = getattr(config.hf_config, "eos_token_id", -1)
        config.eos = eos if isinstance(eos, int) else (eos[0] if eos else -1)
        self.scheduler = Scheduler(config.max_num_seqs, config.max_num_batched_tokens, config.num_kvcache_blocks,
                                   config.eos)
        self.stats = {}

    def add_request(self, prompt, params: SamplingParams) -> Sequence:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("text prompts need a tokenizer in the model directory")
            prompt = self.tokenizer.encode(prompt)
        seq = Sequence(prompt, params)
        self.scheduler.add(seq)
        return seq

    def step(self):
        """One prefill or decode step: (requests, is_prefill, tokens computed, finished requests)."""
        seqs, is_prefill = self.scheduler.schedule()
        computed = sum(len(s) for s in seqs) if is_prefill else len(seqs)
        tokens = self.runner.run(seqs, is_prefill)
        done = self.scheduler.postprocess(seqs, tokens)
        return seqs, is_prefill, computed, done

    def is_finished(self) -> bool:
        return self.scheduler.is_finished()

    def generate(self, prompts, sampling_params, use_tqdm: bool = False) -> list[dict]:
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(prompts)
        seqs = [self.add_request(p, sp) for p, sp in zip(prompts, sampling_params)]
        st = {"prefill_tokens": 0, "prefill_s": 0.0, "decode_tokens": 0, "decode_s": 0.0, "decode_steps": 0,
              "decode_batch_max": 0}
        while not self.is_finished():
            torch.cuda.synchronize()
            t = perf_counter()
            batch, is_prefill, computed, _ = self.step()
            dt = perf_counter() - t  # run() ends with the sampled tokens on the host
            if is_prefill:
                st["prefill_tokens"] += computed
                st["prefill_s"] += dt
            else:
                st["decode_tokens"] += computed
                st["decode_s"] += dt
                st["decode_steps"] += 1
                st["decode_batch_max"] = max(st["decode_batch_max"], len(batch))
        self.stats = st
        out = []
        for s in seqs:
            ids = s.completion_token_ids
            text = self.tokenizer.decode(ids) if self.tokenizer is not None else ""
            out.append({"text": text, "token_ids": ids})
        return out

    def exit(self):
        if getattr(self, "runner", None) is not None:
            self.runner.close()
            self.runner = None
