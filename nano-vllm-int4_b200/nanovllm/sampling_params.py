"""Sampling parameters (the reference's ``nanovllm/sampling_params.py``).

``temperature = 0`` selects greedy decoding, which the end-to-end benchmark
configuration uses; the reference rejects it (``sampling_params.py:10-11``).
"""
from dataclasses import dataclass


@dataclass(slots=True)
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0 (0 is greedy)")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
