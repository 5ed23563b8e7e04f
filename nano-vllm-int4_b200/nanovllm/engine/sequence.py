"""Per-request state of the engine: token ids, the KV pages that hold them, and
the sampling parameters (the role of the reference's
``nanovllm/engine/sequence.py``)."""
from __future__ import annotations

import itertools
from enum import Enum, auto

from nanovllm.sampling_params import SamplingParams

PAGE_TOKENS = 256  # tokens per KV page (Config.kvcache_block_size)


class Status(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    _ids = itertools.count()

    def __init__(self, token_ids: list[int], params: SamplingParams | None = None):
        if not token_ids:
            raise ValueError("a prompt needs at least one token")
        params = params or SamplingParams()
        self.seq_id = next(Sequence._ids)
        self.status = Status.WAITING
        self.token_ids = list(token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.pages: list[int] = []
        self.temperature = params.temperature
        self.max_tokens = params.max_tokens
        self.ignore_eos = params.ignore_eos

    def __len__(self) -> int:
        return len(self.token_ids)

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]

    @property
    def completion_token_ids(self) -> list[int]:
        return self.token_ids[self.num_prompt_tokens:]

    @property
    def num_completion_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def is_finished(self) -> bool:
        return self.status == Status.FINISHED

    def pages_needed(self, tokens: int | None = None) -> int:
        n = len(self) if tokens is None else tokens
        return (n + PAGE_TOKENS - 1) // PAGE_TOKENS

    def slot(self, position: int) -> int:
        """Cache row of the token at `position` (page * PAGE_TOKENS + offset)."""
        return self.pages[position // PAGE_TOKENS] * PAGE_TOKENS + position % PAGE_TOKENS
