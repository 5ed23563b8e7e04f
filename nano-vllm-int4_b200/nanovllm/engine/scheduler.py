"""Batch scheduler and KV page pool (the role of the reference's
``nanovllm/engine/scheduler.py`` and ``block_manager.py``).

Policy: prefill first -- waiting requests are admitted in arrival order while
their whole prompts fit in ``max_num_batched_tokens`` and the page pool; when
no prefill is possible, every running request decodes one token (up to
``max_num_seqs``).  A decoding request that crosses into a new page takes one
from the pool; if the pool is empty, the most recently admitted running
request is preempted (its pages freed, its tokens recomputed later).  Prefix
reuse is not implemented (the benchmark runs with it off), so pages are owned
by one request and freed when it finishes.
"""
from __future__ import annotations

from collections import deque

from nanovllm.engine.sequence import Sequence, Status


class PagePool:
    def __init__(self, num_pages: int):
        if num_pages < 1:
            raise ValueError("the KV cache has no pages")
        self.free = deque(range(num_pages))
        self.num_pages = num_pages

    def take(self, n: int) -> list[int]:
        if n > len(self.free):
            raise RuntimeError("page pool exhausted")
        return [self.free.popleft() for _ in range(n)]

    def give_back(self, pages: list[int]) -> None:
        self.free.extend(pages)


class Scheduler:
    def __init__(self, max_num_seqs: int, max_num_batched_tokens: int, num_pages: int, eos: int):
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.eos = eos
        self.pool = PagePool(num_pages)
        self.waiting: deque[Sequence] = deque()
        self.running: deque[Sequence] = deque()

    def add(self, seq: Sequence) -> None:
        if seq.pages_needed() > self.pool.num_pages:
            raise ValueError("prompt longer than the KV cache")
        self.waiting.append(seq)

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def schedule(self) -> tuple[list[Sequence], bool]:
        """(requests of the next step, whether it is a prefill step)."""
        batch, tokens = [], 0
        while self.waiting and len(batch) < self.max_num_seqs:
            seq = self.waiting[0]
            need = seq.pages_needed()
            if tokens + len(seq) > self.max_num_batched_tokens or need > len(self.pool.free):
                break
            seq.pages = self.pool.take(need)
            seq.status = Status.RUNNING
            tokens += len(seq)
            self.waiting.popleft()
            self.running.append(seq)
            batch.append(seq)
        if batch:
            return batch, True
        if not self.running:
            raise RuntimeError("nothing to schedule")
        batch = []
        while self.running and len(batch) < self.max_num_seqs:
            seq = self.running.popleft()
            # the token this step writes sits at position len(seq) - 1
            if seq.pages_needed() > len(seq.pages):
                while not self.pool.free and self.running:
                    self._preempt(self.running.pop())
                if not self.pool.free:
                    self._preempt(seq)
                    continue
                seq.pages += self.pool.take(1)
            batch.append(seq)
        self.running.extendleft(reversed(batch))
        if not batch:
            raise RuntimeError("KV cache too small for one request")
        return batch, False

    def _preempt(self, seq: Sequence) -> None:
        self.pool.give_back(seq.pages)
        seq.pages = []
        seq.status = Status.WAITING
        self.waiting.appendleft(seq)

    def postprocess(self, batch: list[Sequence], token_ids: list[int]) -> list[Sequence]:
        """Append each request's new token; returns the requests that finished."""
        done = []
        for seq, tok in zip(batch, token_ids):
            seq.token_ids.append(tok)
            if (not seq.ignore_eos and tok == self.eos) or seq.num_completion_tokens >= seq.max_tokens:
                seq.status = Status.FINISHED
                self.pool.give_back(seq.pages)
                seq.pages = []
                self.running.remove(seq)
                done.append(seq)
        return done
