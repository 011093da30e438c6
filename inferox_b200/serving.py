"""Continuous batching: a greedy serving loop over one KvBatch whose requests
arrive and finish at different times. No reference counterpart (its
KvCache holds one sequence, src/model/cache.rs:7-13); each request produces
exactly what Model::generate (src/model/forward.rs:592-612) produces for it
alone: the argmax of the prompt's last logits (the last index among equal
maxima, forward.rs:615-622), then the argmax after feeding each token back.

    srv = Server.for_model(model, slots=16, max_seq=4096)
    rid = srv.submit(prompt_ids, max_tokens=64)
    results = srv.run()            # {request id: generated tokens}

Each step() first admits waiting requests into free slots (first come,
first served: the slot is cleared, the prompt prefilled, its first token
taken), then runs one decode step of every active slot together
(ifx_decode_step_batch_seqs: one read of the weights for all of them). A
request leaves when it has max_tokens tokens or emits `eos`; its slot takes
the next request on the following step. A finished request's last token is
not fed back (the reference feeds it and discards the logits), so a request
needs len(prompt) + max_tokens - 1 cache rows.

Over a paged batch (Server.for_model(..., pages=P): the slots share a pool
of P cache pages) the pool can run dry. A prefill that finds too few pages
leaves its request waiting at the front until a finishing request returns
some; a decode step that finds none preempts the most recently admitted
request (its slot is reset, returning its pages, and it starts again from
its prompt when pages are free), then retries with the others. A restarted
request produces the tokens it would have produced alone.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np


def _pool_empty(e: BaseException) -> bool:
    """The error a paged batch raises when its page pool has no page left."""
    return getattr(e, "name", None) == "OutOfMemory"


def last_argmax(x) -> int:
    """argmax with ties going to the last index (forward.rs:615-622)."""
    x = np.asarray(x)
    return int(x.size - 1 - np.argmax(x[::-1]))


@dataclass
class _Request:
    rid: int
    prompt: np.ndarray
    max_tokens: int
    eos: int | None
    tokens: list = field(default_factory=list)
    done: bool = False
    order: int = 0  # admission count when it took its slot
    restarts: int = 0  # times it was preempted


class Server:
    """Greedy continuous batching over `batch`, any object with KvBatch's
    `batch`, `max_seq`, `prefill`, `decode_step_seqs` and `reset`."""

    def __init__(self, batch):
        self.kb = batch
        self.slots: list[_Request | None] = [None] * batch.batch
        self.used = [False] * batch.batch  # slot ever held a request (needs a reset)
        self.waiting: deque[_Request] = deque()
        self.requests: dict[int, _Request] = {}
        self._next = 0
        self._admitted = 0
        self.steps = 0  # batched decode steps run
        self.preemptions = 0
        # paged: a finished request's slot is reset at once, returning its pages
        self.paged = bool(getattr(batch, "pages", None)) and batch.pages()[1] > 0

    @classmethod
    def for_model(cls, model, slots: int, max_seq: int, pages: int = 0) -> "Server":
        return cls(model.kv_batch(slots, max_seq, pages))

    def submit(self, prompt, max_tokens: int, eos: int | None = None) -> int:
        p = np.ascontiguousarray(prompt, np.uint32)
        if p.size == 0:
            raise ValueError("empty prompt")
        if max_tokens < 1:
            raise ValueError("max_tokens must be at least 1")
        if p.size + max_tokens - 1 > self.kb.max_seq:
            raise ValueError(f"prompt ({p.size}) + max_tokens ({max_tokens}) - 1 exceeds the "
                             f"{self.kb.max_seq}-row cache of a slot")
        r = _Request(self._next, p, max_tokens, eos)
        self._next += 1
        self.requests[r.rid] = r
        self.waiting.append(r)
        return r.rid

    def busy(self) -> bool:
        return bool(self.waiting) or any(s is not None for s in self.slots)

    def result(self, rid: int):
        r = self.requests[rid]
        return list(r.tokens) if r.done else None

    def _finish_if_done(self, slot: int) -> None:
        r = self.slots[slot]
        if len(r.tokens) >= r.max_tokens or (r.eos is not None and r.tokens[-1] == r.eos):
            r.done = True
            self.slots[slot] = None
            if self.paged:
                self.kb.reset(slot)
                self.used[slot] = False

    def _active(self) -> list[int]:
        return [i for i, r in enumerate(self.slots) if r is not None]

    def _admit(self) -> None:
        for slot in range(len(self.slots)):
            if not self.waiting:
                return
            if self.slots[slot] is not None:
                continue
            r = self.waiting.popleft()
            try:
                if self.used[slot]:
                    self.kb.reset(slot)
                self.used[slot] = True
                logits = self.kb.prefill(slot, r.prompt, True)
            except BaseException as e:
                # the request is not lost: it waits at the front again (the
                # slot is reset before its next use)
                self.waiting.appendleft(r)
                if _pool_empty(e) and self._active():
                    return  # pages come back when an active request finishes
                raise
            r.tokens.append(last_argmax(logits[0]))
            r.order = self._admitted
            self._admitted += 1
            self.slots[slot] = r
            self._finish_if_done(slot)

    def _preempt(self, seqs: list[int]) -> None:
        """Return the pages of the most recently admitted of `seqs`; its
        request starts again from its prompt."""
        slot = max(seqs, key=lambda i: self.slots[i].order)
        r = self.slots[slot]
        self.kb.reset(slot)
        r.tokens.clear()
        r.restarts += 1
        self.slots[slot] = None
        self.waiting.appendleft(r)
        self.preemptions += 1

    def step(self) -> int:
        """Admit, then one decode step of every active slot; returns how many
        sequences the step decoded."""
        self._admit()
        while True:
            seqs = self._active()
            if not seqs:
                return 0
            toks = [self.slots[i].tokens[-1] for i in seqs]
            try:
                _, amax = self.kb.decode_step_seqs(seqs, toks, want_logits=False)
                break
            except BaseException as e:
                if not _pool_empty(e) or len(seqs) == 1:
                    raise
                self._preempt(seqs)
        self.steps += 1
        for i, t in zip(seqs, amax):
            self.slots[i].tokens.append(int(t))
            self._finish_if_done(i)
        return len(seqs)

    def run(self) -> dict[int, list]:
        """Steps until every submitted request has finished."""
        while self.busy():
            self.step()
        return {rid: list(r.tokens) for rid, r in self.requests.items()}
