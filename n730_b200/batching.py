"""Continuous batching over the engine's paged KV cache.

The reference generates one prompt at a time and clears its cache per call
(``src-code/inference.py:230-257,723-745``).  Here many requests share one
engine: a request is admitted into a free slot (its prompt prefilled, pages
taken from the KV pool as the sequence grows), every step decodes all active
sequences in one batched call, and a finished request is released: its pages
return to the pool for the next admission.  Decode steps run slots
``[0, n)``, so the active requests are kept in the first slots: a finished
request's slot receives the last active one (``Engine.seq_move``: its row of
page ids and its length move, no KV data does).

Sampling: temperature <= 0 is greedy; otherwise the next tokens are drawn on
the GPU (``n730_model_decode_sample``: temperature + top-p) and only their ids
cross to the host.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np

from .engine import Engine


@dataclass
class Request:
    rid: int
    prompt: np.ndarray
    max_new_tokens: int
    eos: int | None = None
    tokens: list = field(default_factory=list)
    logits: list = field(default_factory=list)   # per emitted token, when the batcher keeps them
    done: bool = False


class ContinuousBatcher:
    def __init__(self, engine: Engine, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0,
                 keep_logits: bool = False):
        self.e = engine
        self.temp, self.top_p, self.seed = temperature, top_p, seed
        self.keep_logits = keep_logits
        self.waiting: deque = deque()
        self.slots: list = []          # active requests; request in slot i decodes as sequence i
        self.finished: dict = {}
        self._next = 0
        page = int(engine.cfg.page_size) or 64
        self.page = page

    # ---- requests ----
    def submit(self, prompt, max_new_tokens: int, eos: int | None = None) -> int:
        p = np.ascontiguousarray(prompt, np.int32).reshape(-1)
        if p.size < 1 or max_new_tokens < 1:
            raise ValueError("a request needs a prompt and at least one new token")
        if p.size + max_new_tokens > self.e.max_ctx:
            raise ValueError(f"prompt {p.size} + {max_new_tokens} tokens exceed the context {self.e.max_ctx}")
        _, total = self.e.kv_pages()
        if self._pages(p.size + max_new_tokens) > total:
            raise ValueError(f"request needs {self._pages(p.size + max_new_tokens)} KV pages, the pool has {total}")
        rid = self._next
        self._next += 1
        self.waiting.append(Request(rid, p, max_new_tokens, eos))
        return rid

    def _pages(self, n: int) -> int:
        return (n + self.page - 1) // self.page

    def _reserved(self) -> int:
        """Pages the active requests may still take (up to their final lengths)."""
        return sum(self._pages(len(r.prompt) + r.max_new_tokens) for r in self.slots)

    def _admit(self):
        """Admit waiting requests while a slot is free and the pool can hold them to completion."""
        _, total = self.e.kv_pages()
        while self.waiting and len(self.slots) < self.e.max_batch:
            r = self.waiting[0]
            if self._reserved() + self._pages(len(r.prompt) + r.max_new_tokens) > total:
                break
            self.waiting.popleft()
            slot = len(self.slots)
            self.slots.append(r)
            logits = self.e.forward(r.prompt, seq=slot)
            self._emit(r, self._pick(logits, r), logits)

    def _pick(self, logits: np.ndarray, r: Request) -> int:
        if self.temp <= 0:
            return int(np.argmax(logits))
        from .inference import sample
        return sample(logits, self.temp, self.top_p, np.random.default_rng((self.seed, r.rid, len(r.tokens))))

    def _emit(self, r: Request, tok: int, logits=None):
        r.tokens.append(int(tok))
        if self.keep_logits and logits is not None:
            r.logits.append(np.array(logits, np.float32))
        if len(r.tokens) >= r.max_new_tokens or (r.eos is not None and tok == r.eos):
            r.done = True

    def _retire(self):
        """Release finished requests; the last active request moves into each freed slot."""
        i = 0
        while i < len(self.slots):
            r = self.slots[i]
            if not r.done:
                i += 1
                continue
            self.e.seq_release(i)
            last = len(self.slots) - 1
            if i != last:
                self.e.seq_move(i, last)
                self.slots[i] = self.slots[last]
            self.slots.pop()
            self.finished[r.rid] = r

    # ---- stepping ----
    def step(self) -> list:
        """Admit what fits, decode one token for every active request, retire finished ones.
        Returns [(rid, token)] of this step's decoded tokens."""
        self._retire()
        self._admit()
        self._retire()  # a request may finish on its first token
        if not self.slots:
            return []
        toks = np.array([r.tokens[-1] for r in self.slots], np.int32)
        out = []
        if self.temp <= 0 or self.keep_logits:
            logits = self.e.decode(toks)
            for r, lg in zip(self.slots, logits):
                t = self._pick(lg, r)
                self._emit(r, t, lg)
                out.append((r.rid, t))
        else:
            nxt = self.e.decode_sample(toks, self.temp, self.top_p, self.seed)
            for r, t in zip(self.slots, nxt):
                self._emit(r, int(t))
                out.append((r.rid, int(t)))
        return out

    def run(self) -> dict:
        """Step until every submitted request has finished; {rid: Request}."""
        while self.waiting or self.slots:
            before = (len(self.waiting), len(self.slots))
            self.step()
            if not self.slots and self.waiting and before == (len(self.waiting), 0):
                raise RuntimeError("a waiting request cannot be admitted (KV pool too small)")
        return self.finished
