"""Continuous batching over the batched decode step (host side).

The reference serves one request at a time (`crates/base-mlx-core/src/model.rs:21-108`;
its server hands each request to `LoadedModel::generate_text`, `engine.rs:149-201`).
`BatchScheduler` keeps up to `max_batch` requests decoding together: a new
request is prefilled on a free cache (its first token comes from the prompt's
last row, as in `generate_text`) and joins the next batched step; every step
carries each active request's newest token through the weights once
(`qw_forward_batch`: one persistent decode step for all rows, each row
attending to its own cache); a request leaves at its EOS or token budget and
its cache goes back to the pool.  Rows of a batched step run the batch-1
decode arithmetic, so every request's tokens equal its own greedy run
whenever it was admitted.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import qwen3_b200 as q

DEFAULT_EOS = (151645, 151643)  # engine.rs:266-272 fallback


@dataclass
class Request:
    rid: int
    prompt: list
    max_new: int
    tokens: list = field(default_factory=list)
    produced: int = 0  # picks so far (a terminating EOS included)
    finish: str = ""   # "stop" (EOS) or "length"
    cache: object = None
    last: int = -1


class BatchScheduler:
    def __init__(self, model: "q.Qwen3", max_batch: int = 8, max_pos: int = 4096, eos=None):
        if not 1 <= max_batch <= 8:
            raise ValueError("max_batch must be 1..8")
        self.model = model
        self.max_batch = max_batch
        self.max_pos = max_pos
        self.eos = set(int(e) for e in (eos if eos is not None else DEFAULT_EOS))
        self.waiting: deque = deque()
        self.active: list = []
        self.done: dict = {}
        self._free: list = []
        self._next_id = 0

    def submit(self, prompt, max_new: int) -> int:
        """Queue a greedy request; returns its id."""
        prompt = [int(t) for t in prompt]
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + max(max_new, 1) > self.max_pos:
            raise q.KvExhausted(q.QW_ERR_KV_EXHAUSTED, "prompt + max_new exceeds the scheduler's cache length")
        rid = self._next_id
        self._next_id += 1
        self.waiting.append(Request(rid, prompt, max(max_new, 1)))
        return rid

    def _cache(self):
        if self._free:
            c = self._free.pop()
            c.reset()
            return c
        return self.model.new_cache(self.max_pos)

    def _retire(self, r: Request, finish: str):
        r.finish = finish
        self.done[r.rid] = r
        self._free.append(r.cache)
        r.cache = None

    def _pick(self, r: Request, tok: int) -> bool:
        """Bookkeeping of one pick (engine.rs:161-173); False once the request is finished."""
        r.produced += 1
        if tok in self.eos:
            self._retire(r, "stop")
            return False
        r.tokens.append(tok)
        r.last = tok
        if r.produced >= r.max_new:
            self._retire(r, "length")
            return False
        return True

    def step(self) -> list:
        """Admit waiting requests into free batch slots (prefill each), then run
        one batched decode step over the active requests.  Returns the
        (request id, token) pairs emitted by this step."""
        emitted = []
        while self.waiting and len(self.active) < self.max_batch:
            r = self.waiting.popleft()
            r.cache = self._cache()
            _, tok = self.model.forward(r.prompt, r.cache, want_logits=False)
            tok = int(tok)
            if self._pick(r, tok):
                self.active.append(r)
            if tok not in self.eos:
                emitted.append((r.rid, tok))
        if not self.active:
            return emitted
        # requests admitted in this step have their first token already; the
        # batched step advances every active request by one token
        toks = [r.last for r in self.active]
        _, am = self.model.forward_batch(toks, [r.cache for r in self.active], want_logits=False)
        still = []
        for r, tok in zip(self.active, am):
            tok = int(tok)
            if tok not in self.eos:
                emitted.append((r.rid, tok))
            if self._pick(r, tok):
                still.append(r)
        self.active = still
        return emitted

    def idle(self) -> bool:
        return not self.waiting and not self.active

    def run(self) -> dict:
        """Step until every submitted request is finished; {id: tokens}."""
        while not self.idle():
            self.step()
        return {rid: r.tokens for rid, r in self.done.items()}

    def close(self):
        for r in self.active:
            if r.cache is not None:
                r.cache.close()
        for c in self._free:
            c.close()
        self.active, self._free = [], []
