"""Greedy and speculative generation loops on the CPU -- TEST INFRASTRUCTURE ONLY.

* ``generate_greedy`` restates ``LoadedModel::generate_text``
  (``crates/base-mlx-core/src/engine.rs:149-193``) with the greedy branch of
  ``pick_next`` (``engine.rs:197-201``) and ``is_eos`` (``engine.rs:266-272``).
* ``spec_generate`` restates ``speculative::generate``
  (``crates/base-mlx-core/src/speculative.rs:57-240``) with the number of
  drafted tokens ``k`` as a parameter (the reference's ``SPEC_K=4`` drafts
  ``k=3``), plus the forced-acceptance hook that the benchmark needs: after
  each draft argmax (``speculative.rs:126``), with probability ``force_p`` the
  drafted token is replaced by the plain-greedy target token for that
  position, ``forced_seq[len(emitted) + slot]``; the uniform draw is
  ``numerics.uniform01(seed, iteration, slot)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import numerics as nm
from .qwen3_ref import Qwen3Ref, argmax_first


@dataclass
class GenResult:
    tokens: list
    completion_tokens: int
    finish_reason: str
    margins: list = field(default_factory=list)  # top1 - top2 logit at every pick


def _margin(logits: np.ndarray) -> float:
    top2 = np.partition(logits, -2)[-2:]
    return float(top2[1] - top2[0])


def generate_greedy(model: Qwen3Ref, prompt, max_new: int, max_pos: int = 4096) -> GenResult:
    cache = model.new_cache(max_pos)
    logits = model.forward(list(prompt), cache)
    out, margins = [], []
    produced = 0
    finish = "length"
    while True:
        nxt = int(argmax_first(logits))
        margins.append(_margin(logits))
        produced += 1
        if model.is_eos(nxt):
            finish = "stop"
            break
        out.append(nxt)
        if produced >= max_new:
            break
        logits = model.forward([nxt], cache)
    return GenResult(out, produced, finish, margins)


@dataclass
class SpecStats:
    iters: int = 0
    proposed: int = 0
    accepted: int = 0
    accepted_per_iter: list = field(default_factory=list)
    proposed_per_iter: list = field(default_factory=list)


def spec_generate(target: Qwen3Ref, draft: Qwen3Ref, prompt, max_new: int, k: int = 3,
                  force_p: float = 0.0, seed: int = 0, forced_seq=None, max_pos: int = 4096):
    """Returns (GenResult, SpecStats)."""
    prompt = list(prompt)
    tc = target.new_cache(max_pos)
    dc = draft.new_cache(max_pos)
    plen = len(prompt)
    tl = target.forward(prompt, tc, return_all=True)
    draft.forward(prompt, dc, return_all=True)
    leader = int(argmax_first(tl[plen - 1]))
    stats = SpecStats()
    if target.is_eos(leader):
        return GenResult([], 0, "stop"), stats
    emitted = [leader]
    finish = "length"
    dlog = draft.forward([leader], dc)
    fp = np.float32(force_p)
    while len(emitted) < max_new:
        drafts = []
        for slot in range(k):
            d = int(argmax_first(dlog))
            if forced_seq is not None and fp > 0:
                pos = len(emitted) + slot
                if pos < len(forced_seq) and nm.uniform01(seed, stats.iters, slot) < fp:
                    d = int(forced_seq[pos])
            drafts.append(d)
            dlog = draft.forward([d], dc)
            if draft.is_eos(d):
                break
        vin = [leader] + drafts
        tlog = target.forward(vin, tc, return_all=True)
        n = len(drafts)
        stats.proposed += n
        stats.iters += 1
        preds = argmax_first(tlog)
        n_acc = 0
        bonus = None
        for i in range(n):
            if int(preds[i]) == drafts[i]:
                n_acc += 1
            else:
                bonus = int(preds[i])
                break
        if bonus is None:
            bonus = int(preds[n])
        stats.accepted += n_acc
        stats.accepted_per_iter.append(n_acc)
        stats.proposed_per_iter.append(n)
        stop = False
        for t in drafts[:n_acc]:
            if len(emitted) >= max_new:
                stop = True
                break
            if target.is_eos(t):
                finish = "stop"
                stop = True
                break
            emitted.append(t)
        if stop:
            break
        if len(emitted) >= max_new:
            break
        if target.is_eos(bonus):
            finish = "stop"
            break
        emitted.append(bonus)
        tc.truncate(plen + len(emitted) - 1)
        dc.truncate(plen + len(emitted) - 1)
        leader = bonus
        dlog = draft.forward([leader], dc)
    return GenResult(emitted, len(emitted), finish), stats
