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
* ``pick_topp`` restates the temperature / top-p branch of ``pick_next``
  (``engine.rs:203-263``) literally -- fp32 division by the temperature,
  softmax with sequential fp32 sums, a stable descending sort, sequential fp32
  cumulative sums for the top-p cutoff, the renormalising sum and the draw
  walk -- with the reference's ``rand::StdRng`` draw (rand 0.8, ChaCha12 seeded
  by ``seed_from_u64``; not vendored) replaced by ``sample_u(seed, counter)``,
  the counter-based generator the CUDA path shares.  ``generate_sampled`` is
  ``generate_text`` with that pick.
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


def sample_u(seed: int, counter: int) -> np.float32:
    """Uniform draw in [0, 1): top 24 bits of splitmix64(seed ^ splitmix64(counter)) / 2^24."""
    h = nm.splitmix64_int((seed & nm.MASK64) ^ nm.splitmix64_int(counter & nm.MASK64))
    return np.float32(h >> 40) * np.float32(1.0 / 16777216.0)


def pick_topp(logits: np.ndarray, temperature: float, top_p: float, u: float, exact: bool = False) -> int:
    """engine.rs:203-263 on one row of (bf16-valued) logits, draw u in [0, 1).

    exact=False is the reference's arithmetic: every sum sequential in fp32
    (which over a long flat tail drifts by up to ~1e-4 of probability mass and
    drops addends below half an ulp).  exact=True keeps the same fp32
    probabilities but sums in fp64 -- the arithmetic of the CUDA path."""
    if not temperature > 0.0:
        return int(argmax_first(np.asarray(logits, np.float32)))
    t = np.float32(max(np.float32(temperature), np.float32(1e-5)))
    p = (np.asarray(logits, np.float32) / t).astype(np.float32)
    mx = np.float32(p.max())
    p = np.exp(p - mx).astype(np.float32)
    acc_t = np.float64 if exact else np.float32
    total = np.float32(np.add.accumulate(p, dtype=acc_t)[-1])  # sequential sum
    p = (p / total).astype(np.float32)
    order = np.argsort(-p, kind="stable")
    top_pf = np.float32(min(max(top_p, 0.0), 1.0))
    cum = np.add.accumulate(p[order], dtype=acc_t)
    hit = np.nonzero(cum >= top_pf)[0]
    cutoff = int(hit[0]) + 1 if len(hit) else len(order)
    top = order[:cutoff]
    acc = np.add.accumulate(p[top], dtype=acc_t)
    renorm = np.float32(acc[-1])
    r = np.float32(np.float32(u) * renorm)
    pos = np.nonzero(acc >= r)[0]
    return int(top[pos[0]]) if len(pos) else int(top[-1])


def generate_sampled(model: Qwen3Ref, prompt, max_new: int, temperature: float, top_p: float, seed: int,
                     same_draw: bool = False, max_pos: int = 4096) -> GenResult:
    """generate_text with the sampled pick; pick i uses sample_u(seed, 0 if same_draw else i)."""
    cache = model.new_cache(max_pos)
    logits = model.forward(list(prompt), cache)
    out = []
    produced = 0
    finish = "length"
    while True:
        nxt = pick_topp(logits, temperature, top_p, sample_u(seed, 0 if same_draw else produced))
        produced += 1
        if model.is_eos(nxt):
            finish = "stop"
            break
        out.append(nxt)
        if produced >= max_new:
            break
        logits = model.forward([nxt], cache)
    return GenResult(out, produced, finish)


# ---- speculative sampling -----------------------------------------------------
# The reference falls back to plain sampled decoding for temperature > 0
# (speculative.rs:65-69).  The CUDA path runs the speculative-sampling rule
# over the sampled pick's distributions; this restates it with the CUDA
# sampler's arithmetic: fp32 softmax of logits / t (fp64 total rounded once),
# top-p nucleus over exact 2^-60 fixed-point masses (descending, ties by lower
# index), P(x) = p_x / mass(nucleus) in fp32; picks and index-order draws on
# the same fixed-point masses; draws from the counter-based generator
# (first token counter 2^40; iteration t: draft slot i 64t + i, acceptance
# 64t + 16 + i, residual / bonus 64t + 32).

_FX = 2.0 ** 60


def draw24(seed: int, counter: int) -> int:
    """Top 24 bits of splitmix64(seed ^ splitmix64(counter)): u = draw24 / 2^24."""
    return nm.splitmix64_int((seed & nm.MASK64) ^ nm.splitmix64_int(counter & nm.MASK64)) >> 40


def fx60(v) -> np.ndarray:
    """Probabilities -> uint64 masses in units of 2^-60 (round half to even; <= 0 -> 0)."""
    v = np.asarray(v, np.float32).astype(np.float64)
    return np.where(v > 0, np.rint(v * _FX), 0.0).astype(np.uint64)


def nucleus(logits, temperature: float, top_p: float):
    """(p, order, n_in, renorm): the fp32 softmax row, its stable descending order,
    the nucleus size and the nucleus mass as fp32."""
    t = np.float32(max(np.float32(temperature), np.float32(1e-5)))
    x = (np.asarray(logits, np.float32) / t).astype(np.float32)
    mx = np.float32(x.max())
    e = np.exp((x - mx).astype(np.float32)).astype(np.float32)
    tot = np.float32(e.astype(np.float64).sum())
    p = (e / tot).astype(np.float32)
    fx = fx60(p)
    T = int(fx60(np.float32(min(max(top_p, 0.0), 1.0))))
    order = np.argsort(-p, kind="stable")
    cum = np.cumsum(fx[order], dtype=np.uint64)
    hit = np.nonzero(cum >= np.uint64(T))[0]
    n_in = int(hit[0]) + 1 if len(hit) else len(order)
    renorm = np.float32(float(int(cum[n_in - 1])) / _FX)
    return p, order, cum, n_in, renorm


def dist_topp(logits, temperature: float, top_p: float) -> np.ndarray:
    """P over the vocabulary: p_x / mass inside the nucleus, 0 outside (fp32)."""
    p, order, _, n_in, renorm = nucleus(logits, temperature, top_p)
    P = np.zeros(len(p), np.float32)
    m = order[:n_in]
    P[m] = (p[m] / renorm).astype(np.float32)
    return P


def pick_fx(logits, temperature: float, top_p: float, U: int) -> int:
    """The sampled pick on fixed-point masses: the first element, in descending
    order, whose cumulative mass reaches u * mass(nucleus); the nucleus's last
    element when rounding walks past it."""
    p, order, cum, n_in, renorm = nucleus(logits, temperature, top_p)
    r = np.float32(np.float32(U * (1.0 / 16777216.0)) * renorm)
    T = np.uint64(int(fx60(r)))
    pos = np.nonzero(cum >= T)[0]
    if len(pos) == 0 and n_in == len(order):
        # the nucleus is the whole row: its last element that carries mass
        nz = np.nonzero(fx60(p[order]))[0]
        return int(order[int(nz[-1]) if len(nz) else 0])
    i = int(pos[0]) if len(pos) else n_in - 1
    return int(order[min(i, n_in - 1)])


def draw_index_order(w: np.ndarray, U: int) -> int:
    """The first index whose inclusive cumulative mass exceeds floor(R * U / 2^24),
    R = the total mass; -1 when R = 0."""
    R = int(np.sum(w, dtype=np.uint64))
    if R == 0:
        return -1
    tgt = (R >> 24) * U + (((R & 0xFFFFFF) * U) >> 24)
    cum = np.cumsum(w, dtype=np.uint64)
    return int(np.nonzero(cum > np.uint64(tgt))[0][0])


def spec_generate_sampled(target, draft, prompt, max_new: int, k: int, temperature: float, top_p: float,
                          seed: int, max_pos: int = 4096):
    """Speculative sampling with the rule above; models need forward(tokens, cache,
    return_all), new_cache(max_pos), is_eos(token) and cache.truncate(n) (Qwen3Ref,
    or a wrapper of the CUDA model).  Returns (GenResult, SpecStats)."""
    prompt = list(prompt)
    tc = target.new_cache(max_pos)
    dc = draft.new_cache(max_pos)
    plen = len(prompt)
    tl = target.forward(prompt, tc, return_all=True)
    draft.forward(prompt, dc, return_all=True)
    leader = pick_fx(tl[plen - 1], temperature, top_p, draw24(seed, 1 << 40))
    stats = SpecStats()
    if target.is_eos(leader):
        return GenResult([], 0, "stop"), stats
    emitted = [leader]
    finish = "length"
    dlog = draft.forward([leader], dc)
    while len(emitted) < max_new:
        it64 = stats.iters * 64
        drafts, Q = [], []
        for slot in range(k):
            Q.append(dist_topp(dlog, temperature, top_p))
            d = pick_fx(dlog, temperature, top_p, draw24(seed, it64 + slot))
            drafts.append(d)
            dlog = draft.forward([d], dc)
            if draft.is_eos(d):
                break
        n = len(drafts)
        tlog = target.forward([leader] + drafts, tc, return_all=True)
        n_acc = 0
        while n_acc < n:
            d = drafts[n_acc]
            P = dist_topp(tlog[n_acc], temperature, top_p)
            u = np.float32(draw24(seed, it64 + 16 + n_acc) * (1.0 / 16777216.0))
            if np.float32(u * Q[n_acc][d]) < P[d]:
                n_acc += 1
            else:
                break
        P = dist_topp(tlog[n_acc], temperature, top_p)
        U = draw24(seed, it64 + 32)
        bonus = -1
        if n_acc < n:
            bonus = draw_index_order(fx60(np.maximum((P - Q[n_acc]).astype(np.float32), np.float32(0.0))), U)
        if bonus < 0:
            bonus = max(draw_index_order(fx60(P), U), 0)
        stats.proposed += n
        stats.iters += 1
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
