"""Speculative sampling on the device (temperature > 0) against the oracle's
restatement (oracle/decode_ref.spec_generate_sampled).

The reference falls back to plain sampled decoding for temperature > 0
(speculative.rs:65-69); the CUDA path runs the rejection rule over the sampled
pick's distributions.  Parity is taken on the device's own logits: the oracle
loop drives the same CUDA models through qw_forward (a row's logits do not
depend on how many rows share its forward, so they equal the ones the device
loop computed), and its acceptance tests, residual draws and picks -- numpy
restatements of the CUDA arithmetic -- must reproduce the device's tokens and
(iterations, proposed, accepted) exactly.
"""
import numpy as np
import pytest

from oracle import synth
from oracle.decode_ref import spec_generate_sampled

pytestmark = pytest.mark.gpu
NOEOS = 1 << 30


class DevModel:
    """The oracle's model interface over a CUDA model (qw_forward).  As a draft
    (fold=True) it runs the device loop's schedule: the prompt's last token is
    held back from the prefill and run with the next token as one 2-row step."""

    def __init__(self, m, fold=False):
        self.m = m
        self.fold = fold
        self.pending = None

    def new_cache(self, max_pos):
        return self.m.new_cache(max_pos)

    def forward(self, tokens, cache, return_all=False):
        tokens = [int(t) for t in tokens]
        if self.fold and len(tokens) > 1 and cache.seq_len == 0:
            self.pending = tokens[-1]
            if len(tokens) > 1:
                self.m.forward(tokens[:-1], cache, want_logits=False)
            return None
        if self.pending is not None:
            tokens = [self.pending] + tokens
            self.pending = None
            lg, _ = self.m.forward_multi(tokens, cache)
            return lg[-1]
        if len(tokens) > 8:
            # prefill: the last row's logits, as the device loop computes them (lm_head on one row)
            lg, _ = self.m.forward(tokens, cache)
            if not return_all:
                return lg
            out = np.zeros((len(tokens), lg.shape[-1]), np.float32)
            out[-1] = lg
            return out
        lg, _ = self.m.forward_multi(tokens, cache)
        return lg if return_all else lg[-1]

    def is_eos(self, t):
        return int(t) == NOEOS


@pytest.fixture(scope="module")
def pair():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    t = q.Qwen3.init_random(cfg, 11, norm_mode="random")
    d = q.Qwen3.init_random(cfg, 12, norm_mode="random")
    yield cfg, t, d
    t.close()
    d.close()


@pytest.mark.parametrize("k,temperature,top_p,seed", [(3, 0.8, 0.9, 5), (4, 1.0, 0.95, 17), (4, 0.6, 1.0, 3)])
def test_spec_sampled_matches_oracle(pair, k, temperature, top_p, seed):
    import qwen3_b200 as q
    cfg, t, d = pair
    prompt = [int(x) for x in np.random.default_rng(seed).integers(0, cfg["vocab_size"], 21)]
    res, st = q.speculative_generate_sampled(t, d, prompt, 40, k=k, temperature=temperature, top_p=top_p,
                                             seed=seed, eos=[NOEOS])
    ref, rst = spec_generate_sampled(DevModel(t), DevModel(d, fold=True), prompt, 40, k, temperature, top_p, seed,
                                     max_pos=512)
    assert res.tokens == ref.tokens
    assert (st.iters, st.proposed, st.accepted) == (rst.iters, rst.proposed, rst.accepted)
    assert 0 < st.accepted < st.proposed  # both outcomes exercised


def test_spec_sampled_identical_draft_accepts_all(pair):
    """Draft = target (same weights): P = Q at every drafted token, so u * Q < P
    always holds and every draft is accepted."""
    import qwen3_b200 as q
    cfg, t, _ = pair
    twin = q.Qwen3.init_random(cfg, 11, norm_mode="random")
    prompt = [int(x) for x in np.random.default_rng(2).integers(0, cfg["vocab_size"], 15)]
    res, st = q.speculative_generate_sampled(t, twin, prompt, 30, k=4, temperature=0.9, top_p=0.9, seed=9,
                                             eos=[NOEOS])
    assert st.accepted == st.proposed and st.proposed > 0
    ref, rst = spec_generate_sampled(DevModel(t), DevModel(twin, fold=True), prompt, 30, 4, 0.9, 0.9, 9, max_pos=512)
    assert res.tokens == ref.tokens
    twin.close()


def test_spec_sampled_temperature_zero_is_greedy_spec(pair):
    import qwen3_b200 as q
    cfg, t, d = pair
    prompt = [int(x) for x in np.random.default_rng(4).integers(0, cfg["vocab_size"], 12)]
    a, sa = q.speculative_generate_sampled(t, d, prompt, 24, k=3, temperature=0.0, top_p=0.9, seed=1, eos=[NOEOS])
    b, sb = q.speculative_generate(t, d, prompt, 24, k=3, eos=[NOEOS])
    assert a.tokens == b.tokens == t.generate_greedy(prompt, 24, eos=[NOEOS]).tokens
    assert (sa.iters, sa.accepted) == (sb.iters, sb.accepted)
