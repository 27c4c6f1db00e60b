"""Sampled decode on the device (engine.rs:149-263 with temperature / top-p)
against the oracle's literal restatement of pick_next (oracle/decode_ref.py),
both drawing u from the same counter-based generator.

* qw_sample_topp on synthetic logits rows against pick_topp(exact=True), the
  same restatement with fp64 sums (the device's arithmetic): >= 97% equal, the
  rest within 1e-6 of cumulative probability mass.  Against the literal fp32
  arithmetic of the reference the picks differ by at most that arithmetic's
  own drift (sequential fp32 cumulative sums over a long flat tail), measured
  per case.
* qw_generate_sampled: every pick equals the oracle's pick on the same logits
  (the device loop's own logits, replayed through qw_forward); top_p = 0 and
  temperature 0 reproduce greedy generation exactly; EOS stops the loop.
"""
import numpy as np
import pytest

from oracle import numerics as nm
from oracle import synth
from oracle.decode_ref import pick_topp, sample_u

pytestmark = pytest.mark.gpu
NOEOS = 1 << 30  # an end-of-sequence id no vocabulary produces: runs go to max_new


def _dev_pick(torch, q, lg_bits, t, top_p, seed, counter):
    dev = torch.device("cuda:0")
    x = torch.from_numpy(lg_bits.view(np.int16).copy()).to(dev)
    probs = torch.zeros(q.sample_scratch_bytes(lg_bits.size) // 4, dtype=torch.float32, device=dev)
    tok = torch.full((1,), -7, dtype=torch.int32, device=dev)
    q.sample_topp(x.data_ptr(), lg_bits.size, t, top_p, seed, counter, probs.data_ptr(), tok.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return int(tok.item())


@pytest.mark.parametrize("V,sigma", [(151936, 1.0), (151936, 6.0), (1000, 3.0)])
def test_sample_topp_matches_oracle(V, sigma):
    import torch
    import qwen3_b200 as q
    rng = np.random.default_rng(V + int(sigma))
    lg = nm.bf16_round((rng.standard_normal(V) * sigma).astype(np.float32))
    bits = nm.f32_to_bf16_bits(lg)
    total = same = 0
    for t, top_p in [(0.7, 0.95), (1.0, 0.5), (1.3, 1.0), (0.8, 0.0)]:
        pr = (lg / np.float32(t)).astype(np.float32)
        pr = np.exp(pr - pr.max()).astype(np.float32)
        pf = (pr / np.float32(np.add.accumulate(pr, dtype=np.float32)[-1])).astype(np.float32)
        order = np.argsort(-pf, kind="stable")
        rank = np.empty(V, np.int64)
        rank[order] = np.arange(V)
        cum64 = np.cumsum(pf[order].astype(np.float64))
        drift = float(np.abs(np.add.accumulate(pf[order], dtype=np.float32) - cum64).max())
        for c in range(24):
            u = sample_u(11, c)
            ref = pick_topp(lg, t, top_p, u, exact=True)
            lit = pick_topp(lg, t, top_p, u)
            got = _dev_pick(torch, q, bits, t, top_p, 11, c)
            total += 1
            same += got == ref
            assert 0 <= got < V
            assert abs(cum64[rank[got]] - cum64[rank[ref]]) <= 1e-6, (t, top_p, c, got, ref)
            assert abs(cum64[rank[got]] - cum64[rank[lit]]) <= drift + 1e-6, (t, top_p, c, got, lit, drift)
            if top_p == 0.0:
                assert got == int(np.argmax(lg))
    assert same / total >= 0.97, same / total


def test_sample_topp_greedy_and_single_entry():
    import torch
    import qwen3_b200 as q
    lg = nm.bf16_round(np.random.default_rng(2).standard_normal(5000).astype(np.float32))
    lg[4321] = lg.max() + 1.0
    assert _dev_pick(torch, q, nm.f32_to_bf16_bits(lg), 0.0, 0.9, 1, 0) == 4321
    one = nm.f32_to_bf16_bits(np.array([0.25], np.float32))
    assert _dev_pick(torch, q, one, 0.9, 0.5, 3, 9) == 0


def _model(cfg, seed=21):
    import qwen3_b200 as q
    return q.Qwen3.init_random(cfg, seed, norm_mode="random")


def _replay_logits(m, prompt, tokens):
    """The logits each pick of a generation saw, through qw_forward (same kernels)."""
    c = m.new_cache(1024)
    try:
        lg, _ = m.forward(prompt, c)
        rows = [lg]
        for tk in tokens[:-1]:
            lg, _ = m.forward([tk], c)
            rows.append(lg)
        return rows
    finally:
        c.close()


@pytest.mark.parametrize("same_draw", [False, True])
def test_generate_sampled_picks_match_oracle(same_draw):
    cfg = synth.tiny_config()
    m = _model(cfg)
    try:
        prompt = np.random.default_rng(4).integers(0, cfg["vocab_size"], 30).tolist()
        t, top_p, seed = 0.9, 0.9, 1234
        res = m.generate_sampled(prompt, 24, temperature=t, top_p=top_p, seed=seed,
                                 same_draw_each_token=same_draw, eos=[NOEOS])
        assert len(res.tokens) == 24 and res.finish_reason == "length"
        rows = _replay_logits(m, prompt, res.tokens)
        picks = [pick_topp(r, t, top_p, sample_u(seed, 0 if same_draw else i)) for i, r in enumerate(rows)]
        mism = sum(a != b for a, b in zip(picks, res.tokens))
        assert mism <= 1, (picks, res.tokens)
        # a different seed samples a different continuation
        other = m.generate_sampled(prompt, 24, temperature=t, top_p=top_p, seed=seed + 1,
                                   same_draw_each_token=same_draw, eos=[NOEOS])
        assert other.tokens != res.tokens
    finally:
        m.close()


def test_generate_sampled_degenerate_cases_equal_greedy():
    cfg = synth.tiny_config()
    m = _model(cfg)
    try:
        prompt = np.random.default_rng(5).integers(0, cfg["vocab_size"], 20).tolist()
        g = m.generate_greedy(prompt, 32, eos=[NOEOS])
        assert m.generate_sampled(prompt, 32, temperature=0.8, top_p=0.0, seed=3, eos=[NOEOS]).tokens == g.tokens
        assert m.generate_sampled(prompt, 32, temperature=0.0, top_p=0.9, seed=3, eos=[NOEOS]).tokens == g.tokens
        # EOS: the greedy token at step 5 made an EOS id stops the loop at its first occurrence
        k = g.tokens.index(g.tokens[5])
        stop = m.generate_sampled(prompt, 32, temperature=0.8, top_p=0.0, seed=3, eos=[g.tokens[5]])
        assert stop.tokens == g.tokens[:k] and stop.finish_reason == "stop" and stop.completion_tokens == k + 1
    finally:
        m.close()


def test_generate_sampled_4b_top_p_zero_is_greedy():
    cfg = dict(synth.QWEN3_4B)
    m = _model(cfg, seed=99)
    try:
        prompt = np.random.default_rng(6).integers(0, cfg["vocab_size"], 64).tolist()
        g = m.generate_greedy(prompt, 32, eos=[NOEOS])
        s = m.generate_sampled(prompt, 32, temperature=0.7, top_p=0.0, seed=8, eos=[NOEOS])
        assert s.tokens == g.tokens
    finally:
        m.close()
