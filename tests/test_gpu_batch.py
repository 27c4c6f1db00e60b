"""Batched greedy decode (benchmark config 5 at batch 8): several independent
sequences decoded together, each with its own cache and position, one
persistent decode step per token for all of them.

Every row of a batched step runs the single-sequence decode step's arithmetic
(the GEMV and RMSNorm summation orders do not depend on the row count, and
each sequence's attention items are the batch-1 items), so each sequence's
tokens and logits must equal its batch-1 run exactly.  The reference serves one
request at a time (model.rs:21-108); its per-request loop is
engine.rs:149-201.
"""
import numpy as np
import pytest

from oracle import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    m = q.Qwen3.init_random(cfg, 11, norm_mode="random")
    yield cfg, m
    m.close()


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [[int(t) for t in rng.integers(0, vocab, n)] for n in lens]


@pytest.mark.parametrize("lens", [[7], [5, 40, 13], [3, 9, 27, 64, 130, 1, 18, 250]])
def test_batch_equals_single_tiny(tiny, lens):
    cfg, m = tiny
    prompts = _prompts(cfg["vocab_size"], lens, 5 + len(lens))
    n_new = 40
    outs, st = m.generate_greedy_batch(prompts, n_new, eos=[1 << 30])
    assert len(outs) == len(prompts)
    for p, o in zip(prompts, outs):
        assert o == m.generate_greedy(p, n_new, eos=[1 << 30]).tokens
    assert st.completion_tokens == n_new * len(prompts)


def test_sub_batches_equal_single(tiny, monkeypatch):
    """A batch larger than one launch carries (forced to 3 rows here, as shared
    memory forces 4 on Qwen3-4B) runs as sub-batches with the same results."""
    cfg, m = tiny
    monkeypatch.setenv("QW_MK_BATCH_ROWS", "3")
    prompts = _prompts(cfg["vocab_size"], [4, 17, 9, 33, 2, 60, 8], 91)
    outs, _ = m.generate_greedy_batch(prompts, 25, eos=[1 << 30])
    for p, o in zip(prompts, outs):
        assert o == m.generate_greedy(p, 25, eos=[1 << 30]).tokens
    bc = [m.new_cache(128) for _ in prompts]
    toks = []
    for p, c in zip(prompts, bc):
        toks.append(m.forward(p, c, want_logits=False)[1])
    lg_b, am_b = m.forward_batch(toks, bc)
    for i, (p, t) in enumerate(zip(prompts, toks)):
        c = m.new_cache(128)
        m.forward(p, c, want_logits=False)
        lg, am = m.forward([t], c)
        assert np.array_equal(lg_b[i], lg) and int(am_b[i]) == am
        c.close()
    for c in bc:
        c.close()


def test_forward_batch_logits_equal_single(tiny):
    cfg, m = tiny
    prompts = _prompts(cfg["vocab_size"], [11, 70, 2, 129], 21)
    bc = [m.new_cache(512) for _ in prompts]
    sc = [m.new_cache(512) for _ in prompts]
    toks = []
    for p, c1, c2 in zip(prompts, bc, sc):
        _, t1 = m.forward(p, c1, want_logits=False)
        _, t2 = m.forward(p, c2, want_logits=False)
        assert t1 == t2
        toks.append(t1)
    for _ in range(3):
        lg_b, am_b = m.forward_batch(toks, bc)
        nxt = []
        for i, (t, c) in enumerate(zip(toks, sc)):
            lg, am = m.forward([t], c)
            assert np.array_equal(lg_b[i], lg), i
            assert int(am_b[i]) == am
            nxt.append(am)
        toks = nxt
    for c1, c2 in zip(bc, sc):
        assert c1.seq_len == c2.seq_len
        for layer in (0, cfg["num_hidden_layers"] - 1):
            assert np.array_equal(c1.read(layer, "k", 0, c1.seq_len), c2.read(layer, "k", 0, c2.seq_len))
            assert np.array_equal(c1.read(layer, "v", 0, c1.seq_len), c2.read(layer, "v", 0, c2.seq_len))
        c1.close()
        c2.close()


def test_batch_eos_stops_one_sequence(tiny):
    cfg, m = tiny
    prompts = _prompts(cfg["vocab_size"], [12, 30], 33)
    ref = [m.generate_greedy(p, 30, eos=[1 << 30]).tokens for p in prompts]
    stop = ref[0][10]  # the first sequence's 11th token becomes an EOS id
    outs, _ = m.generate_greedy_batch(prompts, 30, eos=[stop])
    for r, o in zip(ref, outs):
        want = r[:r.index(stop)] if stop in r else r
        assert o == want


def test_batch_rejects_bad_arguments(tiny):
    import qwen3_b200 as q
    cfg, m = tiny
    c = m.new_cache(64)
    with pytest.raises(q.Error):
        m.forward_batch([1, 2], [c, c])  # one cache twice
    with pytest.raises(q.Error):
        m.generate_greedy_batch([[1]] * 9, 4)  # more than 8 sequences
    with pytest.raises(q.KvExhausted):
        m.generate_greedy_batch([[1, 2, 3]], 100, caches=[c])
    c.close()


def test_batch8_equals_single_4b():
    """Config 5's batch-8 shape on Qwen3-4B: 8 prompts of 512 tokens, 24 tokens each."""
    import qwen3_b200 as q
    cfg = dict(synth.QWEN3_4B)
    m = q.Qwen3.init_random(cfg, 1234, norm_mode="ones")
    prompts = _prompts(cfg["vocab_size"], [512] * 8, 77)
    outs, st = m.generate_greedy_batch(prompts, 24, eos=[1 << 30])
    for p, o in zip(prompts, outs):
        assert o == m.generate_greedy(p, 24, eos=[1 << 30]).tokens
    m.close()
