"""Continuous batching (base-mlx_b200/serving.py): requests admitted while others
are decoding, more requests than batch slots, different budgets and EOS stops.
Every request's tokens must equal its own greedy run (generate_text,
engine.rs:149-201), whatever it shared its batched steps with."""
import numpy as np
import pytest

from oracle import synth

pytestmark = pytest.mark.gpu
NOEOS = 1 << 30


@pytest.fixture(scope="module")
def tiny():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    m = q.Qwen3.init_random(cfg, 11, norm_mode="random")
    yield cfg, m
    m.close()


def test_continuous_batching_equals_solo_runs(tiny):
    from serving import BatchScheduler
    cfg, m = tiny
    rng = np.random.default_rng(8)
    reqs = [([int(t) for t in rng.integers(0, cfg["vocab_size"], n)], mn)
            for n, mn in [(5, 12), (40, 30), (9, 1), (17, 25), (3, 8), (60, 20), (11, 16)]]
    sched = BatchScheduler(m, max_batch=3, max_pos=256, eos=[NOEOS])
    ids = {}
    ids[sched.submit(*reqs[0])] = 0
    ids[sched.submit(*reqs[1])] = 1
    sched.step()
    sched.step()
    for i in range(2, 5):  # arrive mid-flight, more than the free slots
        ids[sched.submit(*reqs[i])] = i
    sched.step()
    for i in range(5, 7):
        ids[sched.submit(*reqs[i])] = i
    out = sched.run()
    for rid, i in ids.items():
        prompt, mn = reqs[i]
        assert out[rid] == m.generate_greedy(prompt, mn, eos=[NOEOS]).tokens, i
        assert sched.done[rid].finish == "length"
    sched.close()


def test_continuous_batching_eos_leaves_the_batch(tiny):
    from serving import BatchScheduler
    cfg, m = tiny
    rng = np.random.default_rng(21)
    prompts = [[int(t) for t in rng.integers(0, cfg["vocab_size"], n)] for n in (7, 13, 22)]
    solo = [m.generate_greedy(p, 20, eos=[NOEOS]).tokens for p in prompts]
    stop = solo[1][6]  # the second request's 7th token is an EOS id
    sched = BatchScheduler(m, max_batch=8, max_pos=128, eos=[stop])
    rids = [sched.submit(p, 20) for p in prompts]
    out = sched.run()
    for rid, s in zip(rids, solo):
        want = s[:s.index(stop)] if stop in s else s
        assert out[rid] == want
    assert sched.done[rids[1]].finish == "stop"
    sched.close()
