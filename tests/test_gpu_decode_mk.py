"""The persistent decode kernel (one cooperative launch per step) against the
per-layer kernel chain and the CPU oracle.

Models created with QW_DECODE_KERNEL=multi in the environment run the kernel
chain; the default is the persistent kernel.  Tolerances: tiny model logits
<= 2e-2 max-abs against the oracle for both paths (shallow model); Qwen3-4B
logits of the two paths within the 4B noise bound (max-abs <= 0.25,
mean-abs <= 0.04) with equal argmax where the top-2 margin exceeds 0.25.
"""
import os

import numpy as np
import pytest

from oracle import synth

pytestmark = pytest.mark.gpu


def _model(cfg, seed, multi):
    import qwen3_b200 as q
    old = os.environ.get("QW_DECODE_KERNEL")
    try:
        if multi:
            os.environ["QW_DECODE_KERNEL"] = "multi"
        else:
            os.environ.pop("QW_DECODE_KERNEL", None)
        return q.Qwen3.init_random(cfg, seed, norm_mode="random")
    finally:
        if old is None:
            os.environ.pop("QW_DECODE_KERNEL", None)
        else:
            os.environ["QW_DECODE_KERNEL"] = old


@pytest.mark.parametrize("rows", [1, 3, 5, 8])
def test_tiny_persistent_vs_chain_and_oracle(rows):
    from oracle.qwen3_ref import Qwen3Ref
    cfg = synth.tiny_config()
    pk = _model(cfg, 31, multi=False)
    ch = _model(cfg, 31, multi=True)
    try:
        ref = Qwen3Ref(cfg, synth.build_tensors(cfg, 31, "random"))
        prompt = list(np.random.default_rng(4).integers(0, cfg["vocab_size"], 70))
        new = list(np.random.default_rng(5).integers(0, cfg["vocab_size"], rows))
        c1, c2, rc = pk.new_cache(256), ch.new_cache(256), ref.new_cache(256)
        pk.forward(prompt, c1, want_logits=False)
        ch.forward(prompt, c2, want_logits=False)
        ref.forward(prompt, rc)
        l1, a1 = pk.forward_multi(new, c1)
        l2, a2 = ch.forward_multi(new, c2)
        r = ref.forward(new, rc, return_all=True)
        assert np.abs(l1 - r).max() <= 2e-2, np.abs(l1 - r).max()
        assert np.abs(l2 - r).max() <= 2e-2, np.abs(l2 - r).max()
        assert list(a1) == list(np.argmax(l1, axis=-1))
        # both paths wrote the same KV rows, up to bf16 rounding noise (the two
        # paths sum the projections in different orders; normalised k, |k| ~ 1)
        from oracle import numerics as nm
        for layer in range(cfg["num_hidden_layers"]):
            for which in ("k", "v"):
                k1 = nm.bf16_bits_to_f32(c1.read(layer, which, 0, 70 + rows))
                k2 = nm.bf16_bits_to_f32(c2.read(layer, which, 0, 70 + rows))
                assert np.abs(k1 - k2).max() <= 0.1 and np.abs(k1 - k2).mean() <= 5e-3, (layer, which)
        assert c1.seq_len == c2.seq_len == 70 + rows
    finally:
        pk.close()
        ch.close()


def test_tiny_persistent_greedy_matches_oracle():
    from oracle.decode_ref import generate_greedy
    from oracle.qwen3_ref import Qwen3Ref
    cfg = synth.tiny_config()
    pk = _model(cfg, 33, multi=False)
    try:
        ref = Qwen3Ref(cfg, synth.build_tensors(cfg, 33, "random"))
        prompt = [5, 17, 200, 3, 999, 42]
        want = generate_greedy(ref, prompt, 40)
        got = pk.generate_greedy(prompt, 40)
        assert got.tokens == want.tokens
    finally:
        pk.close()


def test_4b_persistent_vs_chain():
    cfg = dict(synth.QWEN3_4B)
    pk = _model(cfg, 4243, multi=False)
    ch = _model(cfg, 4243, multi=True)
    try:
        prompt = list(np.random.default_rng(7).integers(0, cfg["vocab_size"], 300))
        c1, c2 = pk.new_cache(1024), ch.new_cache(1024)
        pk.forward(prompt, c1, want_logits=False)
        ch.forward(prompt, c2, want_logits=False)
        for rows in ([17], [1, 2, 3, 4, 5]):
            l1, a1 = pk.forward_multi(rows, c1)
            l2, a2 = ch.forward_multi(rows, c2)
            d = np.abs(l1 - l2)
            assert d.max() <= 0.25 and d.mean() <= 0.04, (d.max(), d.mean())
            for i in range(len(rows)):
                top2 = np.sort(l2[i])[-2:]
                if top2[1] - top2[0] > 0.25:
                    assert a1[i] == a2[i]
    finally:
        pk.close()
        ch.close()
