"""End-to-end parity of the CUDA forward / greedy / spec paths against the oracle on a tiny Qwen3 config.

Logit tolerance: max-abs 2e-2 (the north_star's bf16 bound); token ids,
argmaxes and accepted-length counts must match exactly.
"""
import numpy as np
import pytest

from oracle import numerics as nm, synth
from oracle.decode_ref import generate_greedy, spec_generate
from oracle.qwen3_ref import Qwen3Ref

pytestmark = pytest.mark.gpu

SEED, DSEED = 11, 12


@pytest.fixture(scope="module")
def tiny():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    m = q.Qwen3.init_random(cfg, SEED, norm_mode="random")
    ref = Qwen3Ref(cfg, synth.build_tensors(cfg, SEED, "random"))
    yield cfg, m, ref
    m.close()


@pytest.fixture(scope="module")
def tiny_draft():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    m = q.Qwen3.init_random(cfg, DSEED, norm_mode="random")
    ref = Qwen3Ref(cfg, synth.build_tensors(cfg, DSEED, "random"))
    yield m, ref
    m.close()


def test_device_init_matches_oracle_bits(tiny):
    cfg, m, ref = tiny
    t = synth.build_tensors(cfg, SEED, "random")
    for name in ["model.embed_tokens.weight", "model.embed_tokens.scales", "model.layers.1.mlp.down_proj.biases",
                 "model.layers.0.self_attn.q_norm.weight", "model.layers.1.self_attn.v_proj.weight",
                 "model.norm.weight"]:
        a = t[name]
        got = m.export_tensor(name, a.shape, a.dtype)
        assert np.array_equal(got, a), name


def test_forward_logits_prefill_and_decode(tiny):
    cfg, m, ref = tiny
    prompt = [5, 17, 300, 2, 999, 64, 7, 8, 9, 10, 11, 12]
    c = m.new_cache(256)
    rc = ref.new_cache(256)
    lg, am = m.forward(prompt, c)
    rl = ref.forward(prompt, rc)
    assert np.abs(lg - rl).max() <= 2e-2
    assert am == int(np.argmax(rl))
    for tok in [am, 3, 4]:
        lg, am = m.forward([tok], c)
        rl = ref.forward([tok], rc)
        assert np.abs(lg - rl).max() <= 2e-2
        assert am == int(np.argmax(rl))
    assert c.seq_len == rc.seq_len
    # verify-shaped multi-row forward on a non-empty cache
    lg, am = m.forward_multi([1, 2, 3, 4, 5], c)
    rl = ref.forward([1, 2, 3, 4, 5], rc, return_all=True)
    assert np.abs(lg - rl).max() <= 2e-2
    assert list(am) == list(np.argmax(rl, axis=-1))
    c.close()


def test_kv_cache_contents_and_truncate(tiny):
    cfg, m, ref = tiny
    c = m.new_cache(64)
    rc = ref.new_cache(64)
    m.forward([1, 2, 3, 4, 5, 6, 7, 8, 9, 10], c, want_logits=False)
    ref.forward([1, 2, 3, 4, 5, 6, 7, 8, 9, 10], rc)
    for layer in range(cfg["num_hidden_layers"]):
        k = nm.bf16_bits_to_f32(c.read(layer, "k", 0, 10))
        v = nm.bf16_bits_to_f32(c.read(layer, "v", 0, 10))
        assert np.abs(k - rc.k[layer][:, :10]).max() <= 2e-2
        assert np.abs(v - rc.v[layer][:, :10]).max() <= 2e-2
    c.truncate(20)  # no-op when longer than the cache
    assert c.seq_len == 10
    c.truncate(6)
    rc.truncate(6)
    lg, _ = m.forward([42], c)
    rl = ref.forward([42], rc)
    assert np.abs(lg - rl).max() <= 2e-2
    # slice_update round trip
    upd = nm.f32_to_bf16_bits(np.full((cfg["num_key_value_heads"], 3, 128), 0.5, np.float32))
    c.slice_update(1, "v", upd, 30, 33)
    assert np.array_equal(c.read(1, "v", 30, 33), upd)
    c.reset()
    assert c.seq_len == 0
    c.close()


def test_kv_exhausted_is_an_error(tiny):
    import qwen3_b200 as q
    cfg, m, ref = tiny
    c = m.new_cache(8)
    m.forward([1, 2, 3, 4, 5, 6], c, want_logits=False)
    with pytest.raises(q.KvExhausted):
        m.forward([1, 2, 3], c)
    c.close()


def test_greedy_tokens_match(tiny):
    cfg, m, ref = tiny
    prompt = [1, 2, 3, 4, 5, 6, 7, 8, 9]
    r = generate_greedy(ref, prompt, 24)
    g = m.generate_greedy(prompt, 24)
    assert g.tokens == r.tokens
    assert g.completion_tokens == r.completion_tokens
    assert g.finish_reason == r.finish_reason


def test_greedy_stops_at_eos(tiny):
    cfg, m, ref = tiny
    prompt = [1, 2, 3, 4, 5, 6, 7, 8, 9]
    r = generate_greedy(ref, prompt, 24)
    eos = [r.tokens[5]]
    first = r.tokens.index(eos[0])
    g = m.generate_greedy(prompt, 24, eos=eos)
    assert g.tokens == r.tokens[:first]
    assert g.finish_reason == "stop"
    assert g.completion_tokens == first + 1


@pytest.mark.parametrize("k,p", [(3, 0.0), (4, 0.5), (4, 0.8), (4, 1.0)])
def test_spec_matches_oracle(tiny, tiny_draft, k, p):
    import qwen3_b200 as q
    cfg, m, ref = tiny
    dm, dref = tiny_draft
    prompt = [7, 3, 99, 512, 12, 1, 0, 44]
    plain = generate_greedy(ref, prompt, 40)
    rr, rst = spec_generate(ref, dref, prompt, 40, k=k, force_p=p, seed=3, forced_seq=plain.tokens)
    gr, gst = q.speculative_generate(m, dm, prompt, 40, k=k, force_p=p, seed=3, forced=plain.tokens)
    assert gr.tokens == rr.tokens
    assert gr.tokens == plain.tokens  # greedy spec output == plain greedy
    assert (gst.iters, gst.proposed, gst.accepted) == (rst.iters, rst.proposed, rst.accepted)
