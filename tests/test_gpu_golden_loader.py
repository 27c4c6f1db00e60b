"""CUDA path against the committed golden fixtures, and the safetensors loader
(the tensor-name contract of crates/base-mlx-core/src/model/qwen3.rs:194-295).

* tiny model (seeded, tests/golden/tiny_model.npz): last-row logits within
  2e-2 of the oracle's bf16 logits; greedy tokens, speculative tokens and
  per-iteration accept counts equal to the fixture;
* a checkpoint written in MLX safetensors layout (1 and 3 shards) loads into
  the same bits as the seeded on-device initialisation and decodes the same
  tokens; a missing tensor and an unmapped tensor raise ModelLoad with the
  crate's messages.
"""
import json
import os

import numpy as np
import pytest

from oracle import numerics as nm
from oracle import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def tiny_pair():
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    t = q.Qwen3.init_random(cfg, 11, norm_mode="random")
    d = q.Qwen3.init_random(cfg, 12, norm_mode="random")
    yield cfg, t, d
    d.close()
    t.close()


def test_golden_tiny_on_gpu(tiny_pair):
    import qwen3_b200 as q
    g = np.load(os.path.join(GOLDEN, "tiny_model.npz"))
    cfg, t, d = tiny_pair
    prompt = g["prompt"].tolist()
    c = t.new_cache(64)
    lg, am = t.forward(prompt, c)
    ref = nm.bf16_bits_to_f32(g["logits_bits"])
    assert np.abs(lg - ref).max() <= 2e-2
    assert am == int(np.argmax(ref))
    c.close()
    assert t.generate_greedy(prompt, 16).tokens == g["greedy"].tolist()
    res, st = q.speculative_generate(t, d, prompt, 16, k=4, force_p=0.8, seed=1, forced=g["greedy"].tolist())
    assert res.tokens == g["spec_k4_p08"].tolist()
    assert [st.iters, st.proposed, st.accepted] == g["spec_k4_p08_stats"].tolist()
    res, st = q.speculative_generate(t, d, prompt, 16, k=3, force_p=0.0, seed=1)
    assert res.tokens == g["spec_k3_p0"].tolist()
    assert [st.iters, st.proposed, st.accepted] == g["spec_k3_p0_stats"].tolist()


@pytest.mark.parametrize("shards", [1, 3])
def test_safetensors_checkpoint_loads_same_bits(tmp_path, tiny_pair, shards):
    import qwen3_b200 as q
    cfg, t, _ = tiny_pair
    synth.write_checkpoint(str(tmp_path), cfg, 11, norm_mode="random", shards=shards)
    m = q.Qwen3.load(str(tmp_path))
    try:
        for name in ["model.embed_tokens.weight", "model.layers.1.mlp.down_proj.scales",
                     "model.layers.0.self_attn.k_norm.weight", "model.norm.weight"]:
            ref = synth.build_tensors(cfg, 11, "random")[name]
            assert np.array_equal(m.export_tensor(name, ref.shape, ref.dtype), ref), name
        prompt = [3, 1, 4, 1, 5, 9, 2, 6]
        c1, c2 = m.new_cache(64), t.new_cache(64)
        l1, _ = m.forward(prompt, c1)
        l2, _ = t.forward(prompt, c2)
        assert np.array_equal(l1, l2)
        assert m.generate_greedy(prompt, 12).tokens == t.generate_greedy(prompt, 12).tokens
        c1.close()
        c2.close()
    finally:
        m.close()


def test_safetensors_missing_and_unmapped_tensors(tmp_path):
    import qwen3_b200 as q
    cfg = synth.tiny_config()
    tensors = synth.build_tensors(cfg, 5, "ones")
    missing = dict(tensors)
    del missing["model.layers.1.self_attn.o_proj.biases"]
    synth.write_checkpoint(str(tmp_path / "a"), cfg, 5, tensors=missing)
    with pytest.raises(q.ModelLoad, match="missing tensor"):
        q.Qwen3.load(str(tmp_path / "a"))
    extra = dict(tensors)
    extra["model.layers.0.mlp.extra_proj.weight"] = np.zeros((4, 4), np.uint32)
    synth.write_checkpoint(str(tmp_path / "b"), cfg, 5, tensors=extra)
    with pytest.raises(q.ModelLoad, match="unmapped tensors"):
        q.Qwen3.load(str(tmp_path / "b"))
