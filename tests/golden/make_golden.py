"""Regenerates the golden fixtures in this directory from the CPU oracle.

The reference (Rust over MLX/Metal) cannot run here and ships no fixtures of
its own, so these vectors pin the oracle itself (regression) and serve as
fixed CUDA parity targets.  Run from the repository root:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import numerics as nm  # noqa: E402
from oracle import synth  # noqa: E402
from oracle.decode_ref import generate_greedy, spec_generate  # noqa: E402
from oracle.qwen3_ref import Qwen3Ref, rope_tables  # noqa: E402

TINY_PROMPT = [3, 1, 4, 1, 5, 9, 2, 6]


def fixed_matrix(n: int, k: int) -> np.ndarray:
    """A deterministic, non-random fp32 matrix with varied group ranges (incl. a constant group)."""
    i = np.arange(n, dtype=np.float64)[:, None]
    j = np.arange(k, dtype=np.float64)[None, :]
    w = 0.03 * np.sin(0.7 * i + 0.13 * j) + 0.001 * (j % 7) - 0.0005 * i
    w[1, 64:128] = 0.25  # constant group: scale 0, every q = 0
    return w.astype(np.float32)


def main() -> None:
    # quantizer on a fixed matrix
    w = fixed_matrix(32, 128)
    q, s, b = nm.quantize_groups(w)
    np.savez_compressed(os.path.join(HERE, "quantizer.npz"), w=w, packed=nm.pack_nibbles(q), scales=s, biases=b)

    # seeded weights (the generator shared by numpy, C and CUDA)
    pw, ps, pb = nm.quantized_weight(7, 5, 16, 128)
    np.savez_compressed(os.path.join(HERE, "seeded_weight.npz"), w=pw, scales=ps, biases=pb,
                        norm_random=nm.norm_weight(7, 9, 128, "random"))

    # RoPE tables (theta 1e6, head_dim 128) at a few positions
    cos, sin = rope_tables(4096, 128, 1.0e6)
    pos = np.array([0, 1, 511, 4095])
    np.savez_compressed(os.path.join(HERE, "rope.npz"), positions=pos, cos=cos[pos], sin=sin[pos])

    # tiny model: forward logits, greedy and speculative decoding
    cfg = synth.tiny_config()
    tgt = Qwen3Ref(cfg, synth.build_tensors(cfg, 11, "random"))
    drf = Qwen3Ref(cfg, synth.build_tensors(cfg, 12, "random"))
    cache = tgt.new_cache(64)
    logits = tgt.forward(TINY_PROMPT, cache)
    greedy = generate_greedy(tgt, TINY_PROMPT, 16)
    spec_a, st_a = spec_generate(tgt, drf, TINY_PROMPT, 16, k=4, force_p=0.8, seed=1, forced_seq=greedy.tokens)
    spec_b, st_b = spec_generate(tgt, drf, TINY_PROMPT, 16, k=3, force_p=0.0, seed=1, forced_seq=None)
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), prompt=np.array(TINY_PROMPT, np.int64),
                        logits_bits=nm.f32_to_bf16_bits(logits), greedy=np.array(greedy.tokens, np.int64),
                        spec_k4_p08=np.array(spec_a.tokens, np.int64),
                        spec_k4_p08_stats=np.array([st_a.iters, st_a.proposed, st_a.accepted], np.int64),
                        spec_k4_p08_accepted_per_iter=np.array(st_a.accepted_per_iter, np.int64),
                        spec_k3_p0=np.array(spec_b.tokens, np.int64),
                        spec_k3_p0_stats=np.array([st_b.iters, st_b.proposed, st_b.accepted], np.int64),
                        spec_k3_p0_accepted_per_iter=np.array(st_b.accepted_per_iter, np.int64))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
