"""CPU oracle for the Qwen3 4-bit decode path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package.  The
product (the CUDA library under ``base-mlx_b200/``) never calls into it.

What it restates (paths relative to the flakerimi/base-mlx project root):

* ``crates/base-mlx-core/src/model/qwen3.rs:314-563`` -- ``Qwen3::forward_internal``
  op by op, with bf16 rounding at every MLX op output (qmatmul, rms_norm,
  rope, sdpa, silu, multiply, add) and fp32 inside reductions;
* ``crates/base-mlx-core/src/model/kernels.rs:28-78`` -- ``qkv_block`` / ``mlp_block``;
* ``crates/base-mlx-core/src/engine.rs:149-201,266-272`` -- greedy ``generate_text``,
  ``pick_next`` (greedy branch) and ``is_eos``;
* ``crates/base-mlx-core/src/speculative.rs:57-240`` -- the greedy speculative loop,
  with ``k`` as a runtime parameter (``k=3`` is the reference's ``SPEC_K=4``).

PARITY UNPINNED.  The reference has no tests, fixtures or golden vectors,
and its arithmetic lives in the third-party crates ``mlx-rs 0.25.3`` /
``mlx-sys 0.2.0`` (MLX C++/Metal), which are not vendored and cannot be built
or run on this machine (no Rust toolchain, no Metal).  The oracle is pinned
only by the known-answer tests under ``tests/`` (nibble order, quantizer
round trip, hand-computed RMSNorm / RoPE / attention values) and by the
committed fixtures in ``tests/golden/`` that it generated itself.
"""
