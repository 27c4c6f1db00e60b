"""Seeded random-init Qwen3 checkpoints in MLX layout -- TEST INFRASTRUCTURE ONLY.

Tensor names follow the loader contract of
``crates/base-mlx-core/src/model/qwen3.rs:194-295`` (``model.embed_tokens.*``,
``model.layers.{i}.{input_layernorm,post_attention_layernorm}.weight``,
``.self_attn.{q,k,v,o}_proj.{weight,scales,biases}``,
``.self_attn.{q,k}_norm.weight``, ``.mlp.{gate,up,down}_proj.*``,
``model.norm.weight`` and ``lm_head.*`` when embeddings are untied).

Every tensor has a fixed id (``tensor_id``); its values come from
``numerics.quantized_weight(seed, id, ...)`` / ``numerics.norm_weight``.  The CUDA
library's ``qw_model_init_random`` produces the same bits on the device.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

from . import numerics as nm

# ids of the per-model and per-layer tensors (shared with the CUDA initialiser)
TID_EMBED, TID_FINAL_NORM, TID_LM_HEAD = 0, 1, 2
(L_IN_NORM, L_Q, L_K, L_V, L_Q_NORM, L_K_NORM, L_O, L_POST_NORM,
 L_GATE, L_UP, L_DOWN) = range(11)


def layer_tid(layer: int, kind: int) -> int:
    return 16 + 16 * layer + kind


QWEN3_0_6B = dict(
    model_type="qwen3", hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
    num_attention_heads=16, num_key_value_heads=8, head_dim=128, vocab_size=151936,
    rms_norm_eps=1e-6, rope_theta=1000000.0, tie_word_embeddings=True,
    max_position_embeddings=40960, bos_token_id=151643, eos_token_id=151645,
    quantization=dict(group_size=64, bits=4))

QWEN3_4B = dict(QWEN3_0_6B, hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
                num_attention_heads=32, num_key_value_heads=8)

QWEN3_32B = dict(QWEN3_0_6B, hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
                 num_attention_heads=64, num_key_value_heads=8, tie_word_embeddings=False)


def tiny_config(**over) -> dict:
    """A small Qwen3-shaped config for fast CPU/GPU parity tests."""
    cfg = dict(QWEN3_0_6B, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
               num_attention_heads=4, num_key_value_heads=2, vocab_size=1024,
               bos_token_id=1, eos_token_id=[1000, 1001])
    cfg.update(over)
    return cfg


def _qlin_shapes(cfg):
    H, I = cfg["hidden_size"], cfg["intermediate_size"]
    D = cfg.get("head_dim") or H // cfg["num_attention_heads"]
    Hq, Hkv = cfg["num_attention_heads"], cfg.get("num_key_value_heads") or cfg["num_attention_heads"]
    return {L_Q: ("self_attn.q_proj", Hq * D, H), L_K: ("self_attn.k_proj", Hkv * D, H),
            L_V: ("self_attn.v_proj", Hkv * D, H), L_O: ("self_attn.o_proj", H, Hq * D),
            L_GATE: ("mlp.gate_proj", I, H), L_UP: ("mlp.up_proj", I, H), L_DOWN: ("mlp.down_proj", H, I)}


def iter_tensors(cfg: dict, seed: int, norm_mode: str = "ones"):
    """Yield (name, numpy array) for every tensor of the synthetic checkpoint.

    Quantized weights are uint32, scales/biases and norm weights are uint16
    holding bf16 bits.
    """
    H, V = cfg["hidden_size"], cfg["vocab_size"]
    D = cfg.get("head_dim") or H // cfg["num_attention_heads"]
    w, s, b = nm.quantized_weight(seed, TID_EMBED, V, H)
    yield "model.embed_tokens.weight", w
    yield "model.embed_tokens.scales", s
    yield "model.embed_tokens.biases", b
    shapes = _qlin_shapes(cfg)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        yield f"{p}.input_layernorm.weight", nm.norm_weight(seed, layer_tid(i, L_IN_NORM), H, norm_mode)
        yield f"{p}.post_attention_layernorm.weight", nm.norm_weight(seed, layer_tid(i, L_POST_NORM), H, norm_mode)
        yield f"{p}.self_attn.q_norm.weight", nm.norm_weight(seed, layer_tid(i, L_Q_NORM), D, norm_mode)
        yield f"{p}.self_attn.k_norm.weight", nm.norm_weight(seed, layer_tid(i, L_K_NORM), D, norm_mode)
        for kind, (nme, n, k) in shapes.items():
            w, s, b = nm.quantized_weight(seed, layer_tid(i, kind), n, k)
            yield f"{p}.{nme}.weight", w
            yield f"{p}.{nme}.scales", s
            yield f"{p}.{nme}.biases", b
    yield "model.norm.weight", nm.norm_weight(seed, TID_FINAL_NORM, H, norm_mode)
    if not cfg.get("tie_word_embeddings", False):
        w, s, b = nm.quantized_weight(seed, TID_LM_HEAD, V, H)
        yield "lm_head.weight", w
        yield "lm_head.scales", s
        yield "lm_head.biases", b


def build_tensors(cfg: dict, seed: int, norm_mode: str = "ones", fast: bool = False) -> dict:
    """All tensors of the synthetic checkpoint; fast=True generates the
    quantized weights with the multithreaded C restatement (oracle/synth_ref.c)."""
    if not fast:
        return dict(iter_tensors(cfg, seed, norm_mode))
    out = {}
    for name, arr in iter_tensors_fast(cfg, seed, norm_mode):
        out[name] = arr
    return out


def quantized_weight_c(seed: int, tensor_id: int, n: int, k: int, std: float = 0.02, threads: int = 0):
    """Same as numerics.quantized_weight, computed by oracle/synth_ref.c."""
    import ctypes
    from .qwen3_ref import _lib
    lib = _lib()
    fn = lib.synth_qweight
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_uint64, ctypes.c_float, ctypes.c_int]
    fn.restype = ctypes.c_int
    w = np.empty((n, k // 8), np.uint32)
    s = np.empty((n, k // 64), np.uint16)
    b = np.empty((n, k // 64), np.uint16)
    rc = fn(w.ctypes.data, s.ctypes.data, b.ctypes.data, n, k, 0, 0, k, nm.tensor_key(seed, tensor_id),
            float(nm.normal_scale(std)), threads)
    if rc != 0:
        raise RuntimeError("synth_qweight failed")
    return w, s, b


def iter_tensors_fast(cfg: dict, seed: int, norm_mode: str = "ones"):
    saved = nm.quantized_weight
    try:
        nm.quantized_weight = quantized_weight_c
        yield from iter_tensors(cfg, seed, norm_mode)
    finally:
        nm.quantized_weight = saved


_DT = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.int32): "I32",
       np.dtype(np.float32): "F32"}


def write_safetensors(path: str, tensors: dict) -> None:
    """Minimal safetensors writer (uint16 arrays are written with dtype BF16)."""
    header = {}
    off = 0
    order = sorted(tensors)
    for name in order:
        a = np.ascontiguousarray(tensors[name])
        header[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    header["__metadata__"] = {"format": "mlx"}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in order:
            f.write(np.ascontiguousarray(tensors[name]).tobytes())


def read_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    inv = {"U32": np.uint32, "BF16": np.uint16, "I32": np.int32, "F32": np.float32}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        out[name] = np.frombuffer(data[a:b], dtype=inv[meta["dtype"]]).reshape(meta["shape"]).copy()
    return out


def write_checkpoint(dirpath: str, cfg: dict, seed: int, norm_mode: str = "ones",
                     shards: int = 1, tensors: dict | None = None) -> None:
    """Write config.json + model[-0000i-of-0000n].safetensors in MLX layout."""
    os.makedirs(dirpath, exist_ok=True)
    if tensors is None:
        tensors = build_tensors(cfg, seed, norm_mode)
    names = sorted(tensors)
    per = (len(names) + shards - 1) // shards
    for i in range(shards):
        part = {n: tensors[n] for n in names[i * per:(i + 1) * per]}
        fn = "model.safetensors" if shards == 1 else f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(os.path.join(dirpath, fn), part)
    with open(os.path.join(dirpath, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
