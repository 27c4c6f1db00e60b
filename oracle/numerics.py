"""bf16 rounding, the seeded weight generator and the MLX affine 4-bit format.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

MLX quantized-linear storage, as the reference loads it
(``crates/base-mlx-core/src/model/qwen3.rs:18-42`` and ``kernels.rs:16-18``:
bits=4, group_size=64):

* ``weight``  uint32 [N, K/8]; element k of a row sits in word k//8 at bits
  ``4*(k%8)`` (least-significant nibble first);
* ``scales``  bf16   [N, K/64];
* ``biases``  bf16   [N, K/64];
* dequantised value ``w[n,k] = scales[n,k//64] * q[n,k] + biases[n,k//64]``.

The quantizer below is this project's own (per-group min/max, bias = group
minimum); only the storage format and the dequantisation formula have to
match MLX.  The CUDA initialiser (``init_random`` in the library) computes the
same values bit for bit: every step is a single IEEE fp32 operation with
round-to-nearest-even, or integer arithmetic.
"""
from __future__ import annotations

import math

import numpy as np

GROUP = 64
BITS = 4
MASK64 = (1 << 64) - 1

# ---------------------------------------------------------------- bf16 ---


def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even); result stays float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    r = ((u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, np.uint32(0x7FC00000), r)
    return r.view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    return (bf16_round(a).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


# ------------------------------------------------------- seeded RNG ------

_SM_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_SM_M1 = np.uint64(0xBF58476D1CE4E5B9)
_SM_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(x):
    """splitmix64 finaliser on uint64 arrays (wrapping arithmetic)."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = x + _SM_GAMMA
        z = (z ^ (z >> np.uint64(30))) * _SM_M1
        z = (z ^ (z >> np.uint64(27))) * _SM_M2
        return z ^ (z >> np.uint64(31))


def splitmix64_int(x: int) -> int:
    z = (x + 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def tensor_key(seed: int, tensor_id: int) -> int:
    """Per-tensor stream key: splitmix64(seed ^ splitmix64(tensor_id))."""
    return splitmix64_int((seed & MASK64) ^ splitmix64_int(tensor_id))


# std of the sum of four independent uniform integers on [0, 65535]
_IRWIN_STD = math.sqrt((2.0 ** 32 - 1.0) / 3.0)


def normal_scale(std: float) -> np.float32:
    """fp32 multiplier that turns the centred 4-uniform sum into ~N(0, std)."""
    return np.float32(std / _IRWIN_STD)


def normal_f32(key: int, start: int, count: int, std: float) -> np.ndarray:
    """Approximately normal fp32 values, element e = f(splitmix64(key + e)).

    The value is the Irwin-Hall sum of the four 16-bit fields of the hash,
    centred (an exact int32) and multiplied once by ``normal_scale(std)``.
    """
    idx = np.arange(start, start + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = splitmix64(np.uint64(key) + idx)
    s = ((h & np.uint64(0xFFFF)) + ((h >> np.uint64(16)) & np.uint64(0xFFFF))
         + ((h >> np.uint64(32)) & np.uint64(0xFFFF)) + (h >> np.uint64(48)))
    c = s.astype(np.int64) - 131070
    return c.astype(np.float32) * normal_scale(std)


def uniform01(seed: int, a: int, b: int) -> np.float32:
    """Counter-based uniform in [0,1): top 24 bits of splitmix64(seed ^ splitmix64(a*64+b))."""
    h = splitmix64_int((seed & MASK64) ^ splitmix64_int(a * 64 + b))
    return np.float32((h >> 40) * (1.0 / 16777216.0))


# ------------------------------------------------ affine 4-bit g64 ------


def quantize_groups(w: np.ndarray):
    """Quantize fp32 [N, K] to (q uint8 [N,K], scales bf16-bits [N,K/64], biases bf16-bits).

    scale = bf16((max-min)/15), bias = bf16(min),
    q = clamp(rint((w - bias) / scale), 0, 15), q = 0 where scale == 0.
    """
    n, k = w.shape
    assert k % GROUP == 0
    g = w.reshape(n, k // GROUP, GROUP).astype(np.float32)
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    scale = bf16_round((mx - mn) / np.float32(15.0))
    bias = bf16_round(mn)
    safe = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    q = np.rint((g - bias[..., None]) / safe[..., None])
    q = np.clip(q, 0, 15)
    q = np.where((scale == 0)[..., None], 0, q).astype(np.uint8)
    return q.reshape(n, k), f32_to_bf16_bits(scale), f32_to_bf16_bits(bias)


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """uint8 [N, K] (values 0..15) -> uint32 [N, K/8], element k at bits 4*(k%8)."""
    n, k = q.shape
    q = q.reshape(n, k // 8, 8).astype(np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def unpack_nibbles(w: np.ndarray) -> np.ndarray:
    """uint32 [N, K/8] -> uint8 [N, K]."""
    n, kw = w.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)
    q = (w[..., None].astype(np.uint32) >> shifts) & np.uint32(0xF)
    return q.reshape(n, kw * 8).astype(np.uint8)


def dequantize(w: np.ndarray, scales: np.ndarray, biases: np.ndarray) -> np.ndarray:
    """Exact fp32 dequantisation s*q + b (s*q is exact in fp32; one rounding for +b)."""
    q = unpack_nibbles(w).astype(np.float32)
    n, k = q.shape
    s = bf16_bits_to_f32(scales)
    b = bf16_bits_to_f32(biases)
    qg = q.reshape(n, k // GROUP, GROUP)
    return (qg * s[..., None] + b[..., None]).reshape(n, k).astype(np.float32)


def quantized_weight(seed: int, tensor_id: int, n: int, k: int, std: float = 0.02):
    """Generate the seeded N(0,std) fp32 matrix [n, k] and quantize it (MLX layout)."""
    key = tensor_key(seed, tensor_id)
    w = normal_f32(key, 0, n * k, std).reshape(n, k)
    q, s, b = quantize_groups(w)
    return pack_nibbles(q), s, b


def norm_weight(seed: int, tensor_id: int, n: int, mode: str) -> np.ndarray:
    """RMSNorm weight as bf16 bits: 1.0 ('ones') or bf16(1 + N(0,0.1)) ('random')."""
    if mode == "ones":
        return f32_to_bf16_bits(np.ones(n, np.float32))
    key = tensor_key(seed, tensor_id)
    v = np.float32(1.0) + normal_f32(key, 0, n, 0.1)
    return f32_to_bf16_bits(v)
