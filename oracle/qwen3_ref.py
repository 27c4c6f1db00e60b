"""Qwen3 forward over MLX 4-bit weights, restated on the CPU -- TEST INFRASTRUCTURE ONLY.

Follows ``crates/base-mlx-core/src/model/qwen3.rs:314-563`` op by op.  Every
MLX op output is rounded to bf16 (values are carried as float32 holding bf16
values); reductions run in fp32:

* embedding lookup + dequantize (``qwen3.rs:57-76``): bf16(s*q + b);
* ``qkv_block`` (``kernels.rs:28-46``): rms_norm -> q/k/v quantized_matmul;
* per-head q_norm / k_norm (``qwen3.rs:398-399``), then non-traditional RoPE
  at positions offset..offset+S (``qwen3.rs:401-413``) from a float64
  cos/sin table rounded to fp32;
* in-place KV write at [offset, offset+S) of a [kv_heads, max_pos, 128] cache
  (``qwen3.rs:415-489``);
* SDPA with native GQA, scale 1/sqrt(head_dim), causal mask for S>1 with the
  cached prefix fully visible (``qwen3.rs:491-518``, ``:629-653``);
* o_proj + residual, ``mlp_block`` (``kernels.rs:55-78``) with
  silu(g) = g * sigmoid(g) as two bf16 ops, then * up, down_proj + residual;
* final norm, last row (or every row for ``forward_multi``), lm_head on the
  tied embedding or the untied ``lm_head`` (``qwen3.rs:545-561``).

``quantized_matmul`` is y = bf16(x @ dequant(W)^T) with the exact fp32
dequantisation s*q + b and fp32 accumulation.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import numerics as nm

KV_PREALLOC = 4096  # qwen3.rs:125


def rope_tables(max_pos: int, dim: int, theta: float):
    """cos/sin [max_pos, dim/2] fp32: angle = pos * theta^(-2i/dim), computed in float64."""
    i = np.arange(dim // 2, dtype=np.float64)
    inv = np.power(np.float64(theta), -2.0 * i / dim)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """bf16(x * rsqrt(mean(x^2) + eps) * w); fp32 internally (qwen3.rs:44-55)."""
    x = x.astype(np.float32)
    ms = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    r = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    return nm.bf16_round((x * r) * w.astype(np.float32))


def rope(x: np.ndarray, positions: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Non-interleaved RoPE over the full head dim; x [S, heads, D] -> bf16."""
    half = x.shape[-1] // 2
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    x1 = x[..., :half].astype(np.float32)
    x2 = x[..., half:].astype(np.float32)
    o1 = x1 * c - x2 * s
    o2 = x2 * c + x1 * s
    return nm.bf16_round(np.concatenate([o1, o2], axis=-1))


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, offset: int, scale: float) -> np.ndarray:
    """q [S, Hq, D], k/v [Hkv, T, D] (T = offset + S) -> bf16 [S, Hq*D].

    Scores in fp32, -inf above the shifted diagonal (query i sees keys
    j <= offset + i), softmax in fp32, output rounded once to bf16.
    """
    S, Hq, D = q.shape
    Hkv, T, _ = k.shape
    rep = Hq // Hkv
    out = np.empty((S, Hq, D), np.float32)
    allowed = np.arange(T)[None, :] <= (offset + np.arange(S))[:, None]
    for h in range(Hq):
        g = h // rep
        s = (q[:, h, :].astype(np.float32) @ k[g].astype(np.float32).T) * np.float32(scale)
        s = np.where(allowed, s, np.float32(-np.inf))
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m).astype(np.float32)
        l = p.sum(axis=-1, keepdims=True, dtype=np.float32)
        out[:, h, :] = (p @ v[g].astype(np.float32)) / l
    return nm.bf16_round(out.reshape(S, Hq * D))


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """bf16(bf16(g * bf16(sigmoid(g))) * u) -- kernels.rs:73-74 as three bf16 ops."""
    g = g.astype(np.float32)
    sg = nm.bf16_round(np.float32(1.0) / (np.float32(1.0) + np.exp(-g)))
    a = nm.bf16_round(g * sg)
    return nm.bf16_round(a * u.astype(np.float32))


def argmax_first(logits: np.ndarray) -> np.ndarray:
    """Index of the maximum along the last axis, lowest index on ties."""
    return np.argmax(logits, axis=-1).astype(np.int64)


class QLinearRef:
    """One MLX quantized linear: uint32 weight [N,K/8], bf16 scales/biases [N,K/64]."""

    def __init__(self, w, s, b, backend="numpy"):
        self.w, self.s, self.b = w, s, b
        self.n = w.shape[0]
        self.k = w.shape[1] * 8
        self.backend = backend
        self._deq = None

    def dequant(self) -> np.ndarray:
        if self._deq is None:
            self._deq = nm.dequantize(self.w, self.s, self.b)
        return self._deq

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        if self.backend == "c":
            return nm.bf16_round(qmm_c(x, self.w, self.s, self.b))
        if self.backend == "torch":
            return nm.bf16_round(qmm_torch(x, self.w, self.s, self.b))
        return nm.bf16_round(x @ self.dequant().T)


class KvCacheRef:
    """Per-layer [kv_heads, max_pos, head_dim] bf16 caches + seq_len (qwen3.rs:116-162)."""

    def __init__(self, n_layers, kv_heads, head_dim, max_pos=KV_PREALLOC):
        self.k = [np.zeros((kv_heads, max_pos, head_dim), np.float32) for _ in range(n_layers)]
        self.v = [np.zeros((kv_heads, max_pos, head_dim), np.float32) for _ in range(n_layers)]
        self.seq_len = 0
        self.max_pos = max_pos

    def reset(self):
        self.seq_len = 0

    def truncate(self, target: int):
        """Roll back to the first ``target`` positions; no-op if already shorter."""
        if target < self.seq_len:
            self.seq_len = target


class Qwen3Ref:
    """CPU restatement of ``Qwen3`` (qwen3.rs:165-563)."""

    def __init__(self, cfg: dict, tensors: dict, backend: str = "numpy"):
        self.cfg = cfg
        H = cfg["hidden_size"]
        self.H = H
        self.Hq = cfg["num_attention_heads"]
        self.Hkv = cfg.get("num_key_value_heads") or self.Hq
        self.D = cfg.get("head_dim") or H // self.Hq
        self.L = cfg["num_hidden_layers"]
        self.V = cfg["vocab_size"]
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.theta = float(cfg.get("rope_theta", 10000.0))
        t = tensors
        f = nm.bf16_bits_to_f32

        def ql(p):
            return QLinearRef(t[p + ".weight"], t[p + ".scales"], t[p + ".biases"], backend)

        self.embed = ql("model.embed_tokens")
        self.layers = []
        for i in range(self.L):
            p = f"model.layers.{i}"
            self.layers.append(dict(
                in_norm=f(t[p + ".input_layernorm.weight"]),
                post_norm=f(t[p + ".post_attention_layernorm.weight"]),
                q_norm=f(t[p + ".self_attn.q_norm.weight"]),
                k_norm=f(t[p + ".self_attn.k_norm.weight"]),
                q=ql(p + ".self_attn.q_proj"), k=ql(p + ".self_attn.k_proj"),
                v=ql(p + ".self_attn.v_proj"), o=ql(p + ".self_attn.o_proj"),
                gate=ql(p + ".mlp.gate_proj"), up=ql(p + ".mlp.up_proj"),
                down=ql(p + ".mlp.down_proj")))
        self.norm = f(t["model.norm.weight"])
        self.lm_head = None if cfg.get("tie_word_embeddings", False) else ql("lm_head")
        self.cos, self.sin = rope_tables(KV_PREALLOC, self.D, self.theta)
        eos = cfg.get("eos_token_id")
        self.eos = [] if eos is None else ([eos] if isinstance(eos, int) else list(eos))

    def new_cache(self, max_pos=KV_PREALLOC) -> KvCacheRef:
        if max_pos > self.cos.shape[0]:
            self.cos, self.sin = rope_tables(max_pos, self.D, self.theta)
        return KvCacheRef(self.L, self.Hkv, self.D, max_pos)

    def is_eos(self, tok: int) -> bool:
        """engine.rs:266-272."""
        if self.eos:
            return tok in self.eos
        return tok in (151645, 151643)

    def embed_rows(self, tokens) -> np.ndarray:
        ids = np.asarray(tokens, dtype=np.int64)
        e = self.embed
        rows = nm.dequantize(e.w[ids], e.s[ids], e.b[ids])
        return nm.bf16_round(rows)

    def lm_head_fwd(self, x):
        head = self.lm_head if self.lm_head is not None else self.embed
        return head.forward(x)

    def forward(self, tokens, cache: KvCacheRef, return_all: bool = False, trace=None):
        """Logits (bf16 values as float32): [V] for the last row, or [S, V] if return_all."""
        S = len(tokens)
        off = cache.seq_len
        if off + S > cache.max_pos:
            raise RuntimeError(f"KV cache exhausted: requested {off + S} positions, max {cache.max_pos}")
        pos = np.arange(off, off + S)
        scale = np.float32(1.0) / np.sqrt(np.float32(self.D))
        x = self.embed_rows(tokens)
        if trace is not None:
            trace.append(x.copy())
        for li in range(self.L):
            x = self.layer(li, x, cache, off)
            if trace is not None:
                trace.append(x.copy())
        logits = self.head(x if return_all else x[S - 1:S])
        cache.seq_len += S
        return logits if return_all else logits[0]

    def layer(self, li: int, x: np.ndarray, cache: KvCacheRef, off: int) -> np.ndarray:
        """One decoder layer (qwen3.rs:381-541) on rows x [S, H] at positions
        off..off+S: writes this layer's K/V rows into the cache and returns the
        residual stream after the layer.  The cache's seq_len is not changed."""
        attn = self.attention(li, x, cache, off)
        return self.mlp(li, self.attn_residual(li, x, attn))

    def attention(self, li: int, x: np.ndarray, cache: KvCacheRef, off: int) -> np.ndarray:
        """qkv_block, q/k norm, RoPE, KV write and SDPA (qwen3.rs:381-518): the
        attention output [S, Hq*D] (bf16 values), the o_proj input."""
        ly = self.layers[li]
        S = x.shape[0]
        pos = np.arange(off, off + S)
        scale = np.float32(1.0) / np.sqrt(np.float32(self.D))
        h = rms_norm(x, ly["in_norm"], self.eps)
        q = ly["q"].forward(h).reshape(S, self.Hq, self.D)
        k = ly["k"].forward(h).reshape(S, self.Hkv, self.D)
        v = ly["v"].forward(h).reshape(S, self.Hkv, self.D)
        q = rms_norm(q, ly["q_norm"], self.eps)
        k = rms_norm(k, ly["k_norm"], self.eps)
        q = rope(q, pos, self.cos, self.sin)
        k = rope(k, pos, self.cos, self.sin)
        cache.k[li][:, off:off + S, :] = k.transpose(1, 0, 2)
        cache.v[li][:, off:off + S, :] = v.transpose(1, 0, 2)
        return sdpa(q, cache.k[li][:, :off + S], cache.v[li][:, :off + S], off, scale)

    def attn_residual(self, li: int, x: np.ndarray, attn: np.ndarray) -> np.ndarray:
        """o_proj + residual (qwen3.rs:519-520)."""
        return nm.bf16_round(x + self.layers[li]["o"].forward(attn))

    def mlp(self, li: int, x: np.ndarray) -> np.ndarray:
        """post-attention RMSNorm, mlp_block and residual (kernels.rs:55-78, qwen3.rs:521-541)."""
        ly = self.layers[li]
        h2 = rms_norm(x, ly["post_norm"], self.eps)
        g = ly["gate"].forward(h2)
        u = ly["up"].forward(h2)
        mlp = ly["down"].forward(silu_mul(g, u))
        return nm.bf16_round(x + mlp)

    def head(self, x: np.ndarray) -> np.ndarray:
        """Final RMSNorm and lm_head (qwen3.rs:545-561) of rows x [S, H] -> logits [S, V]."""
        return self.lm_head_fwd(rms_norm(x, self.norm, self.eps))


# ------------------------------------------------------------ C helper ---

_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        here = os.path.dirname(os.path.abspath(__file__))
        path = os.path.join(here, "_build", "libqmm_ref.so")
        if not os.path.exists(path):
            from . import build_oracle
            build_oracle.build()
        lib = ctypes.CDLL(path)
        lib.qmm_ref_f32.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4
        lib.qmm_ref_f32.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def qmm_torch(x, w, s, b) -> np.ndarray:
    """y[M,N] = x[M,K] . dequant(W)^T in fp32 with torch on the CPU: the weight
    is dequantised exactly (s*q + b, one rounding) one 4096-row block at a time
    and multiplied with torch's fp32 matmul (no cache of dequantised weights,
    so a 4B-parameter model fits in host memory).  For long teacher-forced
    sequences where the C loop would take minutes."""
    import torch
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32))
    N, KW = w.shape
    K = KW * 8
    y = torch.empty((xt.shape[0], N), dtype=torch.float32)
    shifts = torch.arange(0, 32, 4, dtype=torch.int64)
    for n0 in range(0, N, 4096):
        n1 = min(N, n0 + 4096)
        wb = torch.from_numpy(np.ascontiguousarray(w[n0:n1]).view(np.int32)).to(torch.int64) & 0xFFFFFFFF
        q = ((wb.unsqueeze(-1) >> shifts) & 0xF).to(torch.float32).reshape(n1 - n0, K // 64, 64)
        sc = torch.from_numpy(nm.bf16_bits_to_f32(s[n0:n1])).unsqueeze(-1)
        bi = torch.from_numpy(nm.bf16_bits_to_f32(b[n0:n1])).unsqueeze(-1)
        deq = (q * sc + bi).reshape(n1 - n0, K)
        y[:, n0:n1] = xt @ deq.T
    return y.numpy()


def qmm_c(x, w, s, b, threads: int = 0) -> np.ndarray:
    """y[M,N] = x[M,K] . dequant(W)^T in fp32 via oracle/qmm_ref.c (multithreaded)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint32)
    s = np.ascontiguousarray(s, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    rc = _lib().qmm_ref_f32(x.ctypes.data, w.ctypes.data, s.ctypes.data, b.ctypes.data,
                            y.ctypes.data, M, N, K, threads)
    if rc != 0:
        raise RuntimeError(f"qmm_ref_f32 failed rc={rc}")
    return y
