"""Python mirror of base-mlx-core's Qwen3 decode API over libqwen3_b200.so (ctypes).

Names and semantics follow the Rust crate (paths relative to the
flakerimi/base-mlx project root):

* ``Qwen3.load`` / ``Qwen3.new_cache`` / ``Qwen3.forward`` / ``Qwen3.forward_multi``
  -- ``Architecture`` in ``crates/base-mlx-core/src/model.rs:21-108``;
* ``KvCache.reset`` / ``KvCache.truncate`` / ``KvCache.seq_len``
  -- ``crates/base-mlx-core/src/model/qwen3.rs:116-162``;
* ``KvCache.slice_update`` -- ``mlx_ext::slice_update`` (``mlx_ext.rs:36-64``) on a cache tensor;
* ``Qwen3.generate_greedy`` -- ``LoadedModel::generate_text`` with temperature 0 (``engine.rs:149-201``);
* ``speculative_generate`` / ``check_compatible`` -- ``speculative.rs:40-286``;
* ``quantized_matmul`` -- ``mlx_rs::ops::quantized_matmul(transpose=true, 64, 4)``.

Errors map onto the crate's ``Error`` enum (``error.rs:6-32``).  There is no
CPU fallback: every compute call goes to the CUDA library and raises when no
usable GPU is present.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwen3_b200.so")

QW_OK = 0
QW_ERR_INVALID_ARG = -1
QW_ERR_INVALID_CONFIG = -2
QW_ERR_MODEL_LOAD = -3
QW_ERR_INFERENCE = -4
QW_ERR_KV_EXHAUSTED = -5
QW_ERR_CUDA = -6
QW_ERR_UNSUPPORTED = -7
QW_ERR_DEVICE_FLAG = -8


class Error(Exception):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class InvalidConfig(Error):
    """Error::InvalidConfig"""


class ModelLoad(Error):
    """Error::ModelLoad"""


class Inference(Error):
    """Error::Inference"""


class KvExhausted(Inference):
    """Error::Inference("KV cache exhausted ...") (qwen3.rs:423-428)"""


class CudaError(Inference):
    """CUDA failure or no usable sm_100 GPU."""


class Unsupported(Error):
    """Shape / format outside what the library supports."""


_ERR = {QW_ERR_INVALID_CONFIG: InvalidConfig, QW_ERR_MODEL_LOAD: ModelLoad, QW_ERR_INFERENCE: Inference,
        QW_ERR_KV_EXHAUSTED: KvExhausted, QW_ERR_CUDA: CudaError, QW_ERR_UNSUPPORTED: Unsupported,
        QW_ERR_DEVICE_FLAG: Inference, QW_ERR_INVALID_ARG: Error}


class ModelInfo(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("tied_embeddings", ctypes.c_int32), ("tp_rank", ctypes.c_int32),
                ("tp_size", ctypes.c_int32), ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("weight_bytes", ctypes.c_uint64)]


class GenStats(ctypes.Structure):
    _fields_ = [("prompt_tokens", ctypes.c_int32), ("completion_tokens", ctypes.c_int32),
                ("finish_reason", ctypes.c_int32), ("pad", ctypes.c_int32),
                ("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double)]


class SpecStats(ctypes.Structure):
    _fields_ = [("iters", ctypes.c_int32), ("proposed", ctypes.c_int32), ("accepted", ctypes.c_int32),
                ("completion_tokens", ctypes.c_int32), ("finish_reason", ctypes.c_int32), ("pad", ctypes.c_int32),
                ("prefill_ms", ctypes.c_double), ("total_ms", ctypes.c_double),
                ("draft_ms_mean", ctypes.c_double), ("verify_ms_mean", ctypes.c_double),
                ("accept_ms_mean", ctypes.c_double)]


_lib = None
P = ctypes.c_void_p
I = ctypes.c_int
U32P = ctypes.POINTER(ctypes.c_uint32)
U16P = ctypes.POINTER(ctypes.c_uint16)

# name -> argtypes; every function returns int
SIGNATURES = {
    "qw_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "qw_version": [ctypes.c_char_p, ctypes.c_size_t],
    "qw_model_load": [ctypes.c_char_p, I, I, I, ctypes.POINTER(P)],
    "qw_model_init_random": [ctypes.c_char_p, ctypes.c_uint64, I, I, I, I, ctypes.POINTER(P)],
    "qw_model_free": [P],
    "qw_model_info_get": [P, ctypes.POINTER(ModelInfo)],
    "qw_model_export_tensor": [P, ctypes.c_char_p, P, ctypes.c_size_t],
    "qw_model_stream": [P, ctypes.POINTER(P)],
    "qw_model_tp_attach": [P, P, I, I],
    "qw_tp_exchange_handle": [P, P, ctypes.c_size_t],
    "qw_tp_exchange_open": [P, P, ctypes.c_size_t],
    "qw_tp_unique_id": [P, ctypes.c_size_t],
    "qw_check_compatible": [P, P],
    "qw_cache_new": [P, I, ctypes.POINTER(P)],
    "qw_cache_free": [P],
    "qw_cache_reset": [P],
    "qw_cache_truncate": [P, I],
    "qw_cache_len": [P, ctypes.POINTER(I)],
    "qw_kv_slice_update": [P, I, I, U16P, I, I],
    "qw_kv_read": [P, I, I, U16P, I, I],
    "qw_forward": [P, P, U32P, I, I, U16P, U32P],
    "qw_forward_trace": [P, P, U32P, I, U16P, U16P, U16P, U16P, U32P],
    "qw_debug_decode_stamps": [P, P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)],
    "qw_generate_greedy": [P, U32P, I, I, U32P, I, U32P, ctypes.POINTER(I), ctypes.POINTER(GenStats)],
    "qw_generate_greedy_batch": [P, ctypes.POINTER(P), I, U32P, ctypes.POINTER(I), I, U32P, I, U32P,
                                 ctypes.POINTER(I), ctypes.POINTER(GenStats)],
    "qw_forward_batch": [P, ctypes.POINTER(P), I, U32P, U16P, U32P],
    "qw_generate_sampled": [P, U32P, I, I, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, I, U32P, I, U32P,
                            ctypes.POINTER(I), ctypes.POINTER(GenStats)],
    "qw_sample_topp": [P, I, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64, P, P, P],
    "qw_spec_generate": [P, P, U32P, I, I, I, ctypes.c_float, ctypes.c_uint64, U32P, I, U32P, I, U32P,
                         ctypes.POINTER(I), ctypes.POINTER(SpecStats)],
    "qw_spec_generate_sampled": [P, P, U32P, I, I, I, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, U32P, I,
                                 U32P, ctypes.POINTER(I), ctypes.POINTER(SpecStats)],
    "qw_quantized_matmul": [P, P, P, P, P, I, I, I, I, I, P],
    "qw_quantized_matmul_argmax_static": [P, P, P, P, P, P, I, I, I, I, I, P],
}


def lib() -> ctypes.CDLL:
    """Load the CUDA library (built in-tree by build.py); raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} not built (run base-mlx_b200/build.py)")
        l = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = l
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(4096)
    lib().qw_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != QW_OK:
        raise _ERR.get(rc, Error)(rc, last_error())


def version() -> str:
    buf = ctypes.create_string_buffer(256)
    check(lib().qw_version(buf, len(buf)))
    return buf.value.decode()


def _u32(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data_as(U32P)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class GenerationResult:
    """crates/base-mlx-core/src/engine.rs:90-101 (token ids instead of text)."""
    tokens: list
    prompt_tokens: int
    completion_tokens: int
    finish_reason: str
    prefill_ms: float = 0.0
    decode_ms: float = 0.0


class KvCache:
    """Device KV cache of one model (qwen3.rs:116-162)."""

    def __init__(self, model: "Qwen3", handle):
        self.model = model
        self.h = handle

    @property
    def seq_len(self) -> int:
        v = ctypes.c_int()
        check(lib().qw_cache_len(self.h, ctypes.byref(v)))
        return v.value

    def reset(self):
        check(lib().qw_cache_reset(self.h))

    def truncate(self, target_seq_len: int):
        check(lib().qw_cache_truncate(self.h, int(target_seq_len)))

    def slice_update(self, layer: int, which: str, update: np.ndarray, start: int, stop: int):
        """cache[layer].{k|v}[:, start:stop, :] = update (bf16 bits [kv_heads, stop-start, head_dim])."""
        u = np.ascontiguousarray(update, dtype=np.uint16)
        check(lib().qw_kv_slice_update(self.h, layer, 1 if which == "v" else 0, u.ctypes.data_as(U16P), start, stop))

    def read(self, layer: int, which: str, start: int, stop: int) -> np.ndarray:
        info = self.model.info
        out = np.empty((info.num_kv_heads // info.tp_size, stop - start, info.head_dim), np.uint16)
        check(lib().qw_kv_read(self.h, layer, 1 if which == "v" else 0, out.ctypes.data_as(U16P), start, stop))
        return out

    def close(self):
        if self.h and self.model.h:
            check(lib().qw_cache_free(self.h))
        self.h = None


class Qwen3:
    """One loaded Qwen3 model on one GPU (one tensor-parallel rank)."""

    def __init__(self, handle):
        self.h = handle
        inf = ModelInfo()
        check(lib().qw_model_info_get(self.h, ctypes.byref(inf)))
        self.info = inf

    @classmethod
    def load(cls, path: str, device: int = 0, tp_rank: int = 0, tp_size: int = 1) -> "Qwen3":
        h = P()
        check(lib().qw_model_load(path.encode(), device, tp_rank, tp_size, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def init_random(cls, cfg: dict, seed: int, norm_mode: str = "ones", device: int = 0, tp_rank: int = 0,
                    tp_size: int = 1) -> "Qwen3":
        h = P()
        check(lib().qw_model_init_random(json.dumps(cfg).encode(), seed & ((1 << 64) - 1),
                                         0 if norm_mode == "ones" else 1, device, tp_rank, tp_size, ctypes.byref(h)))
        return cls(h)

    def close(self):
        if self.h:
            check(lib().qw_model_free(self.h))
            self.h = None

    @property
    def vocab_local(self) -> int:
        inf = self.info
        return inf.vocab if (inf.tied_embeddings or inf.tp_size == 1) else inf.vocab // inf.tp_size

    def stream(self) -> int:
        s = P()
        check(lib().qw_model_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def tp_attach(self, unique_id: bytes, rank: int, size: int):
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        check(lib().qw_model_tp_attach(self.h, ctypes.cast(buf, P), rank, size))

    def export_tensor(self, name: str, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype)
        check(lib().qw_model_export_tensor(self.h, name.encode(), out.ctypes.data, out.nbytes))
        return out

    def new_cache(self, max_pos: int = 4096) -> KvCache:
        h = P()
        check(lib().qw_cache_new(self.h, max_pos, ctypes.byref(h)))
        return KvCache(self, h)

    def _forward(self, tokens, cache: KvCache, all_rows: bool, want_logits: bool):
        ids, ids_p = _u32(tokens)
        rows = len(ids) if all_rows else 1
        logits = np.empty((rows, self.vocab_local), np.uint16) if want_logits else None
        am = np.empty(rows, np.uint32)
        check(lib().qw_forward(self.h, cache.h, ids_p, len(ids), 1 if all_rows else 0,
                               logits.ctypes.data_as(U16P) if want_logits else None, am.ctypes.data_as(U32P)))
        return (bf16_to_f32(logits) if want_logits else None), am

    def forward(self, tokens, cache: KvCache, want_logits: bool = True):
        """Architecture::forward: logits of the last row [vocab] (bf16 values as float32), argmax."""
        lg, am = self._forward(tokens, cache, False, want_logits)
        return (lg[0] if lg is not None else None), int(am[0])

    def forward_multi(self, tokens, cache: KvCache, want_logits: bool = True):
        """Architecture::forward_multi: logits of every row [S, vocab], argmax per row."""
        return self._forward(tokens, cache, True, want_logits)

    def forward_trace(self, tokens, cache: KvCache):
        """forward() that also returns intermediate values as float32: the residual
        stream after the embedding and after every layer [layers + 1, n, hidden],
        the residual after each attention block [layers, n, hidden], each layer's
        attention output [layers, n, heads * head_dim]; then logits [vocab], argmax."""
        ids, ids_p = _u32(tokens)
        inf = self.info
        n = len(ids)
        qd = inf.num_heads // inf.tp_size * inf.head_dim
        res = np.empty((inf.num_layers + 1, n, inf.hidden), np.uint16)
        mid = np.empty((inf.num_layers, n, inf.hidden), np.uint16)
        att = np.empty((inf.num_layers, n, qd), np.uint16)
        logits = np.empty(self.vocab_local, np.uint16)
        am = np.empty(1, np.uint32)
        check(lib().qw_forward_trace(self.h, cache.h, ids_p, n, res.ctypes.data_as(U16P), mid.ctypes.data_as(U16P),
                                     att.ctypes.data_as(U16P), logits.ctypes.data_as(U16P), am.ctypes.data_as(U32P)))
        return bf16_to_f32(res), bf16_to_f32(mid), bf16_to_f32(att), bf16_to_f32(logits), int(am[0])

    def forward_batch(self, tokens, caches, want_logits: bool = True):
        """One batched decode step: tokens[b] at caches[b]'s next position.
        Returns (logits [nseq, vocab] float32 or None, argmax [nseq])."""
        ids, ids_p = _u32(tokens)
        n = len(ids)
        hs = (P * n)(*[c.h for c in caches])
        logits = np.empty((n, self.vocab_local), np.uint16) if want_logits else None
        am = np.empty(n, np.uint32)
        check(lib().qw_forward_batch(self.h, hs, n, ids_p, logits.ctypes.data_as(U16P) if want_logits else None,
                                     am.ctypes.data_as(U32P)))
        return (bf16_to_f32(logits) if want_logits else None), am

    def generate_greedy_batch(self, prompts, max_new: int, caches=None, eos=None):
        """Greedy decode of several prompts at once (one cache each; created
        with room for prompt + max_new when not given).  Returns (list of
        token lists, GenStats)."""
        n = len(prompts)
        own = caches is None
        if own:
            caches = [self.new_cache(len(p) + max(max_new, 1) + 1) for p in prompts]
        flat = np.concatenate([np.asarray(p, np.uint32) for p in prompts])
        fp = flat.ctypes.data_as(U32P)
        lens = (I * n)(*[len(p) for p in prompts])
        mn = max(max_new, 1)
        out = np.empty((n, mn), np.uint32)
        n_out = (I * n)()
        st = GenStats()
        if eos is not None:
            e, ep = _u32(eos)
            ne = len(e)
        else:
            ep, ne = None, 0
        hs = (P * n)(*[c.h for c in caches])
        try:
            check(lib().qw_generate_greedy_batch(self.h, hs, n, fp, lens, max_new, ep, ne, out.ctypes.data_as(U32P),
                                                 n_out, ctypes.byref(st)))
        finally:
            if own:
                for c in caches:
                    c.close()
        return [[int(t) for t in out[b, :n_out[b]]] for b in range(n)], st

    def generate_greedy(self, prompt, max_new: int, eos=None) -> GenerationResult:
        p, pp = _u32(prompt)
        out = np.empty(max(max_new, 1), np.uint32)
        n = ctypes.c_int()
        st = GenStats()
        if eos is not None:
            e, ep = _u32(eos)
            ne = len(e)
        else:
            ep, ne = None, 0
        check(lib().qw_generate_greedy(self.h, pp, len(p), max_new, ep, ne, out.ctypes.data_as(U32P), ctypes.byref(n),
                                       ctypes.byref(st)))
        return GenerationResult([int(t) for t in out[:n.value]], st.prompt_tokens, st.completion_tokens,
                                "stop" if st.finish_reason == 1 else "length", st.prefill_ms, st.decode_ms)

    def generate_sampled(self, prompt, max_new: int, temperature: float = 0.7, top_p: float = 0.95, seed: int = 0,
                         same_draw_each_token: bool = False, eos=None) -> GenerationResult:
        """LoadedModel::generate_text with SamplingParams {temperature, top_p, seed}
        (engine.rs:149-263); temperature <= 0 is greedy."""
        p, pp = _u32(prompt)
        out = np.empty(max(max_new, 1), np.uint32)
        n = ctypes.c_int()
        st = GenStats()
        if eos is not None:
            e, ep = _u32(eos)
            ne = len(e)
        else:
            ep, ne = None, 0
        check(lib().qw_generate_sampled(self.h, pp, len(p), max_new, temperature, top_p, seed & ((1 << 64) - 1),
                                        1 if same_draw_each_token else 0, ep, ne, out.ctypes.data_as(U32P),
                                        ctypes.byref(n), ctypes.byref(st)))
        return GenerationResult([int(t) for t in out[:n.value]], st.prompt_tokens, st.completion_tokens,
                                "stop" if st.finish_reason == 1 else "length", st.prefill_ms, st.decode_ms)


def sample_scratch_bytes(vocab: int) -> int:
    """Size of the device scratch qw_sample_topp needs (zero it before first use)."""
    return 16384 + 4 * vocab


def sample_topp(logits_ptr: int, vocab: int, temperature: float, top_p: float, seed: int, counter: int,
                scratch_ptr: int, token_ptr: int, stream: int = 0) -> None:
    """LoadedModel::pick_next on one device bf16 logits row (engine.rs:195-263);
    writes the picked id to the device int32 at token_ptr."""
    check(lib().qw_sample_topp(logits_ptr, vocab, temperature, top_p, seed & ((1 << 64) - 1),
                               counter & ((1 << 64) - 1), scratch_ptr, token_ptr, stream or None))


def tp_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for a tensor-parallel group."""
    buf = ctypes.create_string_buffer(128)
    check(lib().qw_tp_unique_id(ctypes.cast(buf, P), 128))
    return buf.raw


def tp_share_unique_id(rank: int, group=None, make_id=None) -> bytes:
    """Rank 0 creates the group's NCCL id, every rank returns it: the host-side
    exchange through an initialised torch.distributed process group (any
    backend; gloo suffices, the tensor traffic itself goes through NCCL inside
    the library).  `make_id` replaces tp_unique_id (tests without NCCL)."""
    import torch.distributed as dist
    obj = [(make_id or tp_unique_id)() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise Inference(-1, "tensor-parallel unique id exchange returned a malformed id")
    return bytes(uid)


def tp_init(model: "Qwen3", rank: int, size: int, group=None, peer_reduce: bool = True) -> None:
    """Attach the NCCL communicator of a tensor-parallel group of `size` ranks
    (one process per GPU, model loaded with tp_rank=rank, tp_size=size); with
    peer_reduce, also map every rank's exchange block (CUDA IPC handles shared
    over the host group) so that decode-step reductions run over peer memory."""
    import torch.distributed as dist
    model.tp_attach(tp_share_unique_id(rank, group), rank, size)
    if not peer_reduce:
        return
    buf = ctypes.create_string_buffer(64)
    check(lib().qw_tp_exchange_handle(model.h, buf, 64))
    handles = [None] * size
    dist.all_gather_object(handles, bytes(buf.raw), group=group)
    joined = b"".join(handles)
    if len(joined) != 64 * size:
        raise Inference(-1, "tensor-parallel exchange handles are malformed")
    jb = ctypes.create_string_buffer(joined, len(joined))
    check(lib().qw_tp_exchange_open(model.h, jb, len(joined)))


def check_compatible(target: Qwen3, draft: Qwen3) -> None:
    check(lib().qw_check_compatible(target.h, draft.h))


def speculative_generate(target: Qwen3, draft: Qwen3, prompt, max_new: int, k: int = 3, force_p: float = 0.0,
                         seed: int = 0, forced=None, eos=None):
    """speculative::generate (greedy).  Returns (GenerationResult, SpecStats)."""
    p, pp = _u32(prompt)
    out = np.empty(max(max_new, 1) + 1, np.uint32)
    n = ctypes.c_int()
    st = SpecStats()
    if forced is not None:
        f, fp = _u32(forced)
        nf = len(f)
    else:
        fp, nf = None, 0
    if eos is not None:
        e, ep = _u32(eos)
        ne = len(e)
    else:
        ep, ne = None, 0
    check(lib().qw_spec_generate(target.h, draft.h, pp, len(p), max_new, k, float(force_p), seed & ((1 << 64) - 1),
                                 fp, nf, ep, ne, out.ctypes.data_as(U32P), ctypes.byref(n), ctypes.byref(st)))
    res = GenerationResult([int(t) for t in out[:n.value]], len(p), st.completion_tokens,
                           "stop" if st.finish_reason == 1 else "length", st.prefill_ms, st.total_ms)
    return res, st


def speculative_generate_sampled(target: Qwen3, draft: Qwen3, prompt, max_new: int, k: int = 3,
                                 temperature: float = 0.7, top_p: float = 0.95, seed: int = 0, eos=None):
    """Speculative sampling (rejection rule over the sampled pick's distributions;
    the reference falls back to plain sampling here, speculative.rs:65-69).
    Returns (GenerationResult, SpecStats)."""
    p, pp = _u32(prompt)
    out = np.empty(max(max_new, 1) + 1, np.uint32)
    n = ctypes.c_int()
    st = SpecStats()
    if eos is not None:
        e, ep = _u32(eos)
        ne = len(e)
    else:
        ep, ne = None, 0
    check(lib().qw_spec_generate_sampled(target.h, draft.h, pp, len(p), max_new, k, float(temperature), float(top_p),
                                         seed & ((1 << 64) - 1), ep, ne, out.ctypes.data_as(U32P), ctypes.byref(n),
                                         ctypes.byref(st)))
    res = GenerationResult([int(t) for t in out[:n.value]], len(p), st.completion_tokens,
                           "stop" if st.finish_reason == 1 else "length", st.prefill_ms, st.total_ms)
    return res, st


def quantized_matmul(x_ptr: int, w_ptr: int, s_ptr: int, b_ptr: int, y_ptr: int, M: int, N: int, K: int,
                     group_size: int = 64, bits: int = 4, stream: int = 0) -> None:
    """y[M,N] = x[M,K] . dequant(W)^T on device pointers (MLX layout, bf16 x/y)."""
    check(lib().qw_quantized_matmul(x_ptr, w_ptr, s_ptr, b_ptr, y_ptr, M, N, K, group_size, bits, stream or None))


STATIC_AMAX_SLOTS = 131072  # QW_STATIC_AMAX_SLOTS


def quantized_matmul_argmax_static(x_ptr: int, w_ptr: int, s_ptr: int, b_ptr: int, y_ptr: int, argmax_ptr: int,
                                   M: int, N: int, K: int, group_size: int = 64, bits: int = 4,
                                   stream: int = 0) -> None:
    """Logits head that allocates nothing: y[M,N] (bf16, skipped when y_ptr is 0)
    = x . dequant(W)^T and argmax[m] (int32) on device pointers.  Its scratch
    is a static device array of STATIC_AMAX_SLOTS slots (M * ceil(N/16) must
    fit); concurrent calls on one device race on it.  The first call on a
    device should come before any stream capture."""
    check(lib().qw_quantized_matmul_argmax_static(x_ptr, w_ptr, s_ptr, b_ptr, y_ptr or None, argmax_ptr, M, N, K,
                                                  group_size, bits, stream or None))
