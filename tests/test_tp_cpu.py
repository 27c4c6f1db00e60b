"""Tensor-parallel host logic on CPU, two gloo ranks (no GPU, no NCCL):

* the NCCL unique-id exchange helper (qwen3_b200.tp_share_unique_id) hands
  rank 0's id to every rank;
* the collective plan of the tensor-parallel step, restated in numpy with the
  oracle's quantized linears: o_proj / down_proj split by input columns (K/tp,
  whole 64-groups per rank) with an fp32 sum all-reduce of the partials, and
  the vocab-parallel lm_head argmax as a max all-reduce of packed
  (orderable logit, ~index) keys -- the same key the CUDA epilogue builds
  (amax_key: ties go to the lowest index).  Both must equal the unsplit result.

The library's own sharded load and NCCL collectives run on two GPUs in
tests/test_gpu_tp.py.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import numerics as nm


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _amax_key(v: np.ndarray, idx: np.ndarray) -> np.ndarray:
    u = v.astype(np.float32).view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    u = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (u << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idx.astype(np.uint64))


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist
    import qwen3_b200 as q
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        # 1. unique-id exchange (rank 0's bytes everywhere)
        uid = q.tp_share_unique_id(rank, make_id=lambda: bytes(range(128)))
        res = {"uid_ok": uid == bytes(range(128))}

        # 2. column-split linear + sum all-reduce
        rng = np.random.default_rng(5)
        K, N, M = 512, 96, 3
        w, s, b = nm.quantized_weight(11, 3, N, K)
        x = nm.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
        full = x @ nm.dequantize(w, s, b).T
        kc = K // world
        w_r = w[:, rank * kc // 8:(rank + 1) * kc // 8]
        s_r = s[:, rank * kc // 64:(rank + 1) * kc // 64]
        b_r = b[:, rank * kc // 64:(rank + 1) * kc // 64]
        part = torch.from_numpy((x[:, rank * kc:(rank + 1) * kc] @ nm.dequantize(w_r, s_r, b_r).T).astype(np.float32))
        dist.all_reduce(part, op=dist.ReduceOp.SUM)
        res["colsplit_err"] = float(np.abs(part.numpy() - full).max() / np.abs(full).max())

        # 3. vocab-parallel argmax: max all-reduce of packed keys, lowest index on ties
        V = 64
        logits = nm.bf16_round(rng.standard_normal((M, V)).astype(np.float32))
        logits[1, 7] = logits[1, 40] = 9.0  # tie across the two shards -> index 7
        vl = V // world
        loc = logits[:, rank * vl:(rank + 1) * vl]
        li = np.argmax(loc, axis=1)  # first maximum within the shard
        keys = _amax_key(loc[np.arange(M), li], li + rank * vl)
        kt = torch.from_numpy(keys.view(np.int64).copy())
        # gloo has no unsigned 64-bit max (NCCL's ncclUint64 + ncclMax on the GPU
        # path): gather the keys and take the unsigned maximum
        gathered = [torch.zeros_like(kt) for _ in range(world)]
        dist.all_gather(gathered, kt)
        best = np.max(np.stack([g.numpy().view(np.uint64) for g in gathered]), axis=0)
        idx = (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)
        res["argmax"] = idx.tolist()
        res["argmax_ref"] = np.argmax(logits, axis=1).tolist()
        np.save(os.path.join(out_dir, f"r{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


def test_tp_host_logic_two_gloo_ranks(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(2):
        res = np.load(os.path.join(tmp_path, f"r{r}.npy"), allow_pickle=True).item()
        assert res["uid_ok"]
        assert res["colsplit_err"] < 1e-5, res["colsplit_err"]
        assert res["argmax"] == res["argmax_ref"]
        assert res["argmax"][1] == 7
