"""Tensor parallelism on two GPUs, one process per GPU: the library's sharded
load (tp_rank / tp_size: q/k/v and gate/up rows, o_proj/down_proj columns,
untied lm_head vocabulary rows), the NCCL sum all-reduces after o_proj and
down_proj and the u64 max all-reduce of the vocab-parallel argmax keys,
against the single-GPU model of the same seed on the same inputs.

Tolerances: logits within 2e-2 max-abs (tiny models) / 0.1 (4-layer 0.6B
shapes) -- the split only changes the fp32 summation order of o_proj and
down_proj -- and identical prefill argmaxes and greedy tokens.  Skipped with
fewer than two GPUs.  The NCCL id travels over a gloo process group
(qwen3_b200.tp_init); ranks rendezvous on 127.0.0.1.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import synth

pytestmark = pytest.mark.gpu


def _ngpu() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg, plen, out_dir):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    # single-node boxes without a routable network: NCCL's own bootstrap on loopback
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    import torch
    import torch.distributed as dist
    import qwen3_b200 as q
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    def step(what):  # progress on stdout (pytest -s): shows where a stalled rank stopped
        print(f"[tp rank {rank}] {what}", flush=True)

    try:
        step("process group up")
        m = q.Qwen3.init_random(cfg, 77, norm_mode="random", device=rank, tp_rank=rank, tp_size=world)
        step("shard loaded")
        q.tp_init(m, rank, world)
        step("communicator attached")
        prompt = np.random.default_rng(3).integers(0, cfg["vocab_size"], plen).tolist()
        c = m.new_cache(256)
        lg, am = m.forward_multi(prompt, c)
        c.close()
        step("prefill done")
        gen = m.generate_greedy(prompt, 24)
        step("generation done")
        res = {"argmax": np.asarray(am).tolist(), "last_logits": lg[-1].copy(), "tokens": list(gen.tokens)}
        m.close()
        dist.barrier()
        if rank == 0:
            m1 = q.Qwen3.init_random(cfg, 77, norm_mode="random", device=0)
            c1 = m1.new_cache(256)
            lg1, am1 = m1.forward_multi(prompt, c1)
            c1.close()
            g1 = m1.generate_greedy(prompt, 24)
            res.update(ref_argmax=np.asarray(am1).tolist(), ref_last_logits=lg1[-1].copy(), ref_tokens=list(g1.tokens))
            m1.close()
        np.save(os.path.join(out_dir, f"r{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


CASES = {
    "tiny_tied": (synth.tiny_config(), 40, 2e-2),
    "tiny_untied": (synth.tiny_config(tie_word_embeddings=False), 40, 2e-2),
    "0.6b_4layers": (dict(synth.QWEN3_0_6B, num_hidden_layers=4), 48, 0.1),
}


@pytest.mark.skipif(_ngpu() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("case", sorted(CASES))
def test_tp2_matches_single_gpu(case, tmp_path):
    cfg, plen, tol = CASES[case]
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, cfg, plen, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    r0 = np.load(os.path.join(tmp_path, "r0.npy"), allow_pickle=True).item()
    r1 = np.load(os.path.join(tmp_path, "r1.npy"), allow_pickle=True).item()
    ref = r0["ref_last_logits"]
    V = cfg["vocab_size"]
    if cfg["tie_word_embeddings"]:
        # replicated lm_head: every rank holds the full row
        shards = [(r0["last_logits"], 0), (r1["last_logits"], 0)]
    else:
        shards = [(r0["last_logits"], 0), (r1["last_logits"], V // 2)]
    for lg, off in shards:
        d = np.abs(lg - ref[off:off + len(lg)])
        assert d.max() <= tol, (case, float(d.max()))
    for r in (r0, r1):
        assert r["argmax"] == r0["ref_argmax"], case
        assert r["tokens"] == r0["ref_tokens"], case
