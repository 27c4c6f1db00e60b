"""Tensor parallelism on two GPUs, one process per GPU: the library's sharded
load (tp_rank / tp_size: q/k/v and gate/up rows, o_proj/down_proj columns,
untied lm_head vocabulary rows), the NCCL sum all-reduces after o_proj and
down_proj and the u64 max all-reduce of the vocab-parallel argmax keys,
against the single-GPU model of the same seed on the same inputs.

Tolerances: logits of every prefill row within 2e-2 max-abs (tiny models) /
0.1 (4-layer 0.6B shapes).  The split only changes the fp32 summation order of
o_proj and down_proj, but a partial sum that lands on the other side of a bf16
rounding boundary of the hidden state moves later logits by more than fp32
noise, so a row whose two best logits are closer than that can flip its
argmax.  Every pick (prefill argmax and each greedy token, the latter against
the single-GPU model run teacher-forced on the tensor-parallel tokens) must
therefore lie within 2 x tol of the single-GPU maximum of its row -- which is
exact equality wherever the top-2 gap exceeds 2 x tol -- and the two ranks
must agree bit for bit on argmaxes and tokens.  Skipped with fewer than two
GPUs.  The NCCL id travels over a gloo process group
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
        res = {"argmax": np.asarray(am).tolist(), "logits": np.asarray(lg).copy(), "tokens": list(gen.tokens)}
        m.close()
        dist.barrier()
        if rank == 0:
            m1 = q.Qwen3.init_random(cfg, 77, norm_mode="random", device=0)
            c1 = m1.new_cache(256)
            lg1, am1 = m1.forward_multi(prompt, c1)
            c1.close()
            g1 = m1.generate_greedy(prompt, 24)
            # the single-GPU model teacher-forced on the tensor-parallel tokens:
            # row plen-1+j scores the choice of token j
            c2 = m1.new_cache(256)
            lg2, _ = m1.forward_multi(prompt + list(gen.tokens[:-1]), c2)
            c2.close()
            res.update(ref_argmax=np.asarray(am1).tolist(), ref_logits=np.asarray(lg1).copy(),
                       ref_tokens=list(g1.tokens), ref_forced=np.asarray(lg2)[plen - 1:].copy())
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
    _tp2_case(case, tmp_path)


@pytest.mark.skipif(_ngpu() < 2, reason="needs two GPUs")
def test_tp2_peer_memory_reductions_match_single_gpu(tmp_path, monkeypatch):
    """The decode reductions over peer memory (QW_TP_PUSH=1: the GEMV pushes its
    partial rows to every rank, one kernel per rank sums them) instead of NCCL."""
    monkeypatch.setenv("QW_TP_PUSH", "1")
    _tp2_case("0.6b_4layers", tmp_path)


def _tp2_case(case, tmp_path):
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
    ref = r0["ref_logits"]
    V = cfg["vocab_size"]
    if cfg["tie_word_embeddings"]:
        # replicated lm_head: every rank holds the full rows
        shards = [(r0["logits"], 0), (r1["logits"], 0)]
    else:
        shards = [(r0["logits"], 0), (r1["logits"], V // 2)]
    diffs = [float(np.abs(lg - ref[:, off:off + lg.shape[1]]).max()) for lg, off in shards]
    am, toks = r0["argmax"], r0["tokens"]
    am_exact = sum(a == b for a, b in zip(am, r0["ref_argmax"]))
    tok_exact = sum(a == b for a, b in zip(toks, r0["ref_tokens"]))
    print(f"[tp {case}] logits max-abs diff per rank {diffs}; prefill argmax exact {am_exact}/{len(am)}; "
          f"greedy tokens equal to the single-GPU run {tok_exact}/{len(toks)}")
    assert max(diffs) <= tol, (case, diffs)
    # both ranks hold the same all-reduced state: identical picks
    assert r1["argmax"] == am and r1["tokens"] == toks, case

    def within(rows, picks):
        rows = np.asarray(rows, np.float64)
        got = rows[np.arange(len(picks)), np.asarray(picks)]
        return got >= rows.max(axis=1) - 2 * tol

    assert len(am) == len(ref) and within(ref, am).all(), case
    forced = r0["ref_forced"]
    assert len(toks) == 24 and len(forced) == len(toks) and within(forced, toks).all(), case


def _spec_worker(rank, world, port, out_dir):
    """Speculative decode with a tensor-parallel target and a replicated draft
    (the config-5 spec variant's shape at tiny size): every rank runs the same
    spec loop, the target's verify rows go through the sharded forward and its
    all-reduced argmax, the draft runs whole on each rank."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    import torch
    import torch.distributed as dist
    import qwen3_b200 as q
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        cfg = synth.tiny_config(tie_word_embeddings=False)
        t = q.Qwen3.init_random(cfg, 77, norm_mode="random", device=rank, tp_rank=rank, tp_size=world)
        q.tp_init(t, rank, world)
        d = q.Qwen3.init_random(synth.tiny_config(num_hidden_layers=1), 78, norm_mode="random", device=rank)
        print(f"[tp spec rank {rank}] models up", flush=True)
        prompt = np.random.default_rng(4).integers(0, cfg["vocab_size"], 24).tolist()
        plain = t.generate_greedy(prompt, 32)
        res = {"plain": list(plain.tokens)}
        for k, p in ((4, 0.8), (3, 0.0)):
            r, st = q.speculative_generate(t, d, prompt, 32, k=k, force_p=p, seed=3, forced=plain.tokens)
            res[f"k{k}"] = (list(r.tokens), (st.iters, st.proposed, st.accepted))
        print(f"[tp spec rank {rank}] spec done", flush=True)
        d.close()
        t.close()
        np.save(os.path.join(out_dir, f"s{rank}.npy"), res, allow_pickle=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs two GPUs")
def test_tp2_speculative_matches_tp2_greedy(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_spec_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    s0 = np.load(os.path.join(tmp_path, "s0.npy"), allow_pickle=True).item()
    s1 = np.load(os.path.join(tmp_path, "s1.npy"), allow_pickle=True).item()
    assert s0 == s1  # same tokens and accept counts on both ranks
    for key in ("k4", "k3"):
        toks, (iters, proposed, accepted) = s0[key]
        assert toks == s0["plain"], key  # greedy spec output == plain greedy of the same split target
        assert proposed >= accepted and iters > 0, key
