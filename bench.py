"""Benchmark: Qwen3-4B 4-bit batch-1 greedy decode on B200 (benchmark config 3).

One step = one request of the reference's benchmark shape: a 512-token
seeded-random prompt, prefill, then greedy decode of 300 tokens over a KV
cache pre-allocated to 4096 positions, through qw_generate_greedy (the
LoadedModel::generate_text equivalent).  Weights are random-init (seeded
N(0,0.02) quantized to MLX affine 4-bit g64) generated on the device.

* value  -- decode tok/s as the reference CLI bench defines it
            (crates/base-mlx-cli/src/main.rs:96-179: (n-1) / (total - ttft)),
            taken from CUDA events inside the library (inputs already on the
            device; prefill excluded), summed over the K timed steps and all ranks.
* e2e    -- the same metric through the C ABI with host buffers, timed on the
            host exactly like main.rs: wall(generate 300) - wall(generate 1).
* roofline -- the dominant kernel, decode_step_kernel (the persistent decode
            step: every layer + lm_head in one launch, one launch per token):
            algorithmic bytes per launch (quantized weights + K/V at the mean
            KV length) over its mean duration from the library's CUDA events,
            against the measured HBM copy bandwidth.
* cpu_baseline -- the oracle's CPU restatement of the same path (C qmatmul +
            numpy), rank 0 at N=1 only, on a bounded sample of the workload:
            greedy decode steps at the start and at the end of the 512..811
            KV range (caches pre-filled with seeded K/V; see `sample`).
* extras  -- config2_qmatmul (the standalone quantized matmul at M = 1, 5,
            128, 2048), spec (config 4 at forced acceptance p = 0, 0.5, 0.8,
            1), config1 (Qwen3-0.6B 128 + 128), sampled_decode; at N > 1
            tp_decode (config 5: Qwen3-32B split over all N ranks).

--impl reference times that CPU restatement alone on the same configuration
(the reference itself is Rust over MLX/Metal and cannot be built or run on
this machine; `mlx_probe` records the import attempt).

Multi-GPU: Qwen3-4B fits one GPU, so N GPUs run N independent replicas
(weak scaling, no collective on the data path); value is the sum over ranks
divided by the slowest rank's time.  The tensor-parallel path is measured in
the same run as tp_decode.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "base-mlx_b200"))

PROMPT_LEN, DECODE_TOKENS, KV_PREALLOC, SEED = 512, 300, 4096, 1234
# DRAM bytes read per launch / algorithmic bytes of decode_step_kernel, from an ncu capture
# of the Qwen3-4B layer shapes (4 layers + lm_head; profiles/decode_step_kernel_4b_l4_full.md)
TRAFFIC_RATIO = 1.0043

# Workload shapes (config.json contents of the random-init models)
CFG_0_6B = dict(
    model_type="qwen3", hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
    num_attention_heads=16, num_key_value_heads=8, head_dim=128, vocab_size=151936,
    rms_norm_eps=1e-6, rope_theta=1000000.0, tie_word_embeddings=True,
    max_position_embeddings=40960, bos_token_id=151643, eos_token_id=151645,
    quantization=dict(group_size=64, bits=4))
CFG_4B = dict(CFG_0_6B, hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
              num_attention_heads=32, num_key_value_heads=8)
CFG_32B = dict(CFG_0_6B, hidden_size=5120, intermediate_size=25600, num_hidden_layers=64,
               num_attention_heads=64, num_key_value_heads=8, tie_word_embeddings=False)
TP_PROMPT_LEN, TP_DECODE_TOKENS = 2048, 256  # config 5: 2048-token prompt, greedy decode of 256
REF_TOK_S = 32.75  # the reference's published rate on M2-class Apple Silicon, 300-token greedy decode
METRIC = "Qwen3-4B 4-bit batch-1 decode tok/s (plain & spec k=4); qmatmul HBM GB/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 tensor peak for a kernel timed in isolation (burst figure)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=lambda: self.lines.extend(self.proc.stdout), daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def prompt_ids(vocab: int) -> np.ndarray:
    return np.random.default_rng(SEED).integers(0, vocab, PROMPT_LEN).astype(np.uint32)


# ----------------------------------------------------------------- CPU leg ---

class CpuModel:
    """The oracle's CPU restatement (C qmatmul + numpy) of one benchmark model on
    seeded weights, decoding at the benchmark's KV positions: the cache is filled
    with seeded bf16 K/V rows up to the sample's first position (standing in for
    the prefill, which the decode metric excludes), then greedy decode steps are
    timed."""

    def __init__(self, cfg=None, prompt_len=PROMPT_LEN, decode_tokens=DECODE_TOKENS):
        from oracle import synth
        from oracle.qwen3_ref import Qwen3Ref
        self.cfg = dict(cfg or synth.QWEN3_4B)
        self.prompt_len, self.decode_tokens = prompt_len, decode_tokens
        t0 = time.time()
        self.ref = Qwen3Ref(self.cfg, synth.build_tensors(self.cfg, SEED, "ones", fast=True), backend="c")
        self.build_s = time.time() - t0
        self.start_tok = int(prompt_ids(self.cfg["vocab_size"])[0])

    def _cache_at(self, pos: int, room: int):
        from oracle import numerics as nm
        c = self.ref.new_cache(pos + room)
        rng = np.random.default_rng(SEED + pos)
        for li in range(self.cfg["num_hidden_layers"]):
            for arr in (c.k[li], c.v[li]):
                arr[:, :pos, :] = nm.bf16_round(rng.standard_normal(arr[:, :pos, :].shape, dtype=np.float32))
        c.seq_len = pos
        return c

    def windows(self, n: int):
        """First KV positions of the two timed windows: the start and the end of the
        workload's decode range [prompt_len, prompt_len + decode_tokens)."""
        return (self.prompt_len, self.prompt_len + self.decode_tokens - n)

    def sample(self, n: int) -> float:
        """n greedy decode steps in each window (caches filled untimed); tok/s."""
        secs, toks = 0.0, 0
        for p0 in self.windows(n):
            cache = self._cache_at(p0, n + 1)
            tok = self.start_tok
            t0 = time.time()
            for _ in range(n):
                tok = int(np.argmax(self.ref.forward([tok], cache)))
            secs += time.time() - t0
            toks += n
        return toks / secs

    def describe(self, n: int) -> str:
        w = self.windows(n)
        return (f"oracle CPU restatement (C qmatmul, all host threads, + numpy) of {self.cfg['hidden_size']}-hidden "
                f"Qwen3 on seeded weights: {n} timed greedy decode steps at KV positions {w[0]}-{w[0] + n - 1} and "
                f"{w[1]}-{w[1] + n - 1} (the start and end of the workload's {self.prompt_len}+{self.decode_tokens} "
                f"decode range; caches pre-filled with seeded bf16 K/V, untimed); weight build "
                f"{self.build_s:.1f}s not timed")


def cpu_sample(decode_tokens: int, threads: int):
    cm = CpuModel()
    return cm.sample(decode_tokens), threads, cm.describe(decode_tokens)


def mlx_probe() -> str:
    """Whether the reference's runtime (MLX) imports on this host."""
    r = subprocess.run([sys.executable, "-c", "import mlx.core"], capture_output=True, text=True)
    return "import mlx.core: ok" if r.returncode == 0 else \
        "import mlx.core: " + (r.stderr.strip().splitlines() or ["failed"])[-1]


def workload_config(world: int) -> dict:
    """The benchmark configuration both arms report."""
    return {"workload": "config3: Qwen3-4B 4-bit g64, batch 1, 512-token prompt, greedy decode 300, "
                        "KV pre-allocated 4096 (bf16)",
            "model": "Qwen3-4B (random init)", "prompt_len": PROMPT_LEN,
            "decode_tokens": DECODE_TOKENS, "kv_prealloc": KV_PREALLOC,
            "parallelism": f"replicas x{world}",
            "l2": "no flush: every decode step streams 2.26 GB of weights (> 126 MB L2)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import synth
    threads = os.cpu_count() or 1
    cm = CpuModel()
    per_step = []
    for i in range(args.warmup + args.steps):
        v = cm.sample(args.ref_tokens)
        if i >= args.warmup:
            per_step.append(v)
    desc = cm.describe(args.ref_tokens)
    value = float(np.mean(per_step))
    # config 1 (Qwen3-0.6B, 128-token prompt, greedy decode 128) on the same CPU path
    c1 = CpuModel(synth.QWEN3_0_6B, 128, 128)
    c1.sample(2)
    c1_val = c1.sample(args.ref_tokens)
    line = {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / REF_TOK_S, 4), "dtype": "u4xbf16->f32", "data": "synthetic",
            "config": workload_config(world),
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "config1_cpu": {"tok_s": round(c1_val, 4), "sample": c1.describe(args.ref_tokens)},
            "mlx_probe": mlx_probe(),
            "note": "flakerimi/base-mlx is Rust over mlx-rs/MLX Metal: no Rust toolchain, no MLX and no Metal here, "
                    "so the timed reference is the repository's CPU restatement of the same path (oracle/); each "
                    "step is a bounded sample of the configured workload (cpu_baseline.sample)"}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU leg ---

def qgemv_roofline(q, torch, info, peak_gbs, M=1, with_flops=False):
    """Time the standalone quantized matmul at M rows (the decode GEMV kernel for
    M <= 8) over one layer's 4B shapes + lm_head on rotating weight copies (> L2)
    in a CUDA graph; return achieved GB/s (weights + activations in + outputs)."""
    lib = q.lib()
    dev = torch.device("cuda")
    H, I, V = info.hidden, info.intermediate, info.vocab
    QD, KD = info.num_heads * info.head_dim, info.num_kv_heads * info.head_dim
    shapes = [(H, QD + 2 * KD), (QD, H), (H, 2 * I), (I, H), (H, V)]
    total_bytes, total_flops, launches = 0.0, 0.0, []
    bufs = []
    for K, N in shapes:
        nrep = max(2, int(300e6 // (N * K * 0.5625)) + 1)
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (nrep, N, K // 8), dtype=torch.int32, device=dev)
        s = (torch.rand(nrep, N, K // 64, device=dev) * 0.01).to(torch.bfloat16)
        b = (torch.rand(nrep, N, K // 64, device=dev) * -0.01).to(torch.bfloat16)
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        bufs.append((w, s, b, x, y))
        for i in range(nrep):
            launches.append((x.data_ptr(), w[i].data_ptr(), s[i].data_ptr(), b[i].data_ptr(), y.data_ptr(), N, K))
        total_bytes += nrep * (N * K * 0.5625 + M * (2 * K + 2 * N))
        total_flops += nrep * 2.0 * M * N * K
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        def run_all():
            for (xp, wp, sp, bp, yp, N, K) in launches:
                q.check(lib.qw_quantized_matmul(xp, wp, sp, bp, yp, M, N, K, 64, 4, st.cuda_stream))
        run_all()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            run_all()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 3
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    achieved = total_bytes / sec / 1e9
    del bufs, g
    torch.cuda.empty_cache()
    if with_flops:
        return achieved, len(launches), total_bytes / len(launches), total_flops / sec / 1e12
    return achieved, len(launches), total_bytes / len(launches)


def qgemm_roofline(q, torch, info, M=2048):
    """Time the multi-row quantized matmul (the tcgen05 prefill GEMM, with its
    bf16 -> fp16 activation conversion) over one layer's Qwen3-4B shapes at
    M = 2048 rows; the four shapes' operands (~220 MB) exceed L2.  Returns
    achieved TFLOP/s (2*M*N*K per matmul) and the per-shape times."""
    lib = q.lib()
    dev = torch.device("cuda")
    H, I = info.hidden, info.intermediate
    QD, KD = info.num_heads * info.head_dim, info.num_kv_heads * info.head_dim
    shapes = [(H, QD + 2 * KD), (QD, H), (H, I), (I, H)]
    bufs = []
    for K, N in shapes:
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // 8), dtype=torch.int32, device=dev)
        s = (torch.rand(N, K // 64, device=dev) * 0.01).to(torch.bfloat16)
        b = (torch.rand(N, K // 64, device=dev) * -0.01).to(torch.bfloat16)
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        bufs.append((x, w, s, b, y, N, K))
    st = torch.cuda.Stream()
    per = []
    with torch.cuda.stream(st):
        def one(x, w, s, b, y, N, K):
            q.check(lib.qw_quantized_matmul(x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), y.data_ptr(),
                                            M, N, K, 64, 4, st.cuda_stream))
        for bb in bufs:
            for _ in range(3):
                one(*bb)
        torch.cuda.synchronize()
        reps = 5
        for bb in bufs:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                one(*bb)
            e1.record(st)
            torch.cuda.synchronize()
            per.append(e0.elapsed_time(e1) / reps)
    flops = sum(2.0 * M * N * K for (K, N) in shapes)
    sec = sum(per) / 1e3
    del bufs
    torch.cuda.empty_cache()
    return flops / sec / 1e12, per, shapes


def launches_per_generation(info, prompt_len, decode_tokens):
    """Kernels the library launches for one greedy generation (for gpu_launches):
    the prefill runs the kernel chain (embed; per layer 2 rmsnorm, 4 qgemm,
    q/k-norm+RoPE+KV write, attention; lm_head, argmax finalize, step), every
    decode step is one launch of the persistent decode kernel."""
    L = info.num_layers
    prefill = 1 + 8 * L + 3
    return prefill + (decode_tokens - 1)


def run_ours(args):
    import torch
    import qwen3_b200 as q
    rank, world, local = dist_env()
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300))
    torch.cuda.set_device(local)
    cfg = dict(CFG_4B)
    m = q.Qwen3.init_random(cfg, SEED, norm_mode="ones", device=local)
    info = m.info
    prompt = prompt_ids(cfg["vocab_size"])

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        m.generate_greedy(prompt, DECODE_TOKENS)
    barrier()
    results = []
    with ClockSampler(local) as clk:
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            results.append(m.generate_greedy(prompt, DECODE_TOKENS))
        barrier()
        region = time.perf_counter() - t0
    decode_ms = sum(r.decode_ms for r in results)
    prefill_ms = sum(r.prefill_ms for r in results)
    dec_tokens = sum(max(r.completion_tokens - 1, 0) for r in results)
    gen_tokens = sum(r.completion_tokens for r in results)
    vals = torch.tensor([decode_ms, region, float(dec_tokens), float(gen_tokens)], dtype=torch.float64,
                        device="cuda")
    if dist is not None:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        decode_ms_max, region_max, dec_tokens_all, gen_tokens_all = mx[0].item(), mx[1].item(), sm[2].item(), sm[3].item()
    else:
        decode_ms_max, region_max, dec_tokens_all, gen_tokens_all = decode_ms, region, dec_tokens, gen_tokens
    value = dec_tokens_all / (decode_ms_max / 1e3)

    # e2e through the C ABI with host buffers, the reference CLI bench's way
    e2e_rates = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        full = m.generate_greedy(prompt, DECODE_TOKENS)
        t_full = time.perf_counter() - t0
        t0 = time.perf_counter()
        m.generate_greedy(prompt, 1)
        t_ttft = time.perf_counter() - t0
        e2e_rates.append((full.completion_tokens - 1) / max(t_full - t_ttft, 1e-6))
    e2e_local = float(np.mean(e2e_rates))
    e2e_t = torch.tensor([e2e_local], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.SUM)
    e2e_value = e2e_t.item()

    peak, peak_kind = peaks()
    extra = {}
    cpu = None
    if rank == 0:
        ach, nl, per_launch = qgemv_roofline(q, torch, info, peak)
        # algorithmic bytes of one decode step: all quantized weights + KV read at the mean position
        w_bytes = 0
        H, I, V, L = info.hidden, info.intermediate, info.vocab, info.num_layers
        QD, KD = info.num_heads * info.head_dim, info.num_kv_heads * info.head_dim
        w_bytes = (L * (H * (QD + 2 * KD) + QD * H + 2 * H * I + I * H) + V * H) * 0.5625
        mean_T = PROMPT_LEN + DECODE_TOKENS / 2
        kv_bytes = L * 2 * KD * 2 * mean_T
        step_s = decode_ms / 1e3 / max(dec_tokens, 1)
        # the dominant kernel: one decode_step_kernel launch per token (CUDA events
        # around the decode loop, inside the library)
        step_gbs = (w_bytes + kv_bytes) / step_s / 1e9
        roof = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(step_gbs / peak, 4), "traffic": int(TRAFFIC_RATIO * (w_bytes + kv_bytes)),
                "traffic_source": "ncu dram__bytes_read on the Qwen3-4B layer shapes (4 layers + lm_head, one "
                                  "launch): read/algorithmic 1.0043, applied to these algorithmic bytes "
                                  "(profiles/decode_step_kernel_4b_l4_full.md)",
                "kernel": "decode_step_kernel (persistent decode step: all 36 layers + lm_head in one launch)",
                "bytes_per_launch": int(w_bytes + kv_bytes), "launches_timed": int(dec_tokens),
                "bytes_note": "quantized weights (0.5625 B/param) + bf16 K/V read at the mean KV length 662",
                "peak_source": peak_kind}
        tf, per_ms, shp = qgemm_roofline(q, torch, info)
        tpk, tpk_kind = tensor_peak()
        extra["qgemm_roofline"] = {"bound": "tensor", "achieved": round(tf, 1), "peak": tpk, "unit": "TFLOP/s",
                                   "frac": round(tf / tpk, 4), "peak_source": tpk_kind,
                                   "kernel": "qgemm_tc_kernel (tcgen05 prefill GEMM) + x_to_f16p_kernel, "
                                             "qw_quantized_matmul M=2048 over the 4B layer shapes",
                                   "ms_per_shape": {f"K{K}xN{N}": round(t, 4) for (K, N), t in zip(shp, per_ms)}}
        extra["qgemv_roofline"] = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                                   "frac": round(ach / peak, 4),
                                   "kernel": "qw_quantized_matmul (standalone op, M=1), 4B layer shapes + lm_head",
                                   "bytes_per_launch": int(per_launch), "launches_timed": nl}
        # config 2: the standalone op at the benchmark's row counts, rotating weight copies (> L2)
        c2 = {"M=1": {"GB/s": round(ach, 1), "frac_hbm": round(ach / peak, 4)}}
        for Mr in (5, 128):
            a2, _, _, tf2 = qgemv_roofline(q, torch, info, peak, M=Mr, with_flops=True)
            c2[f"M={Mr}"] = {"GB/s": round(a2, 1), "frac_hbm": round(a2 / peak, 4), "TFLOP/s": round(tf2, 2),
                             "frac_tensor": round(tf2 / tensor_peak()[0], 4)}
        c2["M=2048"] = {"TFLOP/s": round(tf, 1), "frac_tensor": round(tf / tpk, 4)}
        extra["config2_qmatmul"] = {"shapes": "Qwen3-4B q|k|v, o_proj, gate|up, down_proj, lm_head (K, N)",
                                    "rows": c2, "peak_gbs": peak, "peak_tflops": tpk}
        if world == 1 and not args.no_cpu:
            v, cores, desc = cpu_sample(args.cpu_tokens, os.cpu_count() or 1)
            cpu = {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
    if rank == 0 and world == 1:
        # single-GPU extras (at N > 1 the other GPUs would idle meanwhile)
        if args.spec:
            extra["spec"] = spec_measure(q, m, prompt, cfg)
        extra["config1"] = config1_measure(q)
        extra["batch8"] = batch8_measure(q, m)
        # sampled decode (temperature 0.7, top-p 0.95: the reference's SamplingParams defaults):
        # the device pick after every step on the same model and prompt
        rs = m.generate_sampled(prompt, DECODE_TOKENS, temperature=0.7, top_p=0.95, seed=SEED, eos=[1 << 30])
        extra["sampled_decode"] = {"tok_s": round((rs.completion_tokens - 1) / (rs.decode_ms / 1e3), 2),
                                   "temperature": 0.7, "top_p": 0.95, "tokens": rs.completion_tokens}
    m.close()
    if world > 1 and not args.no_tp:
        # config 5 at tp = N on the same ranks: one Qwen3-32B sequence split over all GPUs
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        tp_line = tp_decode_core(2, 3, dist, rank, world, local)
        if rank == 0:
            extra["tp_decode"] = {k: tp_line[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup",
                                                          "scaling", "config", "roofline", "decode_ms_per_token",
                                                          "ttft_ms", "ranks_agree_on_tokens")}
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(region_max * 1e3 / args.steps, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / REF_TOK_S, 3),
                "dtype": "u4xbf16->f32", "data": "synthetic (seeded random-init weights and prompt ids)",
                "config": workload_config(world),
                "roofline": roof, "cpu_baseline": cpu,
                "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                        "h2d_bytes_per_step": PROMPT_LEN * 4, "d2h_bytes_per_step": DECODE_TOKENS * 4 + 40},
                "gpu_launches": launches_per_generation(info, PROMPT_LEN, DECODE_TOKENS) * args.steps,
                "clocks": clk.summary(),
                "decode_ms_per_token": round(decode_ms / max(dec_tokens, 1), 4),
                "ttft_ms": round(prefill_ms / len(results), 3),
                "gen_tok_s_incl_prefill": round(gen_tokens_all / (region_max), 2)}
        line.update(extra)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def spec_measure(q, target, prompt, cfg4):
    """Config 4: 4B target + 0.6B draft, k=4, forced acceptance p in {0, 0.5, 0.8, 1}; and speculative
    sampling (temperature 0.7, top-p 0.95) against plain sampled decode."""
    draft = q.Qwen3.init_random(dict(CFG_0_6B), SEED + 1, norm_mode="ones", device=0)
    plain = target.generate_greedy(prompt, DECODE_TOKENS)
    out = {"k": 4, "plain_decode_tok_s": round((plain.completion_tokens - 1) / (plain.decode_ms / 1e3), 2)}
    for p in (0.0, 0.5, 0.8, 1.0):
        q.speculative_generate(target, draft, prompt, DECODE_TOKENS, k=4, force_p=p, seed=7, forced=plain.tokens)
        res, st = q.speculative_generate(target, draft, prompt, DECODE_TOKENS, k=4, force_p=p, seed=7,
                                         forced=plain.tokens)
        dec_ms = st.total_ms - st.prefill_ms
        out[f"p{p}"] = {"tok_s": round((res.completion_tokens - 1) / (dec_ms / 1e3), 2),
                        "tokens_match_plain": res.tokens == plain.tokens,
                        "iters": st.iters, "accepted": st.accepted, "proposed": st.proposed,
                        "draft_ms_mean": round(st.draft_ms_mean, 3), "verify_ms_mean": round(st.verify_ms_mean, 3),
                        "accept_ms_mean": round(st.accept_ms_mean, 3)}
        out[f"p{p}"]["speedup_vs_plain"] = round(out[f"p{p}"]["tok_s"] / out["plain_decode_tok_s"], 3)
    # speculative sampling (temperature 0.7, top-p 0.95) against plain sampled decode
    ps = target.generate_sampled(prompt, DECODE_TOKENS, temperature=0.7, top_p=0.95, seed=SEED, eos=[1 << 30])
    plain_s = (ps.completion_tokens - 1) / (ps.decode_ms / 1e3)
    q.speculative_generate_sampled(target, draft, prompt, DECODE_TOKENS, k=4, temperature=0.7, top_p=0.95, seed=7,
                                   eos=[1 << 30])
    res, st = q.speculative_generate_sampled(target, draft, prompt, DECODE_TOKENS, k=4, temperature=0.7, top_p=0.95,
                                             seed=7, eos=[1 << 30])
    dec_ms = st.total_ms - st.prefill_ms
    tok_s = (res.completion_tokens - 1) / (dec_ms / 1e3)
    out["sampled_t0.7_p0.95"] = {"tok_s": round(tok_s, 2), "plain_sampled_tok_s": round(plain_s, 2),
                                 "speedup_vs_plain_sampled": round(tok_s / plain_s, 3), "iters": st.iters,
                                 "accepted": st.accepted, "proposed": st.proposed,
                                 "draft_ms_mean": round(st.draft_ms_mean, 3),
                                 "verify_ms_mean": round(st.verify_ms_mean, 3),
                                 "accept_ms_mean": round(st.accept_ms_mean, 3)}
    draft.close()
    return out


def batch8_measure(q, m):
    """Batch-8 greedy decode on the 4B model (config 4's batch-8 row, on one GPU):
    8 seeded 512-token prompts decoded together, 300 tokens each; aggregate
    decode tok/s over all sequences (CUDA events inside the library), and
    whether sequence 0 equals its batch-1 greedy run."""
    rng = np.random.default_rng(SEED + 8)
    prompts = [rng.integers(0, CFG_4B["vocab_size"], PROMPT_LEN).astype(np.uint32) for _ in range(8)]
    m.generate_greedy_batch(prompts, DECODE_TOKENS, eos=[1 << 30])
    runs = [m.generate_greedy_batch(prompts, DECODE_TOKENS, eos=[1 << 30]) for _ in range(2)]
    dec_ms = sum(st.decode_ms for _, st in runs)
    toks = sum(sum(len(o) - 1 for o in outs) for outs, _ in runs)
    same = runs[0][0][0] == m.generate_greedy(prompts[0], DECODE_TOKENS, eos=[1 << 30]).tokens
    return {"workload": "Qwen3-4B 4-bit g64, 8 sequences x (512-token prompt, greedy decode 300), one GPU",
            "decode_tok_s": round(toks / (dec_ms / 1e3), 2), "decode_ms_per_step": round(dec_ms / 2 / (DECODE_TOKENS - 1), 4),
            "rows_per_launch": "sub-batches of up to 4 (shared memory holds every row's staged activations)",
            "seq0_matches_batch1": same}


def config1_measure(q):
    """Config 1: Qwen3-0.6B, 128-token prompt, greedy decode of 128 (decode tok/s
    as main.rs defines it, CUDA events inside the library)."""
    m = q.Qwen3.init_random(dict(CFG_0_6B), SEED, norm_mode="ones", device=0)
    prompt = prompt_ids(CFG_0_6B["vocab_size"])[:128]
    for _ in range(3):
        m.generate_greedy(prompt, 128, eos=[1 << 30])
    rs = [m.generate_greedy(prompt, 128, eos=[1 << 30]) for _ in range(5)]
    dec = sum(r.decode_ms for r in rs) / 1e3
    n = sum(r.completion_tokens - 1 for r in rs)
    m.close()
    return {"workload": "config1: Qwen3-0.6B 4-bit g64, batch 1, 128-token prompt, greedy decode 128",
            "decode_tok_s": round(n / dec, 2), "decode_ms_per_token": round(dec * 1e3 / n, 4),
            "ttft_ms": round(sum(r.prefill_ms for r in rs) / len(rs), 3), "runs": len(rs)}


def profile_qmm(spec: str) -> None:
    """ncu workload: three qw_quantized_matmul calls of one shape "M,K,N"."""
    import torch
    import qwen3_b200 as q
    M, K, N = (int(v) for v in spec.split(","))
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(SEED)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, K // 8), dtype=torch.int64, generator=g).to(torch.int32).to(dev)
    s = (torch.rand(N, K // 64, generator=g) * 0.01 + 0.001).to(torch.bfloat16).to(dev)
    b = (-torch.rand(N, K // 64, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    y = torch.zeros(M, N, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        q.quantized_matmul(x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), y.data_ptr(), M, N, K, stream=st)
    torch.cuda.synchronize()
    print(f"profile_qmm: M={M} K={K} N={N} max|y| {float(y.float().abs().max())}")


def profile_sampled(n: int, model: str) -> None:
    """ncu workload: one sampled generation of n tokens (temperature 0.7, top-p
    0.95) after the prefill, through qw_generate_sampled."""
    import torch
    import qwen3_b200 as q
    cfg = dict(CFG_4B if model == "4b" else CFG_0_6B)
    plen = PROMPT_LEN if model == "4b" else 128
    m = q.Qwen3.init_random(cfg, SEED, norm_mode="ones", device=0)
    r = m.generate_sampled(prompt_ids(cfg["vocab_size"])[:plen].tolist(), n, temperature=0.7, top_p=0.95, seed=SEED,
                           eos=[1 << 30])
    torch.cuda.synchronize()
    print(f"profile_sampled: {model} prefill {plen} + {len(r.tokens)} sampled tokens")


def profile_decode(n: int, model: str, layers: int = 0) -> None:
    """Prefill and n decode steps, one qw_forward each (the ncu workloads): the
    bench model (Qwen3-4B, 512-token prompt) or, for captures that must stay
    small, Qwen3-0.6B with a 128-token prompt; layers > 0 keeps only that many
    decoder layers (the 4B layer shapes at a few hundred MB on the device)."""
    import torch
    import qwen3_b200 as q
    cfg = dict(CFG_4B if model == "4b" else CFG_0_6B)
    if layers > 0:
        cfg["num_hidden_layers"] = layers
    plen = PROMPT_LEN if model == "4b" else 128
    m = q.Qwen3.init_random(cfg, SEED, norm_mode="ones", device=0)
    c = m.new_cache(KV_PREALLOC)
    _, tok = m.forward(prompt_ids(cfg["vocab_size"])[:plen].tolist(), c, want_logits=False)
    for _ in range(n):
        _, tok = m.forward([tok], c, want_logits=False)
    torch.cuda.synchronize()
    print(f"profile_decode: {model} ({cfg['num_hidden_layers']} layers) prefill {plen} + {n} decode steps, "
          f"last token {tok}")


def run_tp_decode(args):
    """Qwen3-32B tensor-parallel batch-1 greedy decode (config 5): ONE sequence
    served by all N ranks, one process per GPU (launched by torchrun; N=1 runs
    the unsplit model).  Each rank loads its shard (q/k/v, gate/up rows;
    o_proj/down_proj columns; lm_head vocabulary rows), the library's own NCCL
    communicator carries the two sum all-reduces per layer and the argmax key
    all-reduce; a gloo group only exchanges the NCCL id and the timings.

    value = decode tok/s of the sequence, (n-1) / decode time, the decode time
    taken from the library's CUDA events and maxed over ranks (strong scaling:
    the work is fixed, N splits it).  roofline: per-rank algorithmic bytes per
    token (its weight shard + its K/V heads at the mean KV length) over the
    per-token time, against the measured HBM copy bandwidth.  NVLS is left off
    (NCCL_NVLS_ENABLE=0): the all-reduces carry 20 KB each, where latency, not
    bandwidth, sets their cost."""
    import datetime
    import torch
    rank, world, local = dist_env()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
    dist = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)
    line = tp_decode_core(args.steps, args.warmup, dist, rank, world, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def tp_decode_core(steps, warmup, dist, rank, world, local):
    """The config-5 measurement over an initialised process group (or none at
    world 1); returns the JSON line's dict on rank 0, None elsewhere."""
    import torch
    import qwen3_b200 as q
    cfg = dict(CFG_32B)
    m = q.Qwen3.init_random(cfg, SEED, norm_mode="ones", device=local, tp_rank=rank, tp_size=world)
    if world > 1:
        q.tp_init(m, rank, world)
    prompt = np.random.default_rng(SEED).integers(0, cfg["vocab_size"], TP_PROMPT_LEN).astype(np.uint32)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(warmup):
        m.generate_greedy(prompt, TP_DECODE_TOKENS)
    barrier()
    results = []
    with ClockSampler(local) as clk:
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            results.append(m.generate_greedy(prompt, TP_DECODE_TOKENS))
        barrier()
        region = time.perf_counter() - t0
    decode_ms = sum(r.decode_ms for r in results)
    prefill_ms = sum(r.prefill_ms for r in results)
    dec_tokens = sum(max(r.completion_tokens - 1, 0) for r in results)
    toks = results[-1].tokens
    nccl_group = dist is not None and dist.get_backend() == "nccl"
    vals = torch.tensor([decode_ms, prefill_ms, region], dtype=torch.float64,
                        device="cuda" if nccl_group else "cpu")
    agree = True
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        got = [None] * world
        dist.all_gather_object(got, toks)
        agree = all(g == toks for g in got)
    decode_ms_max, prefill_ms_max, region_max = (float(v) for v in vals.cpu())
    value = dec_tokens / (decode_ms_max / 1e3)
    line = None
    if rank == 0:
        info = m.info
        H, I, V, L = info.hidden, info.intermediate, info.vocab, info.num_layers
        QD, KD = info.num_heads * info.head_dim, info.num_kv_heads * info.head_dim
        w_full = (L * (H * (QD + 2 * KD) + QD * H + 2 * H * I + I * H) + V * H) * 0.5625
        kv_full = L * 2 * KD * 2 * (TP_PROMPT_LEN + TP_DECODE_TOKENS / 2)
        per_rank = (w_full + kv_full) / world
        tok_s = decode_ms_max / 1e3 / max(dec_tokens, 1)
        gbs = per_rank / tok_s / 1e9
        peak, peak_kind = peaks()
        line = {"metric": "Qwen3-32B 4-bit batch-1 tensor-parallel greedy decode tok/s", "value": round(value, 2),
                "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
                "ms_per_step": round(region_max * 1e3 / steps, 3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "u4xbf16->f32",
                "data": "synthetic (seeded random-init weights and prompt ids)",
                "config": {"workload": f"config5: Qwen3-32B 4-bit g64 (untied lm_head), batch 1, "
                                       f"{TP_PROMPT_LEN}-token prompt, greedy decode {TP_DECODE_TOKENS}",
                           "parallelism": f"tp{world}",
                           "l2": "no flush: every decode step streams its weight shard (> 126 MB L2)"},
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                             "bytes_per_token_per_rank": int(per_rank),
                             "bytes_note": "per-rank share of the quantized weights (0.5625 B/param) and of the "
                                           "bf16 K/V read at the mean KV length 2176"},
                "decode_ms_per_token": round(decode_ms_max / max(dec_tokens, 1), 4),
                "ttft_ms": round(prefill_ms_max / len(results), 3),
                "ranks_agree_on_tokens": agree, "clocks": clk.summary()}
    m.close()
    barrier()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-tokens", type=int, default=8)
    ap.add_argument("--ref-tokens", type=int, default=4)
    ap.add_argument("--no-spec", dest="spec", action="store_false")
    ap.add_argument("--profile-decode", type=int, default=0, metavar="N",
                    help="profiling workload for ncu: weight init, the prefill and N greedy decode steps through "
                         "qw_forward; prints no bench line")
    ap.add_argument("--profile-model", choices=["4b", "0.6b"], default="4b")
    ap.add_argument("--profile-layers", type=int, default=0, metavar="L",
                    help="with --profile-decode: keep only L decoder layers")
    ap.add_argument("--profile-sampled", type=int, default=0, metavar="N",
                    help="profiling workload for ncu: a sampled generation of N tokens; prints no bench line")
    ap.add_argument("--profile-qmm", default="", metavar="M,K,N",
                    help="profiling workload for ncu: three quantized matmuls of one shape; prints no bench line")
    ap.add_argument("--no-tp", action="store_true", help="at N > 1, skip the tp_decode (config 5) measurement")
    ap.add_argument("--tp-decode", action="store_true",
                    help="Qwen3-32B tensor-parallel decode (config 5) over the torchrun ranks; one JSON line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tp_decode:
        run_tp_decode(args)
    elif args.profile_qmm:
        profile_qmm(args.profile_qmm)
    elif args.profile_sampled > 0:
        profile_sampled(args.profile_sampled, args.profile_model)
    elif args.profile_decode > 0:
        profile_decode(args.profile_decode, args.profile_model, args.profile_layers)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
