// The Qwen3 forward step and the device-resident greedy loop.
//
// forward_dev restates crates/base-mlx-core/src/model/qwen3.rs:314-563
// (Qwen3::forward_internal) as a chain of sm_100a kernels on one stream:
//
//   S <= 8 rows (decode / speculative verify):
//     embed -> per layer { qgemv[RMSNorm -> q|k|v] -> attn_decode[q/k norm, RoPE,
//     KV write, split-T attention] -> qgemv[o_proj + residual] ->
//     qgemv[RMSNorm -> gate|up -> SiLU*up] -> qgemv[down_proj + residual] }
//     -> qgemv[final norm -> lm_head -> argmax] -> step_finish
//   S > 8 rows (prefill): the same with rmsnorm + qgemm + qk_norm_rope_kvwrite +
//     attn_prefill kernels.
//
// Every kernel is launched with programmatic dependent launch, so a kernel's
// weight prefetch overlaps the tail of its predecessor.  The KV length lives
// on the device, which lets one captured CUDA graph serve every decode step.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "model.h"

namespace qw {

namespace {

QSeg seg_of(const QLin& q, void* y, int ldy) {
    QSeg s;
    s.w = q.w;
    s.s = q.s;
    s.b = q.b;
    s.y = y;
    s.n = q.n;
    s.ldy = ldy;
    s.rb0 = 0;
    return s;
}

QmmArgs qmm_base(qw_model* m, const bf16* x, int ldx, int M, int K) {
    QmmArgs a;
    std::memset(&a, 0, sizeof(a));
    Workspace& w = m->ws;
    a.x = x;
    a.ldx = ldx;
    a.M = M;
    a.K = K;
    a.eps = m->cfg.eps;
    a.amax_partial = w.amax_partial;
    a.err = m->d_err;
    return a;
}

// QW_PREFILL_GEMM=legacy keeps the multi-row matmuls on the mma.sync kernel.
bool tc_gemm_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("QW_PREFILL_GEMM");
        return !(e && std::strcmp(e, "legacy") == 0);
    }();
    return on;
}

void qmm(qw_model* m, QmmArgs a, cudaStream_t st) {
    if (a.M <= 8 && qgemv_fits(a))
        QW_CUDA(launch_qgemv(a, st, true, m->num_sms));
    else if (a.M <= 8 && (a.norm_w || a.epi == EPI_LOGITS))
        // the fused RMSNorm prologue and the logits epilogue exist in the GEMV only
        throw Error(QW_ERR_INFERENCE, "normed / logits GEMV row of K=" + std::to_string(a.K) +
                                          " exceeds the GEMV's shared-memory slab");
    else if (tc_gemm_enabled() && qgemm_tc_supported(a) && m->ws.xh_bytes >= qgemm_tc_scratch_bytes(a.M, a.K))
        QW_CUDA(launch_qgemm_tc(a, m->ws.xh, m->ws.xh_bytes, st));
    else
        QW_CUDA(launch_qgemm(a, st, m->num_sms));
}

// o_proj / down_proj and, under tensor parallelism, the sum of the ranks'
// partials into the residual stream: over peer memory for decode rows (the
// GEMV pushes its partial rows to every rank, one small kernel sums them), else
// an NCCL all-reduce and a residual add.
void tp_reduce_gemv(qw_model* m, QmmArgs& a, int S, cudaStream_t st) {
    Workspace& w = m->ws;
    if (m->tp_size > 1 && S <= TP_PUSH_ROWS && tp_push_ready(m)) {
        a.epi = EPI_F32_PUSH;
        if (a.M <= 8 && qgemv_fits(a)) {
            tp_push_args(m, a.push);
            QW_CUDA(launch_qgemv(a, st, true, m->num_sms));
            QW_CUDA(launch_tp_push_reduce(m, w.x, S, st));
            return;
        }
        a.epi = EPI_F32;
    }
    qmm(m, a, st);
    if (m->tp_size > 1) {
        tp_allreduce_sum_f32(m, w.f32, (size_t)S * m->cfg.hidden, st);
        QW_CUDA(launch_resid_add_f32(w.x, w.f32, S * m->cfg.hidden, st));
    }
}

}  // namespace

void forward_dev(qw_model* m, qw_cache* c, const int* d_ids, int S, int logits_mode, bool store_logits,
                 int* d_argmax, cudaStream_t st, StepCtl* ctl, int* next_tok, int* out, const int* gate) {
    const Config& cf = m->cfg;
    Workspace& w = m->ws;
    const int H = cf.hidden, D = cf.head_dim, QD = m->hq_l * D, KD = m->hkv_l * D, I = m->inter_l;
    const bool decode = S <= 8;
    const bool tp = m->tp_size > 1;
    if (S > w.cap_rows) throw Error(QW_ERR_INFERENCE, "workspace too small for forward");
    if (decode && !tp && mk_forward(m, c, d_ids, S, logits_mode, store_logits, d_argmax, st, ctl, next_tok, out, gate))
        return;

    QW_CUDA(launch_embed(d_ids, S, m->embed.w, m->embed.s, m->embed.b, H, cf.vocab, w.x, m->d_err, st, true));
    if (m->trace) QW_CUDA(cudaMemcpyAsync(m->trace, w.x, (size_t)S * H * 2, cudaMemcpyDeviceToDevice, st));

    AttnArgs aa;
    std::memset(&aa, 0, sizeof(aa));
    aa.q = w.q;
    aa.k = w.k;
    aa.v = w.v;
    aa.ldq = QD;
    aa.ldk = KD;
    aa.ldv = KD;
    aa.eps = cf.eps;
    aa.rope_cos = m->rope_cos;
    aa.rope_sin = m->rope_sin;
    aa.max_pos = c->max_pos;
    aa.seq_len = c->d_seq_len;
    aa.S = S;
    aa.Hq = m->hq_l;
    aa.Hkv = m->hkv_l;
    aa.scale = 1.0f / sqrtf((float)D);
    aa.part = w.attn_part;
    aa.counters = w.attn_counters;
    aa.out = w.attn;
    aa.ldo = QD;
    aa.nsplit = std::max(1, std::min(2 * m->num_sms, m->num_sms / std::max(1, m->hkv_l)));
    aa.err = m->d_err;

    for (int l = 0; l < cf.layers; ++l) {
        Layer& L = m->layers[l];
        aa.q_norm_w = L.q_norm;
        aa.k_norm_w = L.k_norm;
        aa.kcache = c->kl(l);
        aa.vcache = c->vl(l);
        const bf16* xin = w.x;
        if (!decode) {
            QW_CUDA(launch_rmsnorm(w.x, L.in_norm, w.h, S, H, cf.eps, st));
            xin = w.h;
        }
        {
            QmmArgs a = qmm_base(m, xin, H, S, H);
            if (decode) a.norm_w = L.in_norm;
            a.seg[0] = seg_of(L.q, w.q, QD);
            a.seg[1] = seg_of(L.k, w.k, KD);
            a.seg[2] = seg_of(L.v, w.v, KD);
            a.nseg = 3;
            a.epi = EPI_STORE;
            qmm(m, a, st);
        }
        if (decode) {
            QW_CUDA(launch_attn_decode(aa, st, true));
        } else {
            QW_CUDA(launch_qk_norm_rope_kvwrite(aa, w.qr, st));
            QW_CUDA(launch_attn_prefill(aa, w.qr, st));
        }
        if (m->trace)
            QW_CUDA(cudaMemcpyAsync(m->trace_attn + (size_t)l * S * QD, w.attn, (size_t)S * QD * 2,
                                    cudaMemcpyDeviceToDevice, st));
        {
            QmmArgs a = qmm_base(m, w.attn, QD, S, QD);
            a.seg[0] = seg_of(L.o, tp ? (void*)w.f32 : (void*)w.x, H);
            a.nseg = 1;
            a.epi = tp ? EPI_F32 : EPI_RESID;
            tp_reduce_gemv(m, a, S, st);
        }
        if (m->trace)
            QW_CUDA(cudaMemcpyAsync(m->trace_mid + (size_t)l * S * H, w.x, (size_t)S * H * 2,
                                    cudaMemcpyDeviceToDevice, st));
        xin = w.x;
        if (!decode) {
            QW_CUDA(launch_rmsnorm(w.x, L.post_norm, w.h, S, H, cf.eps, st));
            xin = w.h;
        }
        {
            QmmArgs a = qmm_base(m, xin, H, S, H);
            if (decode) a.norm_w = L.post_norm;
            a.seg[0] = seg_of(L.gate, w.mlp, I);
            a.seg[1] = seg_of(L.up, w.mlp, I);
            a.nseg = 2;
            a.epi = EPI_SWIGLU;
            qmm(m, a, st);
        }
        {
            QmmArgs a = qmm_base(m, w.mlp, I, S, I);
            a.seg[0] = seg_of(L.down, tp ? (void*)w.f32 : (void*)w.x, H);
            a.nseg = 1;
            a.epi = tp ? EPI_F32 : EPI_RESID;
            tp_reduce_gemv(m, a, S, st);
        }
        if (m->trace)
            QW_CUDA(cudaMemcpyAsync(m->trace + (size_t)(l + 1) * S * H, w.x, (size_t)S * H * 2,
                                    cudaMemcpyDeviceToDevice, st));
    }

    if (logits_mode) {
        const int rows = logits_mode == 2 ? S : 1;
        const bf16* xin = w.x + (size_t)(S - rows) * H;
        const bool vocab_split = tp && !cf.tied;
        if (rows > w.cap_logits) throw Error(QW_ERR_INFERENCE, "logits workspace too small");
        if (rows <= 8) {
            QmmArgs a = qmm_base(m, xin, H, rows, H);
            a.norm_w = m->final_norm;
            a.seg[0] = seg_of(m->lm_head, w.logits, m->vocab_l);
            a.nseg = 1;
            a.epi = EPI_LOGITS;
            a.store_logits = store_logits ? 1 : 0;
            a.amax_row_offset = vocab_split ? m->tp_rank * m->vocab_l : 0;
            qmm(m, a, st);
            QW_CUDA(launch_amax_finalize(w.amax_partial, qgemv_row_blocks(a), rows, d_argmax,
                                         vocab_split ? w.amax_keys : nullptr, st));
        } else {
            QW_CUDA(launch_rmsnorm(xin, m->final_norm, w.h, rows, H, cf.eps, st));
            QmmArgs a = qmm_base(m, w.h, H, rows, H);
            a.seg[0] = seg_of(m->lm_head, w.logits, m->vocab_l);
            a.nseg = 1;
            a.epi = EPI_STORE;
            qmm(m, a, st);
            QW_CUDA(launch_argmax_rows(w.logits, rows, m->vocab_l, d_argmax, vocab_split ? w.amax_keys : nullptr,
                                       vocab_split ? m->tp_rank * m->vocab_l : 0, st));
        }
        if (vocab_split) {
            // global argmax across the vocab shards: max over packed (logit, index) keys
            tp_allreduce_max_u64(m, w.amax_keys, (size_t)rows, st);
            QW_CUDA(launch_keys_to_index(w.amax_keys, rows, d_argmax, st));
        }
    }
    QW_CUDA(launch_step_finish(c->d_seq_len, S, d_argmax, ctl, next_tok, out, gate, st, true));
}

void generate_greedy_dev(qw_model* m, qw_cache* c, int n_prompt, int max_new, const std::vector<int>& eos,
                         qw_gen_stats* stats, cudaStream_t st) {
    Workspace& w = m->ws;
    if (n_prompt + max_new > c->max_pos)
        throw Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(n_prompt + max_new) +
                                             " positions, max " + std::to_string(c->max_pos));
    if (max_new > w.out_cap) throw Error(QW_ERR_INVALID_ARG, "max_new too large");
    StepCtl ctl;
    std::memset(&ctl, 0, sizeof(ctl));
    ctl.max_new = max_new;
    ctl.n_eos = (int)std::min<size_t>(eos.size(), 8);
    for (int i = 0; i < ctl.n_eos; ++i) ctl.eos[i] = eos[i];
    QW_CUDA(cudaMemcpyAsync(w.ctl, &ctl, sizeof(ctl), cudaMemcpyHostToDevice, st));
    int zero = 0;
    QW_CUDA(cudaMemcpyAsync(c->d_seq_len, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    c->seq_len = 0;

    cudaEvent_t e0, e1, e2;
    QW_CUDA(cudaEventCreate(&e0));
    QW_CUDA(cudaEventCreate(&e1));
    QW_CUDA(cudaEventCreate(&e2));
    QW_CUDA(cudaEventRecord(e0, st));
    forward_dev(m, c, w.ids, n_prompt, 1, false, w.argmax, st, w.ctl, w.next_tok, w.out);
    QW_CUDA(cudaEventRecord(e1, st));
    if (max_new > 1) {
        if (!c->step_graph || c->step_graph_gen != w.generation) {
            if (c->step_graph) {
                cudaGraphExecDestroy(c->step_graph);
                c->step_graph = nullptr;
            }
            cudaGraph_t g;
            QW_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            try {
                forward_dev(m, c, w.next_tok, 1, 1, false, w.argmax, st, w.ctl, w.next_tok, w.out);
            } catch (...) {
                cudaStreamEndCapture(st, &g);
                throw;
            }
            QW_CUDA(cudaStreamEndCapture(st, &g));
            QW_CUDA(cudaGraphInstantiate(&c->step_graph, g, 0));
            cudaGraphDestroy(g);
            c->step_graph_gen = w.generation;
        }
        for (int i = 1; i < max_new; ++i) QW_CUDA(cudaGraphLaunch(c->step_graph, st));
    }
    QW_CUDA(cudaEventRecord(e2, st));
    QW_CUDA(cudaStreamSynchronize(st));
    QW_CUDA(cudaMemcpy(&ctl, w.ctl, sizeof(ctl), cudaMemcpyDeviceToHost));
    float pf = 0, dc = 0;
    cudaEventElapsedTime(&pf, e0, e1);
    cudaEventElapsedTime(&dc, e1, e2);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    QW_CUDA(cudaMemcpy(&c->seq_len, c->d_seq_len, sizeof(int), cudaMemcpyDeviceToHost));
    if (stats) {
        stats->prompt_tokens = n_prompt;
        stats->completion_tokens = ctl.produced;
        stats->finish_reason = ctl.finish;
        stats->prefill_ms = pf;
        stats->decode_ms = dc;
    }
}

// Batched greedy decode (benchmark config 5 at batch 8): each sequence is
// prefilled on its own (its first token from the prompt's last row), then one
// captured batched step -- every sequence's newest token through the
// persistent kernel as one row, each row attending to its own cache -- is
// replayed max_new - 1 times.  The kernel's last CTA does the bookkeeping
// (per-sequence EOS and output lists, next ids); once every sequence has
// stopped the remaining replays do nothing.  Every row's arithmetic is the
// single-sequence decode step's, so each sequence's tokens equal its batch-1
// greedy run.
void generate_greedy_batch_dev(qw_model* m, qw_cache* const* caches, int nseq, const std::vector<std::vector<int>>& prompts,
                               int max_new, const std::vector<int>& eos, std::vector<std::vector<int>>& outs,
                               qw_gen_stats* stats, cudaStream_t st) {
    Workspace& w = m->ws;
    if (nseq < 1 || nseq > 8) throw Error(QW_ERR_INVALID_ARG, "batch of 1..8 sequences");
    if ((size_t)nseq * max_new > (size_t)w.out_cap) throw Error(QW_ERR_INVALID_ARG, "max_new too large");
    for (int b = 0; b < nseq; ++b) {
        qw_cache* c = caches[b];
        const int n = (int)prompts[b].size();
        if (n + max_new > c->max_pos)
            throw Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(n + max_new) +
                                                 " positions, max " + std::to_string(c->max_pos));
        for (int b2 = 0; b2 < b; ++b2)
            if (caches[b2] == c) throw Error(QW_ERR_INVALID_ARG, "a cache appears twice in the batch");
    }
    cudaEvent_t e0, e1, e2;
    QW_CUDA(cudaEventCreate(&e0));
    QW_CUDA(cudaEventCreate(&e1));
    QW_CUDA(cudaEventCreate(&e2));
    QW_CUDA(cudaEventRecord(e0, st));
    for (int b = 0; b < nseq; ++b) {
        qw_cache* c = caches[b];
        const int zero = 0, n = (int)prompts[b].size();
        QW_CUDA(cudaMemcpyAsync(c->d_seq_len, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
        c->seq_len = 0;
        QW_CUDA(cudaMemcpyAsync(w.ids, prompts[b].data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
        forward_dev(m, c, w.ids, n, 1, false, w.next_tok + b, st, nullptr, nullptr, nullptr);
    }
    int first[8];
    QW_CUDA(cudaMemcpyAsync(first, w.next_tok, (size_t)nseq * 4, cudaMemcpyDeviceToHost, st));
    QW_CUDA(cudaStreamSynchronize(st));
    BatchCtl bc;
    std::memset(&bc, 0, sizeof(bc));
    bc.produced = 1;
    bc.max_new = max_new;
    bc.n_eos = (int)std::min<size_t>(eos.size(), 8);
    for (int i = 0; i < bc.n_eos; ++i) bc.eos[i] = eos[i];
    bool all = true;
    for (int b = 0; b < nseq; ++b) {
        bool is_eos = false;
        for (int i = 0; i < bc.n_eos; ++i) is_eos |= bc.eos[i] == first[b];
        bc.stopped[b] = is_eos;
        if (!is_eos) {
            QW_CUDA(cudaMemcpyAsync(w.out + (size_t)b * max_new, &first[b], 4, cudaMemcpyHostToDevice, st));
            bc.n_out[b] = 1;
        }
        all &= is_eos;
    }
    bc.done = (all || max_new <= 1) ? 1 : 0;
    QW_CUDA(cudaMemcpyAsync(w.bctl, &bc, sizeof(bc), cudaMemcpyHostToDevice, st));
    QW_CUDA(cudaStreamSynchronize(st));  // the host copies above read stack memory
    QW_CUDA(cudaEventRecord(e1, st));
    if (max_new > 1 && !bc.done) {
        // sub-batches of at most mk_batch_rows sequences (shared memory holds every
        // row's staged activations), one launch each per step, sizes balanced
        const int cap = mk_batch_rows(m);
        if (cap < 1) throw Error(QW_ERR_UNSUPPORTED, "this model does not fit the batched decode step");
        const int nch = (nseq + cap - 1) / cap;
        cudaGraph_t g;
        cudaGraphExec_t ge = nullptr;
        QW_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        bool ok = true;
        try {
            for (int ci = 0, b0 = 0; ci < nch; ++ci) {
                const int nc = nseq / nch + (ci < nseq % nch ? 1 : 0);
                MkBatch mb{caches + b0, nc, w.bctl, b0, nseq, ci == nch - 1};
                ok = ok && mk_forward(m, caches[b0], w.next_tok + b0, nc, 2, false, w.argmax, st, nullptr, w.next_tok,
                                      w.out, nullptr, &mb);
                b0 += nc;
            }
        } catch (...) {
            cudaStreamEndCapture(st, &g);
            throw;
        }
        QW_CUDA(cudaStreamEndCapture(st, &g));
        if (!ok) {
            cudaGraphDestroy(g);
            throw Error(QW_ERR_UNSUPPORTED, "this model / batch does not fit the batched decode step");
        }
        QW_CUDA(cudaGraphInstantiate(&ge, g, 0));
        cudaGraphDestroy(g);
        for (int i = 1; i < max_new; ++i) QW_CUDA(cudaGraphLaunch(ge, st));
        QW_CUDA(cudaEventRecord(e2, st));
        QW_CUDA(cudaStreamSynchronize(st));
        cudaGraphExecDestroy(ge);
    } else {
        QW_CUDA(cudaEventRecord(e2, st));
        QW_CUDA(cudaStreamSynchronize(st));
    }
    QW_CUDA(cudaMemcpy(&bc, w.bctl, sizeof(bc), cudaMemcpyDeviceToHost));
    float pf = 0, dc = 0;
    cudaEventElapsedTime(&pf, e0, e1);
    cudaEventElapsedTime(&dc, e1, e2);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    outs.assign(nseq, {});
    std::vector<int> h((size_t)nseq * max_new);
    QW_CUDA(cudaMemcpy(h.data(), w.out, h.size() * 4, cudaMemcpyDeviceToHost));
    int total = 0;
    for (int b = 0; b < nseq; ++b) {
        outs[b].assign(h.begin() + (size_t)b * max_new, h.begin() + (size_t)b * max_new + bc.n_out[b]);
        total += bc.n_out[b] + (bc.stopped[b] ? 1 : 0);
        QW_CUDA(cudaMemcpy(&caches[b]->seq_len, caches[b]->d_seq_len, sizeof(int), cudaMemcpyDeviceToHost));
    }
    if (stats) {
        int np = 0;
        for (int b = 0; b < nseq; ++b) np += (int)prompts[b].size();
        stats->prompt_tokens = np;
        stats->completion_tokens = total;
        stats->finish_reason = 0;
        stats->prefill_ms = pf;
        stats->decode_ms = dc;
    }
}

}  // namespace qw

namespace qw {

// LoadedModel::generate_text with temperature > 0 (engine.rs:149-201, pick_next
// :203-263) as a device loop: prefill with the last row's logits stored, pick
// on the device, then a captured step {forward of the picked token with its
// logits stored, pick} replayed max_new - 1 times.  The pick kernel does the
// loop bookkeeping (EOS, token budget, output list); once it sets `done` the
// replays' forward steps see the gate and do nothing.
void generate_sampled_dev(qw_model* m, qw_cache* c, int n_prompt, int max_new, const std::vector<int>& eos,
                          const SampleCfg& cfg, qw_gen_stats* stats, cudaStream_t st) {
    Workspace& w = m->ws;
    if (m->vocab_l != m->cfg.vocab)
        throw Error(QW_ERR_UNSUPPORTED, "sampled generation needs the whole vocabulary on one rank (untied lm_head "
                                        "is split under tensor parallelism)");
    if (n_prompt + max_new > c->max_pos)
        throw Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(n_prompt + max_new) +
                                             " positions, max " + std::to_string(c->max_pos));
    if (max_new > w.out_cap) throw Error(QW_ERR_INVALID_ARG, "max_new too large");
    StepCtl ctl;
    std::memset(&ctl, 0, sizeof(ctl));
    ctl.max_new = max_new;
    ctl.n_eos = (int)std::min<size_t>(eos.size(), 8);
    for (int i = 0; i < ctl.n_eos; ++i) ctl.eos[i] = eos[i];
    QW_CUDA(cudaMemcpyAsync(w.ctl, &ctl, sizeof(ctl), cudaMemcpyHostToDevice, st));
    QW_CUDA(cudaMemcpyAsync(w.scfg, &cfg, sizeof(cfg), cudaMemcpyHostToDevice, st));
    int zero = 0;
    QW_CUDA(cudaMemcpyAsync(c->d_seq_len, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    c->seq_len = 0;

    SampleArgs sa;
    std::memset(&sa, 0, sizeof(sa));
    sa.logits = w.logits;
    sa.V = m->vocab_l;
    sa.cfg_dev = w.scfg;
    sa.probs = w.probs;
    sa.ctl = w.ctl;
    sa.next_tok = w.next_tok;
    sa.out = w.out;
    sa.ctrl = w.sctrl;
    sa.err = m->d_err;

    cudaEvent_t e0, e1, e2;
    QW_CUDA(cudaEventCreate(&e0));
    QW_CUDA(cudaEventCreate(&e1));
    QW_CUDA(cudaEventCreate(&e2));
    QW_CUDA(cudaEventRecord(e0, st));
    forward_dev(m, c, w.ids, n_prompt, 1, true, w.argmax, st, nullptr, nullptr, nullptr);
    QW_CUDA(launch_sample(sa, st));
    QW_CUDA(cudaEventRecord(e1, st));
    if (max_new > 1) {
        if (!c->sample_graph || c->sample_graph_gen != w.generation) {
            if (c->sample_graph) {
                cudaGraphExecDestroy(c->sample_graph);
                c->sample_graph = nullptr;
            }
            cudaGraph_t g;
            QW_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            try {
                forward_dev(m, c, w.next_tok, 1, 1, true, w.argmax, st, nullptr, nullptr, nullptr, &w.ctl->done);
                QW_CUDA(launch_sample(sa, st));
            } catch (...) {
                cudaStreamEndCapture(st, &g);
                throw;
            }
            QW_CUDA(cudaStreamEndCapture(st, &g));
            QW_CUDA(cudaGraphInstantiate(&c->sample_graph, g, 0));
            cudaGraphDestroy(g);
            c->sample_graph_gen = w.generation;
        }
        for (int i = 1; i < max_new; ++i) QW_CUDA(cudaGraphLaunch(c->sample_graph, st));
    }
    QW_CUDA(cudaEventRecord(e2, st));
    QW_CUDA(cudaStreamSynchronize(st));
    QW_CUDA(cudaMemcpy(&ctl, w.ctl, sizeof(ctl), cudaMemcpyDeviceToHost));
    float pf = 0, dc = 0;
    cudaEventElapsedTime(&pf, e0, e1);
    cudaEventElapsedTime(&dc, e1, e2);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaEventDestroy(e2);
    QW_CUDA(cudaMemcpy(&c->seq_len, c->d_seq_len, sizeof(int), cudaMemcpyDeviceToHost));
    if (stats) {
        stats->prompt_tokens = n_prompt;
        stats->completion_tokens = ctl.produced;
        stats->finish_reason = ctl.finish;
        stats->prefill_ms = pf;
        stats->decode_ms = dc;
    }
}

}  // namespace qw
