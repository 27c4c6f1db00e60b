// Greedy speculative decoding with the accept / rollback step on the device.
//
// Restates crates/base-mlx-core/src/speculative.rs:57-240 (speculative::generate):
//   prefill target and draft on the prompt; leader = target argmax of the last row;
//   per iteration: the draft proposes k tokens (one draft forward per token,
//   stopping the count at a drafted EOS), the target verifies [leader, d1..dk]
//   in one (k+1)-row forward, the longest prefix with draft == target argmax is
//   accepted, the target's token at the first disagreement (or after the last
//   draft) is the bonus, both caches are rewound to prompt + emitted - 1 and the
//   bonus is fed to the draft.
//
// B200 structure: the per-iteration work is three captured CUDA graphs
// (draft: one 2-row draft forward of [token before the leader, leader], then
// k picks with a 1-row draft forward between consecutive picks; verify: target
// forward of k+1 rows; accept: the accept kernel) replayed back to back.  The
// k-th drafted token is never run through the draft here: its KV row, needed
// only when all k are accepted, is the first row of the next iteration's
// 2-row forward, which otherwise rewrites the last kept position with the
// same token (a row's results do not depend on the row count, so the rewrite
// is bit-identical).  k draft forwards per iteration instead of k + 1.
// The accept kernel compares, emits, updates the statistics and rewinds both
// device-side cache lengths, so the host never waits on a token: it only
// polls a mapped "done" flag two iterations behind the GPU.
//
// Rows past a drafted EOS are still verified (their results are ignored and
// their KV slots are rolled back); causal attention makes the first n+1 rows
// identical to a verify of exactly n+1 rows, so results match the reference.
#include <algorithm>
#include <cstring>
#include <functional>

#include "model.h"

namespace qw {

struct SpecCtl {
    int emitted;   // tokens emitted (the leader included)
    int done;
    int finish;    // 0 length, 1 stop
    int iters, proposed, accepted;
    int slot;      // next draft slot of this iteration
    int n_eff;     // drafts counted this iteration (up to and including a drafted EOS)
    int max_new, k, plen;
    float force_p;
    unsigned long long seed;
    int n_forced;
    int n_eos_t, n_eos_d;
    int eos_t[8], eos_d[8];
};

namespace {

QW_DEV bool in_list(const int* l, int n, int t) {
    bool r = false;
    for (int i = 0; i < n; ++i) r |= (l[i] == t);
    return r;
}

// After the prefill: leader = target argmax of the last prompt row; the
// draft's first input pair is (last prompt token, leader) at positions plen-1, plen.
__global__ void spec_init_kernel(SpecCtl* c, const int* t_argmax, int* verify_in, int* draft_in2,
                                 const int* prompt, int* d_seq, int* out, volatile int* host_flag) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    const int leader = t_argmax[0];
    if (in_list(c->eos_t, c->n_eos_t, leader)) {
        c->done = 1;
        c->finish = 1;
    } else {
        out[0] = leader;
        c->emitted = 1;
        if (c->emitted >= c->max_new) c->done = 1;
    }
    verify_in[0] = leader;
    draft_in2[0] = prompt[c->plen - 1];
    draft_in2[1] = leader;
    *d_seq = c->plen - 1;
    c->slot = 0;
    c->n_eff = c->k;
    host_flag[0] = c->done;
    host_flag[1] = c->emitted;
}

// Draft token for the current slot (speculative.rs:125-137) plus the seeded
// forced-acceptance hook of the benchmark.
__global__ void spec_pick_kernel(SpecCtl* c, const int* d_argmax, const int* forced, int* verify_in, int* draft_in) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0 || c->done) return;
    const int slot = c->slot;
    int d = d_argmax[0];
    if (c->force_p > 0.f && forced) {
        const int pos = c->emitted + slot;
        if (pos < c->n_forced) {
            const uint64_t h = splitmix64(c->seed ^ splitmix64((uint64_t)c->iters * 64ull + (uint64_t)slot));
            const float u = (float)(h >> 40) * (1.0f / 16777216.0f);
            if (u < c->force_p) d = forced[pos];
        }
    }
    verify_in[1 + slot] = d;
    *draft_in = d;
    if (slot < c->n_eff && in_list(c->eos_d, c->n_eos_d, d)) c->n_eff = slot + 1;
    c->slot = slot + 1;
}

// speculative.rs:153-239: accept, emit, roll back both caches, set up the next leader.
__global__ void spec_accept_kernel(SpecCtl* c, const int* preds, int* verify_in, int* draft_in2, int* out,
                                   int* t_seq, int* d_seq, volatile int* host_flag) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    if (!c->done) {
        const int n = c->n_eff;
        int n_acc = 0;
        while (n_acc < n && preds[n_acc] == verify_in[1 + n_acc]) ++n_acc;
        const int bonus = preds[n_acc];
        c->proposed += n;
        c->iters += 1;
        c->accepted += n_acc;
        bool stop = false;
        for (int i = 0; i < n_acc && !stop; ++i) {
            const int t = verify_in[1 + i];
            if (c->emitted >= c->max_new) {
                stop = true;
            } else if (in_list(c->eos_t, c->n_eos_t, t)) {
                c->finish = 1;
                stop = true;
            } else {
                out[c->emitted++] = t;
            }
        }
        if (!stop && c->emitted >= c->max_new) stop = true;
        if (!stop && in_list(c->eos_t, c->n_eos_t, bonus)) {
            c->finish = 1;
            stop = true;
        }
        if (stop) {
            c->done = 1;
        } else {
            out[c->emitted++] = bonus;
            const int keep = c->plen + c->emitted - 1;  // the bonus's position
            *t_seq = keep;
            // the draft restarts one position earlier: its next 2-row forward
            // (re)computes the last kept token and runs the bonus
            *d_seq = keep - 1;
            draft_in2[0] = verify_in[n_acc];  // d_{n_acc}, or the old leader when none was accepted
            draft_in2[1] = bonus;
            verify_in[0] = bonus;
            c->slot = 0;
            c->n_eff = c->k;
            if (c->emitted >= c->max_new) c->done = 1;
        }
    }
    host_flag[0] = c->done;
    host_flag[1] = c->emitted;
}

// ---- speculative sampling (temperature > 0) -----------------------------------
// The reference falls back to plain sampled decoding for temperature > 0
// (speculative.rs:65-69; rejection sampling is the missing piece it names).
// This is the speculative-sampling rule over the sampled pick's distributions
// (engine.rs:203-263: softmax of logits / t, top-p nucleus): the drafted token
// d_i ~ Q_i (the draft's pick) is accepted with probability min(1, P_i(d_i) /
// Q_i(d_i)), i.e. when u * Q < P with u = draw(iteration, 16 + i); at the
// first rejection the emitted token is drawn from max(0, P_i - Q_i), after k
// acceptances from P_k (draw(iteration, 32)), so every emitted token follows
// the target's distribution.  Those draws walk the row in index order with
// exact 2^-60 fixed-point masses (the sums do not depend on the order of the
// partial sums).
constexpr int SS_NT = 1024;

QW_DEV uint32_t draw24(unsigned long long seed, unsigned long long counter) {
    return (uint32_t)(splitmix64(seed ^ splitmix64(counter)) >> 40);
}
// P(x) of a nucleus-truncated, renormalised row
QW_DEV float nucleus_p(const float* p, const SpDesc& d, int x) {
    const float v = p[x];
    const float kv = __uint_as_float(d.key);
    const bool in = !d.found || v > kv || (v == kv && x <= d.tie_idx);
    return in ? __fdiv_rn(v, d.renorm) : 0.f;
}
QW_DEV unsigned long long fx60(float v) {
    return v <= 0.f ? 0ull : __double2ull_rn((double)v * 1152921504606846976.0);
}

// Accept / residual draw / emit / roll back (one CTA).  pt: the target's k + 1
// softmax rows and nuclei (rows of the verify), pd / dd: the draft's k rows.
__global__ void __launch_bounds__(SS_NT, 1) spec_sampled_accept_kernel(SpecCtl* c, const float* pt, const SpDesc* dt,
                                                                        const float* pd, const SpDesc* dd, int V,
                                                                        int* verify_in, int* draft_in2, int* out,
                                                                        int* t_seq, int* d_seq,
                                                                        volatile int* host_flag) {
    __shared__ int s_nacc, s_mode, s_tok;
    __shared__ unsigned long long s_scan[SS_NT / 32];
    __shared__ unsigned long long s_R;
    pdl_wait();
    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (c->done) {  // the same value in every thread
        if (tid == 0) {
            host_flag[0] = c->done;
            host_flag[1] = c->emitted;
        }
        return;
    }
    const unsigned long long it64 = (unsigned long long)c->iters * 64ull;
    if (tid == 0) {
        const int n = c->n_eff;
        int n_acc = 0;
        while (n_acc < n) {
            const int d = verify_in[1 + n_acc];
            const float P = nucleus_p(pt + (size_t)n_acc * V, dt[n_acc], d);
            const float Q = nucleus_p(pd + (size_t)n_acc * V, dd[n_acc], d);
            const float u = (float)draw24(c->seed, it64 + 16ull + (unsigned long long)n_acc) * (1.0f / 16777216.0f);
            if (__fmul_rn(u, Q) < P)
                ++n_acc;
            else
                break;
        }
        s_nacc = n_acc;
        s_mode = n_acc < n ? 0 : 1;  // 0: residual of row n_acc, 1: the target's row n_acc
        s_tok = -1;
    }
    __syncthreads();
    const int row = s_nacc;
    const uint32_t U = draw24(c->seed, it64 + 32ull);
    const int chunk = (V + SS_NT - 1) / SS_NT;
    const int x0 = min(V, tid * chunk), x1 = min(V, x0 + chunk);
    const float* P = pt + (size_t)row * V;
    const SpDesc dP = dt[row];
    for (int attempt = 0; attempt < 2; ++attempt) {
        const int mode = s_mode;
        const bool resid = mode == 0;
        const float* Q = pd + (size_t)(resid ? row : 0) * V;
        const SpDesc dQ = dd[resid ? row : 0];
        auto w = [&](int x) -> unsigned long long {
            const float pv = nucleus_p(P, dP, x);
            return resid ? fx60(fmaxf(__fsub_rn(pv, nucleus_p(Q, dQ, x)), 0.f)) : fx60(pv);
        };
        unsigned long long sum = 0ull;
        for (int x = x0; x < x1; ++x) sum += w(x);
        unsigned long long inc = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) s_scan[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            unsigned long long v = s_scan[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            s_scan[lane] = v;
            if (lane == 31) s_R = v;
        }
        __syncthreads();
        const unsigned long long R = s_R;
        if (R == 0ull) {
            // no residual mass (the rows agree to rounding): draw from the target row
            __syncthreads();
            if (tid == 0) s_mode = 1;
            __syncthreads();
            if (!resid) break;
            continue;
        }
        const unsigned long long tgt = (R >> 24) * U + (((R & 0xFFFFFFull) * U) >> 24);  // floor(R U / 2^24) < R
        const unsigned long long excl = (warp > 0 ? s_scan[warp - 1] : 0ull) + inc - sum;
        if (sum > 0ull && excl <= tgt && tgt < excl + sum) {
            unsigned long long acc = excl;
            for (int x = x0; x < x1; ++x) {
                acc += w(x);
                if (acc > tgt) {
                    s_tok = x;
                    break;
                }
            }
        }
        __syncthreads();
        break;
    }
    if (tid != 0) return;
    const int n = c->n_eff, n_acc = s_nacc;
    const int bonus = s_tok < 0 ? 0 : s_tok;
    c->proposed += n;
    c->iters += 1;
    c->accepted += n_acc;
    bool stop = false;
    for (int i = 0; i < n_acc && !stop; ++i) {
        const int t = verify_in[1 + i];
        if (c->emitted >= c->max_new) {
            stop = true;
        } else if (in_list(c->eos_t, c->n_eos_t, t)) {
            c->finish = 1;
            stop = true;
        } else {
            out[c->emitted++] = t;
        }
    }
    if (!stop && c->emitted >= c->max_new) stop = true;
    if (!stop && in_list(c->eos_t, c->n_eos_t, bonus)) {
        c->finish = 1;
        stop = true;
    }
    if (stop) {
        c->done = 1;
    } else {
        out[c->emitted++] = bonus;
        const int keep = c->plen + c->emitted - 1;
        *t_seq = keep;
        *d_seq = keep - 1;
        draft_in2[0] = verify_in[n_acc];
        draft_in2[1] = bonus;
        verify_in[0] = bonus;
        c->slot = 0;
        c->n_eff = c->k;
        if (c->emitted >= c->max_new) c->done = 1;
    }
    host_flag[0] = c->done;
    host_flag[1] = c->emitted;
}

template <typename K, typename... Args>
cudaError_t launch1(K kernel, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// launch1 with a whole-CTA block (the speculative-sampling accept kernel)
template <typename K, typename... Args>
cudaError_t launch_cta(K kernel, int threads, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(threads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

struct SpecState {
    qw_model* draft = nullptr;
    int k = 0, tgen = -1, dgen = -1;
    qw_cache *tc = nullptr, *dc = nullptr;
    cudaGraphExec_t gD = nullptr, gV = nullptr, gA = nullptr;
    SpecCtl* ctl = nullptr;
    int* forced = nullptr;
    int forced_cap = 0;
    int* host_flag = nullptr;  // mapped pinned [done, emitted]
    std::vector<cudaEvent_t> ev;
    // speculative sampling: the draft's k and the target's k + 1 softmax rows,
    // their nuclei (draft first), the draft pick's token; the captured parameters
    bool sampled = false;
    float temperature = 0.f, top_p = 1.f;
    uint64_t seed = 0;
    float* probs = nullptr;
    SpDesc* desc = nullptr;
    int* stok = nullptr;
    size_t probs_cap = 0;
    ~SpecState() {
        for (auto g : {gD, gV, gA})
            if (g) cudaGraphExecDestroy(g);
        if (ctl) cudaFree(ctl);
        if (probs) cudaFree(probs);
        if (desc) cudaFree(desc);
        if (stok) cudaFree(stok);
        if (forced) cudaFree(forced);
        if (host_flag) cudaFreeHost(host_flag);
        for (auto e : ev) cudaEventDestroy(e);
    }
};

cudaGraphExec_t capture(cudaStream_t st, const std::function<void()>& body) {
    cudaGraph_t g;
    QW_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    try {
        body();
    } catch (...) {
        cudaStreamEndCapture(st, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    QW_CUDA(cudaStreamEndCapture(st, &g));
    cudaGraphExec_t ex;
    QW_CUDA(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    return ex;
}

}  // namespace

void spec_state_free(void* p) { delete static_cast<SpecState*>(p); }

void spec_generate_dev(qw_model* t, qw_model* d, const SpecRequest& r, std::vector<int>& out_tokens,
                       qw_spec_stats* stats) {
    if (t == d) throw Error(QW_ERR_INVALID_ARG, "target and draft must be distinct model handles");
    if (t->device != d->device) throw Error(QW_ERR_INVALID_ARG, "target and draft must be on the same device");
    if (r.k < 1 || r.k > 7) throw Error(QW_ERR_INVALID_ARG, "k must be in [1, 7]");
    if (r.n_prompt < 1) throw Error(QW_ERR_INVALID_ARG, "empty prompt");
    const int max_new = std::max(r.max_new, 1);
    const int need = r.n_prompt + max_new + r.k + 2;
    qw_cache* tc = cache_for_generate(t, need);
    qw_cache* dc = cache_for_generate(d, need);
    if (need > tc->max_pos || need > dc->max_pos)
        throw Error(QW_ERR_KV_EXHAUSTED, "KV cache exhausted: requested " + std::to_string(need) + " positions");
    ensure_workspace(t, std::max(r.n_prompt, r.k + 1), r.k + 1);
    ensure_workspace(d, r.n_prompt, 8);
    if (max_new > t->ws.out_cap) throw Error(QW_ERR_INVALID_ARG, "max_new too large");
    cudaStream_t st = t->stream;
    // the draft runs on the target's stream; make sure its own stream is idle
    QW_CUDA(cudaStreamSynchronize(d->stream));

    auto* S = static_cast<SpecState*>(t->spec_state);
    if (!S) {
        S = new SpecState();
        t->spec_state = S;
        QW_CUDA(cudaMalloc(&S->ctl, sizeof(SpecCtl)));
        QW_CUDA(cudaHostAlloc(&S->host_flag, 64, cudaHostAllocMapped));
    }
    if (r.n_forced > S->forced_cap) {
        if (S->forced) cudaFree(S->forced);
        S->forced = nullptr;
        S->forced_cap = std::max(r.n_forced, 1024);
        QW_CUDA(cudaMalloc(&S->forced, (size_t)S->forced_cap * 4));
    }
    Workspace& tw = t->ws;
    Workspace& dw = d->ws;
    int* verify_in = tw.ids;
    int* draft_in2 = dw.next_tok;     // [2]: the 2-row draft input of an iteration
    int* draft_in = dw.next_tok + 2;  // the 1-row draft input after each pick
    int* flag = S->host_flag;
    const int* gate = &S->ctl->done;

    const bool sampled = r.temperature > 0.f;
    const int V = t->vocab_l;
    if (sampled) {
        if (t->vocab_l != t->cfg.vocab || d->vocab_l != V)
            throw Error(QW_ERR_UNSUPPORTED, "speculative sampling needs the whole vocabulary on one rank for target and draft");
        ensure_workspace(d, r.n_prompt, 8);
        const size_t need_p = (size_t)(2 * r.k + 1) * V;
        if (S->probs_cap < need_p) {
            if (S->probs) cudaFree(S->probs);
            if (S->desc) cudaFree(S->desc);
            S->probs = nullptr;
            S->desc = nullptr;
            QW_CUDA(cudaMalloc(&S->probs, need_p * sizeof(float)));
            QW_CUDA(cudaMalloc(&S->desc, (size_t)(2 * 8 + 1) * sizeof(SpDesc)));
            S->probs_cap = need_p;
        }
        if (!S->stok) QW_CUDA(cudaMalloc(&S->stok, 64));
    }
    const bool stale = S->draft != d || S->k != r.k || S->tgen != tw.generation || S->dgen != dw.generation ||
                       S->tc != tc || S->dc != dc || !S->gD || S->sampled != sampled ||
                       (sampled && (S->temperature != r.temperature || S->top_p != r.top_p || S->seed != r.seed));
    if (stale) {
        for (cudaGraphExec_t* g : {&S->gD, &S->gV, &S->gA})
            if (*g) {
                cudaGraphExecDestroy(*g);
                *g = nullptr;
            }
        float* probs_d = S->probs;                      // [k][V]
        float* probs_t = S->probs + (size_t)r.k * V;  // [k + 1][V]
        SpDesc* desc_d = S->desc;
        SpDesc* desc_t = S->desc + 8;
        // one row's softmax and nucleus (and, for the draft, the pick) on the shared control block
        auto sample_row = [&](const bf16* logits, float* probs, SpDesc* desc, int ctr_base, bool draw) {
            SampleArgs sa;
            std::memset(&sa, 0, sizeof(sa));
            sa.logits = logits;
            sa.V = V;
            sa.cfg.temperature = r.temperature;
            sa.cfg.top_p = r.top_p;
            sa.cfg.seed = r.seed;
            sa.probs = probs;
            sa.token_out = S->stok;
            sa.ctrl = dw.sctrl;
            sa.err = t->d_err;
            sa.ctr_iter = &S->ctl->iters;
            sa.ctr_base = ctr_base;
            sa.desc_out = desc;
            sa.no_draw = draw ? 0 : 1;
            sa.gate = gate;
            QW_CUDA(launch_sample(sa, st));
        };
        S->gD = capture(st, [&] {
            forward_dev(d, dc, draft_in2, 2, 1, sampled, dw.argmax, st, nullptr, nullptr, nullptr, gate);
            for (int j = 0; j < r.k; ++j) {
                if (sampled) sample_row(dw.logits, probs_d + (size_t)j * V, desc_d + j, j, true);
                QW_CUDA(launch1(spec_pick_kernel, st, S->ctl, sampled ? (const int*)S->stok : (const int*)dw.argmax,
                                (const int*)S->forced, verify_in, draft_in));
                if (j + 1 < r.k)
                    forward_dev(d, dc, draft_in, 1, 1, sampled, dw.argmax, st, nullptr, nullptr, nullptr, gate);
            }
        });
        S->gV = capture(st, [&] {
            forward_dev(t, tc, verify_in, r.k + 1, 2, sampled, tw.argmax, st, nullptr, nullptr, nullptr, gate);
            if (sampled)
                for (int j = 0; j <= r.k; ++j)
                    sample_row(tw.logits + (size_t)j * V, probs_t + (size_t)j * V, desc_t + j, 0, false);
        });
        S->gA = capture(st, [&] {
            if (sampled)
                QW_CUDA(launch_cta(spec_sampled_accept_kernel, SS_NT, st, S->ctl, (const float*)probs_t,
                                   (const SpDesc*)desc_t, (const float*)probs_d, (const SpDesc*)desc_d, V, verify_in,
                                   draft_in2, tw.out, tc->d_seq_len, dc->d_seq_len, (volatile int*)flag));
            else
                QW_CUDA(launch1(spec_accept_kernel, st, S->ctl, (const int*)tw.argmax, verify_in, draft_in2, tw.out,
                                tc->d_seq_len, dc->d_seq_len, (volatile int*)flag));
        });
        S->sampled = sampled;
        S->temperature = r.temperature;
        S->top_p = r.top_p;
        S->seed = r.seed;
        S->draft = d;
        S->k = r.k;
        S->tgen = tw.generation;
        S->dgen = dw.generation;
        S->tc = tc;
        S->dc = dc;
    }

    SpecCtl h;
    std::memset(&h, 0, sizeof(h));
    h.max_new = max_new;
    h.k = r.k;
    h.plen = r.n_prompt;
    h.force_p = sampled ? 0.f : r.force_p;
    h.seed = r.seed;
    h.n_forced = r.forced ? r.n_forced : 0;
    h.n_eos_t = (int)std::min<size_t>(r.eos_target.size(), 8);
    h.n_eos_d = (int)std::min<size_t>(r.eos_draft.size(), 8);
    for (int i = 0; i < h.n_eos_t; ++i) h.eos_t[i] = r.eos_target[i];
    for (int i = 0; i < h.n_eos_d; ++i) h.eos_d[i] = r.eos_draft[i];
    h.n_eff = r.k;
    flag[0] = 0;
    flag[1] = 0;
    QW_CUDA(cudaMemcpyAsync(S->ctl, &h, sizeof(h), cudaMemcpyHostToDevice, st));
    if (h.n_forced) QW_CUDA(cudaMemcpyAsync(S->forced, r.forced, (size_t)h.n_forced * 4, cudaMemcpyHostToDevice, st));
    QW_CUDA(cudaMemcpyAsync(tw.ids, r.prompt, (size_t)r.n_prompt * 4, cudaMemcpyHostToDevice, st));
    QW_CUDA(cudaMemcpyAsync(dw.ids, r.prompt, (size_t)r.n_prompt * 4, cudaMemcpyHostToDevice, st));
    const int zero = 0;
    QW_CUDA(cudaMemcpyAsync(tc->d_seq_len, &zero, 4, cudaMemcpyHostToDevice, st));
    QW_CUDA(cudaMemcpyAsync(dc->d_seq_len, &zero, 4, cudaMemcpyHostToDevice, st));
    tc->seq_len = dc->seq_len = 0;

    const int max_iters = max_new + 1;
    const size_t nev = 2 + 3 * (size_t)max_iters;
    while (S->ev.size() < nev) {
        cudaEvent_t e;
        QW_CUDA(cudaEventCreate(&e));
        S->ev.push_back(e);
    }
    // prefill: target (last-row logits -> leader), draft (no logits needed)
    QW_CUDA(cudaEventRecord(S->ev[0], st));
    forward_dev(t, tc, tw.ids, r.n_prompt, 1, sampled, tw.argmax, st, nullptr, nullptr, nullptr, nullptr);
    // the draft prefills all but the last prompt token: the first iteration's 2-row
    // draft step runs that token (as every later iteration's 2-row step reruns the
    // last kept token), so each draft KV row after the prompt's first n - 1 comes
    // from the decode step's arithmetic
    if (r.n_prompt > 1)
        forward_dev(d, dc, dw.ids, r.n_prompt - 1, 0, false, dw.argmax, st, nullptr, nullptr, nullptr, nullptr);
    if (sampled) {
        // the first token is drawn from the target's distribution after the prompt (draw counter 2^40)
        SampleArgs sa;
        std::memset(&sa, 0, sizeof(sa));
        sa.logits = tw.logits;
        sa.V = V;
        sa.cfg.temperature = r.temperature;
        sa.cfg.top_p = r.top_p;
        sa.cfg.seed = r.seed;
        sa.probs = S->probs;
        sa.token_out = S->stok;
        sa.ctrl = dw.sctrl;
        sa.err = t->d_err;
        sa.counter = 1ull << 40;
        QW_CUDA(launch_sample(sa, st));
    }
    QW_CUDA(launch1(spec_init_kernel, st, S->ctl, sampled ? (const int*)S->stok : (const int*)tw.argmax, verify_in,
                    draft_in2, (const int*)dw.ids, dc->d_seq_len, tw.out, (volatile int*)flag));
    QW_CUDA(cudaEventRecord(S->ev[1], st));

    int launched = 0;
    for (int it = 0; it < max_iters; ++it) {
        if (it >= 2) {
            QW_CUDA(cudaEventSynchronize(S->ev[2 + 3 * (it - 2) + 2]));
            if (flag[0]) break;
        } else if (it == 1) {
            QW_CUDA(cudaEventSynchronize(S->ev[1]));
            if (flag[0]) break;
        }
        QW_CUDA(cudaGraphLaunch(S->gD, st));
        QW_CUDA(cudaEventRecord(S->ev[2 + 3 * it], st));
        QW_CUDA(cudaGraphLaunch(S->gV, st));
        QW_CUDA(cudaEventRecord(S->ev[2 + 3 * it + 1], st));
        QW_CUDA(cudaGraphLaunch(S->gA, st));
        QW_CUDA(cudaEventRecord(S->ev[2 + 3 * it + 2], st));
        ++launched;
    }
    QW_CUDA(cudaStreamSynchronize(st));
    if (!flag[0]) throw Error(QW_ERR_INFERENCE, "speculative loop did not finish within max_new iterations");
    SpecCtl res;
    QW_CUDA(cudaMemcpy(&res, S->ctl, sizeof(res), cudaMemcpyDeviceToHost));
    out_tokens.resize(res.emitted);
    if (res.emitted) QW_CUDA(cudaMemcpy(out_tokens.data(), tw.out, (size_t)res.emitted * 4, cudaMemcpyDeviceToHost));
    if (stats) {
        float pf = 0, tot = 0;
        cudaEventElapsedTime(&pf, S->ev[0], S->ev[1]);
        double dsum = 0, vsum = 0, asum = 0;
        int counted = 0;
        const cudaEvent_t* E = S->ev.data();
        for (int it = 0; it < launched && it < res.iters; ++it) {
            const cudaEvent_t prev = it == 0 ? E[1] : E[2 + 3 * (it - 1) + 2];
            float a = 0, b = 0, c = 0;
            cudaEventElapsedTime(&a, prev, E[2 + 3 * it]);
            cudaEventElapsedTime(&b, E[2 + 3 * it], E[2 + 3 * it + 1]);
            cudaEventElapsedTime(&c, E[2 + 3 * it + 1], E[2 + 3 * it + 2]);
            dsum += a;
            vsum += b;
            asum += c;
            ++counted;
        }
        const int last = launched > 0 ? 2 + 3 * (launched - 1) + 2 : 1;
        cudaEventElapsedTime(&tot, S->ev[0], S->ev[last]);
        stats->iters = res.iters;
        stats->proposed = res.proposed;
        stats->accepted = res.accepted;
        stats->completion_tokens = res.emitted;
        stats->finish_reason = res.finish;
        stats->prefill_ms = pf;
        stats->total_ms = tot;
        stats->draft_ms_mean = counted ? dsum / counted : 0;
        stats->verify_ms_mean = counted ? vsum / counted : 0;
        stats->accept_ms_mean = counted ? asum / counted : 0;
    }
    set_cache_len(tc, 0);  // target_cache.reset() / draft_cache.reset() (speculative.rs:276-277)
    set_cache_len(dc, 0);
    check_device_err(t);
    check_device_err(d);
}

}  // namespace qw
