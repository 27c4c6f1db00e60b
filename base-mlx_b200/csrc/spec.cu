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
    ~SpecState() {
        for (auto g : {gD, gV, gA})
            if (g) cudaGraphExecDestroy(g);
        if (ctl) cudaFree(ctl);
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

    const bool stale = S->draft != d || S->k != r.k || S->tgen != tw.generation || S->dgen != dw.generation ||
                       S->tc != tc || S->dc != dc || !S->gD;
    if (stale) {
        for (cudaGraphExec_t* g : {&S->gD, &S->gV, &S->gA})
            if (*g) {
                cudaGraphExecDestroy(*g);
                *g = nullptr;
            }
        S->gD = capture(st, [&] {
            forward_dev(d, dc, draft_in2, 2, 1, false, dw.argmax, st, nullptr, nullptr, nullptr, gate);
            for (int j = 0; j < r.k; ++j) {
                QW_CUDA(launch1(spec_pick_kernel, st, S->ctl, (const int*)dw.argmax, (const int*)S->forced, verify_in,
                                draft_in));
                if (j + 1 < r.k)
                    forward_dev(d, dc, draft_in, 1, 1, false, dw.argmax, st, nullptr, nullptr, nullptr, gate);
            }
        });
        S->gV = capture(st, [&] {
            forward_dev(t, tc, verify_in, r.k + 1, 2, false, tw.argmax, st, nullptr, nullptr, nullptr, gate);
        });
        S->gA = capture(st, [&] {
            QW_CUDA(launch1(spec_accept_kernel, st, S->ctl, (const int*)tw.argmax, verify_in, draft_in2, tw.out,
                            tc->d_seq_len, dc->d_seq_len, (volatile int*)flag));
        });
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
    h.force_p = r.force_p;
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
    forward_dev(t, tc, tw.ids, r.n_prompt, 1, false, tw.argmax, st, nullptr, nullptr, nullptr, nullptr);
    forward_dev(d, dc, dw.ids, r.n_prompt, 0, false, dw.argmax, st, nullptr, nullptr, nullptr, nullptr);
    QW_CUDA(launch1(spec_init_kernel, st, S->ctl, (const int*)tw.argmax, verify_in, draft_in2, (const int*)dw.ids,
                    dc->d_seq_len, tw.out, (volatile int*)flag));
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
