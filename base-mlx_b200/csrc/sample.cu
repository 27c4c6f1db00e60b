// Temperature + top-p sampling on the device: the non-greedy branch of
// LoadedModel::pick_next (crates/base-mlx-core/src/engine.rs:203-263), which
// the reference runs on the host after copying the logits out of MLX.
//
// Same distribution, step by step:
//   p = softmax(logits / max(t, 1e-5))                         (engine.rs:212-227)
//   nucleus = the shortest prefix, in descending p with ties by lower index
//             (a stable sort), whose cumulative mass reaches top_p      (:228-240)
//   r = u * sum(nucleus); the first nucleus token whose cumulative mass
//   reaches r                                                   (:241-262)
// The uniform u comes from a counter-based generator shared with the oracle
// (splitmix64 of seed and counter) instead of rand's StdRng.
//
// No sort: both "first rank whose cumulative mass reaches T" questions are
// weighted radix selections over the bit patterns of p (non-negative floats
// order like their bits): four passes of 8-bit digits build per-digit mass
// histograms among the elements that match the digits chosen so far, walking
// digits from the top until the mass reaches the target; ties at the final
// value are then taken in index order with a scan.  Masses are exact integers
// in units of 2^-60 (u64 atomics of per-thread runs): sums do not depend on the
// order of the atomics, so every CTA walks the same histogram to the same
// digit and the picks are deterministic.
//
// Grid: SG_CTAS cooperative CTAs of SG_NT threads (a row of 151,936 entries is
// ~5 per thread per pass).  Passes are separated by a grid barrier on a
// counter in the control block (one red.release per CTA, one acquire poller,
// 2 s bound -> QW_DERR_TIMEOUT); per-CTA partials and the digit histograms
// live in the same block, the histograms in three buffers used round robin
// so that clearing one never races with filling or reading another.
#include "kernels.h"

namespace qw {
namespace {

constexpr int SG_CTAS = 64;
constexpr int SG_NT = 512;
constexpr int SG_NW = SG_NT / 32;
constexpr int SG_HC = 4;  // shared histogram copies (warps w and w + 4k share one)
constexpr unsigned long long SG_TIMEOUT_NS = 2000000000ull;

typedef unsigned long long u64;
constexpr double SP_FX = 1152921504606846976.0;  // 2^60: mass units per unit probability

// Control block of the sampling scratch.  All zero before the first launch;
// every launch leaves `bar` and `exit` at zero again.
struct SpGlobal {
    unsigned bar;   // grid-barrier arrivals of this launch
    unsigned exit;  // CTAs done with this launch
    int token;
    int pad;
    u64 hmass[3][256];
    int hcnt[3][256];
    float pmax[SG_CTAS];
    double psum[SG_CTAS];
    u64 ptot[SG_CTAS];
    int ccnt[SG_CTAS];
};
static_assert(sizeof(SpGlobal) <= QW_SAMPLE_CTRL_BYTES, "sampling control block");

struct SpShared {
    u64 hmass[SG_HC][256];
    int hcnt[SG_HC][256];
    u64 gmass[256];  // the grid's histogram of the current pass, staged for the walk
    int gcnt[256];
    u64 gpart[SG_CTAS];  // per-CTA partials, staged
    int gcntc[SG_CTAS];
    double dred[SG_NW];
    float fred[SG_NW];
    u64 ured[SG_NW];
    int iscan[SG_NW];
    uint32_t key;
    u64 above;
    int n_need;
    int found;
};

QW_DEV u64 to_fx(double v) { return v <= 0.0 ? 0ull : (v >= 8.0 ? (8ull << 60) : __double2ull_rn(v * SP_FX)); }

QW_DEV float sample_u(unsigned long long seed, unsigned long long counter) {
    return (float)(splitmix64(seed ^ splitmix64(counter)) >> 40) * (1.0f / 16777216.0f);
}

QW_DEV unsigned sp_ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
QW_DEV void sp_red_release(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
QW_DEV unsigned long long sp_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid barrier: the block's writes (ordered by the block barrier, published by
// the cumulative release) are visible to every thread after it returns.
QW_DEV void grid_sync(SpGlobal* g, unsigned& target, int* err) {
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) {
        sp_red_release(&g->bar, 1u);
        const unsigned long long t0 = sp_clock();
        while ((int)(sp_ld_acquire(&g->bar) - target) < 0) {
            if (sp_clock() - t0 > SG_TIMEOUT_NS) {
                if (err) atomicOr(err, QW_DERR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

QW_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
QW_DEV u64 warp_sum_u64(u64 v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Fixed-order block reductions; the result is valid in thread 0.
QW_DEV double block_sum_d(double v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_d(v);
    if (lane == 0) s.dred[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < SG_NW; ++w) t += s.dred[w];
    __syncthreads();
    return t;
}
QW_DEV u64 block_sum_u64(u64 v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_u64(v);
    if (lane == 0) s.ured[warp] = v;
    __syncthreads();
    u64 t = 0ull;
    if (threadIdx.x == 0)
        for (int w = 0; w < SG_NW; ++w) t += s.ured[w];
    __syncthreads();
    return t;
}
QW_DEV float block_max_f(float v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) s.fred[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    if (threadIdx.x == 0)
        for (int w = 0; w < SG_NW; ++w) t = fmaxf(t, s.fred[w]);
    __syncthreads();
    return t;
}

// Maximum of the per-CTA partials (after a grid barrier), staged through shared memory.
QW_DEV float grid_max(SpGlobal* g, SpShared& s) {
    if (threadIdx.x < gridDim.x) s.gpart[threadIdx.x] = (u64)__float_as_uint(__ldcg(&g->pmax[threadIdx.x]));
    __syncthreads();
    float m = -INFINITY;
    for (int b = 0; b < (int)gridDim.x; ++b) m = fmaxf(m, __uint_as_float((uint32_t)s.gpart[b]));
    __syncthreads();
    return m;
}

// f(i, x) over this thread's share of a row, grid-strided in 16-byte vectors,
// several loads in flight per thread.  The probability and logit walks map
// element i to the same thread (8 KB of probabilities per CTA per stride is
// 4 K entries, the logit walk's 8 entries per thread x 512 threads), so a
// thread can read back what it wrote in an earlier walk.
template <typename F>
QW_DEV void for_each_prob(const float* p, int V, F f) {
    constexpr int U = 2;
    const int V8 = V & ~7;
    const int gt = gridDim.x * SG_NT;
    for (int base = (blockIdx.x * SG_NT + threadIdx.x) * 8; base < V8; base += gt * 8 * U) {
        float4 v[2 * U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * gt * 8;
            v[2 * u] = j < V8 ? __ldcg(reinterpret_cast<const float4*>(p + j)) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[2 * u + 1] = j < V8 ? __ldcg(reinterpret_cast<const float4*>(p + j + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * gt * 8;
            if (j < V8) {
                f(j, v[2 * u].x);
                f(j + 1, v[2 * u].y);
                f(j + 2, v[2 * u].z);
                f(j + 3, v[2 * u].w);
                f(j + 4, v[2 * u + 1].x);
                f(j + 5, v[2 * u + 1].y);
                f(j + 6, v[2 * u + 1].z);
                f(j + 7, v[2 * u + 1].w);
            }
        }
    }
    for (int j = V8 + blockIdx.x * SG_NT + (int)threadIdx.x; j < V; j += gt) f(j, __ldcg(p + j));
}
template <typename F>
QW_DEV void for_each_logit(const bf16* l, int V, F f) {
    constexpr int U = 2;
    const int V8 = V & ~7;
    const int gt = gridDim.x * SG_NT;
    for (int base = (blockIdx.x * SG_NT + threadIdx.x) * 8; base < V8; base += gt * 8 * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * gt * 8;
            v[u] = j < V8 ? __ldcg(reinterpret_cast<const uint4*>(l + j)) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * gt * 8;
            if (j < V8) {
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    f(j + 2 * e, bits_lo_f(w[e]));
                    f(j + 2 * e + 1, bits_hi_f(w[e]));
                }
            }
        }
    }
    for (int j = V8 + blockIdx.x * SG_NT + (int)threadIdx.x; j < V; j += gt) f(j, bf2f(l[j]));
}

// The value v (as float bits) at which the descending cumulative mass of p
// first reaches T (2^-60 units): mass(p > v) < T <= mass(p >= v); s.n_need =
// how many of the elements equal to v, in index order, that takes.  s.found =
// 0 when the whole mass stays below T.  Only digits holding an element are
// chosen, so T = 0 selects the maximum.  `pass` numbers the grid's histogram
// passes (buffer pass % 3).
QW_DEV void wselect(const float* p, int V, u64 T, SpShared& s, SpGlobal* g, unsigned& target, int& pass, int* err) {
    const int tid = threadIdx.x, warp = tid >> 5;
    uint32_t prefix = 0u, himask = 0u;
    u64 above = 0ull;
    bool found = true;
    for (int d = 0; d < 4; ++d) {
        const int shift = 24 - 8 * d;
        const int buf = pass % 3;
        for (int i = tid; i < SG_HC * 256; i += SG_NT) {
            (&s.hmass[0][0])[i] = 0ull;
            (&s.hcnt[0][0])[i] = 0;
        }
        __syncthreads();
        u64* hm = s.hmass[warp % SG_HC];
        int* hc = s.hcnt[warp % SG_HC];
        int cur = -1, cnt = 0;
        u64 run = 0ull;
        for_each_prob(p, V, [&](int, float f) {
            const uint32_t k = __float_as_uint(f);
            if ((k & himask) != prefix) return;
            const int dg = (int)((k >> shift) & 255u);
            if (dg != cur) {
                if (cur >= 0) {
                    atomicAdd(&hm[cur], run);
                    atomicAdd(&hc[cur], cnt);
                }
                cur = dg;
                run = 0ull;
                cnt = 0;
            }
            run += to_fx((double)f);
            ++cnt;
        });
        if (cur >= 0) {
            atomicAdd(&hm[cur], run);
            atomicAdd(&hc[cur], cnt);
        }
        __syncthreads();
        if (tid < 256) {
            u64 m = 0ull;
            int c = 0;
#pragma unroll
            for (int h = 0; h < SG_HC; ++h) {
                m += s.hmass[h][tid];
                c += s.hcnt[h][tid];
            }
            if (c) {
                atomicAdd(&g->hmass[buf][tid], m);
                atomicAdd(&g->hcnt[buf][tid], c);
            }
        }
        grid_sync(g, target, err);
        if (blockIdx.x == 0) {
            // the buffer of pass + 2 was last read before this barrier
            const int nb = (pass + 2) % 3;
            for (int i = tid; i < 256; i += SG_NT) {
                g->hmass[nb][i] = 0ull;
                g->hcnt[nb][i] = 0;
            }
        }
        ++pass;
        if (tid < 256) {
            s.gmass[tid] = __ldcg(&g->hmass[buf][tid]);
            s.gcnt[tid] = __ldcg(&g->hcnt[buf][tid]);
        }
        __syncthreads();
        if (tid == 0) {
            int pick = -1;
            u64 acc = above;
            for (int dg = 255; dg >= 0; --dg) {
                const int c = s.gcnt[dg];
                if (c == 0) continue;
                const u64 m = s.gmass[dg];
                if (acc + m >= T) {
                    pick = dg;
                    break;
                }
                acc += m;
            }
            s.found = pick >= 0;
            s.key = (uint32_t)(pick < 0 ? 0 : pick);
            s.above = acc;
        }
        __syncthreads();
        found = s.found != 0;
        if (!found) break;  // grid-uniform: every CTA walks the same histogram
        above = s.above;
        prefix |= s.key << shift;
        himask |= 0xFFu << shift;
        __syncthreads();
    }
    __syncthreads();
    if (tid == 0) {
        if (found) {
            const u64 pv = to_fx((double)__uint_as_float(prefix));
            u64 n = 1;
            if (pv > 0ull && T > above + pv) n = (T - above + pv - 1) / pv;  // ceil
            s.n_need = (int)(n < (u64)V ? n : (u64)V);
        } else {
            s.n_need = 0;
        }
        s.found = found;
        s.key = prefix;
        s.above = above;
    }
    __syncthreads();
}

// The n-th (1-based) element whose bits equal `key`, counting in index order
// over the whole grid (the last one when fewer exist), into g->token; -1 when
// none.  Every thread owns a contiguous chunk (a multiple of 4 entries).
QW_DEV void nth_equal(const float* p, int V, uint32_t key, int n, SpShared& s, SpGlobal* g, unsigned& target,
                      int* err) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gt = gridDim.x * SG_NT;
    const int chunk = ((V + gt - 1) / gt + 3) & ~3;
    const int i0 = min(V, (blockIdx.x * SG_NT + tid) * chunk), i1 = min(V, i0 + chunk);
    int c = 0;
    int i = i0;
    for (; i + 4 <= i1; i += 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p + i));
        c += (__float_as_uint(v.x) == key) + (__float_as_uint(v.y) == key) + (__float_as_uint(v.z) == key) +
             (__float_as_uint(v.w) == key);
    }
    for (; i < i1; ++i) c += __float_as_uint(__ldcg(p + i)) == key;
    // inclusive scan of c within the block
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s.iscan[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < SG_NW ? s.iscan[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < SG_NW) s.iscan[lane] = w;
    }
    __syncthreads();
    if (tid == 0) {
        g->ccnt[blockIdx.x] = s.iscan[SG_NW - 1];
        if (blockIdx.x == 0) g->token = -1;
    }
    grid_sync(g, target, err);
    if (tid < (int)gridDim.x) s.gcntc[tid] = __ldcg(&g->ccnt[tid]);
    __syncthreads();
    int before_cta = 0, total = 0;
    for (int b = 0; b < (int)gridDim.x; ++b) {
        const int cb = s.gcntc[b];
        if (b < (int)blockIdx.x) before_cta += cb;
        total += cb;
    }
    const int want = min(n, total);
    const int before = before_cta + (warp > 0 ? s.iscan[warp - 1] : 0) + inc - c;
    if (want > 0 && c > 0 && before < want && want <= before + c) {
        int k = before;
        for (int j = i0; j < i1; ++j) {
            if (__float_as_uint(__ldcg(p + j)) == key && ++k == want) {
                g->token = j;
                break;
            }
        }
    }
    grid_sync(g, target, err);
}

__global__ void __launch_bounds__(SG_NT, 1) sample_kernel(const SampleArgs a) {
    __shared__ SpShared s;
    const int tid = threadIdx.x;
    SpGlobal* g = reinterpret_cast<SpGlobal*>(a.ctrl);
    StepCtl* ctl = a.ctl;
    if (ctl && *reinterpret_cast<volatile int*>(&ctl->done)) return;  // same value in every CTA
    if (a.gate && *reinterpret_cast<const volatile int*>(a.gate)) return;
    const SampleCfg cfg = a.cfg_dev ? *a.cfg_dev : a.cfg;
    const int V = a.V;
    const bf16* lg = a.logits;
    float* p = a.probs;
    unsigned target = 0;
    int pass = 0;
    int token = -1;
    if (blockIdx.x == 0) {
        for (int i = tid; i < 3 * 256; i += SG_NT) {
            (&g->hmass[0][0])[i] = 0ull;
            (&g->hcnt[0][0])[i] = 0;
        }
    }
    if (!(cfg.temperature > 0.f)) {
        // temperature <= 0: greedy argmax, ties to the lowest index (engine.rs:197-202):
        // mark the maxima, take the first mark
        float mx = -INFINITY;
        for_each_logit(lg, V, [&](int, float x) { mx = fmaxf(mx, x); });
        mx = block_max_f(mx, s);
        if (tid == 0) g->pmax[blockIdx.x] = mx;
        grid_sync(g, target, a.err);
        const float gm = grid_max(g, s);
        for_each_logit(lg, V, [&](int i, float x) { p[i] = x == gm ? 1.0f : 0.0f; });
        grid_sync(g, target, a.err);
        nth_equal(p, V, __float_as_uint(1.0f), 1, s, g, target, a.err);
        token = __ldcg(&g->token);
    } else {
        const float t = fmaxf(cfg.temperature, 1e-5f);
        float mx = -INFINITY;
        for_each_logit(lg, V, [&](int, float x) { mx = fmaxf(mx, __fdiv_rn(x, t)); });
        mx = block_max_f(mx, s);
        if (tid == 0) g->pmax[blockIdx.x] = mx;
        grid_sync(g, target, a.err);
        const float gm = grid_max(g, s);
        double se = 0.0;
        for_each_logit(lg, V, [&](int i, float x) {
            const float e = expf(__fsub_rn(__fdiv_rn(x, t), gm));
            p[i] = e;
            se += (double)e;
        });
        se = block_sum_d(se, s);
        if (tid == 0) g->psum[blockIdx.x] = se;
        grid_sync(g, target, a.err);
        if (tid < (int)gridDim.x) s.gpart[tid] = __double_as_longlong(__ldcg(&g->psum[tid]));
        __syncthreads();
        double tot = 0.0;
        for (int b = 0; b < (int)gridDim.x; ++b) tot += __longlong_as_double((long long)s.gpart[b]);
        const float sumf = (float)tot;
        __syncthreads();
        u64 sp = 0ull;
        // same element -> thread map as the exp pass: every thread reads back its own writes
        for_each_logit(lg, V, [&](int i, float) {
            const float q = __fdiv_rn(p[i], sumf);
            p[i] = q;
            sp += to_fx((double)q);
        });
        sp = block_sum_u64(sp, s);
        if (tid == 0) g->ptot[blockIdx.x] = sp;
        grid_sync(g, target, a.err);
        if (tid < (int)gridDim.x) s.gpart[tid] = __ldcg(&g->ptot[tid]);
        __syncthreads();
        u64 ptotal = 0ull;
        for (int b = 0; b < (int)gridDim.x; ++b) ptotal += s.gpart[b];
        __syncthreads();
        // nucleus (engine.rs:228-240)
        const float top_p = fminf(fmaxf(cfg.top_p, 0.f), 1.f);
        wselect(p, V, to_fx((double)top_p), s, g, target, pass, a.err);
        const bool nfound = s.found != 0;
        const uint32_t kp = s.key;
        const int np = s.n_need;
        const u64 renorm = nfound ? s.above + (u64)np * to_fx((double)__uint_as_float(kp)) : ptotal;
        __syncthreads();
        if (a.desc_out) {
            // the nucleus as (value, last included index among the ties, mass)
            int tie = V - 1;
            if (nfound) {
                nth_equal(p, V, kp, np, s, g, target, a.err);
                tie = __ldcg(&g->token);
            }
            if (blockIdx.x == 0 && tid == 0) {
                a.desc_out->key = kp;
                a.desc_out->tie_idx = tie;
                a.desc_out->renorm = (float)((double)renorm / SP_FX);
                a.desc_out->found = nfound ? 1 : 0;
            }
            __syncthreads();
        }
        if (a.no_draw) {
            if (tid == 0 && atomicAdd(&g->exit, 1u) == gridDim.x - 1) {
                g->bar = 0u;
                g->exit = 0u;
            }
            return;
        }
        // categorical draw (engine.rs:241-262)
        const unsigned long long ctr =
            a.ctr_iter ? (unsigned long long)(*a.ctr_iter) * 64ull + (unsigned long long)a.ctr_base
                       : (ctl ? (cfg.same_draw ? 0ull : (unsigned long long)ctl->produced) : a.counter);
        const float r = __fmul_rn(sample_u(cfg.seed, ctr), (float)((double)renorm / SP_FX));
        wselect(p, V, to_fx((double)r), s, g, target, pass, a.err);
        uint32_t kr = s.key;
        int nr = s.n_need;
        const bool rfound = s.found != 0;
        __syncthreads();
        if (!rfound || (nfound && (kr < kp || (kr == kp && nr > np)))) {
            if (nfound) {
                // past the nucleus by rounding: its last element (engine.rs:262)
                kr = kp;
                nr = np;
            } else {
                // the nucleus is the whole vocabulary: its last element with mass
                wselect(p, V, ptotal, s, g, target, pass, a.err);
                kr = s.key;
                nr = s.n_need;
                __syncthreads();
            }
        }
        nth_equal(p, V, kr, nr, s, g, target, a.err);
        token = __ldcg(&g->token);
    }
    if (token < 0) token = 0;
    if (blockIdx.x == 0 && tid == 0) {
        if (ctl) {
            // loop bookkeeping after a pick (engine.rs:161-173); the forward already
            // advanced the cache length
            ctl->produced += 1;
            bool eos = false;
            for (int i = 0; i < ctl->n_eos; ++i) eos |= (ctl->eos[i] == token);
            if (eos) {
                ctl->done = 1;
                ctl->finish = 1;
            } else {
                a.out[ctl->n_out] = token;
                ctl->n_out += 1;
                *a.next_tok = token;
                if (ctl->produced >= ctl->max_new) ctl->done = 1;
            }
        } else {
            *a.token_out = token;
        }
    }
    // the last CTA out re-arms the control block for the next launch
    if (tid == 0 && atomicAdd(&g->exit, 1u) == gridDim.x - 1) {
        g->bar = 0u;
        g->exit = 0u;
    }
}

}  // namespace

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st) {
    if (a.V < 1 || !a.logits || !a.probs || !a.ctrl) return cudaErrorInvalidValue;
    if (!a.ctl && !a.token_out) return cudaErrorInvalidValue;
    if ((uintptr_t)a.logits % 16 != 0 || (uintptr_t)a.probs % 16 != 0 || (uintptr_t)a.ctrl % 16 != 0)
        return cudaErrorMisalignedAddress;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(SG_CTAS);
    cfg.blockDim = dim3(SG_NT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: they meet at grid barriers
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, sample_kernel, a);
}

}  // namespace qw
