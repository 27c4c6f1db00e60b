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
// histograms (fp64, per-thread runs flushed with shared-memory atomics) among
// the elements that match the digits chosen so far, walking digits from the
// top until the mass reaches the target; ties at the final value are then
// taken in index order with a block scan.  One CTA of 1024 threads; about a
// dozen passes over the fp32 probabilities (0.6 MB for Qwen3's vocabulary).
#include "kernels.h"

namespace qw {
namespace {

constexpr int SP_NT = 1024;
constexpr int SP_NW = SP_NT / 32;
constexpr int SP_HC = 8;  // histogram copies (warps w and w + 8k share one)

struct SpShared {
    double hmass[SP_HC][256];
    int hcnt[SP_HC][256];
    double msum[256];
    int csum[256];
    double dred[SP_NW];
    float fred[SP_NW];
    unsigned long long kred[SP_NW];
    int iscan[SP_NW];
    uint32_t key;
    double above;
    int n_need;
    int found;
    int token;
};

QW_DEV float sample_u(unsigned long long seed, unsigned long long counter) {
    return (float)(splitmix64(seed ^ splitmix64(counter)) >> 40) * (1.0f / 16777216.0f);
}

QW_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Fixed-order block reductions (every thread calls; every thread gets the result).
QW_DEV double block_sum_d(double v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum_d(v);
    if (lane == 0) s.dred[warp] = v;
    __syncthreads();
    if (warp == 0) {
        double t = warp_sum_d(s.dred[lane]);
        if (lane == 0) s.dred[0] = t;
    }
    __syncthreads();
    const double r = s.dred[0];
    __syncthreads();
    return r;
}
QW_DEV float block_max_f(float v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) s.fred[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = warp_max(s.fred[lane]);
        if (lane == 0) s.fred[0] = t;
    }
    __syncthreads();
    const float r = s.fred[0];
    __syncthreads();
    return r;
}
QW_DEV unsigned long long block_max_u64(unsigned long long v, SpShared& s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = umax64(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) s.kred[warp] = v;
    __syncthreads();
    if (warp == 0) {
        unsigned long long t = s.kred[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = umax64(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (lane == 0) s.kred[0] = t;
    }
    __syncthreads();
    const unsigned long long r = s.kred[0];
    __syncthreads();
    return r;
}

// The value v (as float bits) at which the descending cumulative mass of p
// first reaches T: mass(p > v) < T <= mass(p >= v), and n_need = how many of
// the elements equal to v, in index order, that takes.  found = 0 when the
// whole mass stays below T.  Only digits holding at least one element are
// chosen, so T <= 0 selects the maximum.
QW_DEV void wselect(const float* p, int V, double T, SpShared& s) {
    const int tid = threadIdx.x, warp = tid >> 5;
    uint32_t prefix = 0u, himask = 0u;
    double above = 0.0;
    for (int d = 0; d < 4; ++d) {
        const int shift = 24 - 8 * d;
        for (int i = tid; i < SP_HC * 256; i += SP_NT) {
            (&s.hmass[0][0])[i] = 0.0;
            (&s.hcnt[0][0])[i] = 0;
        }
        __syncthreads();
        double* hm = s.hmass[warp % SP_HC];
        int* hc = s.hcnt[warp % SP_HC];
        int cur = -1, cnt = 0;
        double run = 0.0;
        for (int i = tid; i < V; i += SP_NT) {
            const float f = p[i];
            const uint32_t k = __float_as_uint(f);
            if ((k & himask) != prefix) continue;
            const int dg = (int)((k >> shift) & 255u);
            if (dg != cur) {
                if (cur >= 0) {
                    atomicAdd(&hm[cur], run);
                    atomicAdd(&hc[cur], cnt);
                }
                cur = dg;
                run = 0.0;
                cnt = 0;
            }
            run += (double)f;
            ++cnt;
        }
        if (cur >= 0) {
            atomicAdd(&hm[cur], run);
            atomicAdd(&hc[cur], cnt);
        }
        __syncthreads();
        if (tid < 256) {
            double m = 0.0;
            int c = 0;
#pragma unroll
            for (int h = 0; h < SP_HC; ++h) {
                m += s.hmass[h][tid];
                c += s.hcnt[h][tid];
            }
            s.msum[tid] = m;
            s.csum[tid] = c;
        }
        __syncthreads();
        if (tid == 0) {
            int pick = -1;
            double a = above;
            for (int dg = 255; dg >= 0; --dg) {
                if (s.csum[dg] == 0) continue;
                if (a + s.msum[dg] >= T) {
                    pick = dg;
                    break;
                }
                a += s.msum[dg];
            }
            s.found = pick >= 0;
            s.key = (uint32_t)(pick < 0 ? 0 : pick);
            s.above = a;
        }
        __syncthreads();
        const bool ok = s.found != 0;
        if (!ok) break;  // block-uniform
        above = s.above;
        prefix |= s.key << shift;
        himask |= 0xFFu << shift;
        __syncthreads();
    }
    if (tid == 0) {
        if (s.found) {
            const double pv = (double)__uint_as_float(prefix);
            long long n = 1;
            if (pv > 0.0 && T - above > pv) n = (long long)ceil((T - above) / pv);
            while (n > 1 && above + (double)(n - 1) * pv >= T) --n;
            s.n_need = (int)min(n, (long long)V);
        } else {
            s.n_need = 0;
        }
        s.key = prefix;
        s.above = above;
    }
    __syncthreads();
}

// Index of the n-th (1-based) element whose bits equal `key`, counting in index
// order; the last such element when there are fewer than n; -1 when none.
QW_DEV int nth_equal(const float* p, int V, uint32_t key, int n, SpShared& s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (V + SP_NT - 1) / SP_NT;
    const int i0 = min(V, tid * chunk), i1 = min(V, i0 + chunk);
    int c = 0;
    for (int i = i0; i < i1; ++i) c += __float_as_uint(p[i]) == key;
    // inclusive scan of c over the block
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s.iscan[warp] = inc;
    if (tid == 0) s.token = -1;
    __syncthreads();
    if (warp == 0) {
        int w = s.iscan[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        s.iscan[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int total = s.iscan[SP_NW - 1];
    const int before = (warp > 0 ? s.iscan[warp - 1] : 0) + inc - c;  // exclusive
    const int want = min(n, total);
    if (want > 0 && c > 0 && before < want && want <= before + c) {
        int k = before;
        for (int i = i0; i < i1; ++i) {
            if (__float_as_uint(p[i]) == key && ++k == want) {
                s.token = i;
                break;
            }
        }
    }
    __syncthreads();
    const int r = s.token;
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(SP_NT, 1) sample_kernel(const SampleArgs a) {
    __shared__ SpShared s;
    pdl_wait();
    const int tid = threadIdx.x;
    StepCtl* ctl = a.ctl;
    if (ctl && *reinterpret_cast<volatile int*>(&ctl->done)) return;
    const SampleCfg cfg = a.cfg_dev ? *a.cfg_dev : a.cfg;
    const int V = a.V;
    const bf16* lg = a.logits;
    int token = 0;
    if (!(cfg.temperature > 0.f)) {
        // temperature <= 0: greedy argmax, ties to the lowest index (engine.rs:197-202)
        unsigned long long best = 0ull;
        for (int i = tid; i < V; i += SP_NT) best = umax64(best, amax_key(bf2f(lg[i]), (uint32_t)i));
        token = (int)amax_key_index(block_max_u64(best, s));
    } else {
        float* p = a.probs;
        const float t = fmaxf(cfg.temperature, 1e-5f);
        float mx = -INFINITY;
        for (int i = tid; i < V; i += SP_NT) mx = fmaxf(mx, __fdiv_rn(bf2f(lg[i]), t));
        mx = block_max_f(mx, s);
        double se = 0.0;
        for (int i = tid; i < V; i += SP_NT) {
            const float e = expf(__fsub_rn(__fdiv_rn(bf2f(lg[i]), t), mx));
            p[i] = e;
            se += (double)e;
        }
        const float sumf = (float)block_sum_d(se, s);
        double sp = 0.0;
        for (int i = tid; i < V; i += SP_NT) {
            const float q = __fdiv_rn(p[i], sumf);
            p[i] = q;
            sp += (double)q;
        }
        const double ptotal = block_sum_d(sp, s);  // also orders the writes above before the reads below
        // nucleus (engine.rs:228-240)
        const float top_p = fminf(fmaxf(cfg.top_p, 0.f), 1.f);
        wselect(p, V, (double)top_p, s);
        const bool nfound = s.found != 0;
        const uint32_t kp = s.key;
        const int np = s.n_need;
        const double renorm = nfound ? s.above + (double)np * (double)__uint_as_float(kp) : ptotal;
        __syncthreads();
        // categorical draw (engine.rs:241-262)
        const unsigned long long ctr = ctl ? (cfg.same_draw ? 0ull : (unsigned long long)ctl->produced) : a.counter;
        const float r = __fmul_rn(sample_u(cfg.seed, ctr), (float)renorm);
        wselect(p, V, (double)r, s);
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
                wselect(p, V, ptotal * (1.0 - 1e-12), s);
                kr = s.key;
                nr = s.n_need;
                __syncthreads();
            }
        }
        token = nth_equal(p, V, kr, nr, s);
        if (token < 0) token = 0;
    }
    if (tid == 0) {
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
    pdl_launch_dependents();
}

}  // namespace

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t st, bool pdl) {
    if (a.V < 1 || !a.logits || !a.probs) return cudaErrorInvalidValue;
    if (!a.ctl && !a.token_out) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(SP_NT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, sample_kernel, a);
}

}  // namespace qw
