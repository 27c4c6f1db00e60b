// Decode / verify attention inside the persistent decode kernel
// (crates/base-mlx-core/src/model/qwen3.rs:398-518: q_norm / k_norm, RoPE,
// in-place KV write, GQA SDPA with the causal mask of :629-653).
//
// Work item = (kv head, split): split s covers the 128 key positions
// [128 s, 128 s + 128) -- fixed boundaries, so a row's summation order does
// not depend on the sequence length or on the number of rows in the launch (a
// (k+1)-row verify equals k+1 single-row decodes bit for bit).  The item
// serves the G = Hq / Hkv query heads of its kv head for the S new rows
// (R = G S rows), or, when the grid has room for more items, a subset of
// them: each row's arithmetic is the same either way, fewer rows per item
// only shorten the item.  Its cached keys / values arrive by two bulk copies (the
// rows are contiguous in the [kv head][position][128] cache), issued while
// the CTA still waits for the other CTAs' q|k|v; the new positions' k / v
// are normalised, rotated and written to the cache by the item that owns
// them and placed into the tile directly.
//
//   scores  thread = (key, dimension quarter): 32 dims of one key against every
//           row, quarter sums joined by a fixed shuffle tree;
//   softmax one warp per row over the item's 128 keys;
//   P.V     thread = (dimension pair, key eighth): 16 keys in order per row,
//           the eight key-eighth sums joined in key order through shared
//           memory;
// then an unnormalised partial (max, sum, o[128]) per row goes to global
// memory and the last item of the kv head to arrive merges the splits in
// split order, fetching every split's statistics and its row's partial
// outputs in one round trip.
#pragma once
#include "attn_decode.cuh"

// diagnostics: globaltimer stamp k of the item (a.prof[k], thread 0)
#define ATTN_STAMP(k)                                                                       \
    do {                                                                                    \
        if (a.prof && tid == 0) {                                                           \
            unsigned long long t_;                                                          \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                          \
            a.prof[(k)] = t_;                                                               \
        }                                                                                   \
    } while (0)

namespace qw {
namespace attn {

constexpr int SPLIT_KEYS = 128;

template <int RMAX>
struct SplitSmem {
    uint64_t bar;                        // the item's bulk copies of cached K and V
    int last;
    float mrow[RMAX], lrow[RMAX];
    __align__(16) float cs[RMAX][HALF];  // RoPE cos / sin rows of the S new positions
    __align__(16) float sn[RMAX][HALF];
    __align__(16) bf16 qn[D], kn[D];     // q_norm / k_norm weights
    __align__(16) bf16 qs[RMAX][D];      // roped queries (bf16 values, as the reference rounds them)
    __align__(16) float sc[RMAX][SPLIT_KEYS];  // scores, then probabilities
    __align__(16) bf16 kt[SPLIT_KEYS][D];
    __align__(16) bf16 vt[SPLIT_KEYS][D];
};

// Splits covering positions [0, T).
QW_DEV int split_count(int T) { return (T + SPLIT_KEYS - 1) / SPLIT_KEYS; }

// Issue the bulk copies of the item's cached rows [j0, min(j0 + 128, off)) of
// K and V (thread 0; the barrier completes when both land) and fetch the step's
// RoPE rows and the q/k norm weights (every thread; NT = 512).  None of it
// depends on this step's q|k|v, so it runs before the phase barrier; the
// caller syncs before any thread waits or reads.
template <int RMAX>
QW_DEV void split_preload(const AttnArgs& a, SplitSmem<RMAX>& sm, int kvh, int split, int off, int tid) {
    for (int i = tid; i < a.S * HALF; i += 512) {
        const int r = i / HALF, c = i - r * HALF;
        sm.cs[r][c] = a.rope_cos[(size_t)(off + r) * HALF + c];
        sm.sn[r][c] = a.rope_sin[(size_t)(off + r) * HALF + c];
    }
    if (tid < D) sm.qn[tid] = a.q_norm_w[tid];
    else if (tid < 2 * D) sm.kn[tid - D] = a.k_norm_w[tid - D];
    if (tid != 0) return;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
    const int j0 = split * SPLIT_KEYS;
    const int nold = max(0, min(j0 + SPLIT_KEYS, off) - j0);
    const uint32_t bytes = (uint32_t)nold * D * 2;
    mbar_arrive_expect_tx(&sm.bar, 2 * bytes);
    if (nold > 0) {
        const size_t base = ((size_t)kvh * a.max_pos + j0) * D;
        bulk_g2s(&sm.kt[0][0], a.kcache + base, bytes, &sm.bar);
        bulk_g2s(&sm.vt[0][0], a.vcache + base, bytes, &sm.bar);
    }
}

// One (kv head, split) item with NT threads (NT = 512).  With SUB it serves
// the query heads qh0_ .. qh0_ + nqh_ - 1 of the kv head's G (fewer than G when
// the grid has room for more items: every row's arithmetic is the same either
// way), its rows being the kv head's rows qh0 S .. (qh0 + nqh) S - 1 and its
// merge counter counters[kvh G + qh0]; without SUB all G (qh0 = 0, merge
// counter counters[kvh]), and the code is the plain per-kv-head item.
// `preloaded`: the cached rows were issued by split_preload (else this issues
// them).
template <int RMAX, int NT, bool SUB, typename Sync>
QW_DEV void split_body(const AttnArgs& a, SplitSmem<RMAX>& sm, const int kvh, const int split, const int nsplit,
                       const int off, const int qh0_, const int nqh_, const int tid, Sync sync, bool preloaded) {
    static_assert(NT == 512, "thread mapping assumes 512 threads");
    constexpr int RQ = (RMAX + 3) / 4;  // rows per row quarter
    const int lane = tid & 31, warp = tid >> 5;
    const int S = a.S, G = a.Hq / a.Hkv;
    const int qh0 = SUB ? qh0_ : 0, nqh = SUB ? nqh_ : G;
    const int R = nqh * S;
    const int T = off + S;
    const int j0 = split * SPLIT_KEYS;
    const int j1 = min(j0 + SPLIT_KEYS, T);
    if (T > a.max_pos || R > RMAX) {
        if (tid == 0) atomicOr(a.err, T > a.max_pos ? QW_DERR_KV_RANGE : QW_DERR_SHAPE);
        return;
    }
    if (!preloaded) {
        split_preload<RMAX>(a, sm, kvh, split, off, tid);
        sync();
    }
    // queries of the G heads: q_norm + RoPE (warp per row)
    for (int r = warp; r < R; r += NT / 32) {
        const int gi = r / S, i = r - gi * S;
        const int h = kvh * G + qh0 + gi, pos = off + i;
        float o[4];
        (void)pos;
        norm_rope_row(a.q + (size_t)i * a.ldq + h * D, sm.qn, a.eps, sm.cs[i], sm.sn[i], lane, o);
        *reinterpret_cast<uint32_t*>(&sm.qs[r][2 * lane]) = pack_bf16x2(o[0], o[1]);
        *reinterpret_cast<uint32_t*>(&sm.qs[r][HALF + 2 * lane]) = pack_bf16x2(o[2], o[3]);
    }
    // new positions inside this split: k_norm + RoPE, cache write, tile row;
    // taken by the warps from the top down, so that with R + S <= 16 they run
    // beside the query rows instead of after them
    for (int p = max(off, j0) + (NT / 32 - 1 - warp); p < j1; p += NT / 32) {
        const int i = p - off;
        float o[4];
        norm_rope_row(a.k + (size_t)i * a.ldk + kvh * D, sm.kn, a.eps, sm.cs[i], sm.sn[i], lane, o);
        const uint32_t k01 = pack_bf16x2(o[0], o[1]), k23 = pack_bf16x2(o[2], o[3]);
        // the cache rows: written once, by the item of the kv head's first query heads
        bf16* kd = a.kcache + ((size_t)kvh * a.max_pos + p) * D;
        if (qh0 == 0) {
            *reinterpret_cast<uint32_t*>(kd + 2 * lane) = k01;
            *reinterpret_cast<uint32_t*>(kd + HALF + 2 * lane) = k23;
        }
        *reinterpret_cast<uint32_t*>(&sm.kt[p - j0][2 * lane]) = k01;
        *reinterpret_cast<uint32_t*>(&sm.kt[p - j0][HALF + 2 * lane]) = k23;
        const uint2 vv = __ldcg(reinterpret_cast<const uint2*>(a.v + (size_t)i * a.ldv + kvh * D + 4 * lane));
        if (qh0 == 0) *reinterpret_cast<uint2*>(a.vcache + ((size_t)kvh * a.max_pos + p) * D + 4 * lane) = vv;
        *reinterpret_cast<uint2*>(&sm.vt[p - j0][4 * lane]) = vv;
    }
    ATTN_STAMP(1);
    // cached rows landed (bounded wait)
    if (!mbar_wait_bounded(&sm.bar, 0) && tid == 0) atomicOr(a.err, QW_DERR_TIMEOUT);
    sync();
    ATTN_STAMP(2);

    // scores: thread = (key k = 8 warp + lane / 4, dimension quarter qq = lane & 3).
    // Quarter qq covers dims [32 qq, 32 qq + 32) as four 16-byte chunks, visited
    // from chunk (2 (k & 1) + qq / 2) & 3 on, so the eight lanes of a quarter-warp
    // read eight different bank groups of K and a warp's query reads are one
    // 128-byte wavefront.  Each row's four quarter sums meet in a fixed shuffle
    // tree, (q0 + q1) + (q2 + q3), identical in all four lanes.
    {
        const int qq = lane & 3, kk = lane >> 2;
        const int k = warp * 8 + kk;
        const int j = j0 + k;
        const int rot = 2 * (kk & 1) + (qq >> 1);
        float kf[4][8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int dc = 4 * qq + ((c + rot) & 3);
            const uint4 u = *reinterpret_cast<const uint4*>(&sm.kt[k][dc * 8]);
            kf[c][0] = bits_lo_f(u.x); kf[c][1] = bits_hi_f(u.x); kf[c][2] = bits_lo_f(u.y); kf[c][3] = bits_hi_f(u.y);
            kf[c][4] = bits_lo_f(u.z); kf[c][5] = bits_hi_f(u.z); kf[c][6] = bits_lo_f(u.w); kf[c][7] = bits_hi_f(u.w);
        }
        for (int r0 = 0; r0 < R; r0 += 4) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                if (r0 + rr < R) {
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int dc = 4 * qq + ((c + rot) & 3);
                        const uint4 qv = *reinterpret_cast<const uint4*>(&sm.qs[r0 + rr][dc * 8]);
                        float s = acc[rr];
                        s = fmaf(bits_lo_f(qv.x), kf[c][0], s); s = fmaf(bits_hi_f(qv.x), kf[c][1], s);
                        s = fmaf(bits_lo_f(qv.y), kf[c][2], s); s = fmaf(bits_hi_f(qv.y), kf[c][3], s);
                        s = fmaf(bits_lo_f(qv.z), kf[c][4], s); s = fmaf(bits_hi_f(qv.z), kf[c][5], s);
                        s = fmaf(bits_lo_f(qv.w), kf[c][6], s); s = fmaf(bits_hi_f(qv.w), kf[c][7], s);
                        acc[rr] = s;
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                float t = acc[rr];
                t += __shfl_xor_sync(0xffffffffu, t, 1);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                acc[rr] = t;
            }
            // lane qq stores row r0 + qq
            const int r = r0 + qq;
            if (r < R) {
                const float dot = qq == 0 ? acc[0] : (qq == 1 ? acc[1] : (qq == 2 ? acc[2] : acc[3]));
                const int i = r % S;
                const bool ok = (j < j1) && (j <= off + i);
                sm.sc[r][k] = ok ? dot * a.scale : -INFINITY;
            }
        }
    }
    sync();
    ATTN_STAMP(5);
    // softmax statistics and probabilities, one warp per row (keys lane, lane + 32, ...)
    for (int r = warp; r < R; r += NT / 32) {
        float s4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) s4[u] = sm.sc[r][lane + 32 * u];
        const float mx = warp_max(fmaxf(fmaxf(s4[0], s4[1]), fmaxf(s4[2], s4[3])));
        float ps = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float p = mx == -INFINITY ? 0.f : expf(s4[u] - mx);
            sm.sc[r][lane + 32 * u] = p;
            ps += p;
        }
        ps = warp_sum(ps);
        if (lane == 0) {
            sm.mrow[r] = mx;
            sm.lrow[r] = ps;
        }
    }
    sync();
    ATTN_STAMP(3);
    // P.V: thread = (dimension pair dp, key eighth ke): keys 16 ke .. 16 ke + 15 in
    // order for rows in groups of 8; the eight key-eighth sums of a (row, dim) meet
    // in shared memory (the K tile's space) in key order.
    const size_t pbase = ((size_t)kvh * nsplit + split) * RMAX + (size_t)qh0 * S;
    {
        const int nk = j1 - j0;
        const int dp = (warp & 1) * 32 + lane, ke = warp >> 1;
        float* red = reinterpret_cast<float*>(&sm.kt[0][0]);  // [8 ke][8 rows][128]
        static_assert(sizeof(sm.kt) >= 8 * 8 * D * sizeof(float), "P.V reduction buffer");
        float2 vv[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            const int key = ke * 16 + t;
            const uint32_t w2 = *reinterpret_cast<const uint32_t*>(&sm.vt[key][2 * dp]);
            vv[t] = key < nk ? make_float2(bits_lo_f(w2), bits_hi_f(w2)) : make_float2(0.f, 0.f);
        }
        const int d = tid & (D - 1), rq = tid >> 7;
        for (int r0 = 0; r0 < R; r0 += 8) {
            float o[8][2];
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
                o[rr][0] = o[rr][1] = 0.f;
                if (r0 + rr < R) {
#pragma unroll
                    for (int t4 = 0; t4 < 4; ++t4) {
                        const float4 p4 = *reinterpret_cast<const float4*>(&sm.sc[r0 + rr][ke * 16 + 4 * t4]);
                        const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            o[rr][0] = fmaf(pp[u], vv[4 * t4 + u].x, o[rr][0]);
                            o[rr][1] = fmaf(pp[u], vv[4 * t4 + u].y, o[rr][1]);
                        }
                    }
                }
            }
            if (r0 > 0) sync();  // the previous row group's sums have been read
#pragma unroll
            for (int rr = 0; rr < 8; ++rr)
                if (r0 + rr < R)
                    *reinterpret_cast<float2*>(&red[(ke * 8 + rr) * D + 2 * dp]) = make_float2(o[rr][0], o[rr][1]);
            sync();
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int rr = rq + 4 * q, r = r0 + rr;
                if (r < R) {
                    float sum = red[rr * D + d];
#pragma unroll
                    for (int e = 1; e < 8; ++e) sum += red[(e * 8 + rr) * D + d];
                    a.part[(pbase + r) * (D + 2) + d] = sum;
                }
            }
        }
    }
    // partial statistics (max, sum) of every row
    if (tid < R) {
        a.part[(pbase + tid) * (D + 2) + D] = sm.mrow[tid];
        a.part[(pbase + tid) * (D + 2) + D + 1] = sm.lrow[tid];
    }
    sync();
    ATTN_STAMP(4);
    unsigned* const counter = &a.counters[SUB ? kvh * G + qh0 : kvh];
    if (tid == 0) sm.last = (atom_add_acq_rel(counter, 1u) == (unsigned)(nsplit - 1));
    sync();
    ATTN_STAMP(7);
    if (!sm.last) return;

    // merge (last split of this kv head): weights e^(m_s - max), sums in split
    // order.  Thread (d, rq) merges rows rq, rq + 4, ...; the first PMAX
    // splits' statistics and partial outputs are fetched in one round trip
    // (every split up to 1024 keys), later splits batch by batch.
    constexpr int PMAX = 8;
    const int d = tid & (D - 1), rq = tid >> 7;
    auto fetch = [&](int s2, int r, float& m_, float& l_, float& o_) {
        const float* pp = &a.part[(((size_t)kvh * nsplit + s2) * RMAX + qh0 * S + r) * (D + 2)];
        m_ = __ldcg(pp + D);
        l_ = __ldcg(pp + D + 1);
        o_ = __ldcg(pp + d);
    };
    for (int q = 0; q < RQ; ++q) {
        const int r = rq + 4 * q;
        if (r >= R) break;
        float m0[PMAX], l0[PMAX], o0[PMAX];
#pragma unroll
        for (int u = 0; u < PMAX; ++u) {
            m0[u] = -INFINITY;
            l0[u] = o0[u] = 0.f;
            if (u < nsplit) fetch(u, r, m0[u], l0[u], o0[u]);
        }
        float M = -INFINITY;
#pragma unroll
        for (int u = 0; u < PMAX; ++u) M = fmaxf(M, m0[u]);
        for (int s2 = PMAX; s2 < nsplit; ++s2)
            M = fmaxf(M, __ldcg(&a.part[(((size_t)kvh * nsplit + s2) * RMAX + qh0 * S + r) * (D + 2) + D]));
        float O = 0.f, L = 0.f;
#pragma unroll
        for (int u = 0; u < PMAX; ++u) {
            if (u < nsplit) {
                const float wgt = m0[u] == -INFINITY ? 0.f : expf(m0[u] - M);
                L = fmaf(l0[u], wgt, L);
                O = fmaf(wgt != 0.f ? o0[u] : 0.f, wgt, O);
            }
        }
        for (int s2 = PMAX; s2 < nsplit; ++s2) {
            float m_, l_, o_;
            fetch(s2, r, m_, l_, o_);
            const float wgt = m_ == -INFINITY ? 0.f : expf(m_ - M);
            L = fmaf(l_, wgt, L);
            O = fmaf(wgt != 0.f ? o_ : 0.f, wgt, O);
        }
        const int gi = r / S, i = r - gi * S;
        a.out[(size_t)i * a.ldo + (kvh * G + qh0 + gi) * D + d] = f2bf(O / L);
    }
    if (tid == 0) *counter = 0u;
}

}  // namespace attn
}  // namespace qw
