// Decode / verify attention body shared by the standalone attention kernel
// (attention.cu) and the persistent decode kernel (decode_mk.cu).  See
// attention.cu for the reference mapping (qwen3.rs:398-518, 629-653).
#pragma once
#include "kernels.h"

namespace qw {
namespace attn {

constexpr int D = 128;
constexpr int HALF = 64;
constexpr int TILE = 64;

// RMSNorm over one 128-wide head row followed by RoPE at position pos.
// Lane l handles dims {2l, 2l+1} and {64+2l, 64+2l+1}; returns the 4 bf16
// results (as floats) in o[0..3] = dims 2l, 2l+1, 64+2l, 64+2l+1.
QW_DEV void norm_rope_row(const bf16* row, const bf16* nw, float eps, const float* cosr, const float* sinr,
                          int lane, float (&o)[4]) {
    // q/k/v rows may have been written by other CTAs of the same (persistent)
    // kernel: read them from L2, not a possibly stale L1 line
    const uint32_t lo = __ldcg(reinterpret_cast<const unsigned int*>(row + 2 * lane));
    const uint32_t hi = __ldcg(reinterpret_cast<const unsigned int*>(row + HALF + 2 * lane));
    float x[4] = {bits_lo_f(lo), bits_hi_f(lo), bits_lo_f(hi), bits_hi_f(hi)};
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)D + eps);
    const uint32_t wlo = *reinterpret_cast<const uint32_t*>(nw + 2 * lane);
    const uint32_t whi = *reinterpret_cast<const uint32_t*>(nw + HALF + 2 * lane);
    const float w[4] = {bits_lo_f(wlo), bits_hi_f(wlo), bits_lo_f(whi), bits_hi_f(whi)};
    float n[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) n[i] = bfr(__fmul_rn(__fmul_rn(x[i], r), w[i]));
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float c = cosr[2 * lane + e], s = sinr[2 * lane + e];
        o[e] = bfr(__fsub_rn(__fmul_rn(n[e], c), __fmul_rn(n[2 + e], s)));
        o[2 + e] = bfr(__fadd_rn(__fmul_rn(n[2 + e], c), __fmul_rn(n[e], s)));
    }
}

// ---------------------------------------------------------------------------
// Decode / verify attention (S <= 8 new rows).  Grid (kv_heads, nsplit): each
// CTA handles the G = Hq/Hkv query heads of one kv head (R = G*S rows) over one
// contiguous slice of key positions, writes an unnormalised partial
// (max, sum, o[128]) per row, and the last CTA of the kv head merges them.
// Cached K/V rows stream through two 64-key shared-memory tiles with 16-byte
// asynchronous copies (K chunks XOR-swizzled by row, so a thread-per-key read
// is bank-conflict free); the new positions' k/v are normalised + rotated by
// the CTA that owns them, written to the cache and placed into the tile
// directly.
// ---------------------------------------------------------------------------
template <int RMAX>
struct DecSmem {
    uint64_t tbar[2];  // tile buffer b: completes when all 128 threads' copies of a tile have landed
    float qs[RMAX][D];
    float sc[RMAX][TILE];
    float mrow[RMAX], lrow[RMAX], alph[RMAX];
    bf16 kt[2][TILE][D];
    bf16 vt[2][TILE][D];
    bf16 nk[8][D], nv[8][D];
    int last;
};

// Cached (old) K/V rows [j0, min(j0 + 64, T, off)) of kv head kvh -> tile buffer
// `buf`, asynchronously.  Old rows do not depend on the current step, so a
// caller may issue the first two tiles early (`preloaded`).  Completion is
// tracked on the buffer's mbarrier (cp.async.mbarrier.arrive.noinc from each
// of the NT threads), not on the threads' cp.async groups, so a caller whose
// threads have other copies in flight does not wait for them.
template <int RMAX, int NT>
QW_DEV void attn_load_tile(const AttnArgs& a, DecSmem<RMAX>& sm, int kvh, int buf, int j0, int T, int off, int tid) {
    const bf16* kbase = a.kcache + (size_t)kvh * a.max_pos * D;
    const bf16* vbase = a.vcache + (size_t)kvh * a.max_pos * D;
    const int nold = max(0, min(j0 + TILE, min(T, off)) - j0);
    for (int idx = tid; idx < nold * 16; idx += NT) {
        const int r = idx >> 4, c = idx & 15;
        cp_async16(&sm.kt[buf][r][(c ^ (r & 15)) * 8], kbase + (size_t)(j0 + r) * D + c * 8);
        cp_async16(&sm.vt[buf][r][c * 8], vbase + (size_t)(j0 + r) * D + c * 8);
    }
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sm.tbar[buf])) : "memory");
}

// (Re)initialise the two tile barriers (NT arrivals each); callers sync after.
template <int RMAX, int NT>
QW_DEV void attn_init_bars(DecSmem<RMAX>& sm, int tid) {
    if (tid == 0) {
        mbar_init(&sm.tbar[0], NT);
        mbar_init(&sm.tbar[1], NT);
        fence_mbar_init();
    }
}

// Tiles of this split CTA (chunks split, split + nsplit, ... of 64 keys).
QW_DEV int attn_ntiles(int T, int split, int nsplit) {
    const int nchunks = (T + TILE - 1) / TILE;
    return split < nchunks ? (nchunks - split + nsplit - 1) / nsplit : 0;
}

// Issue the first two tile loads of attn_decode_body ahead of time (NT threads).
template <int RMAX, int NT, typename Sync>
QW_DEV void attn_decode_preload(const AttnArgs& a, DecSmem<RMAX>& sm, int kvh, int split, int nsplit, int tid,
                                Sync sync) {
    attn_init_bars<RMAX, NT>(sm, tid);
    sync();
    const int off = *a.seq_len;
    const int T = off + a.S;
    if (T > a.max_pos) return;
    const int ntiles = attn_ntiles(T, split, nsplit);
    if (ntiles > 0) attn_load_tile<RMAX, NT>(a, sm, kvh, 0, split * TILE, T, off, tid);
    if (ntiles > 1) attn_load_tile<RMAX, NT>(a, sm, kvh, 1, (split + nsplit) * TILE, T, off, tid);
}

// One (kv head, split) item with NT threads (a multiple of 128).  Work split:
// scores -- thread = (key, row group of NT/64 groups); softmax -- warp per row;
// P.V -- thread = (dim, key quarter of NT/128 quarters), each quarter keeping
// its own rescaled accumulator, the quarters summed in order at the end.  Every
// per-row quantity is computed in an order that depends on neither R nor T.
template <int RMAX, int NT, typename Sync>
QW_DEV void attn_decode_body(const AttnArgs& a, DecSmem<RMAX>& sm, const int kvh, const int split, const int nsplit,
                             const int tid, Sync sync, bool preloaded = false) {
    constexpr int NW = NT / 32;
    constexpr int RG = NT / 64;          // row groups in the score pass
    constexpr int RPT = (RMAX + RG - 1) / RG;
    constexpr int KQ = NT / 128;         // key quarters in the P.V pass
    constexpr int KPQ = TILE / KQ;       // keys per quarter
    const int lane = tid & 31, warp = tid >> 5;
    const int S = a.S, G = a.Hq / a.Hkv, R = G * S;
    const int off = *a.seq_len;
    const int T = off + S;
    if (T > a.max_pos || R > RMAX) {
        if (tid == 0) atomicOr(a.err, T > a.max_pos ? QW_DERR_KV_RANGE : QW_DERR_SHAPE);
        return;
    }
    // Keys are cut into fixed 64-key chunks, chunk c handled by CTA c % nsplit
    // in increasing c.  The summation order of a row therefore does not depend
    // on T: a verify of S rows and S single-row decodes produce bit-identical
    // outputs (chunks past a row's causal limit only add exact zeros).
    const int ntiles = attn_ntiles(T, split, nsplit);
    auto load_tile = [&](int buf, int j0) { attn_load_tile<RMAX, NT>(a, sm, kvh, buf, j0, T, off, tid); };
    if (!preloaded) {
        attn_init_bars<RMAX, NT>(sm, tid);
        sync();
        if (ntiles > 0) load_tile(0, split * TILE);
        if (ntiles > 1) load_tile(1, (split + nsplit) * TILE);
    }

    // queries: q_norm + rope
    for (int r = warp; r < R; r += NW) {
        const int gi = r / S, i = r - gi * S;
        const int h = kvh * G + gi, pos = off + i;
        float o[4];
        norm_rope_row(a.q + (size_t)i * a.ldq + h * D, a.q_norm_w, a.eps, a.rope_cos + (size_t)pos * HALF,
                      a.rope_sin + (size_t)pos * HALF, lane, o);
        sm.qs[r][2 * lane] = o[0];
        sm.qs[r][2 * lane + 1] = o[1];
        sm.qs[r][HALF + 2 * lane] = o[2];
        sm.qs[r][HALF + 2 * lane + 1] = o[3];
    }
    // new keys / values of this CTA's chunks: cache write + local copy
    for (int p = off + warp; p < T; p += NW) {
        if ((p / TILE) % nsplit != split) continue;
        const int i = p - off;
        float o[4];
        norm_rope_row(a.k + (size_t)i * a.ldk + kvh * D, a.k_norm_w, a.eps, a.rope_cos + (size_t)p * HALF,
                      a.rope_sin + (size_t)p * HALF, lane, o);
        const uint32_t k01 = pack_bf16x2(o[0], o[1]), k23 = pack_bf16x2(o[2], o[3]);
        bf16* kd = a.kcache + ((size_t)kvh * a.max_pos + p) * D;
        *reinterpret_cast<uint32_t*>(kd + 2 * lane) = k01;
        *reinterpret_cast<uint32_t*>(kd + HALF + 2 * lane) = k23;
        *reinterpret_cast<uint32_t*>(&sm.nk[i][2 * lane]) = k01;
        *reinterpret_cast<uint32_t*>(&sm.nk[i][HALF + 2 * lane]) = k23;
        const uint2 vv = __ldcg(reinterpret_cast<const uint2*>(a.v + (size_t)i * a.ldv + kvh * D + 4 * lane));
        *reinterpret_cast<uint2*>(a.vcache + ((size_t)kvh * a.max_pos + p) * D + 4 * lane) = vv;
        *reinterpret_cast<uint2*>(&sm.nv[i][4 * lane]) = vv;
    }
    if (tid < RMAX) {
        sm.mrow[tid] = -INFINITY;
        sm.lrow[tid] = 0.f;
    }
    sync();

    const int d = tid & (D - 1), kq = tid / D;  // P.V: dim and key quarter
    float o_acc[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) o_acc[r] = 0.f;

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1, j0 = (split + it * nsplit) * TILE;
        const int hi = min(T, j0 + TILE);
        if (!mbar_wait_bounded(&sm.tbar[buf], (it >> 1) & 1) && tid == 0) atomicOr(a.err, QW_DERR_TIMEOUT);
        // new positions of this tile come from the locally computed rows
        for (int idx = tid; idx < TILE * 16; idx += NT) {
            const int r = idx >> 4, c = idx & 15, j = j0 + r;
            if (j >= off && j < hi) {
                *reinterpret_cast<uint4*>(&sm.kt[buf][r][(c ^ (r & 15)) * 8]) =
                    *reinterpret_cast<const uint4*>(&sm.nk[j - off][c * 8]);
                *reinterpret_cast<uint4*>(&sm.vt[buf][r][c * 8]) = *reinterpret_cast<const uint4*>(&sm.nv[j - off][c * 8]);
            }
        }
        sync();
        // scores: thread -> key (tid & 63), rows par, par + RG, ...
        {
            const int jj = tid & (TILE - 1), par = tid >> 6;
            const int j = j0 + jj;
            float acc[RPT];
#pragma unroll
            for (int q = 0; q < RPT; ++q) acc[q] = 0.f;
            if (j < hi) {
#pragma unroll 4
                for (int dc = 0; dc < D / 8; ++dc) {
                    const uint4 u = *reinterpret_cast<const uint4*>(&sm.kt[buf][jj][(dc ^ (jj & 15)) * 8]);
                    const float kf[8] = {bits_lo_f(u.x), bits_hi_f(u.x), bits_lo_f(u.y), bits_hi_f(u.y),
                                         bits_lo_f(u.z), bits_hi_f(u.z), bits_lo_f(u.w), bits_hi_f(u.w)};
#pragma unroll
                    for (int q = 0; q < RPT; ++q) {
                        const int r = par + RG * q;
                        if (r < R) {
                            const float4 q0 = *reinterpret_cast<const float4*>(&sm.qs[r][dc * 8]);
                            const float4 q1 = *reinterpret_cast<const float4*>(&sm.qs[r][dc * 8 + 4]);
                            float s = acc[q];
                            s = fmaf(q0.x, kf[0], s); s = fmaf(q0.y, kf[1], s);
                            s = fmaf(q0.z, kf[2], s); s = fmaf(q0.w, kf[3], s);
                            s = fmaf(q1.x, kf[4], s); s = fmaf(q1.y, kf[5], s);
                            s = fmaf(q1.z, kf[6], s); s = fmaf(q1.w, kf[7], s);
                            acc[q] = s;
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < RPT; ++q) {
                const int r = par + RG * q;
                if (r < R) {
                    const int i = r % S;
                    const bool ok = (j < hi) && (j <= off + i);
                    sm.sc[r][jj] = ok ? acc[q] * a.scale : -INFINITY;
                }
            }
        }
        sync();
        // online softmax update, one warp per row
        for (int r = warp; r < R; r += NW) {
            const float s0 = sm.sc[r][lane], s1 = sm.sc[r][lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float mold = sm.mrow[r];
            const float mnew = fmaxf(mold, mx);
            float p0 = 0.f, p1 = 0.f, al = 1.f;
            if (mnew != -INFINITY) {
                p0 = expf(s0 - mnew);
                p1 = expf(s1 - mnew);
                al = expf(mold - mnew);
            }
            sm.sc[r][lane] = p0;
            sm.sc[r][lane + 32] = p1;
            const float ps = warp_sum(p0 + p1);
            if (lane == 0) {
                sm.lrow[r] = sm.lrow[r] * al + ps;
                sm.mrow[r] = mnew;
                sm.alph[r] = al;
            }
        }
        sync();
        // o_q[r][d] = o_q*alpha + sum over this quarter's keys of p[r][j] v[j][d]
        {
#pragma unroll
            for (int r = 0; r < RMAX; ++r)
                if (r < R) o_acc[r] *= sm.alph[r];
            const int jlo = kq * KPQ, jhi = min(jlo + KPQ, hi - j0);
            for (int jj = jlo; jj < jhi; ++jj) {
                const float vv = bf2f(sm.vt[buf][jj][d]);
#pragma unroll
                for (int r = 0; r < RMAX; ++r)
                    if (r < R) o_acc[r] = fmaf(sm.sc[r][jj], vv, o_acc[r]);
            }
        }
        sync();
        if (it + 2 < ntiles) load_tile(buf, (split + (it + 2) * nsplit) * TILE);
    }

    // key quarters -> one accumulator per (row, dim), summed in quarter order
    float* comb = reinterpret_cast<float*>(&sm.kt[0][0][0]);  // [KQ][R][D], tiles no longer needed
    if (KQ > 1) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
            if (r < R) comb[((size_t)kq * R + r) * D + d] = o_acc[r];
        sync();
    }
    // partial -> global: thread (dim d, quarter kq) writes rows r = kq, kq + KQ, ...
    const size_t pbase = ((size_t)kvh * nsplit + split) * RMAX;
    for (int r = kq; r < R; r += KQ) {
        float v = 0.f;
        if (KQ > 1) {
            for (int q = 0; q < KQ; ++q) v += comb[((size_t)q * R + r) * D + d];
        } else {
#pragma unroll
            for (int rr = 0; rr < RMAX; ++rr)
                if (rr == r) v = o_acc[rr];
        }
        a.part[(pbase + r) * (D + 2) + d] = v;
    }
    if (tid < R) {
        a.part[(pbase + tid) * (D + 2) + D] = sm.mrow[tid];
        a.part[(pbase + tid) * (D + 2) + D + 1] = sm.lrow[tid];
    }
    sync();
    if (tid == 0) sm.last = (atom_add_acq_rel(&a.counters[kvh], 1u) == (unsigned)(nsplit - 1));
    sync();
    if (!sm.last) return;
    // merge the splits (fixed order) and write bf16 output.  Only splits that
    // own a chunk have data (chunk c -> split c % nsplit); the others would add
    // exact zeros, so skipping them changes no bit.  Split maxima and sums go to
    // the tile buffers (no longer needed): nsplit * R <= 148 * 64 floats.
    const int nact = min(nsplit, (T + TILE - 1) / TILE);
    float* mb = reinterpret_cast<float*>(&sm.kt[0][0][0]);
    float* lb = mb + nsplit * R;
    // decode rows (R <= KQ, one row per thread): the row's split partials are
    // fetched together with the split statistics, one memory round trip
    constexpr int PMAX = 20;
    const bool prefetch = R <= KQ && nact <= PMAX;
    float pre[PMAX];
    if (prefetch && kq < R) {
#pragma unroll
        for (int s2 = 0; s2 < PMAX; ++s2)
            pre[s2] = s2 < nact ? __ldcg(&a.part[(((size_t)kvh * nsplit + s2) * RMAX + kq) * (D + 2) + d]) : 0.f;
    }
    for (int idx = tid; idx < nact * R; idx += NT) {
        const int s2 = idx / R, r = idx - s2 * R;
        const float* pp = a.part + (((size_t)kvh * nsplit + s2) * RMAX + r) * (D + 2);
        mb[idx] = __ldcg(pp + D);
        lb[idx] = __ldcg(pp + D + 1);
    }
    sync();
    if (tid < R) {
        // row tid: global max, then split weights e^(m_s - max) (in place of m_s)
        float mm = -INFINITY;
        for (int s2 = 0; s2 < nact; ++s2) mm = fmaxf(mm, mb[s2 * R + tid]);
        float Lsum = 0.f;
        for (int s2 = 0; s2 < nact; ++s2) {
            const float ms = mb[s2 * R + tid];
            const float f = ms == -INFINITY ? 0.f : expf(ms - mm);
            mb[s2 * R + tid] = f;
            Lsum = fmaf(lb[s2 * R + tid], f, Lsum);
        }
        sm.lrow[tid] = Lsum;
    }
    sync();
    if (prefetch) {
        if (kq < R) {
            const int r = kq;
            float O = 0.f;
#pragma unroll
            for (int s2 = 0; s2 < PMAX; ++s2) {
                if (s2 < nact) {
                    const float wgt = mb[s2 * R + r];
                    O = fmaf(wgt != 0.f ? pre[s2] : 0.f, wgt, O);
                }
            }
            const int gi = r / S, i = r - gi * S;
            a.out[(size_t)i * a.ldo + (kvh * G + gi) * D + d] = f2bf(O / sm.lrow[r]);
        }
        if (tid == 0) a.counters[kvh] = 0u;
        return;
    }
    // thread = (dim, row group); per row, up to 16 splits' partials are loaded together
    for (int r = kq; r < R; r += KQ) {
        float O = 0.f;
        for (int s0 = 0; s0 < nact; s0 += 16) {
            float pv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                pv[j] = (s0 + j < nact && mb[(s0 + j) * R + r] != 0.f)
                            ? __ldcg(&a.part[(((size_t)kvh * nsplit + s0 + j) * RMAX + r) * (D + 2) + d])
                            : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (s0 + j < nact) O = fmaf(pv[j], mb[(s0 + j) * R + r], O);
        }
        const int gi = r / S, i = r - gi * S;
        a.out[(size_t)i * a.ldo + (kvh * G + gi) * D + d] = f2bf(O / sm.lrow[r]);
    }
    if (tid == 0) a.counters[kvh] = 0u;
}

}  // namespace attn
}  // namespace qw
