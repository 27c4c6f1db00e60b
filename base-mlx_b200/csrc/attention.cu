// Attention over the pre-allocated bf16 KV cache, with Qwen3's per-head
// q_norm / k_norm and non-traditional RoPE fused in.
//
// Replaces, per layer, crates/base-mlx-core/src/model/qwen3.rs:
//   :398-399  q_norm / k_norm (RMSNorm over head_dim, fp32 inside, bf16 out)
//   :401-413  fast::rope(dims=128, traditional=false, base=theta, offset)
//   :415-489  mlx_ext::slice_update of k/v into cache[:, offset:offset+S, :]
//   :491-518  fast::scaled_dot_product_attention (native GQA, scale 1/sqrt(128))
//   :629-653  the additive causal mask (query i sees keys j <= offset + i)
//
// Cache layout per layer: K and V each [kv_heads, max_pos, 128] bf16.
// The cache length lives on the device (seq_len) so a captured step graph can
// be replayed at every position; positions past max_pos raise an error flag
// instead of being written.
#include "kernels.h"

namespace qw {
namespace {

constexpr int D = 128;
constexpr int HALF = 64;
constexpr int TILE = 64;

// RMSNorm over one 128-wide head row followed by RoPE at position pos.
// Lane l handles dims {2l, 2l+1} and {64+2l, 64+2l+1}; returns the 4 bf16
// results (as floats) in o[0..3] = dims 2l, 2l+1, 64+2l, 64+2l+1.
QW_DEV void norm_rope_row(const bf16* row, const bf16* nw, float eps, const float* cosr, const float* sinr,
                          int lane, float (&o)[4]) {
    const uint32_t lo = *reinterpret_cast<const uint32_t*>(row + 2 * lane);
    const uint32_t hi = *reinterpret_cast<const uint32_t*>(row + HALF + 2 * lane);
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
    float qs[RMAX][D];
    float sc[RMAX][TILE];
    float mrow[RMAX], lrow[RMAX], alph[RMAX];
    bf16 kt[2][TILE][D];
    bf16 vt[2][TILE][D];
    bf16 nk[8][D], nv[8][D];
    int last;
};

template <int RMAX>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smraw[];
    DecSmem<RMAX>& sm = *reinterpret_cast<DecSmem<RMAX>*>(smraw);
    const int kvh = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S = a.S, G = a.Hq / a.Hkv, R = G * S;

    pdl_wait();
    pdl_launch_dependents();
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
    const int nchunks = (T + TILE - 1) / TILE;
    const int ntiles = split < nchunks ? (nchunks - split + nsplit - 1) / nsplit : 0;
    const bf16* kbase = a.kcache + (size_t)kvh * a.max_pos * D;
    const bf16* vbase = a.vcache + (size_t)kvh * a.max_pos * D;

    // cached (old) rows of a chunk -> shared memory, asynchronously
    auto load_tile = [&](int buf, int j0) {
        const int nold = max(0, min(j0 + TILE, min(T, off)) - j0);
        for (int idx = tid; idx < nold * 16; idx += 128) {
            const int r = idx >> 4, c = idx & 15;
            cp_async16(&sm.kt[buf][r][(c ^ (r & 15)) * 8], kbase + (size_t)(j0 + r) * D + c * 8);
            cp_async16(&sm.vt[buf][r][c * 8], vbase + (size_t)(j0 + r) * D + c * 8);
        }
        cp_async_commit();
    };
    if (ntiles > 0) load_tile(0, split * TILE);
    if (ntiles > 1) load_tile(1, (split + nsplit) * TILE);

    // queries: q_norm + rope
    for (int r = warp; r < R; r += 4) {
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
    for (int p = off + warp; p < T; p += 4) {
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
        const uint2 vv = *reinterpret_cast<const uint2*>(a.v + (size_t)i * a.ldv + kvh * D + 4 * lane);
        *reinterpret_cast<uint2*>(a.vcache + ((size_t)kvh * a.max_pos + p) * D + 4 * lane) = vv;
        *reinterpret_cast<uint2*>(&sm.nv[i][4 * lane]) = vv;
    }
    if (tid < RMAX) {
        sm.mrow[tid] = -INFINITY;
        sm.lrow[tid] = 0.f;
    }
    __syncthreads();

    float o_acc[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) o_acc[r] = 0.f;
    constexpr int RH = (RMAX + 1) / 2;

    for (int it = 0; it < ntiles; ++it) {
        const int buf = it & 1, j0 = (split + it * nsplit) * TILE;
        const int hi = min(T, j0 + TILE);
        if (it + 1 < ntiles)
            cp_async_wait<1>();
        else
            cp_async_wait<0>();
        // new positions of this tile come from the locally computed rows
        for (int idx = tid; idx < TILE * 16; idx += 128) {
            const int r = idx >> 4, c = idx & 15, j = j0 + r;
            if (j >= off && j < hi) {
                *reinterpret_cast<uint4*>(&sm.kt[buf][r][(c ^ (r & 15)) * 8]) =
                    *reinterpret_cast<const uint4*>(&sm.nk[j - off][c * 8]);
                *reinterpret_cast<uint4*>(&sm.vt[buf][r][c * 8]) = *reinterpret_cast<const uint4*>(&sm.nv[j - off][c * 8]);
            }
        }
        __syncthreads();
        // scores: thread -> key (tid & 63), rows of parity (tid >> 6)
        {
            const int jj = tid & (TILE - 1), par = tid >> 6;
            const int j = j0 + jj;
            float acc[RH];
#pragma unroll
            for (int q = 0; q < RH; ++q) acc[q] = 0.f;
            if (j < hi) {
#pragma unroll 4
                for (int dc = 0; dc < D / 8; ++dc) {
                    const uint4 u = *reinterpret_cast<const uint4*>(&sm.kt[buf][jj][(dc ^ (jj & 15)) * 8]);
                    const float kf[8] = {bits_lo_f(u.x), bits_hi_f(u.x), bits_lo_f(u.y), bits_hi_f(u.y),
                                         bits_lo_f(u.z), bits_hi_f(u.z), bits_lo_f(u.w), bits_hi_f(u.w)};
#pragma unroll
                    for (int q = 0; q < RH; ++q) {
                        const int r = par + 2 * q;
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
            for (int q = 0; q < RH; ++q) {
                const int r = par + 2 * q;
                if (r < R) {
                    const int i = r % S;
                    const bool ok = (j < hi) && (j <= off + i);
                    sm.sc[r][jj] = ok ? acc[q] * a.scale : -INFINITY;
                }
            }
        }
        __syncthreads();
        // online softmax update, one warp per row
        for (int r = warp; r < R; r += 4) {
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
        __syncthreads();
        // o[r][d] = o*alpha + sum_j p[r][j] v[j][d]; thread = dim
        {
            const int d = tid;
#pragma unroll
            for (int r = 0; r < RMAX; ++r)
                if (r < R) o_acc[r] *= sm.alph[r];
            const int nj = min(TILE, hi - j0);
            for (int jj = 0; jj < nj; ++jj) {
                const float vv = bf2f(sm.vt[buf][jj][d]);
#pragma unroll
                for (int r = 0; r < RMAX; ++r)
                    if (r < R) o_acc[r] = fmaf(sm.sc[r][jj], vv, o_acc[r]);
            }
        }
        __syncthreads();
        if (it + 2 < ntiles) load_tile(buf, (split + (it + 2) * nsplit) * TILE);
    }

    // partial -> global
    const size_t pbase = ((size_t)kvh * nsplit + split) * RMAX;
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
        if (r < R) a.part[(pbase + r) * (D + 2) + tid] = o_acc[r];
    if (tid < R) {
        a.part[(pbase + tid) * (D + 2) + D] = sm.mrow[tid];
        a.part[(pbase + tid) * (D + 2) + D + 1] = sm.lrow[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sm.last = (atomicAdd(&a.counters[kvh], 1u) == (unsigned)(nsplit - 1));
    __syncthreads();
    if (!sm.last) return;
    __threadfence();
    // merge the splits (fixed order) and write bf16 output.  All split maxima
    // and sums are gathered in one parallel pass; the tile buffers (no longer
    // needed) hold them: nsplit * R <= 148 * 64 floats.
    float* mb = reinterpret_cast<float*>(&sm.kt[0][0][0]);
    float* lb = mb + nsplit * R;
    for (int idx = tid; idx < nsplit * R; idx += 128) {
        const int s2 = idx / R, r = idx - s2 * R;
        const float* pp = a.part + (((size_t)kvh * nsplit + s2) * RMAX + r) * (D + 2);
        mb[idx] = __ldcg(pp + D);
        lb[idx] = __ldcg(pp + D + 1);
    }
    __syncthreads();
    if (tid < R) {
        // row tid: global max, then split weights e^(m_s - max) (in place of m_s)
        float mm = -INFINITY;
        for (int s2 = 0; s2 < nsplit; ++s2) mm = fmaxf(mm, mb[s2 * R + tid]);
        float Lsum = 0.f;
        for (int s2 = 0; s2 < nsplit; ++s2) {
            const float ms = mb[s2 * R + tid];
            const float f = ms == -INFINITY ? 0.f : expf(ms - mm);
            mb[s2 * R + tid] = f;
            Lsum = fmaf(lb[s2 * R + tid], f, Lsum);
        }
        sm.lrow[tid] = Lsum;
    }
    __syncthreads();
    for (int r = 0; r < R; ++r) {
        float O = 0.f;
        for (int s0 = 0; s0 < nsplit; s0 += 8) {
            float pv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                pv[j] = (s0 + j < nsplit && mb[(s0 + j) * R + r] != 0.f)
                            ? __ldcg(&a.part[(((size_t)kvh * nsplit + s0 + j) * RMAX + r) * (D + 2) + tid])
                            : 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < nsplit) O = fmaf(pv[j], mb[(s0 + j) * R + r], O);
        }
        const int gi = r / S, i = r - gi * S;
        a.out[(size_t)i * a.ldo + (kvh * G + gi) * D + tid] = f2bf(O / sm.lrow[r]);
    }
    if (tid == 0) a.counters[kvh] = 0u;
}

// ---------------------------------------------------------------------------
// Prefill helpers (S > 8).
// ---------------------------------------------------------------------------
// One warp per (row, head) item: q heads -> normalised + rotated q (qout),
// k heads -> normalised + rotated into the cache, v heads -> copied into the cache.
__global__ void qk_norm_rope_kvwrite_kernel(const AttnArgs a, bf16* qout) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);
    const int per_row = a.Hq + 2 * a.Hkv;
    if (item >= a.S * per_row) return;
    const int i = item / per_row, hh = item - i * per_row;
    const int off = *a.seq_len;
    const int pos = off + i;
    if (pos >= a.max_pos) {
        if (lane == 0) atomicOr(a.err, QW_DERR_KV_RANGE);
        return;
    }
    const float* cr = a.rope_cos + (size_t)pos * HALF;
    const float* sr = a.rope_sin + (size_t)pos * HALF;
    if (hh < a.Hq) {
        float o[4];
        norm_rope_row(a.q + (size_t)i * a.ldq + hh * D, a.q_norm_w, a.eps, cr, sr, lane, o);
        bf16* d = qout + (size_t)i * (a.Hq * D) + hh * D;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = pack_bf16x2(o[0], o[1]);
        *reinterpret_cast<uint32_t*>(d + HALF + 2 * lane) = pack_bf16x2(o[2], o[3]);
    } else if (hh < a.Hq + a.Hkv) {
        const int kh = hh - a.Hq;
        float o[4];
        norm_rope_row(a.k + (size_t)i * a.ldk + kh * D, a.k_norm_w, a.eps, cr, sr, lane, o);
        bf16* d = a.kcache + ((size_t)kh * a.max_pos + pos) * D;
        *reinterpret_cast<uint32_t*>(d + 2 * lane) = pack_bf16x2(o[0], o[1]);
        *reinterpret_cast<uint32_t*>(d + HALF + 2 * lane) = pack_bf16x2(o[2], o[3]);
    } else {
        const int vh = hh - a.Hq - a.Hkv;
        const uint2 vv = *reinterpret_cast<const uint2*>(a.v + (size_t)i * a.ldv + vh * D + 4 * lane);
        *reinterpret_cast<uint2*>(a.vcache + ((size_t)vh * a.max_pos + pos) * D + 4 * lane) = vv;
    }
}

// Causal attention for S new rows over [0, offset+S): grid (Hq, ceil(S/64)).
// CTA = 64 query rows of one head; 64-key tiles in shared memory (fp32),
// online softmax.  Thread (ty = tid/8, tx = tid%8) owns rows 4ty..4ty+3.
constexpr int PQ = 64, PK = 64, QLD = D + 1, KLD = D + 1, VLD = D + 4, PLD = PK + 1;
__global__ void __launch_bounds__(128) attn_prefill_kernel(const AttnArgs a, const bf16* qr) {
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                // [PQ][QLD]
    float* ks = qs + PQ * QLD;     // [PK][KLD]
    float* vs = ks + PK * KLD;     // [PK][VLD]
    float* ps = vs + PK * VLD;     // [PQ][PLD]
    float* mrow = ps + PQ * PLD;   // [PQ]
    float* lrow = mrow + PQ;
    float* alph = lrow + PQ;
    pdl_wait();
    pdl_launch_dependents();
    const int h = blockIdx.x, G = a.Hq / a.Hkv, kvh = h / G;
    const int i0 = blockIdx.y * PQ;
    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const int off = *a.seq_len;
    const int nrows = min(PQ, a.S - i0);
    if (off + a.S > a.max_pos) return;  // flagged by qk_norm_rope_kvwrite
    for (int u = tid; u < PQ * D; u += 128) {
        const int r = u / D, d = u - r * D;
        qs[r * QLD + d] = (r < nrows) ? bf2f(qr[(size_t)(i0 + r) * (a.Hq * D) + h * D + d]) : 0.f;
    }
    if (tid < PQ) {
        mrow[tid] = -INFINITY;
        lrow[tid] = 0.f;
    }
    float o[4][16];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 16; ++c) o[r][c] = 0.f;
    const int kend = off + i0 + nrows;  // exclusive
    const bf16* kb = a.kcache + (size_t)kvh * a.max_pos * D;
    const bf16* vb = a.vcache + (size_t)kvh * a.max_pos * D;
    for (int j0 = 0; j0 < kend; j0 += PK) {
        __syncthreads();
        for (int u = tid; u < PK * D; u += 128) {
            const int j = u / D, d = u - j * D;
            const bool ok = j0 + j < kend;
            ks[j * KLD + d] = ok ? bf2f(kb[(size_t)(j0 + j) * D + d]) : 0.f;
            vs[j * VLD + d] = ok ? bf2f(vb[(size_t)(j0 + j) * D + d]) : 0.f;
        }
        __syncthreads();
        float s[4][8];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 8; ++c) s[r][c] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            float qv[4], kv[8];
#pragma unroll
            for (int r = 0; r < 4; ++r) qv[r] = qs[(4 * ty + r) * QLD + d];
#pragma unroll
            for (int c = 0; c < 8; ++c) kv[c] = ks[(tx + 8 * c) * KLD + d];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 8; ++c) s[r][c] = fmaf(qv[r], kv[c], s[r][c]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int row = 4 * ty + r, j = j0 + tx + 8 * c;
                const bool ok = (row < nrows) && (j <= off + i0 + row) && (j < kend);
                ps[row * PLD + tx + 8 * c] = ok ? s[r][c] * a.scale : -INFINITY;
            }
        __syncthreads();
        // softmax rows: warp w handles rows w, w+4, ...
        for (int r = tid >> 5; r < PQ; r += 4) {
            const int lane = tid & 31;
            const float s0 = ps[r * PLD + lane], s1 = ps[r * PLD + lane + 32];
            const float mx = warp_max(fmaxf(s0, s1));
            const float mold = mrow[r], mnew = fmaxf(mold, mx);
            float p0 = 0.f, p1 = 0.f, al = 1.f;
            if (mnew != -INFINITY) {
                p0 = expf(s0 - mnew);
                p1 = expf(s1 - mnew);
                al = expf(mold - mnew);
            }
            ps[r * PLD + lane] = p0;
            ps[r * PLD + lane + 32] = p1;
            const float sum = warp_sum(p0 + p1);
            if (lane == 0) {
                lrow[r] = lrow[r] * al + sum;
                mrow[r] = mnew;
                alph[r] = al;
            }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float al = alph[4 * ty + r];
#pragma unroll
            for (int c = 0; c < 16; ++c) o[r][c] *= al;
        }
        for (int j = 0; j < PK; ++j) {
            float pv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) pv[r] = ps[(4 * ty + r) * PLD + j];
            const float4* vr = reinterpret_cast<const float4*>(vs + j * VLD + tx * 16);
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const float4 v = vr[c4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    o[r][4 * c4 + 0] = fmaf(pv[r], v.x, o[r][4 * c4 + 0]);
                    o[r][4 * c4 + 1] = fmaf(pv[r], v.y, o[r][4 * c4 + 1]);
                    o[r][4 * c4 + 2] = fmaf(pv[r], v.z, o[r][4 * c4 + 2]);
                    o[r][4 * c4 + 3] = fmaf(pv[r], v.w, o[r][4 * c4 + 3]);
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = 4 * ty + r;
        if (row >= nrows) continue;
        const float inv = lrow[row];
        bf16* dst = a.out + (size_t)(i0 + row) * a.ldo + h * D + tx * 16;
#pragma unroll
        for (int c = 0; c < 16; c += 2)
            *reinterpret_cast<uint32_t*>(dst + c) = pack_bf16x2(o[r][c] / inv, o[r][c + 1] / inv);
    }
}

template <typename K, typename... Args>
cudaError_t launch(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int RMAX>
cudaError_t launch_decode_t(const AttnArgs& a, cudaStream_t st, bool pdl) {
    const size_t smem = sizeof(DecSmem<RMAX>);
    static bool set = false;
    if (!set) {
        cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<RMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        set = true;
    }
    return launch(attn_decode_kernel<RMAX>, dim3(a.Hkv, a.nsplit), dim3(128), smem, st, pdl, a);
}

}  // namespace

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
    const int R = (a.Hq / a.Hkv) * a.S;
    if (a.S < 1 || a.S > 8 || a.nsplit < 1) return cudaErrorInvalidValue;
    if (R <= 8) return launch_decode_t<8>(a, st, pdl);
    if (R <= 16) return launch_decode_t<16>(a, st, pdl);
    if (R <= 32) return launch_decode_t<32>(a, st, pdl);
    if (R <= 64) return launch_decode_t<64>(a, st, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t launch_qk_norm_rope_kvwrite(const AttnArgs& a, bf16* qout, cudaStream_t st) {
    const int items = a.S * (a.Hq + 2 * a.Hkv);
    return launch(qk_norm_rope_kvwrite_kernel, dim3((items + 3) / 4), dim3(128), 0, st, true, a, qout);
}

cudaError_t launch_attn_prefill(const AttnArgs& a, const bf16* qroped, cudaStream_t st) {
    const size_t smem = (size_t)(PQ * QLD + PK * KLD + PK * VLD + PQ * PLD + 3 * PQ) * sizeof(float);
    static bool set = false;
    if (!set) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        set = true;
    }
    return launch(attn_prefill_kernel, dim3(a.Hq, (a.S + PQ - 1) / PQ), dim3(128), smem, st, true, a, qroped);
}

}  // namespace qw
