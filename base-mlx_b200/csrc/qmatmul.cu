// Quantized matmul y = x . dequant(W)^T for MLX affine 4-bit, group 64 weights.
//
// Replaces mlx_rs::ops::quantized_matmul(x, W, s, b, transpose=true, 64, 4) as
// called from crates/base-mlx-core/src/model/qwen3.rs:30-41 (QLinear) and
// model/kernels.rs:42-44,69-76 (qkv_block / mlp_block).
//
// Both kernels read the MLX layout directly (no repacking): W uint32 [N, K/8]
// (element k at bits 4*(k%8) of word k/8), scales / biases bf16 [N, K/64].
//
// Arithmetic (per output, per group g of 64 inputs):
//     y += s_g * sum_k q_k x_k + b_g * sum_k x_k
// computed on the tensor cores with warp-level mma.m16n8k16 (bf16 in, fp32
// accumulate).  A nibble becomes the bf16 value 128+q with one LOP3
// (nib_pair); the 128*sum(x) excess is removed by seeding the accumulator
// with -128*sum(x), which itself comes from an mma against a constant
// A = 128 (decode) or from the staging pass (prefill).  Every product is
// exact; the per-group scale/bias are applied in fp32.  The accumulator is
// reset per group, so s*q+b never has to be rounded to bf16.
//
// k ordering: lane t of a quad owns elements 16t..16t+15 of each group (words
// 2t and 2t+1 of the row).  nib_pair(w, j) pairs elements (j, j+4) of a word,
// so the activations are permuted the same way (permute16) when they are
// staged into shared memory.
#include <algorithm>

#include "kernels.h"

namespace qw {
namespace {

constexpr int GV_WARPS = 4;
constexpr int GV_THREADS = GV_WARPS * 32;
constexpr int CG = 4;               // groups per chunk (256 inputs)
constexpr int XS_BLOCK_WORDS = 36;  // one (group, column) block: 4 quads x 8 words + 4 pad words

struct Tile {
    const uint32_t* w;
    const bf16* s;
    const bf16* b;
    int row0;
    int nrows;
};

QW_DEV void gv_tiles(const QmmArgs& a, int rb, Tile (&tl)[2], int& si, int& lrb) {
    si = 0;
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (i < a.nseg && rb >= a.seg[i].rb0) si = i;
    lrb = rb - a.seg[si].rb0;
    if (a.epi == EPI_SWIGLU) {
        tl[0] = Tile{a.seg[0].w, a.seg[0].s, a.seg[0].b, lrb * 16, a.seg[0].n};
        tl[1] = Tile{a.seg[1].w, a.seg[1].s, a.seg[1].b, lrb * 16, a.seg[1].n};
    } else {
        const QSeg& sg = a.seg[si];
        tl[0] = Tile{sg.w, sg.s, sg.b, lrb * 32, sg.n};
        tl[1] = Tile{sg.w, sg.s, sg.b, lrb * 32 + 16, sg.n};
    }
}

// Four chained mma over one group for one 16-row tile.  w0/w1: words 2t/2t+1 of
// row g, w2/w3: of row g+8; bq: permuted activations; c seeded with -128*sum(x).
QW_DEV void group_mma(float (&c)[4], uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                      const uint32_t (&bq)[8]) {
    mma_bf16(c, nib_pair(w0, 0), nib_pair(w2, 0), nib_pair(w0, 1), nib_pair(w2, 1), bq[0], bq[1], c);
    mma_bf16(c, nib_pair(w0, 2), nib_pair(w2, 2), nib_pair(w0, 3), nib_pair(w2, 3), bq[2], bq[3], c);
    mma_bf16(c, nib_pair(w1, 0), nib_pair(w3, 0), nib_pair(w1, 1), nib_pair(w3, 1), bq[4], bq[5], c);
    mma_bf16(c, nib_pair(w1, 2), nib_pair(w3, 2), nib_pair(w1, 3), nib_pair(w3, 3), bq[6], bq[7], c);
}

// Stage 16 activations (optionally RMS-normalised) in permuted fragment order.
QW_DEV void stage16(const bf16* src, const bf16* normw, float r, uint32_t* dst, float* sum_out) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4 u0 = s4[0], u1 = s4[1];
    uint32_t X[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    if (normw) {
        const uint4* w4 = reinterpret_cast<const uint4*>(normw);
        uint4 v0 = w4[0], v1 = w4[1];
        uint32_t W[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float lo = __fmul_rn(__fmul_rn(bits_lo_f(X[i]), r), bits_lo_f(W[i]));
            float hi = __fmul_rn(__fmul_rn(bits_hi_f(X[i]), r), bits_hi_f(W[i]));
            X[i] = pack_bf16x2(lo, hi);
        }
    }
    if (sum_out) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s += bits_lo_f(X[i]) + bits_hi_f(X[i]);
        *sum_out = s;
    }
    uint32_t o[8];
    permute16(X, o);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    d4[0] = make_uint4(o[0], o[1], o[2], o[3]);
    d4[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// Final per-element epilogue shared by both kernels (not EPI_LOGITS).
QW_DEV void store_out(const QmmArgs& a, int si, int epi, int row, int feat, int col, float v0, float v1) {
    if (epi == EPI_SWIGLU) {
        const float g = bfr(v0), u = bfr(v1);
        const float sg = bfr(1.0f / (1.0f + expf(-g)));
        const float act = bfr(__fmul_rn(g, sg));
        bf16* y = reinterpret_cast<bf16*>(a.seg[0].y);
        y[(size_t)col * a.seg[0].ldy + feat] = f2bf(__fmul_rn(act, u));
        return;
    }
    const QSeg& sg = a.seg[si];
    const size_t idx = (size_t)col * sg.ldy + row;
    if (epi == EPI_F32) {
        reinterpret_cast<float*>(sg.y)[idx] = v0;
    } else if (epi == EPI_RESID) {
        bf16* y = reinterpret_cast<bf16*>(sg.y);
        y[idx] = f2bf(__fadd_rn(bf2f(y[idx]), bfr(v0)));
    } else {
        reinterpret_cast<bf16*>(sg.y)[idx] = f2bf(v0);
    }
}

// ===========================================================================
// Decode / verify GEMV: M <= 8 activation rows.
// CTA = 32 weight rows (two 16-row mma tiles) x one K slice (gridDim.y splits
// K in units of 8 groups).  At kernel start, before waiting on the previous
// kernel, warp 0 issues bulk copies of the CTA's whole weight slab (row r of
// the slab by lane r, one copy per 8-group stage, one mbarrier per stage) and
// of its scales / biases into shared memory, so every byte the CTA needs is in
// flight at once.  Rows are padded so that a row's stride is 8 mod 32 words:
// the mma fragment loads (lane g,t reads words 2t..2t+1 of rows g and g+8) are
// then bank-conflict free.  Warps take groups of each stage round-robin;
// partial sums are reduced in shared memory, and across K splits by the
// last-arriving CTA (in split order, so the result is deterministic).
// ===========================================================================
struct Gv2Layout {
    int ng, nst, rs, ngp;
    unsigned off_w, off_sb, off_x, off_red, total;
};
constexpr int GV2_MAX_STAGES = 16;  // 128 groups (8192 inputs) per CTA

__host__ __device__ inline Gv2Layout gv2_layout(int ng, int M) {
    Gv2Layout L;
    L.ng = ng;
    L.nst = (ng + 7) / 8;
    const int kw = ng * 8;
    L.rs = kw + ((8 - (kw % 32)) + 32) % 32;
    L.ngp = (ng + 7) & ~7;
    L.off_w = 8 * GV2_MAX_STAGES;
    L.off_sb = L.off_w + 32u * L.rs * 4u;
    L.off_x = L.off_sb + 32u * L.ngp * 4u;
    L.off_red = L.off_x + (unsigned)ng * M * XS_BLOCK_WORDS * 4u;
    L.total = L.off_red + (8 + GV_WARPS * 8 * 32) * 4;
    return L;
}

template <bool SB_BULK>
__global__ void __launch_bounds__(GV_THREADS) qgemv_kernel(const QmmArgs a) {
    extern __shared__ __align__(128) unsigned char smraw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int rb = blockIdx.x, ks = blockIdx.y, nks = gridDim.y;
    const int M = a.M, K = a.K, KW = K / 8, KG = K / 64;
    const int nunits = (KG + 7) / 8;
    const int kg0 = min(KG, 8 * (int)((long long)nunits * ks / nks));
    const int kg1 = min(KG, 8 * (int)((long long)nunits * (ks + 1) / nks));
    const int ng = kg1 - kg0;
    const Gv2Layout L = gv2_layout(ng, M);

    uint64_t* bar = reinterpret_cast<uint64_t*>(smraw);
    uint32_t* W = reinterpret_cast<uint32_t*>(smraw + L.off_w);
    uint16_t* Ssm = reinterpret_cast<uint16_t*>(smraw + L.off_sb);
    uint16_t* Bsm = Ssm + 32 * L.ngp;
    uint32_t* xs = reinterpret_cast<uint32_t*>(smraw + L.off_x);
    float* rnorm = reinterpret_cast<float*>(smraw + L.off_red);
    float* red = rnorm + 8;

    Tile tl[2];
    int si, lrb;
    gv_tiles(a, rb, tl, si, lrb);

    if (threadIdx.x == 0) {
        for (int s = 0; s < L.nst; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Weights are static: put the whole slab in flight before waiting on the
    // previous kernel (programmatic dependent launch).
    if (warp == 0) {
        const int rt = lane >> 4, rr = lane & 15;
        const int row = tl[rt].row0 + rr;
        const bool valid = row < tl[rt].nrows;
        const int nvalid = __popc(__ballot_sync(0xffffffffu, valid));
        for (int s = 0; s < L.nst; ++s) {
            const int gs0 = 8 * s, gsn = min(8, ng - gs0);
            uint32_t bytes = (uint32_t)nvalid * gsn * 32;
            if (SB_BULK && s == 0) bytes += (uint32_t)nvalid * ng * 4;
            if (lane == 0) mbar_arrive_expect_tx(&bar[s], bytes);
            __syncwarp();
            if (valid) {
                bulk_g2s(W + lane * L.rs + gs0 * 8, tl[rt].w + (size_t)row * KW + (size_t)(kg0 + gs0) * 8,
                         (uint32_t)gsn * 32, &bar[s]);
                if (SB_BULK && s == 0) {
                    bulk_g2s(Ssm + lane * L.ngp, tl[rt].s + (size_t)row * KG + kg0, (uint32_t)ng * 2, &bar[0]);
                    bulk_g2s(Bsm + lane * L.ngp, tl[rt].b + (size_t)row * KG + kg0, (uint32_t)ng * 2, &bar[0]);
                }
            }
        }
    }
    if (!SB_BULK) {
        for (int i = threadIdx.x; i < 32 * ng; i += GV_THREADS) {
            const int r = i / ng, gl = i - r * ng;
            const int rt = r >> 4, row = tl[rt].row0 + (r & 15);
            uint16_t sv = 0, bv = 0;
            if (row < tl[rt].nrows) {
                sv = reinterpret_cast<const uint16_t*>(tl[rt].s)[(size_t)row * KG + kg0 + gl];
                bv = reinterpret_cast<const uint16_t*>(tl[rt].b)[(size_t)row * KG + kg0 + gl];
            }
            Ssm[r * L.ngp + gl] = sv;
            Bsm[r * L.ngp + gl] = bv;
        }
    }

    pdl_launch_dependents();
    pdl_wait();

    if (a.norm_w) {
        for (int m = 0; m < M; ++m) {
            float ss = 0.f;
            for (int k = threadIdx.x * 8; k < K; k += GV_THREADS * 8) {
                uint4 u = *reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + k);
                uint32_t X[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float lo = bits_lo_f(X[i]), hi = bits_hi_f(X[i]);
                    ss += lo * lo + hi * hi;
                }
            }
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            if (threadIdx.x == 0) {
                float tot = 0.f;
                for (int w = 0; w < GV_WARPS; ++w) tot += red[w];
                rnorm[m] = 1.0f / sqrtf(tot / (float)K + a.eps);
            }
            __syncthreads();
        }
    }
    {
        const int units = ng * M * 4;
        for (int u = threadIdx.x; u < units; u += GV_THREADS) {
            const int gl = u / (M * 4);
            const int rem = u - gl * M * 4;
            const int m = rem >> 2, tt = rem & 3;
            const int k = (kg0 + gl) * 64 + 16 * tt;
            stage16(a.x + (size_t)m * a.ldx + k, a.norm_w ? a.norm_w + k : nullptr,
                    a.norm_w ? rnorm[m] : 1.f, xs + (size_t)(gl * M + m) * XS_BLOCK_WORDS + tt * 8, nullptr);
        }
    }
    __syncthreads();

    float acc[2][4], bacc[2][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[rt][e] = bacc[rt][e] = 0.f;

    for (int s = 0; s < L.nst; ++s) {
        const bool ok = mbar_wait_bounded(&bar[s], 0);
        if (__syncthreads_or(!ok)) {
            // a transfer never completed: flag it, give the copies another
            // bounded chance to land in this CTA's memory, and leave
            if (threadIdx.x == 0) atomicOr(a.err, QW_DERR_TIMEOUT);
            for (int s2 = s; s2 < L.nst; ++s2) mbar_wait_bounded(&bar[s2], 0);
            return;
        }
        const int gs0 = 8 * s, gsn = min(8, ng - gs0);
        for (int gi = warp; gi < gsn; gi += GV_WARPS) {
            const int gl = gs0 + gi;
            uint32_t bq[8];
            if (g < M) {
                const uint4* p = reinterpret_cast<const uint4*>(xs + (size_t)(gl * M + g) * XS_BLOCK_WORDS + t * 8);
                const uint4 v0 = p[0], v1 = p[1];
                bq[0] = v0.x; bq[1] = v0.y; bq[2] = v0.z; bq[3] = v0.w;
                bq[4] = v1.x; bq[5] = v1.y; bq[6] = v1.z; bq[7] = v1.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) bq[i] = 0u;
            }
            // z = 128 * sum(x) of this group for columns 2t, 2t+1 (rows identical)
            float z[4] = {0.f, 0.f, 0.f, 0.f};
            mma_bf16(z, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, bq[0], bq[1], z);
            mma_bf16(z, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, bq[2], bq[3], z);
            mma_bf16(z, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, bq[4], bq[5], z);
            mma_bf16(z, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, QW_BF16X2_128, bq[6], bq[7], z);
#pragma unroll
            for (int rt = 0; rt < 2; ++rt) {
                const int r0 = rt * 16 + g;
                const uint2 wa = *reinterpret_cast<const uint2*>(W + r0 * L.rs + gl * 8 + 2 * t);
                const uint2 wb = *reinterpret_cast<const uint2*>(W + (r0 + 8) * L.rs + gl * 8 + 2 * t);
                float cc[4] = {-z[0], -z[1], -z[2], -z[3]};
                group_mma(cc, wa.x, wa.y, wb.x, wb.y, bq);
                const float s0 = u16_to_f(Ssm[r0 * L.ngp + gl]), s1 = u16_to_f(Ssm[(r0 + 8) * L.ngp + gl]);
                const float b0 = u16_to_f(Bsm[r0 * L.ngp + gl]), b1 = u16_to_f(Bsm[(r0 + 8) * L.ngp + gl]);
                acc[rt][0] = fmaf(s0, cc[0], acc[rt][0]);
                acc[rt][1] = fmaf(s0, cc[1], acc[rt][1]);
                acc[rt][2] = fmaf(s1, cc[2], acc[rt][2]);
                acc[rt][3] = fmaf(s1, cc[3], acc[rt][3]);
                bacc[rt][0] = fmaf(b0, z[0], bacc[rt][0]);
                bacc[rt][1] = fmaf(b0, z[1], bacc[rt][1]);
                bacc[rt][2] = fmaf(b1, z[2], bacc[rt][2]);
                bacc[rt][3] = fmaf(b1, z[3], bacc[rt][3]);
            }
        }
    }

    // cross-warp reduction (fixed order)
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            red[(warp * 8 + rt * 4 + e) * 32 + lane] = fmaf(bacc[rt][e], 0.0078125f, acc[rt][e]);
    __syncthreads();
    if (warp != 0) return;
    float v[2][4];
#pragma unroll
    for (int rt = 0; rt < 2; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float s = 0.f;
            for (int w = 0; w < GV_WARPS; ++w) s += red[(w * 8 + rt * 4 + e) * 32 + lane];
            v[rt][e] = s;
        }

    if (nks > 1) {
        const size_t pstride = (size_t)a.nrb * 32;
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 2 * t + (e & 1);
                if (col < M)
                    a.partial[((size_t)ks * M + col) * pstride + (size_t)rb * 32 + rt * 16 + g + 8 * (e >> 1)] = v[rt][e];
            }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&a.counters[rb], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != (unsigned)(nks - 1)) return;
        __threadfence();
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 2 * t + (e & 1);
                float s = 0.f;
                if (col < M)
                    for (int k2 = 0; k2 < nks; ++k2)
                        s += __ldcg(&a.partial[((size_t)k2 * M + col) * pstride + (size_t)rb * 32 + rt * 16 + g + 8 * (e >> 1)]);
                v[rt][e] = s;
            }
        if (lane == 0) a.counters[rb] = 0u;
    }

    if (a.epi == EPI_LOGITS) {
        unsigned long long best[2] = {0ull, 0ull};
        const QSeg& sg = a.seg[si];
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = tl[rt].row0 + g + 8 * (e >> 1);
                const int col = 2 * t + (e & 1);
                if (row < tl[rt].nrows && col < M) {
                    const float l = bfr(v[rt][e]);
                    if (a.store_logits) reinterpret_cast<bf16*>(sg.y)[(size_t)col * sg.ldy + row] = f2bf(l);
                    best[e & 1] = umax64(best[e & 1], amax_key(l, (uint32_t)(row + a.amax_row_offset)));
                }
            }
#pragma unroll
        for (int cp = 0; cp < 2; ++cp)
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) best[cp] = umax64(best[cp], __shfl_xor_sync(0xffffffffu, best[cp], o));
        if (g == 0) {
#pragma unroll
            for (int cp = 0; cp < 2; ++cp)
                if (2 * t + cp < M) a.amax_partial[(size_t)rb * M + 2 * t + cp] = best[cp];
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(a.amax_counter, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev != (unsigned)(gridDim.x - 1)) return;
        __threadfence();
        for (int col = 0; col < M; ++col) {
            unsigned long long b = 0ull;
            for (int r = lane; r < (int)gridDim.x; r += 32) b = umax64(b, __ldcg(&a.amax_partial[(size_t)r * M + col]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
            if (lane == 0) {
                a.amax_out[col] = (int)amax_key_index(b);
                if (a.amax_key_out) a.amax_key_out[col] = b;
            }
        }
        if (lane == 0) *a.amax_counter = 0u;
        return;
    }

#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int col = 2 * t + (e & 1);
        if (col >= M) continue;
        if (a.epi == EPI_SWIGLU) {
            const int feat = lrb * 16 + g + 8 * (e >> 1);
            if (feat < a.seg[0].n) store_out(a, si, EPI_SWIGLU, 0, feat, col, v[0][e], v[1][e]);
        } else {
#pragma unroll
            for (int rt = 0; rt < 2; ++rt) {
                const int row = tl[rt].row0 + g + 8 * (e >> 1);
                if (row < tl[rt].nrows) store_out(a, si, a.epi, row, 0, col, v[rt][e], 0.f);
            }
        }
    }
}

// ===========================================================================
// Prefill GEMM: M > 8.  CTA = 4 warps x (16 rows x RT tiles) x 32 columns.
// Activations for a 4-group chunk are staged (permuted, with per-group sums)
// in shared memory; each warp converts its own weight rows in registers.
// ===========================================================================
constexpr int GM_COLS = 32;
constexpr int GM_NT = GM_COLS / 8;

template <int RT>
__global__ void __launch_bounds__(128) qgemm_kernel(const QmmArgs a) {
    __shared__ __align__(16) uint32_t xs[CG * GM_COLS * XS_BLOCK_WORDS];
    __shared__ float xsum[CG * GM_COLS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int rb = blockIdx.x;
    const int c0 = blockIdx.y * GM_COLS;
    const int M = a.M, K = a.K, KW = K / 8, KG = K / 64;

    int si = 0;
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (i < a.nseg && rb >= a.seg[i].rb0) si = i;
    const int lrb = rb - a.seg[si].rb0;
    Tile tl[2];
    if (RT == 2) {
        tl[0] = Tile{a.seg[0].w, a.seg[0].s, a.seg[0].b, lrb * 64 + warp * 16, a.seg[0].n};
        tl[1] = Tile{a.seg[1].w, a.seg[1].s, a.seg[1].b, lrb * 64 + warp * 16, a.seg[1].n};
    } else {
        const QSeg& sg = a.seg[si];
        tl[0] = Tile{sg.w, sg.s, sg.b, lrb * 64 + warp * 16, sg.n};
        tl[1] = tl[0];
    }

    float acc[RT][GM_NT][4], bacc[RT][GM_NT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int nt = 0; nt < GM_NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[rt][nt][e] = bacc[rt][nt][e] = 0.f;

    pdl_wait();
    pdl_launch_dependents();

    const int nchunks = (KG + CG - 1) / CG;
    for (int c = 0; c < nchunks; ++c) {
        const int gb = c * CG;
        const int ng = min(CG, KG - gb);
        // this warp's weights for the chunk (issued before the staging barrier)
        uint2 wv[CG][RT][2];
        uint32_t sbv[CG][RT][2];
#pragma unroll
        for (int gi = 0; gi < CG; ++gi)
#pragma unroll
            for (int rt = 0; rt < RT; ++rt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int row = tl[rt].row0 + g + 8 * h;
                    if (gi < ng && row < tl[rt].nrows) {
                        const size_t r = (size_t)row;
                        wv[gi][rt][h] = *reinterpret_cast<const uint2*>(tl[rt].w + r * KW + (size_t)(gb + gi) * 8 + 2 * t);
                        const uint32_t sv = reinterpret_cast<const unsigned short*>(tl[rt].s)[r * KG + gb + gi];
                        const uint32_t bv = reinterpret_cast<const unsigned short*>(tl[rt].b)[r * KG + gb + gi];
                        sbv[gi][rt][h] = sv | (bv << 16);
                    } else {
                        wv[gi][rt][h] = make_uint2(0u, 0u);
                        sbv[gi][rt][h] = 0u;
                    }
                }
        __syncthreads();
        // stage x[c0 : c0+32, chunk] : 4 groups x 32 cols x 4 quads = 512 units
        for (int u = threadIdx.x; u < CG * GM_COLS * 4; u += 128) {
            const int gl = u / (GM_COLS * 4);
            const int rem = u - gl * GM_COLS * 4;
            const int cl = rem >> 2, tt = rem & 3;
            const int col = c0 + cl;
            float s = 0.f;
            uint32_t* dst = xs + (gl * GM_COLS + cl) * XS_BLOCK_WORDS + tt * 8;
            if (gl < ng && col < M) {
                stage16(a.x + (size_t)col * a.ldx + (gb + gl) * 64 + 16 * tt, nullptr, 1.f, dst, &s);
            } else {
                uint4* d4 = reinterpret_cast<uint4*>(dst);
                d4[0] = make_uint4(0u, 0u, 0u, 0u);
                d4[1] = make_uint4(0u, 0u, 0u, 0u);
            }
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (tt == 0) xsum[gl * GM_COLS + cl] = s;
        }
        __syncthreads();
#pragma unroll
        for (int gi = 0; gi < CG; ++gi) {
            if (gi >= ng) break;
#pragma unroll
            for (int nt = 0; nt < GM_NT; ++nt) {
                const uint4* p = reinterpret_cast<const uint4*>(xs + (gi * GM_COLS + nt * 8 + g) * XS_BLOCK_WORDS + t * 8);
                const uint4 v0 = p[0], v1 = p[1];
                const uint32_t bq[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                const float2 zz = *reinterpret_cast<const float2*>(&xsum[gi * GM_COLS + nt * 8 + 2 * t]);
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    float cc[4] = {-128.f * zz.x, -128.f * zz.y, -128.f * zz.x, -128.f * zz.y};
                    group_mma(cc, wv[gi][rt][0].x, wv[gi][rt][0].y, wv[gi][rt][1].x, wv[gi][rt][1].y, bq);
                    const float s0 = bits_lo_f(sbv[gi][rt][0]), s1 = bits_lo_f(sbv[gi][rt][1]);
                    const float b0 = bits_hi_f(sbv[gi][rt][0]), b1 = bits_hi_f(sbv[gi][rt][1]);
                    acc[rt][nt][0] = fmaf(s0, cc[0], acc[rt][nt][0]);
                    acc[rt][nt][1] = fmaf(s0, cc[1], acc[rt][nt][1]);
                    acc[rt][nt][2] = fmaf(s1, cc[2], acc[rt][nt][2]);
                    acc[rt][nt][3] = fmaf(s1, cc[3], acc[rt][nt][3]);
                    bacc[rt][nt][0] = fmaf(b0, zz.x, bacc[rt][nt][0]);
                    bacc[rt][nt][1] = fmaf(b0, zz.y, bacc[rt][nt][1]);
                    bacc[rt][nt][2] = fmaf(b1, zz.x, bacc[rt][nt][2]);
                    bacc[rt][nt][3] = fmaf(b1, zz.y, bacc[rt][nt][3]);
                }
            }
        }
    }

#pragma unroll
    for (int nt = 0; nt < GM_NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int col = c0 + nt * 8 + 2 * t + (e & 1);
            if (col >= M) continue;
            const int row = tl[0].row0 + g + 8 * (e >> 1);
            if (row >= tl[0].nrows) continue;
            const float v0 = acc[0][nt][e] + bacc[0][nt][e];
            if (RT == 2) {
                const float v1 = acc[RT - 1][nt][e] + bacc[RT - 1][nt][e];
                store_out(a, si, EPI_SWIGLU, 0, row, col, v0, v1);
            } else {
                store_out(a, si, a.epi, row, 0, col, v0, 0.f);
            }
        }
}

template <typename Kern>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                      const QmmArgs& a) {
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
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace

cudaError_t launch_qgemv(QmmArgs a, cudaStream_t st, bool pdl, int num_sms) {
    (void)num_sms;
    if (a.M < 1 || a.M > 8 || a.K <= 0 || a.K % 64 != 0 || a.nseg < 1 || a.nseg > 3)
        return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(qgemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    int nrb = 0;
    if (a.epi == EPI_SWIGLU) {
        if (a.nseg < 2 || a.seg[0].n != a.seg[1].n) return cudaErrorInvalidValue;
        a.seg[0].rb0 = 0;
        a.seg[1].rb0 = 0;
        a.nseg = 2;
        nrb = (a.seg[0].n + 15) / 16;
    } else {
        for (int i = 0; i < a.nseg; ++i) {
            a.seg[i].rb0 = nrb;
            nrb += (a.seg[i].n + 31) / 32;
        }
    }
    a.nrb = nrb;
    const int KG = a.K / 64;
    const int nunits = (KG + 7) / 8;
    // Smallest K split whose weight slab (32 rows x ng groups x 36 B with
    // scales/biases) stays near 28 KB, so several CTAs fit per SM and the
    // kernel's whole weight stream can be in flight at once.
    auto max_ng = [&](int ks) { return std::min(KG, 8 * ((nunits + ks - 1) / ks)); };
    int ks = 1;
    while (ks < nunits && ks < 16 && (32 * max_ng(ks) * 36 > 28 * 1024 || max_ng(ks) > 8 * GV2_MAX_STAGES)) ++ks;
    if (ks > 1 && (a.partial == nullptr || a.counters == nullptr || (size_t)ks * a.M * nrb * 32 > a.partial_cap)) {
        ks = 1;
        if (max_ng(1) > 8 * GV2_MAX_STAGES) return cudaErrorInvalidValue;
    }
    const Gv2Layout L = gv2_layout(max_ng(ks), a.M);
    if (L.total > 200 * 1024) return cudaErrorInvalidValue;
    if (KG % 8 == 0) return launch_ex(qgemv_kernel<true>, dim3(nrb, ks), dim3(GV_THREADS), L.total, st, pdl, a);
    return launch_ex(qgemv_kernel<false>, dim3(nrb, ks), dim3(GV_THREADS), L.total, st, pdl, a);
}

cudaError_t launch_qgemm(QmmArgs a, cudaStream_t st, int num_sms) {
    (void)num_sms;
    if (a.M < 1 || a.K <= 0 || a.K % 64 != 0 || a.nseg < 1 || a.nseg > 3) return cudaErrorInvalidValue;
    if (a.epi == EPI_LOGITS) return cudaErrorInvalidValue;
    int nrb = 0;
    if (a.epi == EPI_SWIGLU) {
        if (a.nseg < 2 || a.seg[0].n != a.seg[1].n) return cudaErrorInvalidValue;
        a.seg[0].rb0 = a.seg[1].rb0 = 0;
        a.nseg = 2;
        nrb = (a.seg[0].n + 63) / 64;
    } else {
        for (int i = 0; i < a.nseg; ++i) {
            a.seg[i].rb0 = nrb;
            nrb += (a.seg[i].n + 63) / 64;
        }
    }
    a.nrb = nrb;
    dim3 grid(nrb, (a.M + GM_COLS - 1) / GM_COLS);
    if (a.epi == EPI_SWIGLU) return launch_ex(qgemm_kernel<2>, grid, dim3(128), 0, st, true, a);
    return launch_ex(qgemm_kernel<1>, grid, dim3(128), 0, st, true, a);
}

}  // namespace qw
