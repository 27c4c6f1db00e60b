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
#include <map>
#include <mutex>
#include <tuple>

#include <cuda_fp16.h>

#include "kernels.h"
#include "qmm_epi.cuh"
#include "smem_attr.h"
#include "tma_map.h"

namespace qw {
namespace {



constexpr int CG = 4;               // groups per chunk (256 inputs)
constexpr int XS_BLOCK_WORDS = 36;  // one (group, column) block: 4 quads x 8 words + 4 pad words

struct Tile {
    const uint32_t* w;
    const bf16* s;
    const bf16* b;
    int row0;
    int nrows;
};

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

// Stage 16 activations (optionally RMS-normalised, rounded to bf16 like the
// reference's rms_norm output) as fp16 in the decode GEMV's fragment order:
// dst[0..3] = even-chain pairs (x0,x4),(x2,x6),(x8,x12),(x10,x14),
// dst[4..7] = odd-chain pairs  (x1,x5),(x3,x7),(x9,x13),(x11,x15).
// bf16 -> fp16 is exact for |x| >= 2^-14; the even / odd sums are taken over
// the converted values so they match what the tensor cores multiply.
QW_DEV void stage16_f16(const bf16* src, const bf16* normw, float r, uint32_t* dst, float& se, float& so) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    const uint4 u0 = s4[0], u1 = s4[1];
    const uint32_t X[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    uint32_t W8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (normw) {
        const uint4* w4 = reinterpret_cast<const uint4*>(normw);
        const uint4 v0 = w4[0], v1 = w4[1];
        W8[0] = v0.x; W8[1] = v0.y; W8[2] = v0.z; W8[3] = v0.w;
        W8[4] = v1.x; W8[5] = v1.y; W8[6] = v1.z; W8[7] = v1.w;
    }
    uint32_t F[8];
    se = 0.f;
    so = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float lo = bits_lo_f(X[i]), hi = bits_hi_f(X[i]);
        if (normw) {
            lo = bfr(__fmul_rn(__fmul_rn(lo, r), bits_lo_f(W8[i])));
            hi = bfr(__fmul_rn(__fmul_rn(hi, r), bits_hi_f(W8[i])));
        }
        const __half2 h = __floats2half2_rn(lo, hi);
        const float2 back = __half22float2(h);
        se += back.x;
        so += back.y;
        F[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    d4[0] = make_uint4(prmt(F[0], F[2], 0x5410), prmt(F[1], F[3], 0x5410), prmt(F[4], F[6], 0x5410),
                       prmt(F[5], F[7], 0x5410));
    d4[1] = make_uint4(prmt(F[0], F[2], 0x7632), prmt(F[1], F[3], 0x7632), prmt(F[4], F[6], 0x7632),
                       prmt(F[5], F[7], 0x7632));
}

// ===========================================================================
// Decode / verify GEMV: M <= 8 activation rows.
// CTA = RT 16-row mma tiles (RT = 2 pairs gate and up rows for the SwiGLU
// epilogue) over the full K.  At kernel start, before waiting on the previous
// kernel, every thread issues 16-byte asynchronous copies of the CTA's weight
// slab, scales and biases into shared memory (consecutive threads copy
// consecutive chunks of a row), one commit group per 8-group stage, so all of
// the CTA's bytes are in flight at once.  Rows are padded to a stride of 8 mod
// 32 words, which makes the fragment loads (lane g,t reads words 2t..2t+1 of
// rows g and g+8) bank-conflict free.  While the weights land, the CTA stages
// its (RMS-normalised) activations in permuted fragment order together with
// per-group sums.  Warps take two groups at a time (independent mma chains);
// their partial sums are reduced in shared memory in a fixed order.
// ===========================================================================
struct GvLayout {
    int nst, rs, ngp;
    unsigned off_sb, off_x, off_xsum, off_red, total;
};

__host__ __device__ inline GvLayout gv_layout(int KG, int M, int RT, int NW) {
    GvLayout L;
    L.nst = (KG + 7) / 8;
    const int kw = KG * 8;
    L.rs = kw + ((8 - (kw % 32)) + 32) % 32;
    L.ngp = (KG + 7) & ~7;
    const int rows = 16 * RT;
    L.off_sb = (unsigned)rows * L.rs * 4u;
    L.off_x = L.off_sb + (unsigned)rows * L.ngp * 4u;
    L.off_xsum = L.off_x + (unsigned)KG * M * XS_BLOCK_WORDS * 4u;
    L.off_red = L.off_xsum + (unsigned)KG * 16 * 4u;
    // rnorm[8] + pad[32], per-warp partials [NW][RT*4*32]
    L.total = L.off_red + (8 + 32 + NW * RT * 128) * 4;
    return L;
}

// cp.async.wait_group needs an immediate operand
QW_DEV void cp_async_wait_dyn(int n) {
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        case 6: cp_async_wait<6>(); break;
        default: cp_async_wait<7>(); break;
    }
}

template <int RT, int NW, bool SB_VEC>
__global__ void __launch_bounds__(NW * 32) qgemv_kernel(const QmmArgs a) {
    constexpr int NT = NW * 32;
    extern __shared__ __align__(128) unsigned char smraw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int rb = blockIdx.x;
    const int M = a.M, K = a.K, KW = K / 8, KG = K / 64;
    const GvLayout L = gv_layout(KG, M, RT, NW);

    uint32_t* W = reinterpret_cast<uint32_t*>(smraw);
    uint16_t* Ssm = reinterpret_cast<uint16_t*>(smraw + L.off_sb);
    uint16_t* Bsm = Ssm + 16 * RT * L.ngp;
    uint32_t* xs = reinterpret_cast<uint32_t*>(smraw + L.off_x);
    float* xsum = reinterpret_cast<float*>(smraw + L.off_xsum);  // [KG][even, odd][8 columns]
    float* rnorm = reinterpret_cast<float*>(smraw + L.off_red);
    float* wred = rnorm + 8 + 32;  // [NW][RT*128]

    // tiles of this CTA
    int si = 0;
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (i < a.nseg && rb >= a.seg[i].rb0) si = i;
    const int lrb = rb - a.seg[si].rb0;
    Tile tl[RT];
    if (RT == 2) {
        tl[0] = Tile{a.seg[0].w, a.seg[0].s, a.seg[0].b, lrb * 16, a.seg[0].n};
        tl[RT - 1] = Tile{a.seg[1].w, a.seg[1].s, a.seg[1].b, lrb * 16, a.seg[1].n};
    } else {
        const QSeg& sg = a.seg[si];
        tl[0] = Tile{sg.w, sg.s, sg.b, lrb * 16, sg.n};
    }

    // Static weights: the whole slab goes in flight before the wait on the
    // previous kernel (programmatic dependent launch).  Weights the previous
    // kernel may write (a.weights_after_wait): L2 prefetch hints before the
    // wait, the copies after it.  Rows past n are left unloaded; their results
    // are never stored.
    const bool after_wait = a.weights_after_wait != 0;
    if (after_wait) {
        if ((int)threadIdx.x < RT) {
            const Tile& tt = tl[threadIdx.x];
            const int nr = min(16, tt.nrows - tt.row0);
            if (nr > 0) {
                prefetch_l2_range(tt.w + (size_t)tt.row0 * KW, (size_t)nr * KW * 4);
                prefetch_l2_range(tt.s + (size_t)tt.row0 * KG, (size_t)nr * KG * 2);
                prefetch_l2_range(tt.b + (size_t)tt.row0 * KG, (size_t)nr * KG * 2);
            }
        }
        // trigger only after the wait: one programmatic launch ahead at most
        pdl_wait();
        pdl_launch_dependents();
    }
    if (KG % 8 == 0) {
        // every stage has 8 groups = 16 chunks of 16 bytes per row: fixed
        // per-thread (row, chunk) slots, advanced by 64 words per stage
        constexpr int CPT = (16 * RT * 16) / NT;
        const uint32_t* src[CPT];
        uint32_t* dst[CPT];
        bool ok[CPT];
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int u = threadIdx.x + i * NT;
            const int r = u >> 4, c = u & 15;
            const int rt = r >> 4, row = tl[rt].row0 + (r & 15);
            ok[i] = row < tl[rt].nrows;
            src[i] = tl[rt].w + (size_t)(ok[i] ? row : 0) * KW + c * 4;
            dst[i] = W + r * L.rs + c * 4;
        }
        for (int s = 0; s < L.nst; ++s) {
#pragma unroll
            for (int i = 0; i < CPT; ++i)
                if (ok[i]) cp_async16(dst[i] + s * 64, src[i] + (size_t)s * 64);
            if (SB_VEC && s == 0) {
                const int nch2 = KG / 8;  // 16-byte chunks of a scale row
                for (int u = threadIdx.x; u < 2 * 16 * RT * nch2; u += NT) {
                    const int which = u / (16 * RT * nch2), rem = u - which * 16 * RT * nch2;
                    const int r = rem / nch2, c = rem - r * nch2;
                    const int rt = r >> 4, row = tl[rt].row0 + (r & 15);
                    if (row < tl[rt].nrows)
                        cp_async16((which ? Bsm : Ssm) + r * L.ngp + c * 8,
                                   (which ? tl[rt].b : tl[rt].s) + (size_t)row * KG + c * 8);
                }
            }
            cp_async_commit();
        }
    } else {
        for (int s = 0; s < L.nst; ++s) {
            const int gs0 = 8 * s, gsn = min(8, KG - gs0);
            const int nch = gsn * 2;
            for (int u = threadIdx.x; u < 16 * RT * nch; u += NT) {
                const int r = u / nch, c = u - r * nch;
                const int rt = r >> 4, row = tl[rt].row0 + (r & 15);
                if (row < tl[rt].nrows)
                    cp_async16(W + r * L.rs + gs0 * 8 + c * 4, tl[rt].w + (size_t)row * KW + (size_t)gs0 * 8 + c * 4);
            }
            cp_async_commit();
        }
    }
    if (!SB_VEC) {
        for (int i = threadIdx.x; i < 16 * RT * KG; i += NT) {
            const int r = i / KG, gl = i - r * KG;
            const int rt = r >> 4, row = tl[rt].row0 + (r & 15);
            uint16_t sv = 0, bv = 0;
            if (row < tl[rt].nrows) {
                sv = reinterpret_cast<const uint16_t*>(tl[rt].s)[(size_t)row * KG + gl];
                bv = reinterpret_cast<const uint16_t*>(tl[rt].b)[(size_t)row * KG + gl];
            }
            Ssm[r * L.ngp + gl] = sv;
            Bsm[r * L.ngp + gl] = bv;
        }
    }
    if (!after_wait) {
        pdl_launch_dependents();
        pdl_wait();
    }

    if (a.norm_w) {
        // sum of squares of every activation row in one pass
        float ss[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) ss[m] = 0.f;
        for (int k = threadIdx.x * 8; k < K; k += NT * 8) {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                if (m < M) {
                    const uint4 u = *reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + k);
                    const uint32_t X[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float lo = bits_lo_f(X[i]), hi = bits_hi_f(X[i]);
                        ss[m] += lo * lo + hi * hi;
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m < M) {
                const float v = warp_sum(ss[m]);
                if (lane == 0) wred[m * NW + warp] = v;
            }
        }
        __syncthreads();
        if (threadIdx.x < M) {
            float tot = 0.f;
            for (int w = 0; w < NW; ++w) tot += wred[threadIdx.x * NW + w];
            rnorm[threadIdx.x] = 1.0f / sqrtf(tot / (float)K + a.eps);
        }
        __syncthreads();
    }
    {
        // stage activations and even / odd group sums; uniform trip count so
        // every lane takes part in the quad shuffles
        const int units = KG * M * 4;
        for (int u0 = 0; u0 < units; u0 += NT) {
            const int u = u0 + threadIdx.x;
            float se = 0.f, so = 0.f;
            int gl = 0, m = 0, tt = 0;
            if (u < units) {
                gl = u / (M * 4);
                const int rem = u - gl * M * 4;
                m = rem >> 2;
                tt = rem & 3;
                const int k = gl * 64 + 16 * tt;
                stage16_f16(a.x + (size_t)m * a.ldx + k, a.norm_w ? a.norm_w + k : nullptr,
                            a.norm_w ? rnorm[m] : 1.f, xs + (size_t)(gl * M + m) * XS_BLOCK_WORDS + tt * 8, se, so);
            }
            se += __shfl_xor_sync(0xffffffffu, se, 1);
            se += __shfl_xor_sync(0xffffffffu, se, 2);
            so += __shfl_xor_sync(0xffffffffu, so, 1);
            so += __shfl_xor_sync(0xffffffffu, so, 2);
            if (u < units && tt == 0) {
                xsum[gl * 16 + m] = se;
                xsum[gl * 16 + 8 + m] = so;
            }
        }
    }

    float acc[RT][4], bacc[RT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[rt][e] = bacc[rt][e] = 0.f;

    // per-lane bases: rows g / g+8 of every tile, activation column g
    const uint32_t* xb = xs + g * XS_BLOCK_WORDS + t * 8;
    const int xstride = M * XS_BLOCK_WORDS;
    const bool has_col = g < M;

    auto do_group = [&](int gl) {
        uint4 be = make_uint4(0u, 0u, 0u, 0u), bo = be;
        if (has_col) {
            const uint4* p = reinterpret_cast<const uint4*>(xb + gl * xstride);
            be = p[0];
            bo = p[1];
        }
        const float2 xe = *reinterpret_cast<const float2*>(xsum + gl * 16 + 2 * t);
        const float2 xo = *reinterpret_cast<const float2*>(xsum + gl * 16 + 8 + 2 * t);
        const float xt0 = xe.x + xo.x, xt1 = xe.y + xo.y;
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
            const int r0 = rt * 16 + g;
            const uint2 wa = *reinterpret_cast<const uint2*>(W + r0 * L.rs + gl * 8 + 2 * t);
            const uint2 wb = *reinterpret_cast<const uint2*>(W + (r0 + 8) * L.rs + gl * 8 + 2 * t);
            const uint32_t wa8x = wa.x >> 8, wb8x = wb.x >> 8, wa8y = wa.y >> 8, wb8y = wb.y >> 8;
            float ce[4], co[4];
            mma_f16(ce, nib_even(wa.x), nib_even(wb.x), nib_even(wa8x), nib_even(wb8x), be.x, be.y, zero4);
            mma_f16(co, nib_odd(wa.x), nib_odd(wb.x), nib_odd(wa8x), nib_odd(wb8x), bo.x, bo.y, zero4);
            mma_f16(ce, nib_even(wa.y), nib_even(wb.y), nib_even(wa8y), nib_even(wb8y), be.z, be.w, ce);
            mma_f16(co, nib_odd(wa.y), nib_odd(wb.y), nib_odd(wa8y), nib_odd(wb8y), bo.z, bo.w, co);
            // 2^24 undoes the subnormal encoding of the nibbles (exact: a power of two)
            const float s0 = u16_to_f(Ssm[r0 * L.ngp + gl]) * QW_NIB_SCALE;
            const float s1 = u16_to_f(Ssm[(r0 + 8) * L.ngp + gl]) * QW_NIB_SCALE;
            const float b0 = u16_to_f(Bsm[r0 * L.ngp + gl]), b1 = u16_to_f(Bsm[(r0 + 8) * L.ngp + gl]);
            // sum q*x = ce + co/16 (odd nibbles entered as 16q)
            acc[rt][0] = fmaf(s0, fmaf(co[0], 0.0625f, ce[0]), acc[rt][0]);
            acc[rt][1] = fmaf(s0, fmaf(co[1], 0.0625f, ce[1]), acc[rt][1]);
            acc[rt][2] = fmaf(s1, fmaf(co[2], 0.0625f, ce[2]), acc[rt][2]);
            acc[rt][3] = fmaf(s1, fmaf(co[3], 0.0625f, ce[3]), acc[rt][3]);
            bacc[rt][0] = fmaf(b0, xt0, bacc[rt][0]);
            bacc[rt][1] = fmaf(b0, xt1, bacc[rt][1]);
            bacc[rt][2] = fmaf(b1, xt0, bacc[rt][2]);
            bacc[rt][3] = fmaf(b1, xt1, bacc[rt][3]);
        }
    };

    for (int s = 0; s < L.nst; ++s) {
        cp_async_wait_dyn(L.nst - 1 - s);
        __syncthreads();
        const int gs0 = 8 * s, gsn = min(8, KG - gs0);
        int gi = warp;
        for (; gi + NW < gsn; gi += 2 * NW) {
            do_group(gs0 + gi);
            do_group(gs0 + gi + NW);
        }
        if (gi < gsn) do_group(gs0 + gi);
    }

    // cross-warp reduction in a fixed order
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e) wred[warp * RT * 128 + (rt * 4 + e) * 32 + lane] = acc[rt][e] + bacc[rt][e];
    __syncthreads();
    if (warp != 0) return;
    float v[RT][4];
#pragma unroll
    for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float sum = 0.f;
            for (int w = 0; w < NW; ++w) sum += wred[w * RT * 128 + (rt * 4 + e) * 32 + lane];
            v[rt][e] = sum;
        }

    if (a.epi == EPI_LOGITS) {
        // bf16 logits (optionally stored) and this CTA's (value, index) maximum
        // per activation row; a separate kernel reduces over the row blocks
        unsigned long long best[2] = {0ull, 0ull};
        const QSeg& sg = a.seg[si];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = tl[0].row0 + g + 8 * (e >> 1);
            const int col = 2 * t + (e & 1);
            if (row < tl[0].nrows && col < M) {
                const float l = bfr(v[0][e]);
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
        return;
    }

#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int col = 2 * t + (e & 1);
        if (col >= M) continue;
        const int row = tl[0].row0 + g + 8 * (e >> 1);
        if (row >= tl[0].nrows) continue;
        if (RT == 2)
            store_out(a, si, EPI_SWIGLU, 0, row, col, v[0][e], v[RT - 1][e]);
        else
            store_out(a, si, a.epi, row, 0, col, v[0][e], 0.f);
    }
    if (a.epi == EPI_F32_PUSH) {
        // arrival (acquire-release): the last CTA's system-scope release then
        // carries every CTA's peer stores to the ranks' flags
        __syncwarp();
        if (lane == 0) {
            unsigned old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.push.ctr) : "memory");
            if (old == gridDim.x - 1) {
                const unsigned ep = *a.push.epoch + 1u;
                for (int q = 0; q < a.push.n; ++q)
                    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.push.flag[q]), "r"(ep) : "memory");
                *a.push.ctr = 0u;
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

// ===========================================================================
// Streaming decode GEMV for the standalone op (M <= 8, one output segment,
// plain bf16 store, no RMSNorm prologue): persistent CTAs, one per SM, walk
// the 16-row tiles tile = blockIdx.x, blockIdx.x + gridDim.x, ...  Each tile's
// weight rows, scales and biases (MLX layout, rows contiguous) arrive by
// 16-byte asynchronous copies spread over all threads (tracked per slot by an
// mbarrier every thread arrives on) into a ring of `ns` tile slots, so a CTA keeps ns tiles in flight while it computes;
// static weights: the first ns tiles are issued before the programmatic-launch
// wait (with a.weights_after_wait only their L2 prefetch hints are).  Activations are staged once per
// CTA (fragment order, as in qgemv_kernel).  Warp w takes the tile's groups
// w, w + 16, ...; the 16 warps' partial sums meet in shared memory in warp
// order (double-buffered: one CTA barrier per tile).
// ===========================================================================
constexpr int GS_NW = 16;
constexpr int GS_NS_MAX = 8;

struct GsLayout {
    unsigned rs, srs, off_s, off_b, stage, off_x, off_xsum, off_red, off_bar, total;
};

__host__ __device__ inline GsLayout gs_layout(int KG, int M, int ns) {
    GsLayout L;
    const int kw = KG * 8;                                // weight words per row
    L.rs = (unsigned)(kw + ((8 - (kw % 32)) + 32) % 32) * 4u;  // row stride = 32 B mod 128 B: conflict-free fragments
    L.srs = (unsigned)((KG * 2 + 15) / 16) * 16u;         // one scale (bias) row
    L.off_s = 16u * L.rs;
    L.off_b = L.off_s + 16u * L.srs;
    L.stage = L.off_b + 16u * L.srs;
    L.off_x = (unsigned)ns * L.stage;
    L.off_xsum = L.off_x + (unsigned)KG * M * XS_BLOCK_WORDS * 4u;
    L.off_red = L.off_xsum + (unsigned)KG * 16u * 4u;
    L.off_bar = L.off_red + 2u * GS_NW * 128u * 4u;
    L.total = L.off_bar + GS_NS_MAX * 8u;
    return L;
}

__global__ void __launch_bounds__(GS_NW * 32, 1) qgemv_stream_kernel(const __grid_constant__ QmmArgs a, int ns,
                                                                      int ntiles) {
    constexpr int NT = GS_NW * 32;
    extern __shared__ __align__(128) unsigned char smraw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M, K = a.K, KW = K / 8, KG = K / 64;
    const GsLayout L = gs_layout(KG, M, ns);
    const QSeg& sg = a.seg[0];
    uint64_t* full = reinterpret_cast<uint64_t*>(smraw + L.off_bar);
    uint32_t* xs = reinterpret_cast<uint32_t*>(smraw + L.off_x);
    float* xsum = reinterpret_cast<float*>(smraw + L.off_xsum);  // [KG][even, odd][8 columns]
    float* red = reinterpret_cast<float*>(smraw + L.off_red);    // [2][GS_NW][4][32]

    // every thread: its 16-byte chunks of tile `tile` (consecutive threads take
    // consecutive chunks of a row) into ring slot `slot`, then one arrival on
    // the slot's barrier once they have landed (the barrier expects NT)
    auto issue = [&](int tile, int slot) {
        const int row0 = tile * 16;
        const int nr = min(16, sg.n - row0);
        unsigned char* base = smraw + (size_t)slot * L.stage;
        const int cw = KW / 4, cs = KG / 8;  // 16-byte chunks per weight row, per scale (bias) row
        const int per_row = cw + 2 * cs;
        for (int c = threadIdx.x; c < nr * per_row; c += NT) {
            const int r = c / per_row, j = c - r * per_row;
            const size_t row = (size_t)row0 + r;
            if (j < cw)
                cp_async16(base + r * L.rs + j * 16, sg.w + row * KW + j * 4);
            else if (j < cw + cs)
                cp_async16(base + L.off_s + r * L.srs + (j - cw) * 16, sg.s + row * KG + (j - cw) * 8);
            else
                cp_async16(base + L.off_b + r * L.srs + (j - cw - cs) * 16, sg.b + row * KG + (j - cw - cs) * 8);
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[slot])) : "memory");
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < ns; ++i) mbar_init(&full[i], NT);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue_first = [&]() {
        for (int i = 0; i < ns; ++i) {
            const int tile = blockIdx.x + i * gridDim.x;
            if (tile < ntiles) issue(tile, i);
        }
    };
    if (a.weights_after_wait) {
        // weights the previous kernel may write: L2 hints only before the wait
        const int tile = blockIdx.x + (int)threadIdx.x * gridDim.x;
        if ((int)threadIdx.x < ns && tile < ntiles) {
            const int row0 = tile * 16, nr = min(16, sg.n - row0);
            prefetch_l2_range(sg.w + (size_t)row0 * KW, (size_t)nr * KW * 4);
            prefetch_l2_range(sg.s + (size_t)row0 * KG, (size_t)nr * KG * 2);
            prefetch_l2_range(sg.b + (size_t)row0 * KG, (size_t)nr * KG * 2);
        }
        pdl_wait();
        pdl_launch_dependents();
        issue_first();
    } else {
        issue_first();
        pdl_launch_dependents();
        pdl_wait();
    }

    {
        // activations and even / odd group sums (uniform trip count: every lane
        // takes part in the quad shuffles)
        const int units = KG * M * 4;
        for (int u0 = 0; u0 < units; u0 += NT) {
            const int u = u0 + threadIdx.x;
            float se = 0.f, so = 0.f;
            int gl = 0, m = 0, tt = 0;
            if (u < units) {
                gl = u / (M * 4);
                const int rem = u - gl * M * 4;
                m = rem >> 2;
                tt = rem & 3;
                stage16_f16(a.x + (size_t)m * a.ldx + gl * 64 + 16 * tt, nullptr, 1.f,
                            xs + (size_t)(gl * M + m) * XS_BLOCK_WORDS + tt * 8, se, so);
            }
            se += __shfl_xor_sync(0xffffffffu, se, 1);
            se += __shfl_xor_sync(0xffffffffu, se, 2);
            so += __shfl_xor_sync(0xffffffffu, so, 1);
            so += __shfl_xor_sync(0xffffffffu, so, 2);
            if (u < units && tt == 0) {
                xsum[gl * 16 + m] = se;
                xsum[gl * 16 + 8 + m] = so;
            }
        }
    }
    __syncthreads();

    const uint32_t* xb = xs + g * XS_BLOCK_WORDS + t * 8;
    const int xstride = M * XS_BLOCK_WORDS;
    const bool has_col = g < M;
    const int rsw = (int)(L.rs / 4), srs2 = (int)(L.srs / 2);
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = 0;; ++i) {
        const int tile = blockIdx.x + i * gridDim.x;
        if (tile >= ntiles) break;
        const int slot = i % ns;
        const bool landed = mbar_wait_bounded(&full[slot], (uint32_t)((i / ns) & 1));
        if (!__syncthreads_and(landed)) {
            if (threadIdx.x == 0 && a.err) atomicOr(a.err, QW_DERR_TIMEOUT);
            break;
        }
        const uint32_t* W = reinterpret_cast<const uint32_t*>(smraw + (size_t)slot * L.stage);
        const uint16_t* Ssm = reinterpret_cast<const uint16_t*>(smraw + (size_t)slot * L.stage + L.off_s);
        const uint16_t* Bsm = reinterpret_cast<const uint16_t*>(smraw + (size_t)slot * L.stage + L.off_b);
        float acc[4] = {0.f, 0.f, 0.f, 0.f}, bacc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int gl = warp; gl < KG; gl += GS_NW) {
            uint4 be = make_uint4(0u, 0u, 0u, 0u), bo = be;
            if (has_col) {
                const uint4* p = reinterpret_cast<const uint4*>(xb + gl * xstride);
                be = p[0];
                bo = p[1];
            }
            const float2 xe = *reinterpret_cast<const float2*>(xsum + gl * 16 + 2 * t);
            const float2 xo = *reinterpret_cast<const float2*>(xsum + gl * 16 + 8 + 2 * t);
            const float xt0 = xe.x + xo.x, xt1 = xe.y + xo.y;
            const uint2 wa = *reinterpret_cast<const uint2*>(W + g * rsw + gl * 8 + 2 * t);
            const uint2 wb = *reinterpret_cast<const uint2*>(W + (g + 8) * rsw + gl * 8 + 2 * t);
            const uint32_t wa8x = wa.x >> 8, wb8x = wb.x >> 8, wa8y = wa.y >> 8, wb8y = wb.y >> 8;
            float ce[4], co[4];
            mma_f16(ce, nib_even(wa.x), nib_even(wb.x), nib_even(wa8x), nib_even(wb8x), be.x, be.y, zero4);
            mma_f16(co, nib_odd(wa.x), nib_odd(wb.x), nib_odd(wa8x), nib_odd(wb8x), bo.x, bo.y, zero4);
            mma_f16(ce, nib_even(wa.y), nib_even(wb.y), nib_even(wa8y), nib_even(wb8y), be.z, be.w, ce);
            mma_f16(co, nib_odd(wa.y), nib_odd(wb.y), nib_odd(wa8y), nib_odd(wb8y), bo.z, bo.w, co);
            const float s0 = u16_to_f(Ssm[g * srs2 + gl]) * QW_NIB_SCALE;
            const float s1 = u16_to_f(Ssm[(g + 8) * srs2 + gl]) * QW_NIB_SCALE;
            const float b0 = u16_to_f(Bsm[g * srs2 + gl]), b1 = u16_to_f(Bsm[(g + 8) * srs2 + gl]);
            acc[0] = fmaf(s0, fmaf(co[0], 0.0625f, ce[0]), acc[0]);
            acc[1] = fmaf(s0, fmaf(co[1], 0.0625f, ce[1]), acc[1]);
            acc[2] = fmaf(s1, fmaf(co[2], 0.0625f, ce[2]), acc[2]);
            acc[3] = fmaf(s1, fmaf(co[3], 0.0625f, ce[3]), acc[3]);
            bacc[0] = fmaf(b0, xt0, bacc[0]);
            bacc[1] = fmaf(b0, xt1, bacc[1]);
            bacc[2] = fmaf(b1, xt0, bacc[2]);
            bacc[3] = fmaf(b1, xt1, bacc[3]);
        }
        float* rb = red + (size_t)(i & 1) * GS_NW * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) rb[warp * 128 + e * 32 + lane] = acc[e] + bacc[e];
        __syncthreads();
        // the slot is free (every warp has read it): refill it with tile i + ns
        const int next = tile + ns * (int)gridDim.x;
        if (next < ntiles) issue(next, slot);
        // outputs (row r, column m) of the tile: the 16 warps' sums in warp order
        if ((int)threadIdx.x < 16 * M) {
            const int r = threadIdx.x / M, m = threadIdx.x - r * M;
            const int ln = 4 * (r & 7) + (m >> 1), e = 2 * (r >> 3) + (m & 1);
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < GS_NW; ++w) sum += rb[w * 128 + e * 32 + ln];
            const int row = tile * 16 + r;
            if (row < sg.n) reinterpret_cast<bf16*>(sg.y)[(size_t)m * sg.ldy + row] = f2bf(sum);
        }
    }
}

// ===========================================================================
// Warp-ring decode GEMV for the standalone op (M <= 8, one output segment,
// plain bf16 store or the lm_head's logits with per-tile argmax keys, no
// RMSNorm prologue, K a multiple of 512): persistent CTAs of NW warps (16, or
// 8 / 4 when the staged activations leave no room for 16 rings), one per SM.
// CTA c takes the 16-row tiles [c*T/C, (c+1)*T/C); the CTA's granules -- one
// granule is a stage of 8 groups (512 inputs) of one tile, tile-major -- are
// split into NW equal contiguous ranges, one per warp.
// A warp streams its range through its own ring of `ns` slots, one TMA box
// per operand: the 16 rows' weight words as two 128-byte-wide boxes with the
// 128-byte swizzle, then 16 x 8 scales and 16 x 8 biases; lane 0 issues the
// four loads, one mbarrier per slot counts the bytes.  Tile row pi(i) =
// (i & 8) | (i & 3) << 1 | (i >> 2) & 1 feeds mma row i, which with the
// swizzle makes every fragment load conflict-free.  A tile the warp covers
// whole is stored straight from its accumulators; a tile split between warps
// leaves one partial per warp in shared memory, summed in warp order by its
// first warp after one CTA barrier.  Against qgemv_kernel this removes the
// per-tile activation staging, copy issue, CTA barriers and cross-warp
// reduction, which bound that kernel's issue rate on wide outputs.
// ===========================================================================
constexpr int WR_NS_MAX = 4;
constexpr int WR_SLOT = 5120;  // two 2 KB weight boxes, 256 B scales, 256 B biases, pad to 1 KB

struct WrMaps {
    CUtensorMap w, s, b;
};

struct WrLayout {
    unsigned off_xsum, off_bar, off_part, off_slots, total;
};

// offsets from the dynamic shared memory base rounded up to 1 KB; total
// includes that rounding slack
__host__ __device__ inline WrLayout wr_layout(int KG, int M, int ns, int nw) {
    WrLayout L;
    L.off_xsum = (unsigned)KG * M * XS_BLOCK_WORDS * 4u;
    L.off_bar = L.off_xsum + (unsigned)KG * 16u * 4u;
    L.off_part = L.off_bar + (unsigned)nw * WR_NS_MAX * 8u;
    L.off_slots = (L.off_part + (unsigned)nw * 2u * 512u + 1023u) & ~1023u;
    L.total = L.off_slots + (unsigned)(nw * ns * WR_SLOT) + 1024u;
    return L;
}

QW_DEV int wr_row(int i) { return (i & 8) | ((i & 3) << 1) | ((i >> 2) & 1); }

// Outputs of one 16-row tile from a warp's fragment sums v (lane g, t: mma
// rows g and g + 8 = tile rows wr_row(g), wr_row(g) + 8; columns 2t, 2t + 1):
// bf16 stores, or for EPI_LOGITS the bf16-rounded logits (stored if asked)
// and the tile's per-column maximum key.  Called by all 32 lanes.
QW_DEV void wr_store_tile(const QmmArgs& a, int tile, const float (&v)[4], int lane) {
    const QSeg& sg = a.seg[0];
    const int g = lane >> 2, t = lane & 3;
    const int rbase = tile * 16 + wr_row(g);
    if (a.epi == EPI_LOGITS) {
        unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int row = rbase + 8 * (e >> 1);
            const int col = 2 * t + (e & 1);
            if (row < sg.n && col < a.M) {
                const float l = bfr(v[e]);
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
                if (2 * t + cp < a.M) a.amax_partial[(size_t)tile * a.M + 2 * t + cp] = best[cp];
        }
        return;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int row = rbase + 8 * (e >> 1);
        const int col = 2 * t + (e & 1);
        if (row < sg.n && col < a.M) reinterpret_cast<bf16*>(sg.y)[(size_t)col * sg.ldy + row] = f2bf(v[e]);
    }
}

template <int NW>
__global__ void __launch_bounds__(NW * 32, 1) qgemv_wr_kernel(const __grid_constant__ QmmArgs a,
                                                               const __grid_constant__ WrMaps maps, int ns,
                                                               int ntiles) {
    constexpr int NT = NW * 32;
    extern __shared__ __align__(1024) unsigned char wr_smem_raw[];
    unsigned char* smraw = reinterpret_cast<unsigned char*>(((uintptr_t)wr_smem_raw + 1023) & ~(uintptr_t)1023);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int M = a.M, KG = a.K / 64, S = KG / 8;
    const WrLayout L = wr_layout(KG, M, ns, NW);
    uint32_t* xs = reinterpret_cast<uint32_t*>(smraw);
    float* xsum = reinterpret_cast<float*>(smraw + L.off_xsum);  // [KG][even, odd][8 columns]
    uint64_t* bar0 = reinterpret_cast<uint64_t*>(smraw + L.off_bar);
    uint64_t* bars = bar0 + warp * WR_NS_MAX;
    float* part = reinterpret_cast<float*>(smraw + L.off_part);  // [warp][first, last][4][32]
    unsigned char* ring = smraw + L.off_slots + (size_t)warp * ns * WR_SLOT;

    // the CTA's tiles [t0, t1) and this warp's granules [gb, ge) of them
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x);
    const int t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    const int gc = (t1 - t0) * S;
    const int gb = (int)((long long)warp * gc / NW), ge = (int)((long long)(warp + 1) * gc / NW);

    // granule j (CTA-local) into slot (j - gb) % ns: lane 0 only
    auto issue = [&](int j) {
        const int tl = j / S, s = j - tl * S;
        const int row0 = (t0 + tl) * 16, k = (j - gb) % ns;
        unsigned char* slot = ring + (size_t)k * WR_SLOT;
        mbar_arrive_expect_tx(&bars[k], 4096u + 512u);
        tma_load_2d(slot, &maps.w, s * 64, row0, &bars[k]);
        tma_load_2d(slot + 2048, &maps.w, s * 64 + 32, row0, &bars[k]);
        tma_load_2d(slot + 4096, &maps.s, s * 8, row0, &bars[k]);
        tma_load_2d(slot + 4352, &maps.b, s * 8, row0, &bars[k]);
    };
    if ((int)threadIdx.x < NW * WR_NS_MAX) {
        mbar_init(&bar0[threadIdx.x], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int npre = min(ns, ge - gb);
    if (a.weights_after_wait) {
        // weights the previous kernel may write: L2 hints only before the wait
        if (lane == 0) {
            for (int i = 0; i < npre; ++i) {
                const int j = gb + i, tl = j / S, s = j - tl * S, row0 = (t0 + tl) * 16;
                tma_prefetch_2d(&maps.w, s * 64, row0);
                tma_prefetch_2d(&maps.w, s * 64 + 32, row0);
                tma_prefetch_2d(&maps.s, s * 8, row0);
                tma_prefetch_2d(&maps.b, s * 8, row0);
            }
        }
        pdl_wait();
        pdl_launch_dependents();
        if (lane == 0)
            for (int i = 0; i < npre; ++i) issue(gb + i);
    } else {
        if (lane == 0)
            for (int i = 0; i < npre; ++i) issue(gb + i);
        pdl_launch_dependents();
        pdl_wait();
    }

    {
        // activations and even / odd group sums (uniform trip count: every lane
        // takes part in the quad shuffles)
        const int units = KG * M * 4;
        for (int u0 = 0; u0 < units; u0 += NT) {
            const int u = u0 + threadIdx.x;
            float se = 0.f, so = 0.f;
            int gl = 0, m = 0, tt = 0;
            if (u < units) {
                gl = u / (M * 4);
                const int rem = u - gl * M * 4;
                m = rem >> 2;
                tt = rem & 3;
                stage16_f16(a.x + (size_t)m * a.ldx + gl * 64 + 16 * tt, nullptr, 1.f,
                            xs + (size_t)(gl * M + m) * XS_BLOCK_WORDS + tt * 8, se, so);
            }
            se += __shfl_xor_sync(0xffffffffu, se, 1);
            se += __shfl_xor_sync(0xffffffffu, se, 2);
            so += __shfl_xor_sync(0xffffffffu, so, 1);
            so += __shfl_xor_sync(0xffffffffu, so, 2);
            if (u < units && tt == 0) {
                xsum[gl * 16 + m] = se;
                xsum[gl * 16 + 8 + m] = so;
            }
        }
    }
    __syncthreads();

    const uint32_t* xb = xs + g * XS_BLOCK_WORDS + t * 8;
    const int xstride = M * XS_BLOCK_WORDS;
    const bool has_col = g < M;
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    // this lane's weight words in a slot: tile row r = wr_row(g) (and r + 8,
    // 1 KB further), words 2t, 2t + 1 of group q at 16-byte chunk
    // (2 (q & 3) + t / 2) ^ (r & 7) of the row in box q / 4
    const int r = wr_row(g);
    uint32_t woff[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) woff[qq] = (uint32_t)(r * 128 + (((2 * qq + (t >> 1)) ^ (r & 7)) << 4) + ((t & 1) << 3));
    const int first_tile = gb / S;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, bacc[4] = {0.f, 0.f, 0.f, 0.f};
    int j = gb;
    for (; j < ge; ++j) {
        const int k = (j - gb) % ns;
        const bool landed = mbar_wait_bounded(&bars[k], (uint32_t)(((j - gb) / ns) & 1));
        if (!__all_sync(0xffffffffu, landed)) {
            if (lane == 0 && a.err) atomicOr(a.err, QW_DERR_TIMEOUT);
            break;
        }
        const int tl = j / S, s = j - tl * S;
        const unsigned char* sp = ring + (size_t)k * WR_SLOT;
        const uint16_t* Ssm = reinterpret_cast<const uint16_t*>(sp + 4096);
        const uint16_t* Bsm = Ssm + 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int gl = s * 8 + q;
            uint4 be = make_uint4(0u, 0u, 0u, 0u), bo = be;
            if (has_col) {
                const uint4* p = reinterpret_cast<const uint4*>(xb + gl * xstride);
                be = p[0];
                bo = p[1];
            }
            const float2 xe = *reinterpret_cast<const float2*>(xsum + gl * 16 + 2 * t);
            const float2 xo = *reinterpret_cast<const float2*>(xsum + gl * 16 + 8 + 2 * t);
            const float xt0 = xe.x + xo.x, xt1 = xe.y + xo.y;
            const unsigned char* wbox = sp + (q >> 2) * 2048 + woff[q & 3];
            const uint2 wa = *reinterpret_cast<const uint2*>(wbox);
            const uint2 wb = *reinterpret_cast<const uint2*>(wbox + 1024);
            const uint32_t wa8x = wa.x >> 8, wb8x = wb.x >> 8, wa8y = wa.y >> 8, wb8y = wb.y >> 8;
            float ce[4], co[4];
            mma_f16(ce, nib_even(wa.x), nib_even(wb.x), nib_even(wa8x), nib_even(wb8x), be.x, be.y, zero4);
            mma_f16(co, nib_odd(wa.x), nib_odd(wb.x), nib_odd(wa8x), nib_odd(wb8x), bo.x, bo.y, zero4);
            mma_f16(ce, nib_even(wa.y), nib_even(wb.y), nib_even(wa8y), nib_even(wb8y), be.z, be.w, ce);
            mma_f16(co, nib_odd(wa.y), nib_odd(wb.y), nib_odd(wa8y), nib_odd(wb8y), bo.z, bo.w, co);
            // 2^24 undoes the subnormal encoding of the nibbles (exact: a power of two)
            const float s0 = u16_to_f(Ssm[r * 8 + q]) * QW_NIB_SCALE;
            const float s1 = u16_to_f(Ssm[(r + 8) * 8 + q]) * QW_NIB_SCALE;
            const float b0 = u16_to_f(Bsm[r * 8 + q]), b1 = u16_to_f(Bsm[(r + 8) * 8 + q]);
            acc[0] = fmaf(s0, fmaf(co[0], 0.0625f, ce[0]), acc[0]);
            acc[1] = fmaf(s0, fmaf(co[1], 0.0625f, ce[1]), acc[1]);
            acc[2] = fmaf(s1, fmaf(co[2], 0.0625f, ce[2]), acc[2]);
            acc[3] = fmaf(s1, fmaf(co[3], 0.0625f, ce[3]), acc[3]);
            bacc[0] = fmaf(b0, xt0, bacc[0]);
            bacc[1] = fmaf(b0, xt1, bacc[1]);
            bacc[2] = fmaf(b1, xt0, bacc[2]);
            bacc[3] = fmaf(b1, xt1, bacc[3]);
        }
        // every lane has read the slot: refill it with the granule ns ahead
        __syncwarp();
        if (lane == 0 && j + ns < ge) {
            fence_proxy_async_smem();
            issue(j + ns);
        }
        if (s == S - 1 || j == ge - 1) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[e] = acc[e] + bacc[e];
                acc[e] = bacc[e] = 0.f;
            }
            if (tl * S >= gb && (tl + 1) * S <= ge) {
                wr_store_tile(a, t0 + tl, v, lane);
            } else {
                float* pp = part + (size_t)(warp * 2 + (tl == first_tile ? 0 : 1)) * 128;
#pragma unroll
                for (int e = 0; e < 4; ++e) pp[e * 32 + lane] = v[e];
            }
        }
    }
    if (j < ge) {
        // timed out: let the loads still in flight into this warp's ring land
        // (bounded) before the CTA can exit
        for (int jj = j + 1; jj < min(ge, j + ns); ++jj)
            (void)mbar_wait_bounded(&bars[(jj - gb) % ns], (uint32_t)(((jj - gb) / ns) & 1));
    }
    __syncthreads();
    // tiles split between warps: the first covering warp (whose range ends
    // inside the tile) sums the partials in warp order
    if (ge > gb) {
        const int tl = (ge - 1) / S;
        if (!((tl + 1) * S <= ge) && gb <= tl * S) {
            float v[4];
            const float* pp = part + (size_t)(warp * 2 + (tl == first_tile ? 0 : 1)) * 128;
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = pp[e * 32 + lane];
            // later warps whose ranges start inside the tile hold it as their first tile
            for (int u = warp + 1; u < NW; ++u) {
                const int ub = (int)((long long)u * gc / NW), ue = (int)((long long)(u + 1) * gc / NW);
                if (ub >= (tl + 1) * S) break;
                if (ue > ub) {
                    const float* up = part + (size_t)(u * 2) * 128;
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] += up[e * 32 + lane];
                }
            }
            wr_store_tile(a, t0 + tl, v, lane);
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

template <int RT, int NW>
cudaError_t launch_qgemv_t(const QmmArgs& a, int nrb, size_t smem, cudaStream_t st, bool pdl) {
    cudaError_t e = ensure_max_dyn_smem(qgemv_kernel<RT, NW, true>, 220 * 1024);
    if (e == cudaSuccess) e = ensure_max_dyn_smem(qgemv_kernel<RT, NW, false>, 220 * 1024);
    if (e != cudaSuccess) return e;
    const int KG = a.K / 64;
    if (KG % 8 == 0) return launch_ex(qgemv_kernel<RT, NW, true>, dim3(nrb), dim3(NW * 32), smem, st, pdl, a);
    return launch_ex(qgemv_kernel<RT, NW, false>, dim3(nrb), dim3(NW * 32), smem, st, pdl, a);
}

// The streaming GEMV when it applies (one plain-store segment, no norm, rows
// longer than 4096 inputs -- where one CTA per tile leaves too few CTAs per SM;
// measured on the Qwen3-4B shapes it is slower than qgemv_kernel for K <= 4096
// -- 16-byte aligned rows and at least two tile slots in shared memory);
// cudaErrorNotSupported otherwise.
cudaError_t launch_qgemv_stream(const QmmArgs& a, cudaStream_t st, bool pdl, int num_sms) {
    if (a.nseg != 1 || a.epi != EPI_STORE || a.norm_w || a.M < 1 || a.M > 8 || a.K % 512 != 0 || a.K <= 4096 ||
        num_sms < 1)
        return cudaErrorNotSupported;
    const QSeg& sg = a.seg[0];
    if (sg.n < 1 || ((uintptr_t)sg.w | (uintptr_t)sg.s | (uintptr_t)sg.b) % 16 != 0) return cudaErrorNotSupported;
    const int KG = a.K / 64;
    int dev = 0, dev_smem = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&dev_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    const GsLayout L1 = gs_layout(KG, a.M, 1);
    const long long fixed = (long long)L1.total - L1.stage;
    const int ns = (int)std::min<long long>(GS_NS_MAX, (dev_smem - fixed) / (long long)L1.stage);
    if (ns < 2) return cudaErrorNotSupported;
    const GsLayout L = gs_layout(KG, a.M, ns);
    e = ensure_max_dyn_smem(qgemv_stream_kernel, (int)L.total);
    if (e != cudaSuccess) return e;
    const int ntiles = (sg.n + 15) / 16;
    const int grid = std::min(ntiles, num_sms);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GS_NW * 32);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, qgemv_stream_kernel, a, ns, ntiles);
}

// Tensor maps of one segment for the warp-ring GEMV (weights: 32-word x
// 16-row boxes, 128-byte swizzle; scales, biases: 8 x 16 boxes), cached by
// (weight, scale and bias pointers, rows, K).
static bool wr_maps(const QSeg& sg, int K, WrMaps& out) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, const void*, const void*, int, int>, WrMaps> cache;
    const auto key = std::make_tuple((const void*)sg.w, (const void*)sg.s, (const void*)sg.b, sg.n, K);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return true;
    }
    WrMaps m;
    const int KW = K / 8, KG = K / 64;
    if (!make_map(&m.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, sg.w, KW, sg.n, 32, 16, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&m.s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sg.s, KG, sg.n, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&m.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sg.b, KG, sg.n, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE))
        return false;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    out = m;
    return true;
}

// The warp-ring GEMV when it applies (one segment, plain store or logits, no
// norm, K a multiple of 512, 16-byte aligned operands, at least
// WR_MIN_TILES_PER_SM tiles per SM, two ring slots per warp in shared
// memory); cudaErrorNotSupported otherwise.
constexpr int WR_MIN_TILES_PER_SM = 1;

cudaError_t launch_qgemv_wr(const QmmArgs& a, cudaStream_t st, bool pdl, int num_sms) {
    if (a.nseg != 1 || (a.epi != EPI_STORE && a.epi != EPI_LOGITS) || a.norm_w || a.M < 1 || a.M > 8 ||
        a.K % 512 != 0 || num_sms < 1 || !encode_fn())
        return cudaErrorNotSupported;
    const QSeg& sg = a.seg[0];
    if (sg.n < 1 || ((uintptr_t)sg.w | (uintptr_t)sg.s | (uintptr_t)sg.b) % 16 != 0) return cudaErrorNotSupported;
    const int ntiles = (sg.n + 15) / 16;
    if (ntiles < WR_MIN_TILES_PER_SM * num_sms) return cudaErrorNotSupported;
    const int KG = a.K / 64;
    int dev = 0, dev_smem = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&dev_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    // 16 warps with two ring slots each when they fit beside the staged
    // activations, else 8, else 4
    int nw = 16, ns = 0;
    for (; nw >= 4; nw /= 2) {
        const long long fixed = (long long)wr_layout(KG, a.M, 0, nw).total;
        ns = (int)std::min<long long>(WR_NS_MAX, (dev_smem - fixed) / (long long)(nw * WR_SLOT));
        if (ns >= 2) break;
    }
    if (nw < 4) return cudaErrorNotSupported;
    WrMaps maps;
    if (!wr_maps(sg, a.K, maps)) return cudaErrorNotSupported;
    const WrLayout L = wr_layout(KG, a.M, ns, nw);
    auto kern = nw == 16 ? qgemv_wr_kernel<16> : nw == 8 ? qgemv_wr_kernel<8> : qgemv_wr_kernel<4>;
    e = ensure_max_dyn_smem(kern, (int)L.total);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min(ntiles, num_sms));
    cfg.blockDim = dim3(nw * 32);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a, maps, ns, ntiles);
}

int qgemv_row_blocks(const QmmArgs& a) {
    if (a.epi == EPI_SWIGLU) return (a.seg[0].n + 15) / 16;
    int nrb = 0;
    for (int i = 0; i < a.nseg; ++i) nrb += (a.seg[i].n + 15) / 16;
    return nrb;
}

bool qgemv_fits(const QmmArgs& a) {
    if (a.M < 1 || a.M > 8 || a.K <= 0 || a.K % 64 != 0) return false;
    const int KG = a.K / 64;
    const int RT = a.epi == EPI_SWIGLU ? 2 : 1;
    const int NW = KG > 48 ? 8 : 4;
    return gv_layout(KG, a.M, RT, NW).total <= 220 * 1024;
}

int qgemv_max_k(int M) {
    int best = 0;
    for (int KG = 1; KG <= 4096; ++KG) {
        const int NW = KG > 48 ? 8 : 4;
        if (gv_layout(KG, M, 1, NW).total <= 220 * 1024) best = KG * 64;
    }
    return best;
}

cudaError_t launch_qgemv(QmmArgs a, cudaStream_t st, bool pdl, int num_sms) {
    if (a.M < 1 || a.M > 8 || a.K <= 0 || a.K % 64 != 0 || a.nseg < 1 || a.nseg > 3)
        return cudaErrorInvalidValue;
    {
        // long rows (K > 4096, few tiles per SM): the streaming GEMV; wide
        // outputs: the warp-ring GEMV (measured faster on the Qwen3-4B shapes)
        const cudaError_t es = launch_qgemv_stream(a, st, pdl, num_sms);
        if (es != cudaErrorNotSupported) return es;
        const cudaError_t ew = launch_qgemv_wr(a, st, pdl, num_sms);
        if (ew != cudaErrorNotSupported) return ew;
    }
    const int RT = a.epi == EPI_SWIGLU ? 2 : 1;
    int nrb = 0;
    if (RT == 2) {
        if (a.nseg < 2 || a.seg[0].n != a.seg[1].n) return cudaErrorInvalidValue;
        a.seg[0].rb0 = 0;
        a.seg[1].rb0 = 0;
        a.nseg = 2;
        nrb = (a.seg[0].n + 15) / 16;
    } else {
        for (int i = 0; i < a.nseg; ++i) {
            a.seg[i].rb0 = nrb;
            nrb += (a.seg[i].n + 15) / 16;
        }
    }
    a.nrb = nrb;
    const int KG = a.K / 64;
    // long rows get 8 warps so each warp keeps a short list of groups
    const int NW = KG > 48 ? 8 : 4;
    const GvLayout L = gv_layout(KG, a.M, RT, NW);
    if (L.total > 220 * 1024) return cudaErrorNotSupported;  // no GEMV form fits: the caller takes the GEMM
    if (RT == 2) return NW == 8 ? launch_qgemv_t<2, 8>(a, nrb, L.total, st, pdl) : launch_qgemv_t<2, 4>(a, nrb, L.total, st, pdl);
    return NW == 8 ? launch_qgemv_t<1, 8>(a, nrb, L.total, st, pdl) : launch_qgemv_t<1, 4>(a, nrb, L.total, st, pdl);
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
