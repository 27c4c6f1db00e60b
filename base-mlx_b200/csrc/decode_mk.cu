// Persistent decode step: the whole Qwen3 forward for S <= MK_MAX_ROWS rows
// (greedy decode and the speculative verify) in one cooperative launch.
//
// It runs what forward_dev otherwise launches as ~5 kernels per layer
// (crates/base-mlx-core/src/model/qwen3.rs:314-563): the embedding lookup
// (:57-76), per layer RMSNorm -> q|k|v (kernels.rs:28-46), attention with
// q/k norm, RoPE, KV write and GQA over the cache (qwen3.rs:398-518),
// o_proj + residual, RMSNorm -> gate|up -> SiLU*up -> down_proj + residual
// (kernels.rs:55-78), the final norm -> lm_head -> argmax (qwen3.rs:78-91,
// engine.rs:197-201) and the greedy step bookkeeping.
//
// Grid = one CTA per SM (cooperative launch: all CTAs are resident), 16 warps.
// Phases are separated by a grid-wide arrival counter; every wait is bounded
// (2 s of globaltimer), after which the launch sets QW_DERR_TIMEOUT, raises an
// abort flag that makes every other wait return, drains its copies and exits.
//
// Weight stream.  At model load every quantized linear is repacked into
// 576-byte granules (16 rows x 64 inputs).  Bytes 0..511 hold the nibbles so
// that lane l (g = l/4, t = l%4) reads one 16-byte word quad (A0, B0, A1, B1)
// that yields, with one shift and four LOP3 per word, the A fragments of the
// group's four mma.m16n8k16 k-steps: steps 0 and 2 take (w & 0x000F000F) |
// 0x64006400 (fp16 1024 + q), steps 1 and 3 take (w & 0x00F000F0) | 0x64006400
// (1024 + 16q), each on two accumulator chains seeded with -1024 * sum(x).
// Bytes 512..575 hold the 16 rows' bf16 scales and biases, 8 bytes per row
// pair (g, g+8).  Work is split stream-K style: every CTA owns an equal
// contiguous range of a phase's (tile, group) pairs and every warp an equal
// contiguous sixteenth of it; tiles split between CTAs are finished by the
// last CTA to arrive, summing partials in CTA order (results do not depend on
// arrival order or on the number of rows).
// Each warp streams its own granule sequence -- across tile, phase and layer
// boundaries, since weights never depend on activations -- through a private
// ring of shared-memory slots with 16-byte cp.async copies, `depth` granules
// ahead of the one it computes, so HBM keeps streaming while the CTA waits at
// a phase barrier.  Copies are committed two granules per group: the fixed
// cost of a commit/wait pair per granule held a copy-only stream near half
// the HBM rate.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "attn_decode.cuh"
#include "model.h"

namespace qw {

namespace {

constexpr int MK_NW = 16;
constexpr int MK_NT = MK_NW * 32;
constexpr int GR_BYTES = 576;  // one granule: 512 B nibbles + 64 B scales/biases
// The GEMV phases stage their activations past the head of the shared union,
// which holds the attention tile mbarriers (attn::DecSmem::tbar, written by
// asynchronous cp.async arrivals): staged data never shares bytes with a
// barrier that an arrival could still update.
constexpr size_t MK_UNI_RESERVED = 128;
constexpr int XW = 36;         // words per (group, column) block of staged activations (32 + 4 pad)
constexpr int SEEDF = 8;       // floats per (group, quad t) seed entry
constexpr unsigned long long MK_TIMEOUT_NS = 2000000000ull;

enum { K_QKV = 0, K_O = 1, K_GU = 2, K_DOWN = 3 };

struct MkLin {
    const unsigned char* w;  // packed granules, tile-major, then group, then sub-tile
    int n_tiles;             // 16-row tiles (gate|up: pair tiles)
    int KG;                  // 64-wide groups along K
    int R16;                 // sub-tiles per tile (1, or 2 for gate|up)
    int seg_stride;          // bound on the tile segments of one warp's range
};

struct MkLayer {
    MkLin lin[4];
    const bf16 *in_norm, *post_norm, *q_norm, *k_norm;
};

struct MkArgs {
    const MkLayer* layers;
    int L;
    MkLin lm;
    const bf16* final_norm;
    const uint32_t* emb_w;
    const bf16* emb_s;
    const bf16* emb_b;
    const int* ids;
    int M, H, I, QD, KD, V;
    float eps;
    bf16 *x, *q, *k, *v, *attn, *mlp;
    AttnArgs aa;  // per-layer fields (norm weights, cache pointers) are set in the kernel
    size_t kv_layer_elems;
    bf16 *kc0, *vc0;
    int logits_rows;  // 0: no lm_head, 1: last row, M: every row
    bf16* logits;
    int store_logits;
    unsigned long long* amax_cta;  // [gridDim.x][8]
    int* argmax;
    int* seq_len;
    StepCtl* ctl;
    int* next_tok;
    int* out;
    const int* gate;
    unsigned* sync;  // [0] phase arrivals, [1] final arrivals, [2] abort flag
    float* part_g;   // [gridDim.x][2][256] partial sums of split tiles
    unsigned* tile_ctr;  // [max tiles] arrivals per split tile (reset by the finisher)
    int* err;
    int depth;       // ring slots per warp (the kernel's DEPTH)
    bf16* trace;     // diagnostics: residual stream after the embedding and every layer, [L + 1][M][H]
    bf16* trace_mid;   // diagnostics: residual after each attention block, [L][M][H]
    bf16* trace_attn;  // diagnostics: attention output of each layer, [L][M][QD]
    unsigned off_union, off_misc, off_tab;
};

struct MkMisc {
    int wft[MK_NW];  // first tile (CTA-local) of each warp's range in the current phase
    float rnorm[8];
    float ssq[MK_NW][8];
    unsigned long long amax[8];
    int bad;
    int last;
};

// ---- device helpers -------------------------------------------------------
QW_DEV unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
QW_DEV void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
QW_DEV unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// mma.m16n8k16 f16 -> f32 without `volatile`, so the compiler can interleave
// the chains of several granules; zero C variant for the first k-step.
QW_DEV void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
QW_DEV void mma_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}
QW_DEV uint32_t lo4(uint32_t w) { return nib_even(w); }  // q * 2^-24 (exact fp16 subnormal)
QW_DEV uint32_t hi4(uint32_t w) { return nib_odd(w); }   // 16q * 2^-24

// Number of GEMV phases in a launch and their descriptors, in stream order:
// layer l -> q|k|v, o, gate|up, down; then lm_head when logits are wanted.
QW_DEV int n_gemv_phases(const MkArgs& a) { return 4 * a.L + (a.logits_rows > 0 ? 1 : 0); }
QW_DEV MkLin phase_lin(const MkArgs& a, int pi) {
    if (pi >= 4 * a.L) return a.lm;
    return a.layers[pi >> 2].lin[pi & 3];
}

// Stream-K partition.  A phase is n_tiles * KG tile-groups (one tile-group =
// the R16 granules of one 64-wide group of one tile).  CTA c owns tile-groups
// [c*N/C, (c+1)*N/C) and warp w of it the w-th sixteenth of that range, so
// every CTA and warp streams the same number of bytes (within one tile-group).
// A tile whose tile-groups are split between CTAs is finished by the last of
// them to arrive, which sums the CTAs' partial sums in CTA order.
QW_DEV int range_lo(int c, int N, int C) { return (int)(((long long)c * N) / C); }
// CTA owning tile-group x
QW_DEV int cta_of(int x, int N, int C) { return (int)(((long long)(x + 1) * C - 1) / N); }

// Per-CTA description of one GEMV phase, built once per launch in shared
// memory so that walking the granule stream needs no global loads.
struct PhaseInfo {
    const unsigned char* w;  // packed granules of the whole linear
    int tg0, tg1;            // this CTA's tile-groups
    int KG, R16;
    int N;                   // tile-groups in the phase
    int seg_stride;
};
static_assert(sizeof(PhaseInfo) == 32, "PhaseInfo layout");

QW_DEV void warp_range(const PhaseInfo& P, int warp, int& wa, int& wb) {
    const int n = P.tg1 - P.tg0;
    wa = P.tg0 + ((warp * n) >> 4);
    wb = P.tg0 + (((warp + 1) * n) >> 4);
}

// Walks a warp's granule sequence: for each phase in order, the warp's
// contiguous range of granules [wa*R16, wb*R16).
struct Cursor {
    const PhaseInfo* tab;
    int np, pi;
    const unsigned char* p;    // next granule
    const unsigned char* end;  // end of the warp's range in phase pi

    QW_DEV void enter(int warp) {
        while (pi < np) {
            const PhaseInfo& P = tab[pi];
            int wa, wb;
            warp_range(P, warp, wa, wb);
            p = P.w + (size_t)wa * P.R16 * GR_BYTES;
            end = P.w + (size_t)wb * P.R16 * GR_BYTES;
            if (p < end) return;
            ++pi;
        }
    }
    QW_DEV void init(const PhaseInfo* t, int n, int warp) {
        tab = t;
        np = n;
        pi = 0;
        enter(warp);
    }
    QW_DEV bool done() const { return pi >= np; }
    QW_DEV void advance(int warp) {
        p += GR_BYTES;
        if (p >= end) {
            ++pi;
            enter(warp);
        }
    }
};

// Issue the copies of the producer cursor's next two granules into the slot
// pair at `dst` (one commit group per pair; fewer granules, or an empty group,
// once the stream has ended).  Every lane walks the cursor in lockstep.
QW_DEV void issue_pair(Cursor& pc, int warp, int lane, unsigned char* dst) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        if (!pc.done()) {
            cp_async16(dst + u * GR_BYTES + 16 * lane, pc.p + 16 * lane);
            if (lane < 4) cp_async16(dst + u * GR_BYTES + 512 + 16 * lane, pc.p + 512 + 16 * lane);
            pc.advance(warp);
        }
    }
    cp_async_commit();
}

// ---- activation staging ----------------------------------------------------
// x' for one GEMV phase: per (group gl, column m) a block of XW words, words
// t*8 + 2j + h = fp16 pair (x[64gl+16j+2t+8h], x[..+1]); per (gl, quad t)
// SEEDF floats {-1024*lo(2t), -1024*lo(2t+1), -1024*hi(2t), -1024*hi(2t+1),
// sum(2t), sum(2t+1)}, lo/hi = sums over k-steps {0,2} / {1,3}.
// Source: rows [row0, row0+Mx) of a bf16 matrix (ld) or of the embedding.
struct StageSrc {
    const bf16* x;     // null -> embedding rows of ids[row0 + m]
    int ld;
    int row0;
    const bf16* norm;  // optional RMSNorm weight
};

QW_DEV void load16(const MkArgs& a, const StageSrc& s, int m, int k, float (&v)[16]) {
    if (s.x) {
        const uint4* p = reinterpret_cast<const uint4*>(s.x + (size_t)(s.row0 + m) * s.ld + k);
        const uint4 u0 = __ldcg(p), u1 = __ldcg(p + 1);
        const uint32_t X[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[2 * i] = bits_lo_f(X[i]);
            v[2 * i + 1] = bits_hi_f(X[i]);
        }
    } else {
        // QEmbedding::lookup: bf16(s * q + b) of the token's row
        int tok = a.ids[s.row0 + m];
        if (tok < 0 || tok >= a.V) tok = 0;
        const int KW = a.H / 8, KG = a.H / 64;
        const uint32_t* wr = a.emb_w + (size_t)tok * KW + k / 8;
        const float sc = u16_to_f(reinterpret_cast<const unsigned short*>(a.emb_s)[(size_t)tok * KG + k / 64]);
        const float bi = u16_to_f(reinterpret_cast<const unsigned short*>(a.emb_b)[(size_t)tok * KG + k / 64]);
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const uint32_t word = wr[wi];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[8 * wi + e] = bfr(fmaf(sc, (float)((word >> (4 * e)) & 0xF), bi));
        }
    }
}

// Convert one unit (16 values of column m, k-step j of group gl) into its
// fragment words and return the sum of the converted values.
QW_DEV float stage_unit(const float (&v)[16], int gl, int m, int j, int Mx, uint32_t* xs) {
    float sum = 0.f;
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        const float2 back = __half22float2(hh);
        sum += back.x + back.y;
        h[i] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    uint32_t* blk = xs + (size_t)(gl * Mx + m) * XW;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        blk[t * 8 + 2 * j] = h[t];          // (x[16j+2t], x[16j+2t+1])
        blk[t * 8 + 2 * j + 1] = h[t + 4];  // (x[16j+2t+8], x[16j+2t+9])
    }
    return sum;
}

// j-quads share (gl, m): lo = steps 0+2, hi = steps 1+3 (every lane of the warp
// takes part in the shuffles).
QW_DEV void stage_seeds(float sum, bool valid, int gl, int m, int j, float* seeds) {
    const float pair = sum + __shfl_xor_sync(0xffffffffu, sum, 2);
    const float tot = pair + __shfl_xor_sync(0xffffffffu, pair, 1);
    if (valid && j < 2) {
        float* e = seeds + (size_t)(gl * 4 + (m >> 1)) * SEEDF;
        e[2 * j + (m & 1)] = -1024.f * pair;  // j = 0: lo, j = 1: hi
        if (j == 0) e[4 + (m & 1)] = tot;
    }
}

QW_DEV void apply_norm(const StageSrc& s, float r, int k, float (&v)[16]) {
    const uint4* wp = reinterpret_cast<const uint4*>(s.norm + k);
    const uint4 w0 = wp[0], w1 = wp[1];
    const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = bfr(__fmul_rn(__fmul_rn(v[2 * i], r), bits_lo_f(W[i])));
        v[2 * i + 1] = bfr(__fmul_rn(__fmul_rn(v[2 * i + 1], r), bits_hi_f(W[i])));
    }
}

// Unit u -> (group, column, k-step); units are ordered (gl, m, j).
QW_DEV void unit_coords(int u, int Mx, int& gl, int& m, int& j) {
    j = u & 3;
    const int gm = u >> 2;
    gl = gm / Mx;
    m = gm - gl * Mx;
}

// The 16 bf16 values of a unit as 8 packed words (the staged values are exact
// bf16: rows of a bf16 matrix or bf16-rounded embedding entries).
QW_DEV void load16_packed(const MkArgs& a, const StageSrc& s, int m, int k, uint32_t (&X)[8]) {
    if (s.x) {
        const uint4* p = reinterpret_cast<const uint4*>(s.x + (size_t)(s.row0 + m) * s.ld + k);
        const uint4 u0 = __ldcg(p), u1 = __ldcg(p + 1);
        X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
        X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
    } else {
        float v[16];
        load16(a, s, m, k, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) X[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    }
}
QW_DEV float sumsq_packed(const uint32_t (&X)[8]) {
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float lo = bits_lo_f(X[i]), hi = bits_hi_f(X[i]);
        q = fmaf(lo, lo, q);
        q = fmaf(hi, hi, q);
    }
    return q;
}
QW_DEV void unpack16(const uint32_t (&X)[8], float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = bits_lo_f(X[i]);
        v[2 * i + 1] = bits_hi_f(X[i]);
    }
}

QW_DEV void stage_acts(const MkArgs& a, const StageSrc& s, int K, int Mx, uint32_t* xs, float* seeds, float* sq,
                       MkMisc& mm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KG = K / 64;
    const int units = KG * Mx * 4;
    if (s.norm && units <= 2 * MK_NT) {
        // RMSNorm in one pass over x: each thread keeps its (at most two) units
        // in registers while the per-row sums of squares are reduced
        uint32_t X0[8], X1[8];
        int gl0 = 0, m0 = 0, j0 = 0, gl1 = 0, m1 = 0, j1 = 0;
        const int u0 = tid, u1 = tid + MK_NT;
        if (u0 < units) {
            unit_coords(u0, Mx, gl0, m0, j0);
            load16_packed(a, s, m0, gl0 * 64 + 16 * j0, X0);
            sq[u0] = sumsq_packed(X0);
        }
        if (u1 < units) {
            unit_coords(u1, Mx, gl1, m1, j1);
            load16_packed(a, s, m1, gl1 * 64 + 16 * j1, X1);
            sq[u1] = sumsq_packed(X1);
        }
        __syncthreads();
        if (warp < Mx) {
            // row `warp`: its KG*4 units, lane-strided, then a fixed shuffle tree
            float q = 0.f;
            for (int i = lane; i < KG * 4; i += 32) q += sq[((i >> 2) * Mx + warp) * 4 + (i & 3)];
            q = warp_sum(q);
            if (lane == 0) mm.rnorm[warp] = 1.0f / sqrtf(q / (float)K + a.eps);
        }
        __syncthreads();
        float sum0 = 0.f, sum1 = 0.f;
        if (u0 < units) {
            float v[16];
            unpack16(X0, v);
            apply_norm(s, mm.rnorm[m0], gl0 * 64 + 16 * j0, v);
            sum0 = stage_unit(v, gl0, m0, j0, Mx, xs);
        }
        stage_seeds(sum0, u0 < units, gl0, m0, j0, seeds);
        if (u1 - lane < units) {  // warp-uniform: some lane of this warp has a unit
            if (u1 < units) {
                float v[16];
                unpack16(X1, v);
                apply_norm(s, mm.rnorm[m1], gl1 * 64 + 16 * j1, v);
                sum1 = stage_unit(v, gl1, m1, j1, Mx, xs);
            }
            stage_seeds(sum1, u1 < units, gl1, m1, j1, seeds);
        }
        return;
    }
    if (s.norm) {
        // RMSNorm statistics: fp32 sum of squares per row
        float ss[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) ss[m] = 0.f;
        for (int k = tid * 16; k < K; k += MK_NT * 16) {
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                if (m < Mx) {
                    float v[16];
                    load16(a, s, m, k, v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) ss[m] = fmaf(v[i], v[i], ss[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m < Mx) {
                const float w = warp_sum(ss[m]);
                if (lane == 0) mm.ssq[warp][m] = w;
            }
        }
        __syncthreads();
        if (tid < Mx) {
            float tot = 0.f;
            for (int w = 0; w < MK_NW; ++w) tot += mm.ssq[w][tid];
            mm.rnorm[tid] = 1.0f / sqrtf(tot / (float)K + a.eps);
        }
        __syncthreads();
    }
    for (int ub = 0; ub < units; ub += MK_NT) {
        const int u = ub + tid;
        float sum = 0.f;
        int gl = 0, m = 0, j = 0;
        if (u < units) {
            unit_coords(u, Mx, gl, m, j);
            const int k = gl * 64 + 16 * j;
            float v[16];
            load16(a, s, m, k, v);
            if (s.norm) apply_norm(s, mm.rnorm[m], k, v);
            sum = stage_unit(v, gl, m, j, Mx, xs);
        }
        stage_seeds(sum, u < units, gl, m, j, seeds);
    }
}

// ---- grid phase barrier ----------------------------------------------------
QW_DEV bool cta_wait(const MkArgs& a, unsigned target, MkMisc& mm) {
    if (threadIdx.x == 0 && !mm.bad) {
        const unsigned long long t0 = globaltimer();
        unsigned it = 0;
        while ((int)(ld_acquire_u32(a.sync) - target) < 0) {
            if ((++it & 31u) == 0) {
                if (*reinterpret_cast<volatile unsigned*>(a.sync + 2)) {
                    mm.bad = 1;
                    break;
                }
                if (globaltimer() - t0 > MK_TIMEOUT_NS) {
                    atomicOr(a.err, QW_DERR_TIMEOUT);
                    atomicExch(a.sync + 2, 1u);
                    mm.bad = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();  // the acquire above, then this barrier, orders every thread's reads
    return !*reinterpret_cast<volatile int*>(&mm.bad);
}
// Block barrier, then one release-add: publishes every thread's earlier writes
// (the barrier orders them before the release, which is cumulative).
QW_DEV void cta_arrive(const MkArgs& a) {
    __syncthreads();
    if (threadIdx.x == 0) red_release_add(a.sync, 1u);
}

// Diagnostics: copy n bf16 values (a multiple of 8) from src to dst.
QW_DEV void trace_copy_n(const bf16* src_, bf16* dst_, int n) {
    const uint4* src = reinterpret_cast<const uint4*>(src_);
    uint4* dst = reinterpret_cast<uint4*>(dst_);
    for (int i = threadIdx.x; i < n / 8; i += MK_NT) dst[i] = __ldcg(src + i);
}
// the residual stream (final for layer l - 1) into trace[l]
QW_DEV void trace_copy(const MkArgs& a, int l) { trace_copy_n(a.x, a.trace + (size_t)l * a.M * a.H, a.M * a.H); }

// Attention items run on the whole CTA (taken by whole CTAs only).
struct BlockSync {
    QW_DEV void operator()() const { __syncthreads(); }
};

// Staged activations of one group for this lane: B fragments of the four
// k-steps and the per-column seed terms.
struct GAct {
    uint4 xa, xb;   // (step 0, step 1) and (step 2, step 3) B fragment pairs
    float z0, z1;   // -(1024 lo + 64 hi) for columns 2t, 2t+1
    float sx0, sx1; // sum(x) for columns 2t, 2t+1
};
QW_DEV GAct load_act(const uint32_t* xs_lane, const float* seeds_lane, int gl, int col_stride) {
    GAct r;
    const uint32_t* xp = xs_lane + (size_t)gl * col_stride;
    r.xa = *reinterpret_cast<const uint4*>(xp);
    r.xb = *reinterpret_cast<const uint4*>(xp + 4);
    const float* sp = seeds_lane + (size_t)gl * 4 * SEEDF;
    const float4 sd = *reinterpret_cast<const float4*>(sp);
    const float2 sx = *reinterpret_cast<const float2*>(sp + 4);
    r.z0 = fmaf(sd.z, 0.0625f, sd.x);
    r.z1 = fmaf(sd.w, 0.0625f, sd.y);
    r.sx0 = sx.x;
    r.sx1 = sx.y;
    return r;
}
// One granule: four mma over the group's k-steps (two chains: 1024+q and
// 1024+16q), then acc += s * sum(q x) + b * sum(x) per row and column.
QW_DEV void granule_mma(const unsigned char* gp, int lane, const GAct& x, float (&acc)[4]) {
    const int g = lane >> 2;
    const uint4 wv = *reinterpret_cast<const uint4*>(gp + 16 * lane);
    const uint2 sb = *reinterpret_cast<const uint2*>(gp + 512 + 8 * g);
    const uint32_t a8 = wv.x >> 8, b8 = wv.y >> 8, c8 = wv.z >> 8, d8 = wv.w >> 8;
    float cl[4], ch[4];
    mma_zero(cl, lo4(wv.x), lo4(a8), lo4(wv.y), lo4(b8), x.xa.x, x.xa.y);
    mma_zero(ch, hi4(wv.x), hi4(a8), hi4(wv.y), hi4(b8), x.xa.z, x.xa.w);
    mma_acc(cl, lo4(wv.z), lo4(c8), lo4(wv.w), lo4(d8), x.xb.x, x.xb.y);
    mma_acc(ch, hi4(wv.z), hi4(c8), hi4(wv.w), hi4(d8), x.xb.z, x.xb.w);
    // the chains hold q*x * 2^-24 (k-steps 0, 2) and 16q*x * 2^-24 (k-steps 1, 3)
    const float s0 = bits_lo_f(sb.x) * QW_NIB_SCALE, b0 = bits_hi_f(sb.x);
    const float s1 = bits_lo_f(sb.y) * QW_NIB_SCALE, b1 = bits_hi_f(sb.y);
    const float s016 = s0 * 0.0625f, s116 = s1 * 0.0625f;
    acc[0] = fmaf(s0, cl[0], fmaf(s016, ch[0], fmaf(b0, x.sx0, acc[0])));
    acc[1] = fmaf(s0, cl[1], fmaf(s016, ch[1], fmaf(b0, x.sx1, acc[1])));
    acc[2] = fmaf(s1, cl[2], fmaf(s116, ch[2], fmaf(b1, x.sx0, acc[2])));
    acc[3] = fmaf(s1, cl[3], fmaf(s116, ch[3], fmaf(b1, x.sx1, acc[3])));
}

// ---- one GEMV phase --------------------------------------------------------
// Computes the CTA's items of phase `pi` from its ring, then the epilogue.
// Epilogue of one output element (tile row `row`, column m) with the final
// fp32 sums v[sub].
template <int KIND>
QW_DEV void store_elem(const MkArgs& a, bool lm, int row, int m, const float (&v)[2], unsigned long long (&best)[8]) {
    if (KIND == K_GU && !lm) {
        const float gv = bfr(v[0]), uv = bfr(v[1]);
        const float sg = bfr(1.0f / (1.0f + expf(-gv)));
        const float act = bfr(__fmul_rn(gv, sg));
        a.mlp[(size_t)m * a.I + row] = f2bf(__fmul_rn(act, uv));
    } else if (lm) {
        const float l = bfr(v[0]);
        if (a.store_logits) a.logits[(size_t)m * a.V + row] = f2bf(l);
        const unsigned long long key = amax_key(l, (uint32_t)row);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j == m) best[j] = umax64(best[j], key);
    } else if (KIND == K_QKV) {
        if (row < a.QD)
            a.q[(size_t)m * a.QD + row] = f2bf(v[0]);
        else if (row < a.QD + a.KD)
            a.k[(size_t)m * a.KD + row - a.QD] = f2bf(v[0]);
        else
            a.v[(size_t)m * a.KD + row - a.QD - a.KD] = f2bf(v[0]);
    } else {
        bf16* y = a.x + (size_t)m * a.H + row;
        *y = f2bf(__fadd_rn(bf2f(__ldcg(y)), bfr(v[0])));
    }
}

// One GEMV phase: each warp computes its granule range from its ring, writing
// one partial per tile segment to shared memory (red: [warp][segment][sub][128]);
// then the CTA reduces the segments of each tile in warp order and either
// stores the outputs (tiles it owns completely) or hands its partial to the
// CTA that finishes a split tile.
template <int KIND, int DEPTH>
QW_DEV void gemv_phase(const MkArgs& a, const PhaseInfo& P, int Mx, uint32_t* xs, float* seeds, float* red,
                       Cursor& pc, unsigned& gpos, unsigned char* ring, bool lm, MkMisc& mm) {
    constexpr int R16 = KIND == K_GU ? 2 : 1;
    constexpr int NS = DEPTH / 2;  // slot pairs per warp, one commit group each
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int KG = P.KG;
    const int seg_stride = P.seg_stride;
    const int mcol = min(g, Mx - 1);
    const int col_stride = Mx * XW;
    const uint32_t* xs_lane = xs + (size_t)mcol * XW + t * 8;
    const float* seeds_lane = seeds + (size_t)t * SEEDF;
    unsigned char* wring = ring + (size_t)warp * DEPTH * GR_BYTES;
    auto gptr = [&](int u) { return wring + (size_t)((gpos + u) & (DEPTH - 1)) * GR_BYTES; };
    // refill the slot pair of chunk c (granules 2c, 2c+1) with the chunk NS ahead
    auto refill = [&](unsigned c) { issue_pair(pc, warp, lane, wring + (size_t)(c % NS) * 2 * GR_BYTES); };

    int wa, wb;
    warp_range(P, warp, wa, wb);
    if (lane == 0) mm.wft[warp] = (wa - P.tg0) / KG;
    int seg = 0;
    for (int tg = wa; tg < wb; ++seg) {
        // one tile segment: tile-groups [tg, se) of tile `tile`
        const int tile = tg / KG;
        const int se = min(wb, (tile + 1) * KG);
        const int gl0 = tg - tile * KG;
        const int ng = (se - tg) * R16;
        float acc[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
        int gi = 0;
        // four granules per step: independent mma chains in flight
        for (; gi + 4 <= ng; gi += 4) {
            // groups newer than the last pair these four granules touch may stay pending
            if ((gpos & 1) == 0)
                cp_async_wait<NS - 2>();
            else
                cp_async_wait<NS - 3>();
            __syncwarp();
            if (R16 == 1) {
                const int gl = gl0 + gi;
                const GAct x0 = load_act(xs_lane, seeds_lane, gl, col_stride);
                const GAct x1 = load_act(xs_lane, seeds_lane, gl + 1, col_stride);
                const GAct x2 = load_act(xs_lane, seeds_lane, gl + 2, col_stride);
                const GAct x3 = load_act(xs_lane, seeds_lane, gl + 3, col_stride);
                granule_mma(gptr(0), lane, x0, acc[0]);
                granule_mma(gptr(1), lane, x1, acc[1]);
                granule_mma(gptr(2), lane, x2, acc[2]);
                granule_mma(gptr(3), lane, x3, acc[3]);
            } else {
                const int gl = gl0 + gi / 2;
                const GAct x0 = load_act(xs_lane, seeds_lane, gl, col_stride);
                const GAct x1 = load_act(xs_lane, seeds_lane, gl + 1, col_stride);
                granule_mma(gptr(0), lane, x0, acc[0]);
                granule_mma(gptr(1), lane, x0, acc[1]);
                granule_mma(gptr(2), lane, x1, acc[2]);
                granule_mma(gptr(3), lane, x1, acc[3]);
            }
            __syncwarp();
            // refill the two pairs whose second granule was just consumed
            if ((gpos & 1) == 0) {
                refill(gpos / 2);
                refill(gpos / 2 + 1);
            } else {
                refill((gpos - 1) / 2);
                refill((gpos + 1) / 2);
            }
            gpos += 4;
        }
        for (; gi < ng; ++gi) {
            if ((gpos & 1) == 0) cp_async_wait<NS - 1>();
            __syncwarp();
            const GAct x0 = load_act(xs_lane, seeds_lane, gl0 + gi / R16, col_stride);
            if ((gi & 3) == 0) granule_mma(gptr(0), lane, x0, acc[0]);
            else if ((gi & 3) == 1) granule_mma(gptr(0), lane, x0, acc[1]);
            else if ((gi & 3) == 2) granule_mma(gptr(0), lane, x0, acc[2]);
            else granule_mma(gptr(0), lane, x0, acc[3]);
            __syncwarp();
            if (gpos & 1) refill((gpos - 1) / 2);
            gpos += 1;
        }
        // partial accumulators combined in a fixed order (sub-tile = granule parity)
        float* r0 = red + ((size_t)(warp * seg_stride + seg) * R16 * 32 + lane) * 4;
        if (R16 == 1) {
            *reinterpret_cast<float4*>(r0) = make_float4((acc[0][0] + acc[1][0]) + (acc[2][0] + acc[3][0]),
                                                         (acc[0][1] + acc[1][1]) + (acc[2][1] + acc[3][1]),
                                                         (acc[0][2] + acc[1][2]) + (acc[2][2] + acc[3][2]),
                                                         (acc[0][3] + acc[1][3]) + (acc[2][3] + acc[3][3]));
        } else {
            *reinterpret_cast<float4*>(r0) =
                make_float4(acc[0][0] + acc[2][0], acc[0][1] + acc[2][1], acc[0][2] + acc[2][2], acc[0][3] + acc[2][3]);
            *reinterpret_cast<float4*>(r0 + 128) =
                make_float4(acc[1][0] + acc[3][0], acc[1][1] + acc[3][1], acc[1][2] + acc[3][2], acc[1][3] + acc[3][3]);
        }
        tg = se;
    }
    __syncthreads();

    // ---- epilogue -------------------------------------------------------------
    const int C = gridDim.x, c = blockIdx.x;
    const int tfirst = P.tg0 / KG, tlast = (P.tg1 - 1) / KG;
    const int ntl = P.tg1 > P.tg0 ? tlast - tfirst + 1 : 0;
    // CTA partial of tile (tfirst + tl), element (sub, lane slot ln, e): warps in order
    const int tg0 = P.tg0, nrange = P.tg1 - P.tg0;
    auto cta_part = [&](int tl, int sub, int ln, int e) {
        const int lo = (tfirst + tl) * KG - tg0, hi = lo + KG;  // tile's tile-groups, CTA-relative
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < MK_NW; ++w) {
            const int xa = (w * nrange) >> 4, xb = ((w + 1) * nrange) >> 4;
            if (xa < xb && xa < hi && xb > lo) {
                const int sg = (tfirst + tl) - (tfirst + mm.wft[w]);
                v += red[((size_t)(w * seg_stride + sg) * R16 + sub) * 32 * 4 + ln * 4 + e];
            }
        }
        return v;
    };
    unsigned long long best[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) best[j] = 0ull;
    if (lm) {
        if (tid < 8) mm.amax[tid] = 0ull;
        __syncthreads();
    }
    // 1. tiles owned completely: outputs now
    const int nout = ntl * 16 * Mx;
    for (int o = tid; o < nout; o += MK_NT) {
        const int m = o % Mx, rr = o / Mx, r = rr & 15, tl = rr >> 4;
        const int tile = tfirst + tl;
        if (tile * KG < P.tg0 || (tile + 1) * KG > P.tg1) continue;  // split tile
        const int ln = 4 * (r & 7) + (m >> 1), e = 2 * (r >> 3) + (m & 1);
        float v[2] = {cta_part(tl, 0, ln, e), R16 == 2 ? cta_part(tl, 1, ln, e) : 0.f};
        store_elem<KIND>(a, lm, tile * 16 + r, m, v, best);
    }
    // 2. split tiles (at most the first and the last): publish this CTA's
    //    partial; the last CTA to arrive sums them in CTA order
    for (int side = 0; side < 2; ++side) {
        const int tl = side == 0 ? 0 : ntl - 1;
        if (ntl == 0 || (side == 1 && ntl == 1)) break;
        const int tile = tfirst + tl;
        if (tile * KG >= P.tg0 && (tile + 1) * KG <= P.tg1) continue;  // owned completely
        float* slotp = a.part_g + ((size_t)c * 2 + side) * 256;
        for (int i = tid; i < R16 * 128; i += MK_NT) {
            const int sub = i >> 7, ln = (i >> 2) & 31, e = i & 3;
            slotp[i] = cta_part(tl, sub, ln, e);
        }
        __syncthreads();
        // CTAs with a non-empty share of this tile (empty ranges exist when N < C)
        const int cf = cta_of(tile * KG, P.N, C), cl = cta_of((tile + 1) * KG - 1, P.N, C);
        int ncov = 0;
        for (int cc = cf; cc <= cl; ++cc) ncov += range_lo(cc, P.N, C) < range_lo(cc + 1, P.N, C);
        if (tid == 0) mm.last = atom_add_acq_rel(&a.tile_ctr[tile], 1u) == (unsigned)(ncov - 1);
        __syncthreads();
        if (mm.last) {
            for (int o = tid; o < 16 * Mx; o += MK_NT) {
                const int m = o % Mx, r = o / Mx;
                const int ln = 4 * (r & 7) + (m >> 1), e = 2 * (r >> 3) + (m & 1);
                float v[2] = {0.f, 0.f};
                for (int cc = cf; cc <= cl; ++cc) {
                    if (range_lo(cc, P.N, C) >= range_lo(cc + 1, P.N, C)) continue;
                    const int sd = (tile == range_lo(cc, P.N, C) / KG) ? 0 : 1;
                    const float* sp = a.part_g + ((size_t)cc * 2 + sd) * 256;
                    v[0] += __ldcg(sp + ln * 4 + e);
                    if (R16 == 2) v[1] += __ldcg(sp + 128 + ln * 4 + e);
                }
                store_elem<KIND>(a, lm, tile * 16 + r, m, v, best);
            }
            if (tid == 0) a.tile_ctr[tile] = 0u;
        }
        __syncthreads();
    }
    if (lm) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            if (m < Mx) {
                unsigned long long b = best[m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, off));
                if (lane == 0 && b) atomicMax(&mm.amax[m], b);
            }
        }
        __syncthreads();
        if (tid < Mx) a.amax_cta[(size_t)blockIdx.x * 8 + tid] = mm.amax[tid];
    }
}

// ---- the kernel ------------------------------------------------------------
template <int RMAX, int DEPTH>
__global__ void __launch_bounds__(MK_NT, 1) decode_step_kernel(const MkArgs a) {
    extern __shared__ __align__(128) unsigned char sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    MkMisc& mm = *reinterpret_cast<MkMisc*>(sm + a.off_misc);
    unsigned char* ring = sm;
    unsigned char* uni = sm + a.off_union;
    const int C = gridDim.x;

    // a finished greedy loop / spec loop turns the remaining replays into no-ops
    if ((a.gate && *a.gate) || (a.ctl && a.ctl->done)) return;
    if (tid == 0) {
        mm.bad = 0;
        mm.last = 0;
    }

    // this CTA's share of every GEMV phase
    PhaseInfo* tab = reinterpret_cast<PhaseInfo*>(sm + a.off_tab);
    const int np = n_gemv_phases(a);
    for (int pi = tid; pi < np; pi += MK_NT) {
        const MkLin lin = phase_lin(a, pi);
        PhaseInfo P;
        P.w = lin.w;
        P.N = lin.n_tiles * lin.KG;
        // whole tiles per CTA: no tile is split between CTAs
        P.tg0 = range_lo(blockIdx.x, lin.n_tiles, C) * lin.KG;
        P.tg1 = range_lo(blockIdx.x + 1, lin.n_tiles, C) * lin.KG;
        P.KG = lin.KG;
        P.R16 = lin.R16;
        P.seg_stride = lin.seg_stride;
        tab[pi] = P;
    }
    __syncthreads();

    // prime the ring: `depth` granules per warp in flight
    Cursor pc;
    pc.init(tab, np, warp);
    for (int i = 0; i < DEPTH / 2; ++i) issue_pair(pc, warp, lane, ring + ((size_t)warp * DEPTH + 2 * i) * GR_BYTES);
    unsigned gpos = 0;
    __syncthreads();

    const int M = a.M;
    unsigned arrivals = 0;  // completed phases (grid barrier target = arrivals * C)
    bool ok = true;
    for (int l = 0; l < a.L && ok; ++l) {
        const MkLayer& Ly = a.layers[l];
        // ---- q|k|v (x = embedding rows at layer 0)
        {
            const MkLin lin = Ly.lin[K_QKV];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            if (l > 0) ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            StageSrc s{l == 0 ? nullptr : a.x, a.H, 0, Ly.in_norm};
            stage_acts(a, s, a.H, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            if (l == 0 && blockIdx.x == 0) {
                // the residual stream starts as the embedding rows
                for (int u = tid; u < M * (a.H / 16); u += MK_NT) {
                    const int m = u / (a.H / 16), k = (u % (a.H / 16)) * 16;
                    float v[16];
                    StageSrc e{nullptr, 0, 0, nullptr};
                    load16(a, e, m, k, v);
                    uint32_t w8[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) w8[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
                    uint4* d = reinterpret_cast<uint4*>(a.x + (size_t)m * a.H + k);
                    d[0] = make_uint4(w8[0], w8[1], w8[2], w8[3]);
                    d[1] = make_uint4(w8[4], w8[5], w8[6], w8[7]);
                    if (a.trace) {
                        uint4* t = reinterpret_cast<uint4*>(a.trace + (size_t)m * a.H + k);
                        t[0] = d[0];
                        t[1] = d[1];
                    }
                }
            }
            if (l > 0 && a.trace && blockIdx.x == 0) trace_copy(a, l);
            __syncthreads();
            gemv_phase<K_QKV, DEPTH>(a, tab[4 * l + K_QKV], M, xs, seeds, red, pc, gpos, ring, false, mm);
            // the attention tiles' cached K/V rows do not depend on this step:
            // start loading them before waiting for the other CTAs' q|k|v
            __syncthreads();
            if ((int)blockIdx.x < a.aa.Hkv * a.aa.nsplit) {
                AttnArgs aa = a.aa;
                aa.kcache = a.kc0 + (size_t)l * a.kv_layer_elems;
                aa.vcache = a.vc0 + (size_t)l * a.kv_layer_elems;
                attn::attn_decode_preload<RMAX, MK_NT>(aa, *reinterpret_cast<attn::DecSmem<RMAX>*>(uni),
                                                       blockIdx.x / a.aa.nsplit, blockIdx.x % a.aa.nsplit,
                                                       a.aa.nsplit, tid, BlockSync{});
            }
            cta_arrive(a);
            ++arrivals;
        }
        // ---- attention
        {
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            if ((int)blockIdx.x < a.aa.Hkv * a.aa.nsplit) {
                AttnArgs aa = a.aa;
                aa.q_norm_w = Ly.q_norm;
                aa.k_norm_w = Ly.k_norm;
                aa.kcache = a.kc0 + (size_t)l * a.kv_layer_elems;
                aa.vcache = a.vc0 + (size_t)l * a.kv_layer_elems;
                attn::DecSmem<RMAX>& asm_ = *reinterpret_cast<attn::DecSmem<RMAX>*>(uni);
                attn::attn_decode_body<RMAX, MK_NT>(aa, asm_, blockIdx.x / a.aa.nsplit, blockIdx.x % a.aa.nsplit,
                                                    a.aa.nsplit, tid, BlockSync{}, true);
            }
            cta_arrive(a);
            ++arrivals;
        }
        // ---- o_proj + residual
        {
            const MkLin lin = Ly.lin[K_O];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            if (a.trace && blockIdx.x == 0) trace_copy_n(a.attn, a.trace_attn + (size_t)l * a.M * a.QD, a.M * a.QD);
            StageSrc s{a.attn, a.QD, 0, nullptr};
            stage_acts(a, s, a.QD, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            __syncthreads();
            gemv_phase<K_O, DEPTH>(a, tab[4 * l + K_O], M, xs, seeds, red, pc, gpos, ring, false, mm);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- gate|up + SwiGLU
        {
            const MkLin lin = Ly.lin[K_GU];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            if (a.trace && blockIdx.x == 0) trace_copy_n(a.x, a.trace_mid + (size_t)l * a.M * a.H, a.M * a.H);
            StageSrc s{a.x, a.H, 0, Ly.post_norm};
            stage_acts(a, s, a.H, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            __syncthreads();
            gemv_phase<K_GU, DEPTH>(a, tab[4 * l + K_GU], M, xs, seeds, red, pc, gpos, ring, false, mm);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- down + residual
        {
            const MkLin lin = Ly.lin[K_DOWN];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            StageSrc s{a.mlp, a.I, 0, nullptr};
            stage_acts(a, s, a.I, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            __syncthreads();
            gemv_phase<K_DOWN, DEPTH>(a, tab[4 * l + K_DOWN], M, xs, seeds, red, pc, gpos, ring, false, mm);
            cta_arrive(a);
            ++arrivals;
        }
    }
    // ---- final norm -> lm_head -> per-CTA argmax
    if (ok && a.logits_rows > 0) {
        const MkLin lin = a.lm;
        const int rows = a.logits_rows;
        uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
        float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * rows * XW * 4);
        float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
        ok = cta_wait(a, arrivals * C, mm);
        if (ok && a.trace && blockIdx.x == 0) trace_copy(a, a.L);
        if (ok) {
            StageSrc s{a.x, a.H, M - rows, a.final_norm};
            stage_acts(a, s, a.H, rows, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            __syncthreads();
            gemv_phase<K_O, DEPTH>(a, tab[4 * a.L], rows, xs, seeds, red, pc, gpos, ring, true, mm);
        }
    }
    // no copy may still be landing in shared memory when the CTA exits
    cp_async_wait<0>();
    __syncthreads();

    // ---- last CTA: argmax over CTAs, step bookkeeping, counter reset
    if (tid == 0) mm.last = atom_add_acq_rel(a.sync + 1, 1u) == (unsigned)(C - 1);
    __syncthreads();
    if (!mm.last) return;
    const bool aborted = *reinterpret_cast<volatile unsigned*>(a.sync + 2) != 0;
    if (!aborted && a.logits_rows > 0 && warp == 0) {
        for (int m = 0; m < a.logits_rows; ++m) {
            unsigned long long b = 0ull;
            for (int c = lane; c < C; c += 32) b = umax64(b, __ldcg(a.amax_cta + (size_t)c * 8 + m));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, off));
            if (lane == 0) a.argmax[m] = (int)amax_key_index(b);
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (!aborted) {
            // step_finish_kernel semantics (misc.cu)
            if (a.ctl == nullptr) {
                *a.seq_len += M;
            } else {
                StepCtl* ctl = a.ctl;
                *a.seq_len += M;
                const int tok = a.argmax[0];
                ctl->produced += 1;
                bool eos = false;
                for (int i = 0; i < ctl->n_eos; ++i) eos |= (ctl->eos[i] == tok);
                if (eos) {
                    ctl->done = 1;
                    ctl->finish = 1;
                } else {
                    a.out[ctl->n_out] = tok;
                    ctl->n_out += 1;
                    *a.next_tok = tok;
                    if (ctl->produced >= ctl->max_new) ctl->done = 1;
                }
            }
        }
        if (aborted)
            for (int h = 0; h < a.aa.Hkv; ++h) a.aa.counters[h] = 0u;
        a.sync[0] = 0u;
        a.sync[1] = 0u;
        a.sync[2] = 0u;  // visible to the next launch at kernel completion
    }
}

// ---- weight packing ----------------------------------------------------------
struct PackSeg {
    const uint32_t* w;
    const bf16* s;
    const bf16* b;
    int rows;
};
struct PackArgs {
    PackSeg seg[3];
    int nseg;
    int pair;  // gate|up: sub-tile 0 from seg[0], 1 from seg[1]
    int K;
    int n_tiles;
    unsigned char* dst;
};

// One warp per granule.
__global__ void mk_pack_kernel(const PackArgs p) {
    const int KG = p.K / 64, KW = p.K / 8, R16 = p.pair ? 2 : 1;
    const long long gran = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const long long total = (long long)p.n_tiles * KG * R16;
    if (gran >= total) return;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int sub = (int)(gran % R16);
    const long long tg = gran / R16;
    const int gl = (int)(tg % KG);
    const int tile = (int)(tg / KG);
    auto src_row = [&](int r16, int& seg) {
        int gr = tile * 16 + r16;
        seg = 0;
        if (p.pair) {
            seg = sub;
        } else {
            while (seg + 1 < p.nseg && gr >= p.seg[seg].rows) {
                gr -= p.seg[seg].rows;
                ++seg;
            }
        }
        return gr;
    };
    int slo, shi;
    const int rlo = src_row(g, slo), rhi = src_row(g + 8, shi);
    auto nib = [&](int seg, int row, int k) -> uint32_t {
        return (p.seg[seg].w[(size_t)row * KW + k / 8] >> (4 * (k % 8))) & 0xFu;
    };
    uint32_t words[4];
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
            const int ka = gl * 64 + 16 * (2 * pp) + 2 * t + 8 * hb;
            const int kb = gl * 64 + 16 * (2 * pp + 1) + 2 * t + 8 * hb;
            words[2 * pp + hb] = nib(slo, rlo, ka) | (nib(slo, rlo, kb) << 4) | (nib(shi, rhi, ka) << 8) |
                                 (nib(shi, rhi, kb) << 12) | (nib(slo, rlo, ka + 1) << 16) |
                                 (nib(slo, rlo, kb + 1) << 20) | (nib(shi, rhi, ka + 1) << 24) |
                                 (nib(shi, rhi, kb + 1) << 28);
        }
    }
    unsigned char* d = p.dst + (size_t)gran * GR_BYTES;
    *reinterpret_cast<uint4*>(d + 16 * lane) = make_uint4(words[0], words[1], words[2], words[3]);
    if (lane < 4) {
        uint32_t sbw[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = 2 * lane + h;
            int s0, s1;
            const int ra = src_row(r, s0), rb = src_row(r + 8, s1);
            const unsigned short* S0 = reinterpret_cast<const unsigned short*>(p.seg[s0].s);
            const unsigned short* B0 = reinterpret_cast<const unsigned short*>(p.seg[s0].b);
            const unsigned short* S1 = reinterpret_cast<const unsigned short*>(p.seg[s1].s);
            const unsigned short* B1 = reinterpret_cast<const unsigned short*>(p.seg[s1].b);
            sbw[2 * h] = (uint32_t)S0[(size_t)ra * KG + gl] | ((uint32_t)B0[(size_t)ra * KG + gl] << 16);
            sbw[2 * h + 1] = (uint32_t)S1[(size_t)rb * KG + gl] | ((uint32_t)B1[(size_t)rb * KG + gl] << 16);
        }
        *reinterpret_cast<uint4*>(d + 512 + 16 * lane) = make_uint4(sbw[0], sbw[1], sbw[2], sbw[3]);
    }
}

// Upper bound on the tiles one warp's range touches: a warp owns at most
// ceil(ceil(N / C) / 16) tile-groups, which span at most (n - 1) / KG + 2 tiles.
int seg_bound(int n_tiles, int KG, int C) {
    const int per_cta = ((n_tiles + C - 1) / C) * KG;
    const int per_warp = (per_cta + MK_NW - 1) / MK_NW;
    return std::max(1, (per_warp - 1) / KG + 2);
}

size_t lin_bytes(int n_tiles, int KG, int R16) { return (size_t)n_tiles * KG * R16 * GR_BYTES; }

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct MkState {
    void* packed = nullptr;
    size_t packed_bytes = 0;
    MkLayer* d_layers = nullptr;
    std::vector<MkLayer> layers;
    MkLin lm{};
    unsigned* sync = nullptr;
    unsigned long long* amax_cta = nullptr;
    float* part_g = nullptr;
    unsigned* tile_ctr = nullptr;
    int C = 0;
    bool attr_set[6] = {false, false, false, false, false, false};
};

void mk_free(qw_model* m) {
    if (!m->mk) return;
    MkState* s = m->mk;
    if (s->packed) cudaFree(s->packed);
    if (s->d_layers) cudaFree(s->d_layers);
    if (s->sync) cudaFree(s->sync);
    if (s->amax_cta) cudaFree(s->amax_cta);
    if (s->part_g) cudaFree(s->part_g);
    if (s->tile_ctr) cudaFree(s->tile_ctr);
    delete s;
    m->mk = nullptr;
}

// Repack the model's quantized linears for the persistent decode kernel.
// Returns without enabling it when the model does not fit its constraints.
void mk_prepare(qw_model* m) {
    mk_free(m);
    const Config& cf = m->cfg;
    if (m->tp_size != 1 || cf.head_dim != 128) return;
    const int H = cf.hidden, QD = m->hq_l * 128, KD = m->hkv_l * 128, I = m->inter_l, V = m->vocab_l;
    if (H % 64 || QD % 64 || I % 64 || H % 16 || (QD + 2 * KD) % 16 || I % 16 || V % 16) return;
    if (m->num_sms < m->hkv_l) return;
    const char* env = getenv("QW_DECODE_KERNEL");
    if (env && std::string(env) == "multi") return;

    MkState* s = new MkState();
    m->mk = s;
    const int C = m->num_sms;
    s->C = C;
    const int L = cf.layers;
    // packed arena
    const size_t b_qkv = lin_bytes((QD + 2 * KD) / 16, H / 64, 1), b_o = lin_bytes(H / 16, QD / 64, 1),
                 b_gu = lin_bytes(I / 16, H / 64, 2), b_down = lin_bytes(H / 16, I / 64, 1),
                 b_lm = lin_bytes(V / 16, H / 64, 1);
    s->packed_bytes = (b_qkv + b_o + b_gu + b_down) * L + b_lm;
    QW_CUDA(cudaSetDevice(m->device));
    QW_CUDA(cudaMalloc(&s->packed, s->packed_bytes));
    unsigned char* p = static_cast<unsigned char*>(s->packed);
    auto pack = [&](const QLin* segs, int nseg, bool pair, int K, int n_tiles, MkLin& out) {
        PackArgs pa;
        std::memset(&pa, 0, sizeof(pa));
        for (int i = 0; i < nseg; ++i) pa.seg[i] = PackSeg{segs[i].w, segs[i].s, segs[i].b, segs[i].n};
        pa.nseg = nseg;
        pa.pair = pair ? 1 : 0;
        pa.K = K;
        pa.n_tiles = n_tiles;
        pa.dst = p;
        const int R16 = pair ? 2 : 1;
        const long long grans = (long long)n_tiles * (K / 64) * R16;
        mk_pack_kernel<<<(unsigned)((grans + 7) / 8), 256, 0, m->stream>>>(pa);
        QW_CUDA(cudaGetLastError());
        out.w = p;
        out.n_tiles = n_tiles;
        out.KG = K / 64;
        out.R16 = R16;
        out.seg_stride = seg_bound(n_tiles, K / 64, C);
        p += lin_bytes(n_tiles, K / 64, R16);
    };
    s->layers.resize(L);
    for (int l = 0; l < L; ++l) {
        Layer& Lw = m->layers[l];
        MkLayer& ml = s->layers[l];
        const QLin qkv[3] = {Lw.q, Lw.k, Lw.v};
        pack(qkv, 3, false, H, (QD + 2 * KD) / 16, ml.lin[K_QKV]);
        pack(&Lw.o, 1, false, QD, H / 16, ml.lin[K_O]);
        const QLin gu[2] = {Lw.gate, Lw.up};
        pack(gu, 2, true, H, I / 16, ml.lin[K_GU]);
        pack(&Lw.down, 1, false, I, H / 16, ml.lin[K_DOWN]);
        ml.in_norm = Lw.in_norm;
        ml.post_norm = Lw.post_norm;
        ml.q_norm = Lw.q_norm;
        ml.k_norm = Lw.k_norm;
    }
    pack(&m->lm_head, 1, false, H, V / 16, s->lm);
    QW_CUDA(cudaMalloc(&s->d_layers, sizeof(MkLayer) * L));
    QW_CUDA(cudaMemcpyAsync(s->d_layers, s->layers.data(), sizeof(MkLayer) * L, cudaMemcpyHostToDevice, m->stream));
    QW_CUDA(cudaMalloc(&s->sync, 4 * sizeof(unsigned)));
    QW_CUDA(cudaMemsetAsync(s->sync, 0, 4 * sizeof(unsigned), m->stream));
    QW_CUDA(cudaMalloc(&s->amax_cta, (size_t)C * 8 * sizeof(unsigned long long)));
    QW_CUDA(cudaMalloc(&s->part_g, (size_t)C * 2 * 256 * sizeof(float)));
    int max_tiles = s->lm.n_tiles;
    for (int k = 0; k < 4; ++k) max_tiles = std::max(max_tiles, s->layers[0].lin[k].n_tiles);
    QW_CUDA(cudaMalloc(&s->tile_ctr, (size_t)max_tiles * sizeof(unsigned)));
    QW_CUDA(cudaMemsetAsync(s->tile_ctr, 0, (size_t)max_tiles * sizeof(unsigned), m->stream));
    QW_CUDA(cudaStreamSynchronize(m->stream));
}

namespace {

static_assert(offsetof(attn::DecSmem<8>, tbar) + sizeof(uint64_t) * 2 <= MK_UNI_RESERVED,
              "attention mbarriers must sit in the reserved head of the union");

template <int RMAX>
size_t mk_union_bytes(const MkState* s, int M, int rows, int C) {
    size_t u = sizeof(attn::DecSmem<RMAX>);
    // staged x', seeds, per-warp partials and (RMSNorm phases) per-unit sums of squares
    auto need = [&](const MkLin& lin, int Mx, bool norm) {
        return (size_t)lin.KG * Mx * XW * 4 + (size_t)lin.KG * 4 * SEEDF * 4 +
               (size_t)MK_NW * lin.seg_stride * lin.R16 * 512 + (norm ? (size_t)lin.KG * Mx * 4 * 4 : 0);
    };
    for (int k = 0; k < 4; ++k) u = std::max(u, MK_UNI_RESERVED + need(s->layers[0].lin[k], M, k == K_QKV || k == K_GU));
    if (rows > 0) u = std::max(u, MK_UNI_RESERVED + need(s->lm, rows, true));
    return (u + 127) & ~(size_t)127;
}

template <int RMAX, int DEPTH>
void mk_launch_d(qw_model* m, MkArgs& a, cudaStream_t st, size_t smem, int max_smem, bool& attr_set) {
    if (!attr_set) {
        QW_CUDA(cudaFuncSetAttribute(decode_step_kernel<RMAX, DEPTH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     max_smem));
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->mk->C);
    cfg.blockDim = dim3(MK_NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QW_CUDA(cudaLaunchKernelEx(&cfg, decode_step_kernel<RMAX, DEPTH>, a));
}

// Ring depth 16 granules per warp when shared memory allows, else 8.
template <int RMAX>
bool mk_launch_t(qw_model* m, MkArgs& a, cudaStream_t st, int slot_idx) {
    MkState* s = m->mk;
    int max_smem = 0;
    QW_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    const size_t uni = mk_union_bytes<RMAX>(s, a.M, a.logits_rows, s->C);
    const int np = 4 * a.L + (a.logits_rows > 0 ? 1 : 0);
    const size_t misc_struct = (sizeof(MkMisc) + 127) & ~(size_t)127;
    const size_t misc = misc_struct + (((size_t)np * sizeof(PhaseInfo) + 127) & ~(size_t)127);
    const long long room = (long long)max_smem - (long long)uni - (long long)misc;
    const long long per_depth = (long long)MK_NW * GR_BYTES;
    int depth = room >= 16 * per_depth ? 16 : (room >= 8 * per_depth ? 8 : 0);
    // QW_MK_DEPTH=8 caps the ring depth (profiling / testing both kernel forms)
    if (const char* e = std::getenv("QW_MK_DEPTH"))
        if (std::atoi(e) == 8 && depth == 16) depth = 8;
    if (depth == 0) return false;
    a.depth = depth;
    a.off_union = (unsigned)((size_t)MK_NW * depth * GR_BYTES);  // a multiple of 128
    a.off_misc = a.off_union + (unsigned)uni;
    a.off_tab = a.off_misc + (unsigned)misc_struct;
    const size_t smem = a.off_misc + misc;
    if (depth == 16)
        mk_launch_d<RMAX, 16>(m, a, st, smem, max_smem, s->attr_set[2 * slot_idx]);
    else
        mk_launch_d<RMAX, 8>(m, a, st, smem, max_smem, s->attr_set[2 * slot_idx + 1]);
    return true;
}

}  // namespace

bool mk_forward(qw_model* m, qw_cache* c, const int* d_ids, int S, int logits_mode, bool store_logits,
                int* d_argmax, cudaStream_t st, StepCtl* ctl, int* next_tok, int* out, const int* gate) {
    MkState* s = m->mk;
    if (!s || S < 1 || S > 8) return false;
    const Config& cf = m->cfg;
    Workspace& w = m->ws;
    const int G = m->hq_l / m->hkv_l, R = G * S;
    if (R > 32) return false;
    const int rows = logits_mode == 0 ? 0 : (logits_mode == 2 ? S : 1);
    if (rows > w.cap_logits || S > w.cap_rows) return false;

    MkArgs a;
    std::memset(&a, 0, sizeof(a));
    a.layers = s->d_layers;
    a.L = cf.layers;
    a.lm = s->lm;
    a.final_norm = m->final_norm;
    a.emb_w = m->embed.w;
    a.emb_s = m->embed.s;
    a.emb_b = m->embed.b;
    a.ids = d_ids;
    a.M = S;
    a.H = cf.hidden;
    a.I = m->inter_l;
    a.QD = m->hq_l * 128;
    a.KD = m->hkv_l * 128;
    a.V = m->vocab_l;
    a.eps = cf.eps;
    a.x = w.x;
    a.q = w.q;
    a.k = w.k;
    a.v = w.v;
    a.attn = w.attn;
    a.mlp = w.mlp;
    AttnArgs& aa = a.aa;
    aa.q = w.q;
    aa.k = w.k;
    aa.v = w.v;
    aa.ldq = a.QD;
    aa.ldk = a.KD;
    aa.ldv = a.KD;
    aa.eps = cf.eps;
    aa.rope_cos = m->rope_cos;
    aa.rope_sin = m->rope_sin;
    aa.max_pos = c->max_pos;
    aa.seq_len = c->d_seq_len;
    aa.S = S;
    aa.Hq = m->hq_l;
    aa.Hkv = m->hkv_l;
    aa.scale = 1.0f / sqrtf(128.0f);
    aa.part = w.attn_part;
    aa.counters = w.attn_counters;
    aa.out = w.attn;
    aa.ldo = a.QD;
    aa.nsplit = std::max(1, s->C / m->hkv_l);
    aa.err = m->d_err;
    a.kv_layer_elems = (size_t)m->hkv_l * c->max_pos * 128;
    a.kc0 = c->k;
    a.vc0 = c->v;
    a.logits_rows = rows;
    a.logits = w.logits;
    a.store_logits = store_logits ? 1 : 0;
    a.amax_cta = s->amax_cta;
    a.argmax = d_argmax;
    a.seq_len = c->d_seq_len;
    a.ctl = ctl;
    a.next_tok = next_tok;
    a.out = out;
    a.gate = gate;
    a.sync = s->sync;
    a.part_g = s->part_g;
    a.tile_ctr = s->tile_ctr;
    a.err = m->d_err;
    a.trace = m->trace;
    a.trace_mid = m->trace_mid;
    a.trace_attn = m->trace_attn;
    if (R <= 8) return mk_launch_t<8>(m, a, st, 0);
    if (R <= 16) return mk_launch_t<16>(m, a, st, 1);
    return mk_launch_t<32>(m, a, st, 2);
}

}  // namespace qw
