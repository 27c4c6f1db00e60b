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
// Grid = one CTA per SM (cooperative launch: all CTAs are resident) of 16
// warps.  Phases are separated by a grid-wide arrival counter; every wait is
// bounded (2 s of globaltimer), after which the launch sets QW_DERR_TIMEOUT,
// raises an abort flag that makes every other wait return, drains its copies
// and exits.
//
// Weight stream.  At model load every quantized linear is repacked into
// 576-byte granules (16 rows x 64 inputs).  Bytes 0..511 hold the nibbles so
// that lane l (g = l/4, t = l%4) reads one 16-byte word quad (A0, B0, A1, B1)
// that yields, with one shift and four LOP3 per word, the A fragments of the
// group's four mma.m16n8k16 k-steps: steps 0 and 2 take (w & 0x000F000F) |
// 0x64006400 (fp16 1024 + q), steps 1 and 3 take (w & 0x00F000F0) | 0x64006400
// (1024 + 16q), each on two accumulator chains seeded with -1024 * sum(x).
// The nibbles reach the tensor core as exact fp16 subnormals (q * 2^-24 and,
// for the high nibble of a byte, 16q * 2^-24, whose k-steps take x/16), so the
// fp32 accumulation carries no offset to cancel.  Bytes 512..575 hold the 16
// rows' bf16 scales (pre-multiplied by 2^24 at packing, exact) and biases,
// 8 bytes per row pair (g, g+8).  Every CTA owns whole 16-row tiles of a phase
// and every warp an equal contiguous sixteenth of the CTA's (tile, group)
// pairs; tile partial sums are combined across warps in warp order (results
// do not depend on the number of rows).
// Weight stream: weights never depend on activations, so each warp walks its
// own granule sequence across tile, phase and layer boundaries and copies it,
// R granules (2.3 KB) per bulk copy (cp.async.bulk through the TMA engine,
// completion counted on an mbarrier), into a private ring of four stages: the
// moment the warp has consumed a stage, its lane 0 issues the copy of the
// stage four ahead into the freed slot.  HBM keeps streaming while the warps
// wait at a phase barrier, a copy costs the warp a handful of instructions per
// 2.3 KB, and nothing polls for free slots.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "attn_split.cuh"
#include "model.h"
#include "smem_attr.h"

namespace qw {

namespace {

#ifndef QW_MK_NW
#define QW_MK_NW 16
#endif
constexpr int MK_NW = QW_MK_NW;           // compute warps
constexpr int MK_NT = MK_NW * 32;         // compute threads (the named barrier's count)
constexpr int MK_NSLOT = 4;               // stage barriers per warp (the most stages a ring has)
// ring stages per warp for stages of R granules (the ring holds 16 granules, 8 for R = 2)
__host__ __device__ constexpr int mk_ns(int R) { return R >= 8 ? 2 : 4; }
constexpr int GR_BYTES = 576;  // one granule: 512 B nibbles + 64 B scales/biases
// The GEMV phases stage their activations past the head of the shared union,
// which holds the attention item's mbarrier (attn::SplitSmem::bar, written by
// asynchronous cp.async arrivals): staged data never shares bytes with a
// barrier that an arrival could still update.
constexpr size_t MK_UNI_RESERVED = 128;
constexpr int XW = 36;         // words per (group, column) block of staged activations (32 + 4 pad)
constexpr int SEEDF = 2;       // floats per (group, quad t) entry: sum(x) of columns 2t, 2t+1
constexpr unsigned long long MK_TIMEOUT_NS = 2000000000ull;
#ifndef QW_MK_POLL_NS
#define QW_MK_POLL_NS 64  // back-off between polls of the phase counter
#endif

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

// One sequence of a batched step: its cache and sequence length.
struct MkSeq {
    bf16 *kc0, *vc0;        // layer 0's K / V cache
    int* seq_len;           // device sequence length
    int max_pos;
    size_t kv_layer_elems;  // elements per layer of one cache
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
    int* err;
    bf16* trace;     // diagnostics: residual stream after the embedding and every layer, [L + 1][M][H]
    bf16* trace_mid;   // diagnostics: residual after each attention block, [L][M][H]
    bf16* trace_attn;  // diagnostics: attention output of each layer, [L][M][QD]
    unsigned long long* prof;  // diagnostics: phase timing stamps (see MK_STAMP), or null
    // batched step (nseq > 0): row m is the one new token of sequence m, which
    // attends to its own cache at its own position; otherwise the M rows are
    // consecutive positions of one sequence (kc0 / vc0 / seq_len above)
    int nseq;
    MkSeq seqs[8];
    size_t part_seq_stride;  // attention partial floats per sequence
    BatchCtl* bctl;
    int b0;          // the launch's first sequence within the whole batch (bookkeeping index)
    int btotal;      // sequences in the whole batch
    int bfinalize;   // this launch completes the step (step count, done flag)
    unsigned off_union, off_misc, off_tab;
};

// A compute warp's weight stream: where its next bulk copy starts.  Stage s of
// the warp's sequence (R granules, never spanning two phases) goes to ring slot
// s % NS (NS = mk_ns(R)); the warp's lane 0 issues it right after the warp has
// consumed stage s - NS from that slot, so copies run NS stages ahead of
// the computation, across tile, phase and layer boundaries (weights never
// depend on activations), and no thread ever polls for a free slot.
struct IssueCur {
    int pi;          // phase of the next copy (np: stream exhausted)
    int gi, ge;      // next granule and end of the warp's range in that phase
    unsigned stage;  // stages issued so far
};

struct MkMisc {
    int wft[MK_NW];  // first tile (CTA-local) of each warp's range in the current phase
    int2 wr[MK_NW];  // each warp's range of tile-groups in the current phase, CTA-relative
    float rnorm[8];
    float ssq[MK_NW][8];
    unsigned long long amax[8];
    int bad;
    int last;
    int seq;  // the cache's sequence length at launch (constant until the last CTA's bookkeeping)
    IssueCur ic[MK_NW];  // each warp's weight-stream cursor (lane 0)
    int seqb[8];   // batched step: each sequence's length at launch
    int ibase[9];  // batched step: first attention item of each sequence; ibase[nseq] = items
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

// Per-CTA description of one GEMV phase, built once per launch in shared
// memory so that walking the granule stream needs no global loads.
struct PhaseInfo {
    const unsigned char* w;  // packed granules of the whole linear
    const bf16* norm;        // a norm weight read by this layer's steps: q|k|v phase: input RMSNorm;
                             // o phase: q_norm; gate|up phase: post-attention RMSNorm; down phase:
                             // k_norm; lm_head phase: the final norm
    int tg0, tg1;            // this CTA's tile-groups
    int KG, R16;
    int N;                   // tile-groups in the phase
    int seg_stride;
};
static_assert(sizeof(PhaseInfo) == 40, "PhaseInfo layout");

QW_DEV void warp_range(const PhaseInfo& P, int warp, int& wa, int& wb) {
    const int n = P.tg1 - P.tg0;
    wa = P.tg0 + (warp * n) / MK_NW;
    wb = P.tg0 + ((warp + 1) * n) / MK_NW;
}

// Bounded mbarrier wait (4 s of globaltimer, or the launch's abort flag); the
// slow path is out of line so the weight loop keeps its registers.
__device__ __noinline__ bool mbar_wait_mk_slow(uint64_t* bar, uint32_t parity, const unsigned* abort_flag) {
    const unsigned long long t0 = globaltimer();
    for (unsigned it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*reinterpret_cast<const volatile unsigned*>(abort_flag)) return false;
            if (globaltimer() - t0 > 2 * MK_TIMEOUT_NS) return false;
        }
    }
}
QW_DEV bool mbar_wait_mk(uint64_t* bar, uint32_t parity, const unsigned* abort_flag) {
    return mbar_try_wait(bar, parity) || mbar_wait_mk_slow(bar, parity, abort_flag);
}

QW_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Advance to the next non-empty range of warp w, from phase c.pi on.
QW_DEV void issue_enter(IssueCur& c, const PhaseInfo* tab, int np, int w) {
    for (; c.pi < np; ++c.pi) {
        int wa, wb;
        warp_range(tab[c.pi], w, wa, wb);
        c.gi = wa * tab[c.pi].R16;
        c.ge = wb * tab[c.pi].R16;
        if (c.gi < c.ge) return;
    }
}

// Lane 0: issue the warp's next stage, if the stream has one (out of line: it
// runs once per stage and keeps its registers out of the weight loop).
template <int R>
__device__ __noinline__ void issue_next(IssueCur& c, const PhaseInfo* tab, int np, int w, unsigned char* ring, uint64_t* fullb) {
    if (c.pi >= np) return;
    constexpr int NS = mk_ns(R);
    const unsigned slot = c.stage % NS;
    uint64_t* fb = fullb + w * MK_NSLOT + slot;
    const int n = min(R, c.ge - c.gi);
    mbar_arrive_expect_tx(fb, (uint32_t)(n * GR_BYTES));
    bulk_g2s(ring + ((size_t)w * NS + slot) * R * GR_BYTES, tab[c.pi].w + (size_t)c.gi * GR_BYTES,
             (uint32_t)(n * GR_BYTES), fb);
    c.gi += n;
    ++c.stage;
    if (c.gi >= c.ge) {
        ++c.pi;
        issue_enter(c, tab, np, w);
    }
}

// ---- activation staging ----------------------------------------------------
// x' for one GEMV phase: per (group gl, column m) a block of XW words, words
// t*8 + 2j + h = fp16 pair (x[64gl+16j+2t+8h], x[..+1]), divided by 16 for the
// odd k-steps j (their nibbles enter the tensor core as 16q); per (gl, quad t)
// SEEDF floats {sum(x) of column 2t, of column 2t+1} for the bias term.
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
    const float f = (j & 1) ? 0.0625f : 1.0f;  // exact power-of-two scaling
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        sum += v[2 * i] + v[2 * i + 1];
        const __half2 hh = __floats2half2_rn(v[2 * i] * f, v[2 * i + 1] * f);
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

// The four k-step units of (gl, m) sit in one lane quad: their sum is sum(x)
// of the group and column (every lane of the warp takes part in the shuffles).
QW_DEV void stage_seeds(float sum, bool valid, int gl, int m, int j, float* seeds) {
    const float pair = sum + __shfl_xor_sync(0xffffffffu, sum, 2);
    const float tot = pair + __shfl_xor_sync(0xffffffffu, pair, 1);
    if (valid && j == 0) seeds[(size_t)(gl * 4 + (m >> 1)) * SEEDF + (m & 1)] = tot;
}

QW_DEV void load_norm16(const StageSrc& s, int k, uint32_t (&W)[8]) {
    const uint4* wp = reinterpret_cast<const uint4*>(s.norm + k);
    const uint4 w0 = wp[0], w1 = wp[1];
    W[0] = w0.x; W[1] = w0.y; W[2] = w0.z; W[3] = w0.w;
    W[4] = w1.x; W[5] = w1.y; W[6] = w1.z; W[7] = w1.w;
}
QW_DEV void apply_norm_w(const uint32_t (&W)[8], float r, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[2 * i] = bfr(__fmul_rn(__fmul_rn(v[2 * i], r), bits_lo_f(W[i])));
        v[2 * i + 1] = bfr(__fmul_rn(__fmul_rn(v[2 * i + 1], r), bits_hi_f(W[i])));
    }
}
QW_DEV void apply_norm(const StageSrc& s, float r, int k, float (&v)[16]) {
    uint32_t W[8];
    load_norm16(s, k, W);
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

// Block barrier of the 16 warps (named barrier 1).
QW_DEV void csync() { asm volatile("bar.sync 1, %0;" ::"n"(MK_NT) : "memory"); }

QW_DEV void stage_acts(const MkArgs& a, const StageSrc& s, int K, int Mx, uint32_t* xs, float* seeds, float* sq,
                       MkMisc& mm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KG = K / 64;
    const int units = KG * Mx * 4;
    if (s.norm) {
        // RMSNorm statistics, the same summation order for every row count:
        // per-unit sums of squares, then per row its units lane-strided and a
        // fixed shuffle tree.  With one unit per thread the unit (values and
        // norm weights, fetched together: one memory round trip) stays in
        // registers for the second pass; otherwise the second pass reloads.
        const bool keep = units <= MK_NT;
        uint32_t X0[8], W0[8];
        int gl0 = 0, m0 = 0, j0 = 0;
        for (int u = tid; u < units; u += MK_NT) {
            int gl, m, j;
            unit_coords(u, Mx, gl, m, j);
            uint32_t X[8];
            load16_packed(a, s, m, gl * 64 + 16 * j, X);
            if (keep) {
                load_norm16(s, gl * 64 + 16 * j, W0);
#pragma unroll
                for (int i = 0; i < 8; ++i) X0[i] = X[i];
                gl0 = gl;
                m0 = m;
                j0 = j;
            }
            sq[u] = sumsq_packed(X);
        }
        csync();
        if (warp < Mx) {
            float q = 0.f;
            for (int i = lane; i < KG * 4; i += 32) q += sq[((i >> 2) * Mx + warp) * 4 + (i & 3)];
            q = warp_sum(q);
            if (lane == 0) mm.rnorm[warp] = 1.0f / sqrtf(q / (float)K + a.eps);
        }
        csync();
        if (keep) {
            float sum0 = 0.f;
            if (tid < units) {
                float v[16];
                unpack16(X0, v);
                apply_norm_w(W0, mm.rnorm[m0], v);
                sum0 = stage_unit(v, gl0, m0, j0, Mx, xs);
            }
            stage_seeds(sum0, tid < units, gl0, m0, j0, seeds);
            return;
        }
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
            __nanosleep(QW_MK_POLL_NS);
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
    csync();  // the acquire above, then this barrier, orders every thread's reads
    return !*reinterpret_cast<volatile int*>(&mm.bad);
}
// Block barrier, then one release-add: publishes every thread's earlier writes
// (the barrier orders them before the release, which is cumulative).
QW_DEV void cta_arrive(const MkArgs& a) {
    csync();
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
struct CSync {
    QW_DEV void operator()() const { csync(); }
};

// Staged activations of one group for this lane: B fragments of the four
// k-steps (odd steps as x/16) and sum(x) of columns 2t, 2t+1.
struct GAct {
    uint4 xa, xb;  // (step 0, step 1) and (step 2, step 3) B fragment pairs
    float2 sx;
};
// One granule's four mma over the group's k-steps, one chain: c = 2^-24 * sum(q x)
// per row (g, g+8) and column (2t, 2t+1).
QW_DEV void granule_mma(const uint4 wv, const GAct& x, float (&c)[4]) {
    const uint32_t a8 = wv.x >> 8, b8 = wv.y >> 8, c8 = wv.z >> 8, d8 = wv.w >> 8;
    mma_zero(c, lo4(wv.x), lo4(a8), lo4(wv.y), lo4(b8), x.xa.x, x.xa.y);
    mma_acc(c, hi4(wv.x), hi4(a8), hi4(wv.y), hi4(b8), x.xa.z, x.xa.w);
    mma_acc(c, lo4(wv.z), lo4(c8), lo4(wv.w), lo4(d8), x.xb.x, x.xb.y);
    mma_acc(c, hi4(wv.z), hi4(c8), hi4(wv.w), hi4(d8), x.xb.z, x.xb.w);
}
// acc += (2^24 s) * c + b * sum(x) for rows g (s0, b0) and g + 8 (s1, b1).
QW_DEV void granule_epi(const uint2 sb, const float (&c)[4], const float2 sx, float (&acc)[4]) {
    const float s0 = bits_lo_f(sb.x), b0 = bits_hi_f(sb.x);
    const float s1 = bits_lo_f(sb.y), b1 = bits_hi_f(sb.y);
    acc[0] = fmaf(s0, c[0], fmaf(b0, sx.x, acc[0]));
    acc[1] = fmaf(s0, c[1], fmaf(b0, sx.y, acc[1]));
    acc[2] = fmaf(s1, c[2], fmaf(b1, sx.x, acc[2]));
    acc[3] = fmaf(s1, c[3], fmaf(b1, sx.y, acc[3]));
}

// ---- one GEMV phase --------------------------------------------------------
// Computes the CTA's items of phase `pi` from its ring, then the epilogue.
// Epilogue of one output element (tile row `row`, column m) with the final
// fp32 sums v[sub].
template <int KIND>
QW_DEV void store_elem(const MkArgs& a, bool lm, int row, int m, const float (&v)[2], unsigned long long (&best)[8],
                       float resid) {
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
        a.x[(size_t)m * a.H + row] = f2bf(__fadd_rn(resid, bfr(v[0])));
    }
}

// ---- optional timing stamps --------------------------------------------------
// With a stamp buffer (MkArgs::prof, set by the QW_MK_PROFILE environment
// variable), thread 0 of each CTA records globaltimer at points of every
// phase: prof[(cta * MK_PROF_PHASES + phase) * MK_PROF_SLOTS + k], k = 0 after the phase
// barrier, 1 after activation staging, 2 first weight stage ready, 3 own
// weight loop done, 4 all warps' loops done, 5 epilogue done, 6 before
// arriving, 8 weight loop entered (warp 0), 9 weight loop left (warp 0).  Phase 5l + {0..4} = layer l's q|k|v, attention, o, gate|up, down;
// 5L = lm_head.  Read back with qw_debug_mk_prof.
constexpr int MK_PROF_PHASES = 4 * 64 * 2 + 2;
constexpr int MK_PROF_SLOTS = 16;
#define MK_STAMP(ph, k)                                                                                      \
    do {                                                                                                     \
        if (a.prof && threadIdx.x == 0 && (ph) < MK_PROF_PHASES)                                             \
            a.prof[((size_t)blockIdx.x * MK_PROF_PHASES + (ph)) * MK_PROF_SLOTS + (k)] = globaltimer();      \
    } while (0)

template <int KIND>
QW_DEV void gemv_epilogue(const MkArgs& a, const PhaseInfo& P, int Mx, const float* red, bool lm,
                                           MkMisc& mm);

// Explicit shared-memory accesses on 32-bit shared addresses (the weight loop
// below is a separate function: a generic pointer would cost it the shared path).
QW_DEV uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
QW_DEV uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
QW_DEV float2 lds64f(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
QW_DEV void sts128f(uint32_t a, float x, float y, float z, float w) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}

// Where a warp's weight loop reads and writes in shared memory (32-bit shared addresses).
struct LoopSmem {
    uint32_t xs;     // this lane's staged activations of group 0 (column min(g, M-1), quad t)
    uint32_t seeds;  // this lane's sum(x) entry of group 0
    uint32_t col;    // bytes between the staged activations of consecutive groups
    uint32_t ring;   // this warp's ring
    uint32_t fb;     // this warp's stage barriers
    uint32_t red;    // this warp's partials: segment s, sub-tile u at red + (s * R16 + u) * 512 + 16 * lane
};

// The warp's weight loop over granules [gi, gend) of the phase (tile segments
// end every per_tile granules): waits for its ring stages, computes four
// granules per batch (their weights loaded together), writes one partial per
// tile segment, and has lane 0 refill every consumed slot with the stage
// NS ahead.  Granules enter their sub-tile's accumulator in phase order.
// Out of line, so the kernel's own live state never competes with the loop
// for registers.
template <int KIND, int R>
__device__ __noinline__ unsigned gemv_loop(const unsigned* abort_flag, int* err, const LoopSmem sm, int gi, const int gend,
                                       const int per_tile, const int KG, unsigned stage, IssueCur* ic,
                                       const PhaseInfo* tab, int np, unsigned char* ring, uint64_t* fullb,
                                       unsigned long long* prof_slot) {
    constexpr int R16 = KIND == K_GU ? 2 : 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2;
    constexpr int NS = mk_ns(R);
    int seg_end = (gi / per_tile + 1) * per_tile;
    uint32_t red = sm.red + 16 * lane;
    float acc[R16][4];
#pragma unroll
    for (int u = 0; u < R16; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
    auto flush = [&]() {
#pragma unroll
        for (int u = 0; u < R16; ++u) {
            sts128f(red + u * 512, acc[u][0], acc[u][1], acc[u][2], acc[u][3]);
            acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
        }
        red += R16 * 512;
    };
    bool first = true;
    if (prof_slot && threadIdx.x == 0) prof_slot[6] = globaltimer();
    while (gi < gend) {
        const int n = min(R, gend - gi);
        const uint32_t slot = stage % NS;
        uint64_t* bar = reinterpret_cast<uint64_t*>(fullb) + warp * MK_NSLOT + slot;
        if (!mbar_wait_mk(bar, (stage / NS) & 1, abort_flag)) {
            if (lane == 0) {
                atomicOr(err, QW_DERR_TIMEOUT);
                atomicExch(const_cast<unsigned*>(abort_flag), 1u);
            }
            break;
        }
        if (first && prof_slot && lane == 0) *prof_slot = globaltimer();
        first = false;
        const uint32_t sp = sm.ring + slot * (R * GR_BYTES);
        // a stage starts at an even granule when R16 == 2 (ranges and stages are whole pairs)
        int gl = (gi / R16) % KG;
        uint4 xa = lds128(sm.xs + gl * sm.col), xb = lds128(sm.xs + gl * sm.col + 16);
        float2 sx = lds64f(sm.seeds + gl * 32);
        // the stage's granules in batches of at most 4 (weights of a batch loaded together)
        constexpr int RB = R > 4 ? 4 : R;
#pragma unroll 1
        for (int jb = 0; jb < n; jb += RB) {
            uint4 wv[RB];
#pragma unroll
            for (int j = 0; j < RB; ++j)
                if (jb + j < n) wv[j] = lds128(sp + (jb + j) * GR_BYTES + 16 * lane);
#pragma unroll
            for (int j = 0; j < RB; ++j) {
                const int jj = jb + j;
                if (jj < n) {
                    if (gi + jj == seg_end) {
                        flush();
                        seg_end += per_tile;
                    }
                    if (jj > 0 && (R16 == 1 || (jj & 1) == 0)) {
                        if (++gl == KG) gl = 0;
                        xa = lds128(sm.xs + gl * sm.col);
                        xb = lds128(sm.xs + gl * sm.col + 16);
                        sx = lds64f(sm.seeds + gl * 32);
                    }
                    GAct x;
                    x.xa = xa;
                    x.xb = xb;
                    x.sx = sx;
                    float c[4];
                    granule_mma(wv[j], x, c);
                    const uint2 sb = lds64(sp + jj * GR_BYTES + 512 + 8 * g);
                    granule_epi(sb, c, sx, acc[R16 == 2 ? (j & 1) : 0]);
                }
            }
        }
        // the slot is free: refill it with the stage NS ahead
        __syncwarp();
        if (lane == 0) {
            fence_proxy_async_smem();
            issue_next<R>(*ic, tab, np, warp, ring, fullb);
        }
        gi += n;
        ++stage;
    }
    flush();
    if (prof_slot && threadIdx.x == 0) prof_slot[7] = globaltimer();
    return stage;
}

// One GEMV phase: each warp computes its granule range from its ring, writing
// one partial per tile segment to shared memory (red: [warp][segment][sub][128]);
// then the CTA reduces the segments of each tile in warp order and stores the
// outputs.  Granules enter their sub-tile's accumulator in phase order (the
// granules' own mma chains are independent, so this costs no latency): the
// summation order depends only on the warp's range, never on the stage size R.
template <int KIND, int R>
QW_DEV void gemv_phase(const MkArgs& a, const PhaseInfo& P, int Mx, uint32_t* xs, float* seeds, float* red,
                       unsigned& stage, unsigned char* ring, uint64_t* fullb, IssueCur& ic, const PhaseInfo* tab,
                       int np, bool lm, MkMisc& mm, int prof_id) {
    (void)prof_id;
    constexpr int R16 = KIND == K_GU ? 2 : 1;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int KG = P.KG;
    const int seg_stride = P.seg_stride;
    const int mcol = min(g, Mx - 1);
    const int col_stride = Mx * XW;
    const uint32_t* xs_lane = xs + (size_t)mcol * XW + t * 8;
    const float* seeds_lane = seeds + (size_t)t * SEEDF;
    const unsigned char* wring = ring + (size_t)warp * mk_ns(R) * R * GR_BYTES;
    uint64_t* fb = fullb + warp * MK_NSLOT;

    int wa, wb;
    warp_range(P, warp, wa, wb);
    if (lane == 0) {
        mm.wft[warp] = (wa - P.tg0) / KG;
        mm.wr[warp] = make_int2(wa - P.tg0, wb - P.tg0);
    }
    const int per_tile = KG * R16;  // granules of one tile
    LoopSmem ls;
    ls.xs = smem_u32(xs_lane);
    ls.seeds = smem_u32(seeds_lane);
    ls.col = (uint32_t)col_stride * 4;
    ls.ring = smem_u32(wring);
    ls.fb = smem_u32(fb);
    ls.red = smem_u32(red + (size_t)warp * seg_stride * R16 * 128);
    if (wa < wb)
        stage = gemv_loop<KIND, R>(a.sync + 2, a.err, ls, wa * R16, wb * R16, per_tile, KG, stage, &ic, tab, np, ring,
                           fullb, a.prof ? a.prof + ((size_t)blockIdx.x * MK_PROF_PHASES + prof_id) * MK_PROF_SLOTS + 2 : nullptr);
    MK_STAMP(prof_id, 3);
    csync();
    MK_STAMP(prof_id, 4);
    gemv_epilogue<KIND>(a, P, Mx, red, lm, mm);
    MK_STAMP(prof_id, 5);
}

// The CTA's outputs of one GEMV phase from the warps' tile-segment partials.
template <int KIND>
QW_DEV void gemv_epilogue(const MkArgs& a, const PhaseInfo& P, int Mx, const float* red, bool lm,
                                           MkMisc& mm) {
    constexpr int R16 = KIND == K_GU ? 2 : 1;
    const int tid = threadIdx.x, lane = tid & 31;
    const int KG = P.KG;
    const int seg_stride = P.seg_stride;
    // ---- epilogue -------------------------------------------------------------
    const int tfirst = P.tg0 / KG, tlast = (P.tg1 - 1) / KG;
    const int ntl = P.tg1 > P.tg0 ? tlast - tfirst + 1 : 0;
    // CTA partial of tile (tfirst + tl), element (sub, lane slot ln, e): warps in order
    const int tg0 = P.tg0;
    auto cta_part = [&](int tl, int sub, int ln, int e) {
        const int lo = (tfirst + tl) * KG - tg0, hi = lo + KG;  // tile's tile-groups, CTA-relative
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < MK_NW; ++w) {
            const int2 xr = mm.wr[w];
            if (xr.x < xr.y && xr.x < hi && xr.y > lo) {
                const int sg = tl - mm.wft[w];
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
        csync();
    }
    // every tile of the phase is owned by one CTA: outputs (thread per element;
    // the residual read is issued before the reduction so its latency overlaps it)
    const int nout = ntl * 16 * Mx;
    for (int o = tid; o < nout; o += MK_NT) {
        const int m = o % Mx, rr = o / Mx, r = rr & 15, tl = rr >> 4;
        const int row = (tfirst + tl) * 16 + r;
        const int ln = 4 * (r & 7) + (m >> 1), e = 2 * (r >> 3) + (m & 1);
        float resid = 0.f;
        if ((KIND == K_O || KIND == K_DOWN) && !lm) resid = bf2f(__ldcg(a.x + (size_t)m * a.H + row));
        float v[2] = {cta_part(tl, 0, ln, e), R16 == 2 ? cta_part(tl, 1, ln, e) : 0.f};
        store_elem<KIND>(a, lm, row, m, v, best, resid);
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
        csync();
        if (tid < Mx) a.amax_cta[(size_t)blockIdx.x * 8 + tid] = mm.amax[tid];
    }
}

// ---- attention items ---------------------------------------------------------
// Items of one launch: (kv head, query-head group, split) of the sequence, or,
// in a batched step, (sequence, kv head, split) in sequence order with all G
// query heads per item.  A multi-row (verify) launch gives its items the fewest
// query heads (a divisor of G) for which every item still has a CTA of its
// own: fewer rows per item shorten the attention phase, whose slowest item
// every CTA waits for (5-row verify on Qwen3-4B: 3.00 -> 2.80 ms).  A one-row
// step keeps all G per item: more, smaller items measured slower there
// (Qwen3-4B 497 -> 486 tok/s, Qwen3-0.6B 1027 -> 967 tok/s).
template <bool SUB>
QW_DEV int attn_heads_per_item(const MkArgs& a, int nsp) {
    const int G = a.aa.Hq / a.aa.Hkv;
    if (SUB && a.M >= 2)
        for (int h = 1; h < G; ++h)
            if (G % h == 0 && a.aa.Hkv * (G / h) * nsp <= (int)gridDim.x) return h;
    return G;
}
template <bool SUB>
QW_DEV int attn_items(const MkArgs& a, const MkMisc& mm) {
    if (a.nseq > 0) return mm.ibase[a.nseq];
    const int nsp = attn::split_count(mm.seq + a.M);
    if (!SUB) return a.aa.Hkv * nsp;
    return a.aa.Hkv * (a.aa.Hq / a.aa.Hkv / attn_heads_per_item<SUB>(a, nsp)) * nsp;
}
// Item `it` of layer l: its kv head, split, split count, first new position,
// query heads [qh0, qh0 + nqh) of the kv head, and the attention arguments of
// its sequence.
struct AttnItem {
    int kvh, split, nsp, off, qh0, nqh;
};
template <bool SUB>
QW_DEV AttnItem attn_item(const MkArgs& a, const MkMisc& mm, int l, int it, const bf16* qn, const bf16* kn,
                          AttnArgs& aa) {
    aa = a.aa;
    aa.q_norm_w = qn;
    aa.k_norm_w = kn;
    AttnItem r;
    if (a.nseq == 0) {
        r.off = mm.seq;
        r.nsp = attn::split_count(mm.seq + a.M);
        aa.kcache = a.kc0 + (size_t)l * a.kv_layer_elems;
        aa.vcache = a.vc0 + (size_t)l * a.kv_layer_elems;
        if (!SUB) {
            r.kvh = it / r.nsp;
            r.split = it - r.kvh * r.nsp;
            r.qh0 = 0;
            r.nqh = a.aa.Hq / a.aa.Hkv;
            return r;
        }
        r.nqh = attn_heads_per_item<SUB>(a, r.nsp);
        const int per_kvh = (a.aa.Hq / a.aa.Hkv / r.nqh) * r.nsp;
        r.kvh = it / per_kvh;
        const int rem = it - r.kvh * per_kvh;
        const int qg = rem / r.nsp;
        r.split = rem - qg * r.nsp;
        r.qh0 = qg * r.nqh;
        return r;
    }
    int b = 0;
    while (b + 1 < a.nseq && it >= mm.ibase[b + 1]) ++b;
    const int j = it - mm.ibase[b];
    r.off = mm.seqb[b];
    r.nsp = attn::split_count(r.off + 1);
    r.kvh = j / r.nsp;
    r.split = j - r.kvh * r.nsp;
    r.qh0 = 0;
    r.nqh = a.aa.Hq / a.aa.Hkv;
    const MkSeq& sq = a.seqs[b];
    aa.q = a.q + (size_t)b * a.QD;
    aa.k = a.k + (size_t)b * a.KD;
    aa.v = a.v + (size_t)b * a.KD;
    aa.out = a.attn + (size_t)b * a.QD;
    aa.S = 1;
    aa.max_pos = sq.max_pos;
    aa.kcache = sq.kc0 + (size_t)l * sq.kv_layer_elems;
    aa.vcache = sq.vc0 + (size_t)l * sq.kv_layer_elems;
    aa.part = a.aa.part + (size_t)b * a.part_seq_stride;
    aa.counters = a.aa.counters + (size_t)b * a.aa.Hq;
    return r;
}

// ---- the kernel ------------------------------------------------------------
template <int RMAX, int R>
__global__ void __launch_bounds__(MK_NT, 1) decode_step_kernel(const __grid_constant__ MkArgs a) {
    // attention items with fewer query heads only in the multi-row (verify)
    // instantiations: the one-row kernel keeps the plain per-kv-head items
    constexpr bool RMAX_SUB = RMAX > 8;
    extern __shared__ __align__(128) unsigned char sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    MkMisc& mm = *reinterpret_cast<MkMisc*>(sm + a.off_misc);
    unsigned char* ring = sm;
    uint64_t* fullb = reinterpret_cast<uint64_t*>(sm + (size_t)MK_NW * mk_ns(R) * R * GR_BYTES);
    unsigned char* uni = sm + a.off_union;
    const int C = gridDim.x;

    // a finished greedy loop / spec loop turns the remaining replays into no-ops
    if ((a.gate && *a.gate) || (a.ctl && a.ctl->done) || (a.bctl && a.bctl->done)) return;
    if (tid == 0) {
        mm.bad = 0;
        mm.last = 0;
        if (a.nseq > 0) {
            mm.seq = 0;
            mm.ibase[0] = 0;
            for (int b = 0; b < a.nseq; ++b) {
                mm.seqb[b] = *a.seqs[b].seq_len;
                mm.ibase[b + 1] = mm.ibase[b] + a.aa.Hkv * attn::split_count(mm.seqb[b] + 1);
            }
        } else {
            mm.seq = *a.seq_len;
        }
        for (int i = 0; i < MK_NW * MK_NSLOT; ++i) mbar_init(&fullb[i], 1);
        fence_mbar_init();
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
        if (pi >= 4 * a.L) {
            P.norm = a.final_norm;
        } else {
            const MkLayer& Ly = a.layers[pi >> 2];
            const int k = pi & 3;
            P.norm = k == K_QKV ? Ly.in_norm : k == K_O ? Ly.q_norm : k == K_GU ? Ly.post_norm : Ly.k_norm;
        }
        tab[pi] = P;
    }
    __syncthreads();  // the phase table and the stage barriers are ready

    // every warp starts its weight stream: the first NS stages in flight (the
    // warp's issue cursor lives in shared memory: only lane 0 touches it)
    IssueCur& ic = mm.ic[warp];
    unsigned stage = 0;  // stages consumed
    if (lane == 0) {
        ic = IssueCur{0, 0, 0, 0u};
        issue_enter(ic, tab, np, warp);
        for (int i = 0; i < mk_ns(R); ++i) issue_next<R>(ic, tab, np, warp, ring, fullb);
    }

    const int M = a.M;
    unsigned arrivals = 0;  // completed phases (grid barrier target = arrivals * C)
    bool ok = true;
    for (int l = 0; l < a.L && ok; ++l) {
        // this layer's norm weights, from the shared-memory phase table
#define in_norm (tab[4 * l + K_QKV].norm)
#define q_norm (tab[4 * l + K_O].norm)
#define post_norm (tab[4 * l + K_GU].norm)
#define k_norm (tab[4 * l + K_DOWN].norm)
        // ---- q|k|v (x = embedding rows at layer 0)
        {
            const PhaseInfo& lin = tab[4 * l + K_QKV];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            if (l > 0) ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            MK_STAMP(5 * l, 0);
            StageSrc s{l == 0 ? nullptr : a.x, a.H, 0, in_norm};
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
            csync();
            MK_STAMP(5 * l, 1);
            gemv_phase<K_QKV, R>(a, tab[4 * l + K_QKV], M, xs, seeds, red, stage, ring, fullb, ic, tab, np, false, mm,
                                 5 * l + 0);
            // the attention tiles' cached K/V rows do not depend on this step:
            // start loading them before waiting for the other CTAs' q|k|v
            csync();
            {
                // this CTA's first attention item: issue its cached K/V rows now
                if ((int)blockIdx.x < attn_items<RMAX_SUB>(a, mm)) {
                    AttnArgs aa;
                    const AttnItem ai = attn_item<RMAX_SUB>(a, mm, l, blockIdx.x, q_norm, k_norm, aa);
                    attn::split_preload<RMAX>(aa, *reinterpret_cast<attn::SplitSmem<RMAX>*>(uni), ai.kvh, ai.split,
                                              ai.off, tid);
                }
            }
            MK_STAMP(5 * l, 6);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- attention
        {
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            MK_STAMP(5 * l + 1, 0);
            {
                attn::SplitSmem<RMAX>& asm_ = *reinterpret_cast<attn::SplitSmem<RMAX>*>(uni);
                const int items = attn_items<RMAX_SUB>(a, mm);
                for (int it = blockIdx.x; it < items; it += C) {
                    AttnArgs aa;
                    const AttnItem ai = attn_item<RMAX_SUB>(a, mm, l, it, q_norm, k_norm, aa);
                    aa.prof = a.prof ? a.prof + ((size_t)blockIdx.x * MK_PROF_PHASES + 5 * l + 1) * MK_PROF_SLOTS
                                     : nullptr;
                    attn::split_body<RMAX, MK_NT, RMAX_SUB>(aa, asm_, ai.kvh, ai.split, ai.nsp, ai.off, ai.qh0,
                                                            ai.nqh, tid, CSync{}, it == (int)blockIdx.x);
                    csync();
                }
            }
            MK_STAMP(5 * l + 1, 6);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- o_proj + residual
        {
            const PhaseInfo& lin = tab[4 * l + K_O];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            MK_STAMP(5 * l + 2, 0);
            if (a.trace && blockIdx.x == 0) trace_copy_n(a.attn, a.trace_attn + (size_t)l * a.M * a.QD, a.M * a.QD);
            StageSrc s{a.attn, a.QD, 0, nullptr};
            stage_acts(a, s, a.QD, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            csync();
            MK_STAMP(5 * l + 2, 1);
            gemv_phase<K_O, R>(a, tab[4 * l + K_O], M, xs, seeds, red, stage, ring, fullb, ic, tab, np, false, mm,
                                 5 * l + 2);
            MK_STAMP(5 * l + 2, 6);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- gate|up + SwiGLU
        {
            const PhaseInfo& lin = tab[4 * l + K_GU];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            MK_STAMP(5 * l + 3, 0);
            if (a.trace && blockIdx.x == 0) trace_copy_n(a.x, a.trace_mid + (size_t)l * a.M * a.H, a.M * a.H);
            StageSrc s{a.x, a.H, 0, post_norm};
            stage_acts(a, s, a.H, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            csync();
            MK_STAMP(5 * l + 3, 1);
            gemv_phase<K_GU, R>(a, tab[4 * l + K_GU], M, xs, seeds, red, stage, ring, fullb, ic, tab, np, false, mm,
                                 5 * l + 3);
            MK_STAMP(5 * l + 3, 6);
            cta_arrive(a);
            ++arrivals;
        }
        // ---- down + residual
        {
            const PhaseInfo& lin = tab[4 * l + K_DOWN];
            uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
            float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * M * XW * 4);
            float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
            ok = cta_wait(a, arrivals * C, mm);
            if (!ok) break;
            MK_STAMP(5 * l + 4, 0);
            StageSrc s{a.mlp, a.I, 0, nullptr};
            stage_acts(a, s, a.I, M, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            csync();
            MK_STAMP(5 * l + 4, 1);
            gemv_phase<K_DOWN, R>(a, tab[4 * l + K_DOWN], M, xs, seeds, red, stage, ring, fullb, ic, tab, np, false, mm,
                                 5 * l + 4);
            MK_STAMP(5 * l + 4, 6);
            cta_arrive(a);
            ++arrivals;
        }
    }
#undef in_norm
#undef q_norm
#undef post_norm
#undef k_norm
    // ---- final norm -> lm_head -> per-CTA argmax
    if (ok && a.logits_rows > 0) {
        const PhaseInfo& lin = tab[4 * a.L];
        const int rows = a.logits_rows;
        uint32_t* xs = reinterpret_cast<uint32_t*>(uni + MK_UNI_RESERVED);
        float* seeds = reinterpret_cast<float*>(uni + MK_UNI_RESERVED + (size_t)lin.KG * rows * XW * 4);
        float* red = seeds + (size_t)lin.KG * 4 * SEEDF;
        ok = cta_wait(a, arrivals * C, mm);
        MK_STAMP(5 * a.L, 0);
        if (ok && a.trace && blockIdx.x == 0) trace_copy(a, a.L);
        if (ok) {
            StageSrc s{a.x, a.H, M - rows, tab[4 * a.L].norm};
            stage_acts(a, s, a.H, rows, xs, seeds, red + (size_t)MK_NW * lin.seg_stride * lin.R16 * 128, mm);
            csync();
            MK_STAMP(5 * a.L, 1);
            gemv_phase<K_O, R>(a, tab[4 * a.L], rows, xs, seeds, red, stage, ring, fullb, ic, tab, np, true, mm, 5 * a.L);
            MK_STAMP(5 * a.L, 6);
        }
    }
    // no copy may still be landing in shared memory when the CTA exits: after an
    // abort, wait (bounded) for the bulk copies this warp issued but never consumed
    cp_async_wait<0>();
    if (lane == 0) {
        for (unsigned s2 = stage; s2 < ic.stage; ++s2) {
            const unsigned long long t0 = globaltimer();
            while (!mbar_test(&fullb[warp * MK_NSLOT + s2 % mk_ns(R)], (s2 / mk_ns(R)) & 1))
                if (globaltimer() - t0 > 2 * MK_TIMEOUT_NS) break;
        }
    }
    csync();

    // ---- last CTA: argmax over CTAs, step bookkeeping, counter reset
    if (tid == 0) mm.last = atom_add_acq_rel(a.sync + 1, 1u) == (unsigned)(C - 1);
    csync();
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
    csync();
    if (tid == 0) {
        if (!aborted && a.nseq > 0) {
            // batched step: every sequence advanced by its one row
            for (int b = 0; b < a.nseq; ++b) *a.seqs[b].seq_len += 1;
            if (a.bctl) {
                BatchCtl* bc = a.bctl;
                for (int b = 0; b < a.nseq; ++b) {
                    const int tok = a.argmax[b], g = a.b0 + b;
                    if (!bc->stopped[g]) {
                        bool eos = false;
                        for (int i = 0; i < bc->n_eos; ++i) eos |= (bc->eos[i] == tok);
                        if (eos)
                            bc->stopped[g] = 1;
                        else
                            a.out[(size_t)g * bc->max_new + bc->n_out[g]++] = tok;
                    }
                    a.next_tok[g] = tok;
                }
                if (a.bfinalize) {
                    bc->produced += 1;
                    bool all = true;
                    for (int g = 0; g < a.btotal; ++g) all &= bc->stopped[g] != 0;
                    if (all || bc->produced >= bc->max_new) bc->done = 1;
                }
            }
        } else if (!aborted) {
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
            for (int h = 0; h < a.aa.Hq * (a.nseq > 0 ? a.nseq : 1); ++h) a.aa.counters[h] = 0u;
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
            // scales times 2^24 (exact in bf16): the nibbles enter the tensor core as q * 2^-24
            const uint32_t sa = f_to_bf16bits(u16_to_f(S0[(size_t)ra * KG + gl]) * QW_NIB_SCALE);
            const uint32_t sc = f_to_bf16bits(u16_to_f(S1[(size_t)rb * KG + gl]) * QW_NIB_SCALE);
            sbw[2 * h] = sa | ((uint32_t)B0[(size_t)ra * KG + gl] << 16);
            sbw[2 * h + 1] = sc | ((uint32_t)B1[(size_t)rb * KG + gl] << 16);
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
    unsigned long long* prof = nullptr;  // QW_MK_PROFILE: phase timing stamps
    unsigned long long* amax_cta = nullptr;
    int C = 0;
};

void mk_free(qw_model* m) {
    if (!m->mk) return;
    MkState* s = m->mk;
    if (s->packed) cudaFree(s->packed);
    if (s->d_layers) cudaFree(s->d_layers);
    if (s->sync) cudaFree(s->sync);
    if (s->prof) cudaFree(s->prof);
    if (s->amax_cta) cudaFree(s->amax_cta);
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
    if (std::getenv("QW_MK_PROFILE")) {
        const size_t pb = (size_t)C * MK_PROF_PHASES * MK_PROF_SLOTS * sizeof(unsigned long long);
        QW_CUDA(cudaMalloc(&s->prof, pb));
        QW_CUDA(cudaMemsetAsync(s->prof, 0, pb, m->stream));
    }
    QW_CUDA(cudaStreamSynchronize(m->stream));
}

namespace {

static_assert(offsetof(attn::SplitSmem<8>, bar) + sizeof(uint64_t) <= MK_UNI_RESERVED,
              "attention mbarriers must sit in the reserved head of the union");

template <int RMAX>
size_t mk_union_bytes(const MkState* s, int M, int rows, int C) {
    size_t u = sizeof(attn::SplitSmem<RMAX>);
    // staged x', seeds, per-warp partials and (RMSNorm phases) per-unit sums of squares
    auto need = [&](const MkLin& lin, int Mx, bool norm) {
        return (size_t)lin.KG * Mx * XW * 4 + (size_t)lin.KG * 4 * SEEDF * 4 +
               (size_t)MK_NW * lin.seg_stride * lin.R16 * 512 + (norm ? (size_t)lin.KG * Mx * 4 * 4 : 0);
    };
    for (int k = 0; k < 4; ++k) u = std::max(u, MK_UNI_RESERVED + need(s->layers[0].lin[k], M, k == K_QKV || k == K_GU));
    if (rows > 0) u = std::max(u, MK_UNI_RESERVED + need(s->lm, rows, true));
    return (u + 127) & ~(size_t)127;
}

template <int RMAX, int R>
void mk_launch_d(qw_model* m, MkArgs& a, cudaStream_t st, size_t smem, int max_smem) {
    QW_CUDA(ensure_max_dyn_smem(decode_step_kernel<RMAX, R>, max_smem));
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
    QW_CUDA(cudaLaunchKernelEx(&cfg, decode_step_kernel<RMAX, R>, a));
}

// Ring of 16 granules per warp in stages of 4 (or 8), or 8 granules in stages
// of 2, as the phases' sizes and shared memory allow.
template <int RMAX>
bool mk_launch_t(qw_model* m, MkArgs& a, cudaStream_t st) {
    MkState* s = m->mk;
    int max_smem = 0;
    QW_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    const size_t uni = mk_union_bytes<RMAX>(s, a.M, a.logits_rows, s->C);
    const int np = 4 * a.L + (a.logits_rows > 0 ? 1 : 0);
    const size_t misc_struct = (sizeof(MkMisc) + 127) & ~(size_t)127;
    const size_t misc = misc_struct + (((size_t)np * sizeof(PhaseInfo) + 127) & ~(size_t)127);
    const size_t bars = MK_NW * MK_NSLOT * sizeof(uint64_t);  // stage barriers (512 B)
    const long long room = (long long)max_smem - (long long)uni - (long long)misc - (long long)bars;
    // ring bytes for stages of r granules
    auto ring_bytes = [](int r) { return (long long)MK_NW * mk_ns(r) * r * GR_BYTES; };
    // Stage size: the loops stream faster with larger stages, but the weight
    // loop's register footprint then leaves the kernel body fewer registers
    // across the call (its spills cost a round trip per phase).  Measured on
    // Qwen3-4B / 0.6B: stages of 4 where a warp's share of a layer phase
    // averages 4 granules or more, else 2.  QW_MK_STAGE = 2 / 4 / 8 forces a
    // form (profiling, testing every kernel form).
    const MkLayer& L0 = s->layers[0];
    long long gran = 0;
    for (int k = 0; k < 4; ++k) gran += (long long)L0.lin[k].n_tiles * L0.lin[k].KG * L0.lin[k].R16;
    const double per_warp = (double)gran / 4.0 / ((double)s->C * MK_NW);
    int r = per_warp >= 4.0 ? 4 : 2;
    if (const char* e = std::getenv("QW_MK_STAGE")) {
        const int want = std::atoi(e);
        if (want == 2 || want == 4 || want == 8) r = want;
    }
    if (room < ring_bytes(r)) r = room >= ring_bytes(2) ? 2 : 0;
    if (r == 0) return false;
    a.off_union = (unsigned)(ring_bytes(r) + bars);  // a multiple of 128
    a.off_misc = a.off_union + (unsigned)uni;
    a.off_tab = a.off_misc + (unsigned)misc_struct;
    const size_t smem = a.off_misc + misc;
    if (r == 8)
        mk_launch_d<RMAX, 8>(m, a, st, smem, max_smem);
    else if (r == 4)
        mk_launch_d<RMAX, 4>(m, a, st, smem, max_smem);
    else
        mk_launch_d<RMAX, 2>(m, a, st, smem, max_smem);
    return true;
}

}  // namespace

int mk_batch_rows(qw_model* m) {
    MkState* s = m->mk;
    if (!s) return 0;
    int max_smem = 0;
    QW_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    const int G = m->hq_l / m->hkv_l;
    const int np = 4 * m->cfg.layers + 1;
    const size_t misc = ((sizeof(MkMisc) + 127) & ~(size_t)127) + (((size_t)np * sizeof(PhaseInfo) + 127) & ~(size_t)127);
    const size_t bars = MK_NW * MK_NSLOT * sizeof(uint64_t);
    const size_t ring2 = (size_t)MK_NW * mk_ns(2) * 2 * GR_BYTES;
    int best = 0;
    for (int M = 1; M <= 8; ++M) {
        const size_t uni = G <= 8 ? mk_union_bytes<8>(s, M, M, s->C)
                                  : (G <= 16 ? mk_union_bytes<16>(s, M, M, s->C) : mk_union_bytes<32>(s, M, M, s->C));
        if (uni + misc + bars + ring2 <= (size_t)max_smem) best = M;
    }
    // QW_MK_BATCH_ROWS caps it (testing the sub-batched form on small models)
    if (const char* e = std::getenv("QW_MK_BATCH_ROWS")) {
        const int cap = std::atoi(e);
        if (cap >= 1 && cap < best) best = cap;
    }
    return best;
}

size_t mk_prof_read(const qw_model* m, void* dst, size_t bytes) {
    const MkState* s = m->mk;
    if (!s || !s->prof) return 0;
    const size_t pb = (size_t)s->C * MK_PROF_PHASES * MK_PROF_SLOTS * sizeof(unsigned long long);
    if (bytes < pb) return 0;
    QW_CUDA(cudaMemcpy(dst, s->prof, pb, cudaMemcpyDeviceToHost));
    return pb;
}

bool mk_forward(qw_model* m, qw_cache* c, const int* d_ids, int S, int logits_mode, bool store_logits,
                int* d_argmax, cudaStream_t st, StepCtl* ctl, int* next_tok, int* out, const int* gate,
                const MkBatch* batch) {
    MkState* s = m->mk;
    if (batch) {
        if (batch->nseq < 1 || batch->nseq > 8) return false;
        S = batch->nseq;
        c = batch->caches[0];
    }
    if (!s || S < 1 || S > 8) return false;
    const Config& cf = m->cfg;
    Workspace& w = m->ws;
    const int G = m->hq_l / m->hkv_l, R = G * (batch ? 1 : S);
    if (R > 32) return false;
    const int rmax = R <= 8 ? 8 : (R <= 16 ? 16 : 32);
    const int rows = logits_mode == 0 ? 0 : (logits_mode == 2 ? S : 1);
    if (rows > w.cap_logits || S > w.cap_rows) return false;
    // attention partials: [sequence][kv head][128-key split][rmax rows][130] must fit
    // the workspace's [kv head][2 * SMs][64 rows][130] buffer
    int max_pos = c->max_pos;
    if (batch)
        for (int b = 0; b < batch->nseq; ++b) max_pos = std::max(max_pos, batch->caches[b]->max_pos);
    const long long part_seq = (long long)m->hkv_l * ((max_pos + attn::SPLIT_KEYS - 1) / attn::SPLIT_KEYS) * rmax * 130;
    if (part_seq * (batch ? batch->nseq : 1) > (long long)m->hkv_l * 2 * m->num_sms * 64 * 130) return false;

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
    a.err = m->d_err;
    a.trace = m->trace;
    a.trace_mid = m->trace_mid;
    a.trace_attn = m->trace_attn;
    a.prof = s->prof;
    if (batch) {
        a.nseq = batch->nseq;
        a.bctl = batch->bctl;
        a.b0 = batch->b0;
        a.btotal = batch->btotal > 0 ? batch->btotal : batch->nseq;
        a.bfinalize = batch->finalize ? 1 : 0;
        a.part_seq_stride = (size_t)part_seq;
        for (int b = 0; b < batch->nseq; ++b) {
            const qw_cache* cb = batch->caches[b];
            a.seqs[b].kc0 = cb->k;
            a.seqs[b].vc0 = cb->v;
            a.seqs[b].seq_len = cb->d_seq_len;
            a.seqs[b].max_pos = cb->max_pos;
            a.seqs[b].kv_layer_elems = (size_t)m->hkv_l * cb->max_pos * 128;
        }
        a.trace = a.trace_mid = a.trace_attn = nullptr;
    }
    if (R <= 8) return mk_launch_t<8>(m, a, st);
    if (R <= 16) return mk_launch_t<16>(m, a, st);
    return mk_launch_t<32>(m, a, st);
}

}  // namespace qw

