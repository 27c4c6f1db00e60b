// Prefill / multi-row quantized matmul on the 5th-generation tensor cores:
// y[M, N] = x[M, K] . dequant(W)^T for MLX affine 4-bit, group-64 weights
// (the M > 8 rows of mlx_rs::ops::quantized_matmul(x, W, s, b, transpose=true,
// 64, 4) as called from crates/base-mlx-core/src/model/qwen3.rs:30-41 and
// model/kernels.rs:42-44,69-76 during prefill and forward_multi).
//
// Tile: 128 output features (the MMA M) x 128 or 256 activation rows (the MMA N), fp32
// accumulators in tensor memory (TMEM), K walked one 64-wide quantization group
// per stage.  Operands are fp16, K-major, in the 128-byte-swizzled canonical
// layout (one 128-byte row per tile row, its eight 16-byte chunks XOR-permuted
// by row % 8, 1 KB per 8 rows).
//
//   * activations: converted once per call from bf16 to fp16 by
//     x_to_f16p_kernel (exact for |x| in fp16 range), the eight elements of
//     every 8-wide K chunk stored in the order (0,4,1,5,2,6,3,7), rows
//     zero-padded to a multiple of 128; one TMA tensor load (128B swizzle)
//     per stage brings the 128 x 64 tile.
//   * weights: one TMA tensor load per stage of the packed words (128 rows x
//     32 bytes, rows past N zero-filled) and, every 8 stages, of the scales and
//     biases (128 rows x 8 groups); producer threads dequantize: nibble pairs
//     (j, j+4) of a word become the fp16 pair 1024+q with one LOP3, 1024 is
//     subtracted exactly, and w = q*s + b is one fused half2 FMA (a single
//     rounding to fp16).  The pair order matches the activation permutation.
//
// Roles (320 threads): warps 0-7 dequantize into a two-deep operand ring and
// then run the epilogue; lane 0 of warp 8 issues tcgen05.mma (4 per stage per
// 128-row weight tile) and releases stages with tcgen05.commit; lane 0 of
// warp 9 issues the TMA loads into an L-deep load ring.  Warp 8 owns the TMEM
// allocation.  Producers only touch shared memory, so the proxy fence that
// publishes their operand tile never waits on an outstanding global copy.
// Every wait is bounded: a lost arrival sets QW_DERR_TIMEOUT and the CTA
// still releases its TMEM and exits.
//
// RT = 2 runs the gate and up projections of the MLP in one CTA (two TMEM
// accumulators) for the fused SiLU(gate) * up epilogue.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "kernels.h"
#include "qmm_epi.cuh"
#include "smem_attr.h"
#include "tma_map.h"

namespace qw {
namespace {

constexpr int TC_BM = 128;            // output features per tile (MMA M)
constexpr int TC_BN_MAX = 256;        // activation rows per tile (MMA N): 128 or 256
constexpr int TC_PT = 256;            // producer threads (warps 0-7)
constexpr int TC_NT = TC_PT + 64;     // + MMA warp + TMA warp
constexpr int TC_LMAX = 8;            // deepest load ring
constexpr int TC_SMEM_MAX = 232448;   // opt-in shared memory per block
constexpr unsigned long long TC_TIMEOUT_NS = 2000000000ull;

// Shared-memory plan (bytes from the 1 KB-aligned base; every tile 1 KB aligned):
//   [0, 1024)            mbarriers + TMEM address
//   A ring   2 x RT x 16 KB   dequantized weights (fp16, swizzled)
//   SB ring  2 x RT x 4 KB    scales [128][8] bf16 then biases [128][8] bf16
//   load ring L x (16 KB activations + RT x 4 KB packed words)
template <int RT, int BN>
struct TcPlan {
    static constexpr int A_TILE = TC_BM * 128;
    static constexpr int A_OFF = 1024;
    static constexpr int SB_OFF = A_OFF + 2 * RT * A_TILE;
    static constexpr int SB_SLOT = RT * 4096;
    static constexpr int LD_OFF = SB_OFF + 2 * SB_SLOT;
    static constexpr int LD_SLOT = BN * 128 + RT * 4096;
    static constexpr int L = (TC_SMEM_MAX - 1024 - LD_OFF) / LD_SLOT > TC_LMAX ? TC_LMAX
                                                                                : (TC_SMEM_MAX - 1024 - LD_OFF) / LD_SLOT;
    static constexpr int SMEM = LD_OFF + L * LD_SLOT + 1024;  // + base alignment slack
    static constexpr uint32_t TMEM_COLS = RT * BN;
};

// TMA tensor maps of one launch: activations, then per segment the packed
// words, scales and biases.
struct TcMaps {
    CUtensorMap x;
    CUtensorMap w[3], s[3], b[3];
};

// Instruction descriptor (kind::f16): fp32 accumulate, fp16 A and B, both
// K-major, N = BN, M = TC_BM.
template <int BN>
__host__ __device__ constexpr uint32_t tc_idesc() {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 1 KB between
// 8-row groups, descriptor version 1.  A K-step of 16 elements inside the
// 128-byte row advances the start address by 32 bytes.
QW_DEV uint64_t tc_sdesc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

QW_DEV unsigned long long tc_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded mbarrier wait (2 s of wall time).
QW_DEV bool tc_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = tc_clock();
    while (!mbar_try_wait(bar, parity))
        if (tc_clock() - t0 > TC_TIMEOUT_NS) return false;
    return true;
}

QW_DEV void tc_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
QW_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
QW_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QW_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int BN>
QW_DEV void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(tc_idesc<BN>()), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
QW_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
QW_DEV void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
QW_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// (1024 + q_j, 1024 + q_{j+4}) as an fp16 pair, q_j = nibble j of w
QW_DEV uint32_t nib_f16x2(uint32_t w) { return (w & 0x000F000Fu) | 0x64006400u; }

template <int RT, int BN>
__global__ void __launch_bounds__(TC_NT, 1) qgemm_tc_kernel(const QmmArgs a, const __grid_constant__ TcMaps maps) {
    using P = TcPlan<RT, BN>;
    constexpr int L = P::L;
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)tc_smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* ld_full = reinterpret_cast<uint64_t*>(smem);   // [L] TMA -> producers, MMA
    uint64_t* ld_empty = ld_full + TC_LMAX;                   // [L] MMA -> TMA
    uint64_t* a_full = ld_empty + TC_LMAX;                    // [2] producers -> MMA
    uint64_t* a_empty = a_full + 2;                           // [2] MMA -> producers
    uint64_t* sb_full = a_empty + 2;                          // [2] TMA -> producers
    uint64_t* sb_empty = sb_full + 2;                         // [2] producers -> TMA
    uint64_t* done = sb_empty + 2;                            // accumulators final
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KG = a.K / 64;
    const int rb = blockIdx.x, t0 = blockIdx.y * BN;
    // this CTA's groups [g0, g0 + nl): all of K, or whole 8-group chunks of a K split
    const int nch = KG / 8, zs = (int)gridDim.z, z = (int)blockIdx.z;
    const int g0 = 8 * (z * nch / zs), nl = 8 * ((z + 1) * nch / zs) - g0;

    // segment of this row block (q | k | v of the fused qkv launch, or one)
    int si = 0;
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (RT == 1 && i < a.nseg && rb >= a.seg[i].rb0) si = i;
    const int n0 = (rb - a.seg[si].rb0) * TC_BM;

    auto A_of = [&](int slot, int rt) { return smem + P::A_OFF + (slot * RT + rt) * P::A_TILE; };
    auto SB_of = [&](int slot, int rt) { return smem + P::SB_OFF + slot * P::SB_SLOT + rt * 4096; };
    auto X_of = [&](int slot) { return smem + P::LD_OFF + slot * P::LD_SLOT; };
    auto W_of = [&](int slot, int rt) { return smem + P::LD_OFF + slot * P::LD_SLOT + BN * 128 + rt * 4096; };

    if (tid == 0) {
        for (int s = 0; s < L; ++s) {
            mbar_init(ld_full + s, 1);
            mbar_init(ld_empty + s, 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(a_full + s, TC_PT);
            mbar_init(a_empty + s, 1);
            mbar_init(sb_full + s, 1);
            mbar_init(sb_empty + s, TC_PT);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    pdl_wait();

    bool ok = true;
    if (warp < 8) {
        // ---- producers: packed words -> fp16 operand tile --------------------------
        const int row = tid & 127, half = tid >> 7;
        const __half2 k1024 = __float2half2_rn(1024.f);
        for (int gi = 0; gi < nl; ++gi) {
            // gi counts this CTA's groups (rings and parities); chunks start at multiples of 8
            const int ls = gi % L, as = gi & 1, c = gi >> 3;
            if (ok && (gi & 7) == 0 && !tc_wait(sb_full + (c & 1), (c >> 1) & 1)) ok = false;
            if (ok && !tc_wait(ld_full + ls, (gi / L) & 1)) ok = false;
            if (ok && gi >= 2 && !tc_wait(a_empty + as, ((gi - 2) >> 1) & 1)) ok = false;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                const uint4 wr = *reinterpret_cast<const uint4*>(W_of(ls, rt) + row * 32 + half * 16);
                const unsigned short* sbp = reinterpret_cast<const unsigned short*>(SB_of(c & 1, rt));
                const float sf = __uint_as_float((uint32_t)sbp[row * 8 + (gi & 7)] << 16);
                const float bf = __uint_as_float((uint32_t)sbp[1024 + row * 8 + (gi & 7)] << 16);
                const __half2 s2 = __float2half2_rn(sf), b2 = __float2half2_rn(bf);
                const uint32_t wv[4] = {wr.x, wr.y, wr.z, wr.w};
                unsigned char* ad = A_of(as, rt) + row * 128;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    uint32_t o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t h = nib_f16x2(wv[u] >> (4 * j));
                        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&h), k1024);
                        const __half2 r = __hfma2(q, s2, b2);
                        o[j] = *reinterpret_cast<const uint32_t*>(&r);
                    }
                    *reinterpret_cast<uint4*>(ad + (((half * 4 + u) ^ (row & 7)) << 4)) =
                        make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            fence_proxy_async();
            tc_arrive(a_full + as);
            if ((gi & 7) == 7) tc_arrive(sb_empty + (c & 1));
        }
    } else if (warp == 8) {
        if (lane == 0) {
            // ---- MMA issuer ------------------------------------------------------------
            for (int gi = 0; gi < nl; ++gi) {
                const int ls = gi % L, as = gi & 1;
                if (!tc_wait(a_full + as, (gi >> 1) & 1) || !tc_wait(ld_full + ls, (gi / L) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t xb = smem_u32(X_of(ls));
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    const uint32_t ab = smem_u32(A_of(as, rt));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        tc_mma<BN>(tmem + rt * BN, tc_sdesc_sw128(ab + 32 * j), tc_sdesc_sw128(xb + 32 * j),
                               (gi | j) != 0 ? 1u : 0u);
                }
                tc_commit(a_empty + as);
                tc_commit(ld_empty + ls);
            }
            tc_commit(done);
        }
    } else if (lane == 0) {
        // ---- TMA issuer ----------------------------------------------------------------
        const CUtensorMap* wmap[RT];
        const CUtensorMap* smap[RT];
        const CUtensorMap* bmap[RT];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
            const int sg = RT == 2 ? rt : si;
            wmap[rt] = &maps.w[sg];
            smap[rt] = &maps.s[sg];
            bmap[rt] = &maps.b[sg];
        }
        for (int gi = 0; gi < nl; ++gi) {
            const int ls = gi % L, gk = g0 + gi;  // gk: the group's index in K
            if ((gi & 7) == 0) {
                const int c = gi >> 3, ck = gk >> 3;
                if (c >= 2 && !tc_wait(sb_empty + (c & 1), ((c - 2) >> 1) & 1)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(sb_full + (c & 1), RT * 4096);
#pragma unroll
                for (int rt = 0; rt < RT; ++rt) {
                    tma_load_2d(SB_of(c & 1, rt), smap[rt], ck * 8, n0, sb_full + (c & 1));
                    tma_load_2d(SB_of(c & 1, rt) + 2048, bmap[rt], ck * 8, n0, sb_full + (c & 1));
                }
            }
            if (gi >= L && !tc_wait(ld_empty + ls, ((gi - L) / L) & 1)) {
                ok = false;
                break;
            }
            mbar_arrive_expect_tx(ld_full + ls, BN * 128 + RT * 4096);
            tma_load_2d(X_of(ls), &maps.x, gk * 64, t0, ld_full + ls);
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) tma_load_2d(W_of(ls, rt), wmap[rt], gk * 8, n0, ld_full + ls);
        }
    }
    pdl_launch_dependents();

    // ---- epilogue: TMEM -> registers -> outputs --------------------------------------
    if (warp < 8) {
        if (!tc_wait(done, 0)) ok = false;
        tc_fence_after();
        const int lq = warp & 3, ch = warp >> 2;
        const int n = n0 + 32 * lq + lane;
        const bool nvalid = n < a.seg[RT == 2 ? 0 : si].n;
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
            const int c0 = ch * (BN / 2) + cc * 16;
            float v[RT][16];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) tc_ld16(tmem + ((uint32_t)(32 * lq) << 16) + rt * BN + c0, v[rt]);
            tc_wait_ld();
            if (ok && nvalid) {
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int t = t0 + c0 + c;
                    if (t >= a.M) break;
                    if (RT == 2)
                        store_out(a, 0, EPI_SWIGLU, 0, n, t, v[0][c], v[RT - 1][c]);
                    else if (a.ksplit > 1)
                        a.kpart[((size_t)z * a.M + t) * a.seg[0].n + n] = v[0][c];
                    else
                        store_out(a, si, a.epi, n, 0, t, v[0][c], 0.f);
                }
            }
        }
    }
    if (!ok) atomicOr(a.err, QW_DERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::TMEM_COLS)
                     : "memory");
    }
}

// bf16 [M, ldx] -> fp16 [Mpad, K], each 8-wide K chunk permuted to
// (0,4,1,5,2,6,3,7), rows M..Mpad-1 zero.
__global__ void x_to_f16p_kernel(const bf16* __restrict__ x, int ldx, int M, int Mpad, int K, __half* __restrict__ xh) {
    const int cpr = K / 8;
    const long long total = (long long)Mpad * cpr;
    pdl_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / cpr), c = (int)(i - (long long)row * cpr);
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (row < M) {
            const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)row * ldx + (size_t)c * 8);
            const uint32_t X[4] = {u.x, u.y, u.z, u.w};
            float f[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                f[2 * j] = bits_lo_f(X[j]);
                f[2 * j + 1] = bits_hi_f(X[j]);
            }
            const __half2 h0 = __floats2half2_rn(f[0], f[4]), h1 = __floats2half2_rn(f[1], f[5]);
            const __half2 h2 = __floats2half2_rn(f[2], f[6]), h3 = __floats2half2_rn(f[3], f[7]);
            o = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                           *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
        }
        *reinterpret_cast<uint4*>(xh + (size_t)row * K + (size_t)c * 8) = o;
    }
    pdl_launch_dependents();
}

// Sum of a K split's fp32 partials in split order, then the epilogue.
__global__ void ksplit_reduce_kernel(const QmmArgs a) {
    const int N = a.seg[0].n;
    const long long total = (long long)a.M * N, plane = total;
    pdl_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        float v = __ldcg(a.kpart + i);
        for (int z = 1; z < a.ksplit; ++z) v += __ldcg(a.kpart + (size_t)z * plane + i);
        const int t = (int)(i / N), n = (int)(i - (long long)t * N);
        store_out(a, 0, a.epi, n, 0, t, v, 0.f);
    }
    pdl_launch_dependents();
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Weight-side maps depend only on (weight, scale and bias pointers, rows, K):
// cached across calls.
struct SegMaps {
    CUtensorMap w, s, b;
};
bool seg_maps(const QSeg& sg, int K, SegMaps& out) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, const void*, const void*, int, int>, SegMaps> cache;
    const auto key = std::make_tuple((const void*)sg.w, (const void*)sg.s, (const void*)sg.b, sg.n, K);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return true;
    }
    SegMaps m;
    const int KW = K / 8, KG = K / 64;
    if (!make_map(&m.w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, sg.w, KW, sg.n, 8, TC_BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&m.s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sg.s, KG, sg.n, 8, TC_BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&m.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sg.b, KG, sg.n, 8, TC_BM, CU_TENSOR_MAP_SWIZZLE_NONE))
        return false;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    out = m;
    return true;
}

template <int RT, int BN>
cudaError_t launch_tc_t(const QmmArgs& a, const TcMaps& maps, dim3 grid, cudaStream_t st) {
    const cudaError_t e = ensure_max_dyn_smem(qgemm_tc_kernel<RT, BN>, (int)TcPlan<RT, BN>::SMEM);
    if (e != cudaSuccess) return e;
    return launch_pdl(qgemm_tc_kernel<RT, BN>, grid, dim3(TC_NT), (size_t)TcPlan<RT, BN>::SMEM, st, a, maps);
}

}  // namespace

size_t qgemm_tc_scratch_bytes(int M, int K) { return (size_t)((M + TC_BN_MAX - 1) / TC_BN_MAX) * TC_BN_MAX * K * 2; }

bool qgemm_tc_supported(const QmmArgs& a) {
    if (a.M < 9 || a.K < 128 || a.K % 128 != 0 || a.nseg < 1 || a.nseg > 3) return false;
    if (a.epi == EPI_LOGITS || a.norm_w) return false;
    if (a.ldx % 8 != 0) return false;
    if (a.epi == EPI_SWIGLU && (a.nseg < 2 || a.seg[0].n != a.seg[1].n)) return false;
    // TMA: 16-byte aligned bases, row strides a multiple of 16 bytes (K/64
    // groups of bf16 scales per row -> K a multiple of 512)
    if (a.K % 512 != 0 || (uintptr_t)a.x % 16 != 0 || !encode_fn()) return false;
    const int ns = a.epi == EPI_SWIGLU ? 2 : a.nseg;
    for (int i = 0; i < ns; ++i)
        if ((uintptr_t)a.seg[i].w % 16 != 0 || (uintptr_t)a.seg[i].s % 16 != 0 || (uintptr_t)a.seg[i].b % 16 != 0)
            return false;
    return true;
}

int qgemm_tc_ksplit(const QmmArgs& a, int num_sms) {
    if (!qgemm_tc_supported(a) || a.nseg != 1 || num_sms < 1) return 1;
    if (a.epi != EPI_STORE && a.epi != EPI_F32 && a.epi != EPI_RESID) return 1;
    if (std::getenv("QW_TC_BN")) return 1;  // a forced tile width is taken as given
    const int tiles = (a.seg[0].n + TC_BM - 1) / TC_BM * ((a.M + 127) / 128);
    if (tiles * 2 > num_sms) return 1;
    return std::max(1, std::min(a.K / 512, num_sms / tiles));
}

size_t qgemm_tc_ksplit_bytes(const QmmArgs& a, int ksplit) {
    return ksplit > 1 ? (size_t)ksplit * a.M * a.seg[0].n * sizeof(float) : 0;
}

cudaError_t launch_qgemm_tc(QmmArgs a, void* scratch, size_t scratch_bytes, cudaStream_t st, int ksplit) {
    if (!qgemm_tc_supported(a)) return cudaErrorInvalidValue;
    if (ksplit < 1 || ksplit > a.K / 512 || (ksplit > 1 && (a.nseg != 1 || a.epi == EPI_SWIGLU ||
                                                           a.epi == EPI_LOGITS || a.epi == EPI_F32_PUSH)))
        return cudaErrorInvalidValue;
    a.ksplit = ksplit;
    a.kpart = nullptr;
    if (ksplit > 1) {
        const size_t xb = (qgemm_tc_scratch_bytes(a.M, a.K) + 255) & ~(size_t)255;
        if (!scratch || scratch_bytes < xb + qgemm_tc_ksplit_bytes(a, ksplit)) return cudaErrorInvalidValue;
        a.kpart = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + xb);
    }
    // 256 activation rows per tile when that still gives every SM a tile, else 128
    // (QW_TC_BN=128|256 forces one); x is padded to a multiple of 256 rows either way
    const int Mpad = (a.M + TC_BN_MAX - 1) / TC_BN_MAX * TC_BN_MAX;
    if (!scratch || scratch_bytes < qgemm_tc_scratch_bytes(a.M, a.K)) return cudaErrorInvalidValue;
    __half* xh = static_cast<__half*>(scratch);
    int nrb = 0;
    if (a.epi == EPI_SWIGLU) {
        a.seg[0].rb0 = a.seg[1].rb0 = 0;
        a.nseg = 2;
        nrb = (a.seg[0].n + TC_BM - 1) / TC_BM;
    } else {
        for (int i = 0; i < a.nseg; ++i) {
            a.seg[i].rb0 = nrb;
            nrb += (a.seg[i].n + TC_BM - 1) / TC_BM;
        }
    }
    a.nrb = nrb;
    const long long chunks = (long long)Mpad * (a.K / 8);
    const int cblocks = (int)std::min<long long>((chunks + 255) / 256, 148 * 8);
    cudaError_t e = launch_pdl(x_to_f16p_kernel, dim3(cblocks), dim3(256), 0, st, a.x, a.ldx, a.M, Mpad, a.K, xh);
    if (e != cudaSuccess) return e;
    int BN = (long long)nrb * (Mpad / 256) >= 148 ? 256 : 128;
    if (const char* e = std::getenv("QW_TC_BN")) BN = std::atoi(e) == 256 ? 256 : 128;
    if (ksplit > 1) BN = 128;
    TcMaps maps;
    std::memset(&maps, 0, sizeof(maps));
    if (!make_map(&maps.x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, a.K, Mpad, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    for (int i = 0; i < a.nseg; ++i) {
        SegMaps sm;
        if (!seg_maps(a.seg[i], a.K, sm)) return cudaErrorInvalidValue;
        maps.w[i] = sm.w;
        maps.s[i] = sm.s;
        maps.b[i] = sm.b;
    }
    const dim3 grid(nrb, (a.M + BN - 1) / BN, ksplit);
    if (ksplit > 1) {
        e = launch_tc_t<1, 128>(a, maps, grid, st);
        if (e != cudaSuccess) return e;
        const long long total = (long long)a.M * a.seg[0].n;
        const int rblocks = (int)std::min<long long>((total + 255) / 256, 148 * 8);
        return launch_pdl(ksplit_reduce_kernel, dim3(rblocks), dim3(256), 0, st, a);
    }
    if (BN == 256) {
        if (a.epi == EPI_SWIGLU) return launch_tc_t<2, 256>(a, maps, grid, st);
        return launch_tc_t<1, 256>(a, maps, grid, st);
    }
    if (a.epi == EPI_SWIGLU) return launch_tc_t<2, 128>(a, maps, grid, st);
    return launch_tc_t<1, 128>(a, maps, grid, st);
}

}  // namespace qw
