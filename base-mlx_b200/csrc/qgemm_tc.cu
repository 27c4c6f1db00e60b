// Prefill / multi-row quantized matmul on the 5th-generation tensor cores:
// y[M, N] = x[M, K] . dequant(W)^T for MLX affine 4-bit, group-64 weights
// (the M > 8 rows of mlx_rs::ops::quantized_matmul(x, W, s, b, transpose=true,
// 64, 4) as called from crates/base-mlx-core/src/model/qwen3.rs:30-41 and
// model/kernels.rs:42-44,69-76 during prefill and forward_multi).
//
// Tile: 128 output features (the MMA M) x 128 activation rows (the MMA N), fp32
// accumulators in tensor memory (TMEM), K walked one 64-wide quantization group
// per pipeline stage.  Operands are fp16, K-major, in the no-swizzle canonical
// layout (8 rows x 16 bytes per core matrix, core matrices of one 8-row block
// contiguous along K: LBO 128 B between the two K halves of an MMA, SBO 1 KB
// between 8-row blocks).
//
//   * activations: converted once per call from bf16 to fp16 by
//     x_to_f16p_kernel (exact for |x| in fp16 range), with the eight elements
//     of every 8-wide K chunk stored in the order (0,4,1,5,2,6,3,7) and rows
//     zero-padded to a multiple of 128; 16-byte cp.async copies then place
//     each chunk directly in its core-matrix row.
//   * weights: 16-byte cp.async copies of the packed words and 4-byte copies of
//     the (scale, bias) pairs into a raw stage; each producer thread then
//     dequantizes its own 32 weights: nibble pairs (j, j+4) of a word become
//     the fp16 pair 1024+q with one LOP3, 1024 is subtracted exactly, and
//     w = q*s + b is one fused half2 FMA (single rounding to fp16).  The
//     pair order matches the activation permutation above.
//
// Roles (288 threads): warps 0-7 are producers (copies, dequantization) and
// afterwards the epilogue; lane 0 of warp 8 issues tcgen05.mma (4 per stage
// per 128-row weight tile) and signals stage release / completion through
// tcgen05.commit on mbarriers; warp 8 owns the TMEM allocation.  Every wait
// is bounded: a lost arrival sets QW_DERR_TIMEOUT and the CTA still releases
// its TMEM and exits.
//
// RT = 2 runs the gate and up projections of the MLP in one CTA (two TMEM
// accumulators) for the fused SiLU(gate) * up epilogue.
#include <cuda_fp16.h>

#include <algorithm>

#include "kernels.h"
#include "qmm_epi.cuh"

namespace qw {
namespace {

constexpr int TC_BM = 128;            // output features per tile (MMA M)
constexpr int TC_BN = 128;            // activation rows per tile (MMA N)
constexpr int TC_PT = 256;            // producer threads
constexpr int TC_NT = TC_PT + 32;     // + the MMA warp
constexpr unsigned long long TC_TIMEOUT_NS = 2000000000ull;

template <int RT>
struct TcCfg {
    static constexpr int A_BYTES = RT * TC_BM * 64 * 2;   // fp16 weight operand
    static constexpr int B_BYTES = TC_BN * 64 * 2;        // fp16 activation operand
    static constexpr int W_BYTES = RT * TC_BM * 32;       // packed words of one group
    static constexpr int SB_BYTES = RT * 2 * TC_BM * 8;   // (scale pair, bias pair) per row and half
    static constexpr int STAGE = A_BYTES + B_BYTES + W_BYTES + SB_BYTES;
    static constexpr int S = RT == 1 ? 4 : 3;             // pipeline depth
    static constexpr int CTRL = 256;                      // mbarriers + TMEM address
    static constexpr int SMEM = CTRL + S * STAGE + 128;   // + alignment slack
    static constexpr uint32_t TMEM_COLS = RT * TC_BN;
};

// Instruction descriptor (kind::f16): fp32 accumulate, fp16 A and B, both
// K-major, N = TC_BN, M = TC_BM.
constexpr uint32_t TC_IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(TC_BN >> 3) << 17) |
                              ((uint32_t)(TC_BM >> 4) << 24);

// Shared-memory matrix descriptor, no swizzle, K-major (descriptor version 1).
QW_DEV uint64_t tc_sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
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
QW_DEV void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
QW_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
QW_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QW_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

QW_DEV void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
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

template <int RT>
__global__ void __launch_bounds__(TC_NT, 1) qgemm_tc_kernel(const QmmArgs a, const __half* __restrict__ xh) {
    using C = TcCfg<RT>;
    extern __shared__ unsigned char tc_smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)tc_smem_raw + 127) & ~(uintptr_t)127);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);   // [S] producers -> MMA
    uint64_t* empty = full + 4;                           // [S] MMA -> producers
    uint64_t* done = full + 8;                            // accumulators final
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 12);
    unsigned char* stages = smem + C::CTRL;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K, KG = K / 64, KW = K / 8;
    const int rb = blockIdx.x, t0 = blockIdx.y * TC_BN;

    // segment of this row block (q | k | v of the fused qkv launch, or one)
    int si = 0;
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (RT == 1 && i < a.nseg && rb >= a.seg[i].rb0) si = i;
    const int n0 = (rb - a.seg[si].rb0) * TC_BM;

    if (tid == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(full + s, TC_PT);
            mbar_init(empty + s, 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    pdl_wait();

    auto A_of = [&](int slot, int rt) { return stages + (size_t)slot * C::STAGE + rt * (TC_BM * 64 * 2); };
    auto B_of = [&](int slot) { return stages + (size_t)slot * C::STAGE + C::A_BYTES; };
    auto W_of = [&](int slot, int rt) {
        return stages + (size_t)slot * C::STAGE + C::A_BYTES + C::B_BYTES + rt * (TC_BM * 32);
    };
    auto SB_of = [&](int slot, int rt) {
        return stages + (size_t)slot * C::STAGE + C::A_BYTES + C::B_BYTES + C::W_BYTES + rt * (2 * TC_BM * 8);
    };

    bool ok = true;
    if (warp < 8) {
        // ---- producers -------------------------------------------------------
        const int row = tid & 127, half = tid >> 7;
        const uint32_t* wrow[RT];
        const bf16* srow[RT];
        const bf16* brow[RT];
        bool valid[RT];
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
            const QSeg& sg = a.seg[RT == 2 ? rt : si];
            const int n = n0 + row;
            valid[rt] = n < sg.n;
            const int nn = valid[rt] ? n : 0;
            wrow[rt] = sg.w + (size_t)nn * KW + 4 * half;
            srow[rt] = sg.s + (size_t)nn * KG;
            brow[rt] = sg.b + (size_t)nn * KG;
        }
        const __half* xrow = xh + (size_t)t0 * K;

        auto issue = [&](int gi) {
            const int slot = gi % C::S;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                unsigned char* wd = W_of(slot, rt) + row * 32 + half * 16;
                unsigned char* sd = SB_of(slot, rt) + (half * TC_BM + row) * 8;
                if (valid[rt]) {
                    cp_async16(wd, wrow[rt] + (size_t)gi * 8);
                    cp_async4(sd, srow[rt] + (gi & ~1));
                    cp_async4(sd + 4, brow[rt] + (gi & ~1));
                } else {
                    *reinterpret_cast<uint4*>(wd) = make_uint4(0u, 0u, 0u, 0u);
                    *reinterpret_cast<uint2*>(sd) = make_uint2(0u, 0u);
                }
            }
            unsigned char* bd = B_of(slot);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = tid + TC_PT * u;
                const int tt = (q & 7) + 8 * (q >> 6), j = (q >> 3) & 7;
                cp_async16(bd + (tt >> 3) * 1024 + j * 128 + (tt & 7) * 16, xrow + (size_t)tt * K + gi * 64 + j * 8);
            }
        };

#pragma unroll
        for (int i = 0; i < C::S - 1; ++i) {
            if (i < KG) issue(i);
            cp_async_commit();
        }
        const __half2 k1024 = __float2half2_rn(1024.f);
        for (int gi = 0; gi < KG; ++gi) {
            const int ni = gi + C::S - 1;
            if (ni < KG) {
                // slot of stage ni last held stage gi-1: its MMAs must have finished
                if (gi >= 1 && ok && !tc_wait(empty + (gi - 1) % C::S, ((gi - 1) / C::S) & 1)) ok = false;
                issue(ni);
            }
            cp_async_commit();
            cp_async_wait<C::S - 1>();
            const int slot = gi % C::S;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                const uint4 wr = *reinterpret_cast<const uint4*>(W_of(slot, rt) + row * 32 + half * 16);
                const uint2 sbp = *reinterpret_cast<const uint2*>(SB_of(slot, rt) + (half * TC_BM + row) * 8);
                const uint32_t sh = (gi & 1) ? 16u : 0u;
                const float sf = __uint_as_float(((sbp.x >> sh) & 0xFFFFu) << 16);
                const float bf = __uint_as_float(((sbp.y >> sh) & 0xFFFFu) << 16);
                const __half2 s2 = __float2half2_rn(sf), b2 = __float2half2_rn(bf);
                const uint32_t wv[4] = {wr.x, wr.y, wr.z, wr.w};
                unsigned char* ad = A_of(slot, rt) + (row >> 3) * 1024 + (row & 7) * 16;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    uint32_t o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t h = nib_f16x2(wv[u] >> (4 * j));
                        __half2 q = __hsub2(*reinterpret_cast<__half2*>(&h), k1024);
                        __half2 r = __hfma2(q, s2, b2);
                        o[j] = *reinterpret_cast<uint32_t*>(&r);
                    }
                    *reinterpret_cast<uint4*>(ad + (half * 4 + u) * 128) = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            fence_proxy_async();
            tc_arrive(full + slot);
        }
        cp_async_wait<0>();
    } else if (lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------
        for (int gi = 0; gi < KG; ++gi) {
            const int slot = gi % C::S;
            if (!tc_wait(full + slot, (gi / C::S) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t bbase = smem_u32(B_of(slot));
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                const uint32_t abase = smem_u32(A_of(slot, rt));
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    tc_mma(tmem + rt * TC_BN, tc_sdesc(abase + j * 256, 128, 1024), tc_sdesc(bbase + j * 256, 128, 1024),
                           (gi | j) != 0 ? 1u : 0u);
            }
            tc_commit(empty + slot);
        }
        tc_commit(done);
    }
    pdl_launch_dependents();

    // ---- epilogue: TMEM -> registers -> outputs --------------------------------
    if (warp < 8) {
        if (!tc_wait(done, 0)) ok = false;
        tc_fence_after();
        const int lq = warp & 3, ch = warp >> 2;
        const int r = 32 * lq + lane;
        const int n = n0 + r;
        const bool nvalid = n < a.seg[RT == 2 ? 0 : si].n;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
            const int c0 = ch * 64 + cc * 16;
            float v[RT][16];
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) tc_ld16(tmem + ((uint32_t)(32 * lq) << 16) + rt * TC_BN + c0, v[rt]);
            tc_wait_ld();
            if (ok && nvalid) {
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const int t = t0 + c0 + c;
                    if (t >= a.M) break;
                    if (RT == 2)
                        store_out(a, 0, EPI_SWIGLU, 0, n, t, v[0][c], v[RT - 1][c]);
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS)
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

template <int RT>
cudaError_t launch_tc_t(const QmmArgs& a, const __half* xh, dim3 grid, cudaStream_t st) {
    static bool set = false;
    if (!set) {
        const cudaError_t e =
            cudaFuncSetAttribute(qgemm_tc_kernel<RT>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<RT>::SMEM);
        if (e != cudaSuccess) return e;
        set = true;
    }
    return launch_pdl(qgemm_tc_kernel<RT>, grid, dim3(TC_NT), (size_t)TcCfg<RT>::SMEM, st, a, xh);
}

}  // namespace

size_t qgemm_tc_scratch_bytes(int M, int K) { return (size_t)((M + TC_BN - 1) / TC_BN) * TC_BN * K * 2; }

bool qgemm_tc_supported(const QmmArgs& a) {
    if (a.M < 9 || a.K < 128 || a.K % 128 != 0 || a.nseg < 1 || a.nseg > 3) return false;
    if (a.epi == EPI_LOGITS || a.norm_w) return false;
    if (a.ldx % 8 != 0) return false;
    if (a.epi == EPI_SWIGLU && (a.nseg < 2 || a.seg[0].n != a.seg[1].n)) return false;
    if ((uintptr_t)a.x % 16 != 0) return false;
    const int ns = a.epi == EPI_SWIGLU ? 2 : a.nseg;
    for (int i = 0; i < ns; ++i)  // 16-byte word copies, 4-byte scale / bias pair copies
        if ((uintptr_t)a.seg[i].w % 16 != 0 || (uintptr_t)a.seg[i].s % 4 != 0 || (uintptr_t)a.seg[i].b % 4 != 0)
            return false;
    return true;
}

cudaError_t launch_qgemm_tc(QmmArgs a, void* scratch, size_t scratch_bytes, cudaStream_t st) {
    if (!qgemm_tc_supported(a)) return cudaErrorInvalidValue;
    const int Mpad = (a.M + TC_BN - 1) / TC_BN * TC_BN;
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
    const dim3 grid(nrb, Mpad / TC_BN);
    if (a.epi == EPI_SWIGLU) return launch_tc_t<2>(a, xh, grid, st);
    return launch_tc_t<1>(a, xh, grid, st);
}

}  // namespace qw
