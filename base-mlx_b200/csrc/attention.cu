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
#include "attn_decode.cuh"
#include "smem_attr.h"

namespace qw {
namespace {

using namespace attn;

// CUDA-core block barrier for the standalone kernel (128 threads).
struct CtaSync {
    QW_DEV void operator()() const { __syncthreads(); }
};

template <int RMAX>
__global__ void __launch_bounds__(128) attn_decode_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) unsigned char smraw[];
    DecSmem<RMAX>& sm = *reinterpret_cast<DecSmem<RMAX>*>(smraw);
    pdl_wait();
    pdl_launch_dependents();
    attn_decode_body<RMAX, 128>(a, sm, blockIdx.x, blockIdx.y, gridDim.y, threadIdx.x, CtaSync{});
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
    const cudaError_t e = ensure_max_dyn_smem(attn_decode_kernel<RMAX>, (int)smem);
    if (e != cudaSuccess) return e;
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
    const cudaError_t e = ensure_max_dyn_smem(attn_prefill_kernel, (int)smem);
    if (e != cudaSuccess) return e;
    return launch(attn_prefill_kernel, dim3(a.Hq, (a.S + PQ - 1) / PQ), dim3(128), smem, st, true, a, qroped);
}

}  // namespace qw
