// Small kernels of the decode path: embedding gather + dequant, RMSNorm (prefill
// path), row argmax, tensor-parallel residual add, step bookkeeping and the
// seeded random-weight initialiser.
#include "kernels.h"

namespace qw {
namespace {

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

// QEmbedding::lookup (crates/base-mlx-core/src/model/qwen3.rs:57-76):
// x[i, :] = bf16(s * q + b) of row ids[i] of the quantized table.
__global__ void embed_kernel(const int* ids, const uint32_t* w, const bf16* s, const bf16* b, int H,
                             int vocab, bf16* x, int* err) {
    pdl_wait();
    pdl_launch_dependents();
    const int i = blockIdx.x;
    int tok = ids[i];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) atomicOr(err, QW_DERR_TOKEN_RANGE);
        tok = 0;
    }
    const int KW = H / 8, KG = H / 64;
    const uint32_t* wr = w + (size_t)tok * KW;
    const unsigned short* sr = reinterpret_cast<const unsigned short*>(s) + (size_t)tok * KG;
    const unsigned short* br = reinterpret_cast<const unsigned short*>(b) + (size_t)tok * KG;
    for (int j = threadIdx.x; j < KW; j += blockDim.x) {
        const uint32_t word = wr[j];
        const float sc = u16_to_f(sr[j / 8]), bi = u16_to_f(br[j / 8]);
        uint32_t o[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const float lo = fmaf(sc, (float)((word >> (8 * p)) & 0xF), bi);
            const float hi = fmaf(sc, (float)((word >> (8 * p + 4)) & 0xF), bi);
            o[p] = pack_bf16x2(lo, hi);
        }
        *reinterpret_cast<uint4*>(x + (size_t)i * H + 8 * j) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// RmsNorm::forward (qwen3.rs:44-55): y = bf16((x * rsqrt(mean(x^2) + eps)) * w).
__global__ void rmsnorm_kernel(const bf16* x, const bf16* w, bf16* y, int H, float eps) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float red[32];
    __shared__ float rs;
    const bf16* xr = x + (size_t)blockIdx.x * H;
    float ss = 0.f;
    for (int k = threadIdx.x; k < H; k += blockDim.x) {
        const float v = bf2f(xr[k]);
        ss += v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
        rs = 1.0f / sqrtf(tot / (float)H + eps);
    }
    __syncthreads();
    const float r = rs;
    for (int k = threadIdx.x; k < H; k += blockDim.x)
        y[(size_t)blockIdx.x * H + k] = f2bf(__fmul_rn(__fmul_rn(bf2f(xr[k]), r), bf2f(w[k])));
}

// argmax over bf16 logits rows, lowest index on ties (engine.rs:197-201, speculative.rs:168).
__global__ void argmax_rows_kernel(const bf16* logits, int V, int* out, unsigned long long* keys, int off) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned long long red[32];
    const bf16* r = logits + (size_t)blockIdx.x * V;
    unsigned long long best = 0ull;
    for (int j = threadIdx.x; j < V; j += blockDim.x) best = umax64(best, amax_key(bf2f(r[j]), (uint32_t)(j + off)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) b = umax64(b, red[i]);
        out[blockIdx.x] = (int)amax_key_index(b);
        if (keys) keys[blockIdx.x] = b;
    }
}

// Final argmax over the per-CTA maxima of the lm_head GEMV (one CTA).
__global__ void amax_finalize_kernel(const unsigned long long* partial, int nrb, int M, int* out,
                                     unsigned long long* keys) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned long long red[32];
    for (int m = 0; m < M; ++m) {
        unsigned long long b = 0ull;
        for (int r0 = threadIdx.x; r0 < nrb; r0 += blockDim.x * 4) {
            unsigned long long kv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int r = r0 + j * blockDim.x;
                kv[j] = r < nrb ? partial[(size_t)r * M + m] : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) b = umax64(b, kv[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long bb = 0ull;
            for (int i = 0; i < (int)(blockDim.x >> 5); ++i) bb = umax64(bb, red[i]);
            out[m] = (int)amax_key_index(bb);
            if (keys) keys[m] = bb;
        }
        __syncthreads();
    }
}

__global__ void keys_to_index_kernel(const unsigned long long* keys, int n, int* out) {
    pdl_wait();
    pdl_launch_dependents();
    const int i = threadIdx.x;
    if (i < n) out[i] = (int)amax_key_index(keys[i]);
}

// x = bf16(x + bf16(p)) where p is the all-reduced fp32 partial of a
// row-parallel projection (tensor-parallel o_proj / down_proj).
__global__ void resid_add_f32_kernel(bf16* x, const float* p, int n) {
    pdl_wait();
    pdl_launch_dependents();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        x[i] = f2bf(__fadd_rn(bf2f(x[i]), bfr(p[i])));
}

// After a forward of S rows: advance the device-side cache length, and for a
// device-resident greedy loop (engine.rs:161-173) record the picked token.
// While *gate is non-zero (a finished generation) nothing changes.
__global__ void step_finish_kernel(int* seq_len, int S, const int* argmax, StepCtl* ctl, int* next_tok,
                                   int* out, const int* gate) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    if (gate && *gate) return;
    if (ctl == nullptr) {
        *seq_len += S;
        return;
    }
    if (ctl->done) return;
    *seq_len += S;
    const int tok = argmax[0];  // the greedy loop computes logits of the last row only
    ctl->produced += 1;
    bool eos = false;
    for (int i = 0; i < ctl->n_eos; ++i) eos |= (ctl->eos[i] == tok);
    if (eos) {
        ctl->done = 1;
        ctl->finish = 1;
        return;
    }
    out[ctl->n_out] = tok;
    ctl->n_out += 1;
    *next_tok = tok;
    if (ctl->produced >= ctl->max_new) ctl->done = 1;
}

// Seeded weights, identical to oracle/numerics.py: element e of the full
// [rows_full, Kfull] tensor is c(e) * mult with c the centred sum of the four
// 16-bit fields of splitmix64(key + e); each 64-group is quantized with
// scale = bf16((max-min)/15), bias = bf16(min), q = clamp(rint((w-bias)/scale), 0, 15).
QW_DEV float seeded_value(uint64_t key, uint64_t e, float mult) {
    const uint64_t h = splitmix64(key + e);
    const int s4 = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
    return __fmul_rn((float)(s4 - 131070), mult);
}

__global__ void init_qweight_kernel(uint32_t* w, bf16* s, bf16* b, int rows, int K, int row0, int k0,
                                    int Kfull, uint64_t key, float mult) {
    const int KG = K / 64;
    const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (long long)rows * KG) return;
    const int r = (int)(gid / KG), gl = (int)(gid % KG);
    const uint64_t base = (uint64_t)(row0 + r) * (uint64_t)Kfull + (uint64_t)(k0 + gl * 64);
    float mn = 3.0e38f, mx = -3.0e38f;
    for (int i = 0; i < 64; ++i) {
        const float v = seeded_value(key, base + i, mult);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    const float scale = bfr(__fdiv_rn(__fsub_rn(mx, mn), 15.0f));
    const float bias = bfr(mn);
    for (int j = 0; j < 8; ++j) {
        uint32_t word = 0;
        for (int i = 0; i < 8; ++i) {
            float q = 0.f;
            if (scale != 0.f) {
                const float v = seeded_value(key, base + j * 8 + i, mult);
                q = rintf(__fdiv_rn(__fsub_rn(v, bias), scale));
                q = fminf(fmaxf(q, 0.f), 15.f);
            }
            word |= ((uint32_t)q) << (4 * i);
        }
        w[(size_t)r * (K / 8) + gl * 8 + j] = word;
    }
    s[(size_t)r * KG + gl] = f2bf(scale);
    b[(size_t)r * KG + gl] = f2bf(bias);
}

__global__ void init_norm_kernel(bf16* w, int n, uint64_t key, float mult, int ones) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    w[i] = ones ? f2bf(1.0f) : f2bf(__fadd_rn(1.0f, seeded_value(key, (uint64_t)i, mult)));
}

}  // namespace

cudaError_t launch_embed(const int* ids, int S, const uint32_t* w, const bf16* s, const bf16* b, int H,
                         int vocab, bf16* x, int* err, cudaStream_t st, bool pdl) {
    if (H % 64 != 0 || S < 1) return cudaErrorInvalidValue;
    return launch(embed_kernel, dim3(S), dim3(128), 0, st, pdl, ids, w, s, b, H, vocab, x, err);
}

cudaError_t launch_rmsnorm(const bf16* x, const bf16* w, bf16* y, int S, int H, float eps, cudaStream_t st) {
    return launch(rmsnorm_kernel, dim3(S), dim3(256), 0, st, true, x, w, y, H, eps);
}

cudaError_t launch_argmax_rows(const bf16* logits, int rows, int V, int* out, unsigned long long* keys_out,
                               int index_offset, cudaStream_t st) {
    return launch(argmax_rows_kernel, dim3(rows), dim3(1024), 0, st, true, logits, V, out, keys_out, index_offset);
}

cudaError_t launch_amax_finalize(const unsigned long long* partial, int nrb, int M, int* out,
                                 unsigned long long* keys_out, cudaStream_t st) {
    return launch(amax_finalize_kernel, dim3(1), dim3(1024), 0, st, true, partial, nrb, M, out, keys_out);
}

cudaError_t launch_keys_to_index(const unsigned long long* keys, int n, int* out, cudaStream_t st) {
    return launch(keys_to_index_kernel, dim3(1), dim3(((n + 31) / 32) * 32), 0, st, true, keys, n, out);
}

cudaError_t launch_resid_add_f32(bf16* x, const float* p, int n, cudaStream_t st) {
    const int blocks = (n + 255) / 256;
    return launch(resid_add_f32_kernel, dim3(blocks < 1024 ? blocks : 1024), dim3(256), 0, st, true, x, p, n);
}

cudaError_t launch_step_finish(int* seq_len, int S, const int* argmax, StepCtl* ctl, int* next_tok, int* out,
                               const int* gate, cudaStream_t st, bool pdl) {
    return launch(step_finish_kernel, dim3(1), dim3(32), 0, st, pdl, seq_len, S, argmax, ctl, next_tok, out, gate);
}

cudaError_t launch_init_qweight(uint32_t* w, bf16* s, bf16* b, int rows, int K, int row0, int k0, int Kfull,
                                uint64_t key, float mult, cudaStream_t st) {
    if (K % 64 != 0) return cudaErrorInvalidValue;
    const long long groups = (long long)rows * (K / 64);
    const int blocks = (int)((groups + 255) / 256);
    init_qweight_kernel<<<blocks, 256, 0, st>>>(w, s, b, rows, K, row0, k0, Kfull, key, mult);
    return cudaGetLastError();
}

cudaError_t launch_init_norm(bf16* w, int n, uint64_t key, float mult, int ones, cudaStream_t st) {
    init_norm_kernel<<<(n + 255) / 256, 256, 0, st>>>(w, n, key, mult, ones);
    return cudaGetLastError();
}

}  // namespace qw
