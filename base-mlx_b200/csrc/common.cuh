// Shared device helpers for the sm_100a Qwen3 4-bit decode kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

typedef __nv_bfloat16 bf16;

#define QW_DEV __device__ __forceinline__

// Device-side error flag bits (qw_model::d_err).  A kernel that detects an
// out-of-range index records a bit here and skips the access instead of
// faulting; the host turns a non-zero flag into QW_ERR_DEVICE_FLAG.
enum : int {
    QW_DERR_KV_RANGE = 1,     // KV write/read position >= max_pos
    QW_DERR_TOKEN_RANGE = 2,  // token id >= vocab
    QW_DERR_SHAPE = 4,        // kernel launched with an unsupported shape
    QW_DERR_TIMEOUT = 8,      // a bounded wait on an asynchronous copy gave up
};

QW_DEV float bf2f(bf16 v) { return __bfloat162float(v); }
QW_DEV bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
// round an fp32 value to the nearest bf16 and return it as fp32
QW_DEV float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

QW_DEV float bits_lo_f(uint32_t w) { return __uint_as_float(w << 16); }
QW_DEV float bits_hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
QW_DEV float u16_to_f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
QW_DEV uint16_t f_to_bf16bits(float v) {
    bf16 b = __float2bfloat16_rn(v);
    return *reinterpret_cast<uint16_t*>(&b);
}
QW_DEV uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f_to_bf16bits(lo) | ((uint32_t)f_to_bf16bits(hi) << 16);
}

// ---- programmatic dependent launch (sm_90+) -------------------------------
// Every kernel of a forward calls pdl_wait() before touching data written by
// the previous kernel; weight prefetches (static data) may run before it.
QW_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QW_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- warp-level tensor core op -----------------------------------------
// D[16x8] (fp32) = A[16x16] (bf16, row) * B[16x8] (bf16, col) + C.
// Fragment ownership (lane = 4*g + t): a0:(g, 2t..2t+1) a1:(g+8, 2t..) a2:(g, 2t+8..)
// a3:(g+8, 2t+8..); b0:(k=2t..2t+1, n=g) b1:(k=2t+8.., n=g); c0,c1:(g, 2t..2t+1) c2,c3:(g+8, ..).
QW_DEV void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                     uint32_t b0, uint32_t b1, const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// ---- 4-bit nibbles -> bf16 pairs ----------------------------------------
// For a packed word w (element i at bits 4i), nib_pair(w, j) is a bf16x2
// register holding (128 + q_j, 128 + q_{j+4}): the nibble is dropped into the
// low mantissa bits of bf16 128.0 (0x4300), which represents 128 + q exactly.
QW_DEV uint32_t nib_pair(uint32_t w, int j) {
    return ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
}
// bf16x2 (128.0, 128.0): the A operand whose product with B yields 128 * sum(x).
#define QW_BF16X2_128 0x43004300u

// fp16 variant used by the decode GEMVs: a nibble left in the low mantissa
// bits of an fp16 with a zero exponent field is the subnormal q * 2^-24, and
// one at bits 4-7 is 16q * 2^-24, both exact.  The eight nibbles of a word
// become four fp16 pairs with one shift and four ANDs, and the tensor core
// multiplies the exact small integers q (scaled by 2^-24, folded back into
// the group scale) -- no offset, so the fp32 accumulation carries no
// cancellation:
//   nib_even(w, 0) = (e0, e4), nib_even(w, 8) = (e2, e6)      [q * 2^-24]
//   nib_odd (w, 0) = (e1, e5), nib_odd (w, 8) = (e3, e7)      [16q * 2^-24]
QW_DEV uint32_t nib_even(uint32_t w) { return w & 0x000F000Fu; }
QW_DEV uint32_t nib_odd(uint32_t w) { return w & 0x00F000F0u; }
// 2^24 and 2^20: the factors that turn the subnormal products back into q*x and 16q*x
#define QW_NIB_SCALE 16777216.0f
#define QW_NIB_SCALE_ODD 1048576.0f

// D[16x8] (fp32) = A[16x16] (fp16, row) * B[16x8] (fp16, col) + C (same fragment layout as mma_bf16).
QW_DEV void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                    const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// byte permute (PRMT)
QW_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Rearrange 16 consecutive bf16 values (8 words X0..X7, value 2i in the low
// half of Xi) into the B-fragment order used with nib_pair():
// out = {(x0,x4),(x1,x5),(x2,x6),(x3,x7),(x8,x12),(x9,x13),(x10,x14),(x11,x15)}
QW_DEV void permute16(const uint32_t (&X)[8], uint32_t (&o)[8]) {
    o[0] = prmt(X[0], X[2], 0x5410);
    o[1] = prmt(X[0], X[2], 0x7632);
    o[2] = prmt(X[1], X[3], 0x5410);
    o[3] = prmt(X[1], X[3], 0x7632);
    o[4] = prmt(X[4], X[6], 0x5410);
    o[5] = prmt(X[4], X[6], 0x7632);
    o[6] = prmt(X[5], X[7], 0x5410);
    o[7] = prmt(X[5], X[7], 0x7632);
}

// ---- argmax keys ----------------------------------------------------------
// 64-bit key ordering (value desc, index asc): max over keys is the argmax
// with the lowest index winning ties (MLX argmax semantics).
QW_DEV unsigned long long amax_key(float v, uint32_t idx) {
    uint32_t u = __float_as_uint(v);
    if ((u << 1) == 0u) u = 0u;  // -0.0 and +0.0 are the same value: the lower index wins between them
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
QW_DEV uint32_t amax_key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull); }
QW_DEV unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }

QW_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
QW_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- inter-CTA publication ------------------------------------------------
// atom.add with acquire-release semantics at GPU scope.  Called by one thread
// after a block barrier, it publishes the whole block's earlier writes (the
// barrier orders them before the release, and release is cumulative) and,
// for the CTA that sees the final count, orders the block's later reads
// (after another block barrier) after every earlier publisher's writes.
QW_DEV unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// ---- shared-memory staging: bulk copies (TMA engine) + mbarriers --------
QW_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

QW_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
QW_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// one arrival that also raises the barrier's expected transaction bytes
QW_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// global -> shared bulk copy (16-byte aligned addresses, size a multiple of 16),
// completion counted on `bar` in bytes.  One destination CTA; the source is
// always this GPU's own memory.
QW_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
QW_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Generic-proxy accesses of shared memory (a consumed ring slot) ordered before
// the bulk copy (async proxy) that refills it.
QW_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Bounded wait: gives up after ~2^22 polls (each try_wait already suspends
// for a while), so a lost transfer becomes an error flag instead of a hang.
QW_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Ampere-style 16-byte asynchronous copies (used where each thread places its
// own chunk, e.g. swizzled tiles).  Waiting is done by the hardware.
QW_DEV void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
QW_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// L2 prefetch hint for the 16-byte-aligned interior of [p, p + bytes) in
// pieces of at most 32 KB.  A hint only: reads issued after it still see
// every write that reaches L2 before them, so it may run ahead of the
// programmatic-launch wait even for data the previous kernel writes.
QW_DEV void prefetch_l2_range(const void* p, size_t bytes) {
    uintptr_t b = ((uintptr_t)p + 15) & ~(uintptr_t)15;
    const uintptr_t e = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
    while (b < e) {
        const uint32_t n = (uint32_t)((e - b) < 32768 ? (e - b) : 32768);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b), "r"(n) : "memory");
        b += n;
    }
}
template <int N>
QW_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- seeded generator shared with the CPU oracle ------------------------
QW_DEV uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
