/* Seeded random-init quantized weights, restated in C -- TEST INFRASTRUCTURE ONLY.
 *
 * Same values as oracle/numerics.py::quantized_weight (and the CUDA
 * initialiser): element e of a [rows_full, Kfull] tensor is
 * fp32(c(e)) * mult with c(e) the centred sum of the four 16-bit fields of
 * splitmix64(key + e); each 64-element group is quantized with
 * scale = bf16((max-min)/15), bias = bf16(min),
 * q = clamp(rint((w - bias) / scale), 0, 15), packed 8 per uint32 (element k
 * at bits 4*(k%8)).  Used by the CPU baseline to build a full-size model
 * without the GPU.  Every step is a single IEEE fp32 operation (compiled
 * without -ffast-math and without FMA contraction).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline float seeded(uint64_t key, uint64_t e, float mult) {
    const uint64_t h = splitmix64(key + e);
    const int s4 = (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
    volatile float c = (float)(s4 - 131070);
    return c * mult;
}

static inline uint16_t f2bf(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Fill w [rows, K/8], s/b [rows, K/64] with rows row0.. and columns k0.. of the full tensor. */
int synth_qweight(uint32_t* w, uint16_t* s, uint16_t* b, int rows, int K, int row0, int k0, int Kfull,
                  uint64_t key, float mult, int threads) {
    if (K % 64) return -1;
    const int KG = K / 64;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (long long gid = 0; gid < (long long)rows * KG; ++gid) {
        const int r = (int)(gid / KG), gl = (int)(gid % KG);
        const uint64_t base = (uint64_t)(row0 + r) * (uint64_t)Kfull + (uint64_t)(k0 + gl * 64);
        float v[64];
        float mn = 3.0e38f, mx = -3.0e38f;
        for (int i = 0; i < 64; ++i) {
            v[i] = seeded(key, base + i, mult);
            mn = v[i] < mn ? v[i] : mn;
            mx = v[i] > mx ? v[i] : mx;
        }
        volatile float span = mx - mn;
        const float scale = bf2f(f2bf(span / 15.0f));
        const float bias = bf2f(f2bf(mn));
        for (int j = 0; j < 8; ++j) {
            uint32_t word = 0;
            for (int i = 0; i < 8; ++i) {
                float q = 0.f;
                if (scale != 0.f) {
                    volatile float d = v[j * 8 + i] - bias;
                    q = rintf(d / scale);
                    q = q < 0.f ? 0.f : (q > 15.f ? 15.f : q);
                }
                word |= ((uint32_t)q) << (4 * i);
            }
            w[(size_t)r * (K / 8) + gl * 8 + j] = word;
        }
        s[(size_t)r * KG + gl] = f2bf(scale);
        b[(size_t)r * KG + gl] = f2bf(bias);
    }
    return 0;
}
