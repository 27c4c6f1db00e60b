/* CPU restatement of MLX quantized_matmul(x, W, s, b, transpose=true, 64, 4).
 *
 * TEST INFRASTRUCTURE ONLY: used by the oracle (tests) and as the timed CPU
 * baseline of bench.py.  Never linked into the product library.
 *
 * Reference call sites: crates/base-mlx-core/src/model/qwen3.rs:30-41 (QLinear)
 * and kernels.rs:42-44,69-76.  y[m,n] = sum_k x[m,k] * (s[n,k/64]*q[n,k] + b[n,k/64])
 * with the dequantised weight formed exactly in fp32 (s*q is exact, one
 * rounding for +b) and an fp32 accumulator per output.  Element k of row n is
 * nibble k%8 (least significant first) of word W[n, k/8].
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

int qmm_ref_f32(const float* x, const uint32_t* w, const uint16_t* scales,
                const uint16_t* biases, float* y, int M, int N, int K, int threads) {
    if (K % 64 != 0 || M < 0 || N < 0) return -1;
    const int kw = K / 8, kg = K / 64;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        float wrow[64];
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int n = 0; n < N; ++n) {
            const uint32_t* wr = w + (size_t)n * kw;
            float acc[16];
            int mcap = M < 16 ? M : 16;
            for (int m0 = 0; m0 < M; m0 += mcap) {
                int mm = (M - m0) < mcap ? (M - m0) : mcap;
                for (int i = 0; i < mm; ++i) acc[i] = 0.f;
                for (int g = 0; g < kg; ++g) {
                    float s = bf16_to_f32(scales[(size_t)n * kg + g]);
                    float b = bf16_to_f32(biases[(size_t)n * kg + g]);
                    for (int j = 0; j < 8; ++j) {
                        uint32_t word = wr[g * 8 + j];
                        for (int i = 0; i < 8; ++i) {
                            float q = (float)((word >> (4 * i)) & 0xFu);
                            wrow[j * 8 + i] = s * q + b;
                        }
                    }
                    for (int i = 0; i < mm; ++i) {
                        const float* xr = x + (size_t)(m0 + i) * K + g * 64;
                        float a = acc[i];
                        for (int k = 0; k < 64; ++k) a += xr[k] * wrow[k];
                        acc[i] = a;
                    }
                }
                for (int i = 0; i < mm; ++i) y[(size_t)(m0 + i) * N + n] = acc[i];
            }
        }
    }
    return 0;
}
