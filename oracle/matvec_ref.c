/* C restatement of the reference's fused MXFP4 matvec -- TEST INFRASTRUCTURE ONLY.
 *
 * Restates the Metal kernel body of air_llm/kernels/metal/mxfp4_matvec.py:29-63:
 * one output out[m][n] per loop iteration, walking packed row n byte by byte; each
 * byte yields elements 2j (low nibble) and 2j+1 (high nibble); the E8M0 scale is
 * built by placing the byte in a float's exponent field (byte << 23); magnitudes come
 * from the E2M1 table, the sign from bit 3; two fp32 fma per byte into one fp32
 * accumulator, in k order. The only change is the outer loop: OpenMP threads over
 * output rows n instead of one GPU thread per (n, m).
 *
 * Used by tests as the exact-order numeric check of the reference kernel, and by
 * bench.py as the timed CPU baseline ("port" of the reference path).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static const float kE2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

static inline float e8m0_to_f32(uint8_t b) {
    uint32_t bits = ((uint32_t)b) << 23;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* 3 when the x86-64-v3 clone of k3o_mxfp4_matvec runs on this host, else 2. */
int k3o_isa_level(void) {
    __builtin_cpu_init();
    return __builtin_cpu_supports("x86-64-v3") ? 3 : 2;
}

int k3o_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* x fp32 [M][K]; packed u8 [N][K/2]; scales u8 [N][K/32]; out fp32 [M][N].
 * threads <= 0 uses the OpenMP default. Returns 0, or 1 on a bad shape.
 * Two clones, picked at load time by the CPU's features: x86-64-v3 (fmaf as the FMA3
 * instruction) where the host has it, the x86-64-v2 baseline elsewhere. Both compute the
 * same fused multiply-adds in the same order. */
__attribute__((target_clones("arch=x86-64-v3", "default")))
int k3o_mxfp4_matvec(const float* x, int64_t M, int64_t K, const uint8_t* packed,
                     const uint8_t* scales, int64_t N, float* out, int threads) {
    if (M <= 0 || N <= 0 || K <= 0 || (K % 32) != 0) return 1;
    const int64_t KB = K / 2, KS = K / 32;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        const uint8_t* prow = packed + n * KB;
        const uint8_t* srow = scales + n * KS;
        for (int64_t m = 0; m < M; ++m) {
            const float* xrow = x + m * K;
            float acc = 0.0f;
            for (int64_t kb = 0; kb < KB; ++kb) {
                const uint8_t b = prow[kb];
                const int64_t k0 = kb << 1;
                const float scale = e8m0_to_f32(srow[k0 >> 5]);
                const uint8_t lo = b & 0x0F, hi = (b >> 4) & 0x0F;
                float v0 = kE2M1[lo & 7] * scale;
                float v1 = kE2M1[hi & 7] * scale;
                if (lo & 8) v0 = -v0;
                if (hi & 8) v1 = -v1;
                acc = fmaf(xrow[k0], v0, acc);
                acc = fmaf(xrow[k0 + 1], v1, acc);
            }
            out[m * N + n] = acc;
        }
    }
    return 0;
}
