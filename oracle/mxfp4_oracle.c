/*
 * CPU oracle for the MXFP4 expert kernels. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
 * library, and only as the checker. The product path (lazylora_b200) never links it and
 * has no CPU fallback.
 *
 * It restates the arithmetic of the reference's native kernels
 * (lazy_lora/native/mxfp4_gemm.c) in plain C:
 *   - E2M1 code table and E8M0 exponent rule, bytes >= 253 contribute zero
 *     (mxfp4_gemm.c:33-43; the same rule as streaming/expert_streamer.py:63,139-142)
 *   - row decode, element 2j in the low nibble of byte j, one scale per 32 columns
 *     (mxfp4_gemm.c:45-62)
 *   - y[M,R] = x[M,K] . W^T                        (mxfp4_gemm,   mxfp4_gemm.c:64-94)
 *   - y[M,K] += dy[M,R] . W   (accumulates into y)  (mxfp4_gemm_t, mxfp4_gemm.c:96-129)
 *   - out[R,K] = W                                   (mxfp4_dequant, mxfp4_gemm.c:142-150)
 * Differences, on purpose: dot products accumulate in double (the reference keeps eight
 * float partial sums), and K is not limited to 4096 (the reference's stack tile is, see
 * mxfp4_gemm.c:72). Both only tighten the check.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static const float kE2M1[16] = {0.f, .5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                 -0.f, -.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

/* 2^(b-127) for b < 253, else 0 (damaged group / E8M0 NaN). */
static inline float e8m0_value(uint8_t b)
{
    return b >= 253 ? 0.f : ldexpf(1.f, (int)b - 127);
}

static inline float w_at(const uint8_t *packed, const uint8_t *scales, int K, int r, int k)
{
    const uint8_t byte = packed[(size_t)r * (K / 2) + k / 2];
    const uint8_t code = (k & 1) ? (byte >> 4) : (byte & 0x0F);
    return kE2M1[code] * e8m0_value(scales[(size_t)r * (K / 32) + k / 32]);
}

void oracle_mxfp4_dequant(float *out, const uint8_t *packed, const uint8_t *scales, int K, int R)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < R; r++)
        for (int k = 0; k < K; k++)
            out[(size_t)r * K + k] = w_at(packed, scales, K, r, k);
}

void oracle_mxfp4_gemm(float *y, const float *x, const uint8_t *packed, const uint8_t *scales,
                       int M, int K, int R)
{
#pragma omp parallel
    {
        float *w = (float *)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(dynamic, 4)
        for (int r = 0; r < R; r++) {
            for (int k = 0; k < K; k++) w[k] = w_at(packed, scales, K, r, k);
            for (int m = 0; m < M; m++) {
                const float *xm = x + (size_t)m * K;
                double acc = 0.0;
                for (int k = 0; k < K; k++) acc += (double)xm[k] * (double)w[k];
                y[(size_t)m * R + r] = (float)acc;
            }
        }
        free(w);
    }
}

void oracle_mxfp4_gemm_t(float *y, const float *dy, const uint8_t *packed, const uint8_t *scales,
                         int M, int K, int R)
{
    /* Each thread owns a block of output columns k, so no reduction across threads. */
#pragma omp parallel for schedule(static)
    for (int k0 = 0; k0 < K; k0 += 32) {
        double acc[32];
        for (int m = 0; m < M; m++) {
            for (int c = 0; c < 32; c++) acc[c] = 0.0;
            for (int r = 0; r < R; r++) {
                const double d = dy[(size_t)m * R + r];
                if (d == 0.0) continue;
                for (int c = 0; c < 32 && k0 + c < K; c++)
                    acc[c] += d * (double)w_at(packed, scales, K, r, k0 + c);
            }
            for (int c = 0; c < 32 && k0 + c < K; c++)
                y[(size_t)m * K + k0 + c] += (float)acc[c];
        }
    }
}

int oracle_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
