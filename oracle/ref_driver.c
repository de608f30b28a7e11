/*
 * ref_driver.c -- TEST INFRASTRUCTURE ONLY: drives the reference's own
 * hand-written x86-64 kernels (assembled by oracle/ref_asm.py from the
 * reference's sources/x86_64/*.S) through operations, so that their outputs
 * pin the oracle and make the golden fixtures.
 *
 * The driving follows the reference:
 *   refk_mul_mat      mul_mat.cc:306-366 (compute_shared_weights): the weights
 *                     widened FP16 -> FP32 into panels of 16 columns over all
 *                     of K, [panel][k][16] (gemm.cc:23-110); the rows of x
 *                     packed per k-stretch of 256 into panels of 6,
 *                     [panel][kc][6]; each 6 x 16 tile by
 *                     sdasm_gemm_6x16_avx2, accumulating after the first
 *                     stretch; edge tiles through a scratch tile
 *                     (gemm.cc:tile_part).
 *   refk_gated_gelu   fusion.cc:290-310: sdasm_gated_gelu_avx2 over the
 *                     multiples of 16, the rest by the C++ form's gelu()
 *                     (scalar_math.h:60-63).
 *   refk_exponentials attention.cc:287-301: sdasm_exponentials_avx2 over a
 *                     panel [key][16], n a multiple of 8.
 * Nothing here is the reference's code: it is this project's restatement of
 * how the reference calls its kernels.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { KC = 256, MR = 6, NR = 16 };

void sdasm_gemm_6x16_avx2(int64_t kc, const float *a, const float *b, float *c, int64_t ldc, int64_t accumulate);
void sdasm_gated_gelu_avx2(float *out, const float *x, const float *gate, int64_t n);
void sdasm_exponentials_avx2(float *s, int64_t n, const float *max, double *total);

static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            exp = 127 - 15 + 1;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                --exp;
            }
            bits = sign | (exp << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

static void *aligned(size_t bytes) {
    void *p = NULL;
    if (posix_memalign(&p, 64, bytes ? bytes : 64) != 0) return NULL;
    return p;
}

/* y[m][n] = sum_k x[m][k] w16[n][k]; x (M, K), w16 (N, K), y (M, N). */
int refk_mul_mat(const uint16_t *w16, int N, int K, const float *x, int M, float *y) {
    const int npanels = (N + NR - 1) / NR;
    float *wp = aligned(sizeof(float) * (size_t)npanels * NR * K);
    float *ap = aligned(sizeof(float) * (size_t)((M + MR - 1) / MR) * MR * KC);
    float tile[MR * NR] __attribute__((aligned(64)));
    if (!wp || !ap) return 1;
    for (int p = 0; p < npanels; ++p)
        for (int k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int n = p * NR + j;
                wp[((size_t)p * K + k) * NR + j] = n < N ? half_to_float(w16[(size_t)n * K + k]) : 0.0f;
            }
    for (int k0 = 0; k0 < K; k0 += KC) {
        const int kc = K - k0 < KC ? K - k0 : KC;
        for (int i0 = 0; i0 < M; i0 += MR)
            for (int k = 0; k < kc; ++k)
                for (int i = 0; i < MR; ++i) {
                    const int m = i0 + i;
                    ap[((size_t)(i0 / MR) * kc + k) * MR + i] = m < M ? x[(size_t)m * K + k0 + k] : 0.0f;
                }
        for (int p = 0; p < npanels; ++p) {
            const float *b = wp + ((size_t)p * K + k0) * NR;
            const int cols = N - p * NR < NR ? N - p * NR : NR;
            for (int i0 = 0; i0 < M; i0 += MR) {
                const float *a = ap + (size_t)(i0 / MR) * kc * MR;
                const int rows = M - i0 < MR ? M - i0 : MR;
                float *c = y + (size_t)i0 * N + p * NR;
                if (rows == MR && cols == NR) {
                    sdasm_gemm_6x16_avx2(kc, a, b, c, (int64_t)N * 4, k0 > 0);
                } else {
                    sdasm_gemm_6x16_avx2(kc, a, b, tile, NR * 4, 0);
                    for (int i = 0; i < rows; ++i)
                        for (int j = 0; j < cols; ++j)
                            c[(size_t)i * N + j] = k0 > 0 ? c[(size_t)i * N + j] + tile[i * NR + j] : tile[i * NR + j];
                }
            }
        }
    }
    free(wp);
    free(ap);
    return 0;
}

/* scalar_math.h:34-63: the C++ form's exponential and GELU, for the tail. */
static float c_exponential(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.73f);
    const float magic = 12582912.0f;
    const float z = fmaf(x, 1.44269504088896341f, magic);
    const float n = z - magic;
    float r = fmaf(n, -0.693359375f, x);
    r = fmaf(n, 2.12194440e-4f, r);
    float p = 1.9875691500e-4f;
    p = fmaf(p, r, 1.3981999507e-3f);
    p = fmaf(p, r, 8.3334519073e-3f);
    p = fmaf(p, r, 4.1665795894e-2f);
    p = fmaf(p, r, 1.6666665459e-1f);
    p = fmaf(p, r, 5.0000001201e-1f);
    p = fmaf(p * r, r, r) + 1.0f;
    int32_t zi;
    memcpy(&zi, &z, 4);
    const uint32_t e = (uint32_t)(zi - 0x4b400000 + 127) << 23;
    float s;
    memcpy(&s, &e, 4);
    return p * s;
}

static float c_gelu(float x) {
    const float yv = x * fmaf(0.044715f * x, x, 1.0f);
    return x / (1.0f + c_exponential(-1.5957691216057308f * yv));
}

void refk_gated_gelu(float *out, const float *x, const float *gate, int64_t n) {
    const int64_t whole = n / 16 * 16;
    if (whole > 0) sdasm_gated_gelu_avx2(out, x, gate, whole);
    for (int64_t k = whole; k < n; ++k) out[k] = x[k] * c_gelu(gate[k]);
}

/* s: a panel [n][16] (32-byte aligned by the caller), n a multiple of 8. */
void refk_exponentials(float *s, int64_t n, const float *max, double *total) {
    sdasm_exponentials_avx2(s, n, max, total);
}

/* The C++ form's exponential, for comparison. */
void refk_c_exponential(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = c_exponential(x[i]);
}
