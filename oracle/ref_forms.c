/*
 * ref_forms.c -- TEST INFRASTRUCTURE ONLY: a CPU restatement of the
 * reference's single-precision forms of the hot-path operations, used as the
 * timed CPU baseline (bench.py's cpu_baseline leg and its --impl reference
 * arm) and by the tests as a second checker.  Nothing in the library links or
 * calls it.
 *
 * Each function follows the reference's algorithm, in plain C that GCC
 * vectorises, parallelised with OpenMP over the reference's work items:
 *   rf_mul_mat   mul_mat.cc:306-366 -- y[m][n] = sum_k x[m][k] w[n][k]: the
 *                weights widened FP16 -> FP32 into panels of 16 columns per
 *                k-stretch of 256 (gemm.cc:23-110), a 6 x 16 register tile
 *                accumulated by FMA over the stretch (microkernel.cc:51-69)
 *                and added to the output stretch after stretch;
 *   rf_conv2d    conv2d.cc:231-316, 512-599 -- the direct convolution as the
 *                same product, the columns of the image packed per block of
 *                output positions (implicit GEMM, no im2col buffer);
 *   rf_attention attention.cc:858-1064 -- per head and block of 32 queries:
 *                scaled scores, their maximum, exponentials (the Cephes-form
 *                exponential of scalar_math.h:34-51) summed in double, the
 *                values summed by them, one reciprocal per query at the end;
 *   rf_group_norm norm.cc:100-140 -- mean and variance in double, two passes,
 *                then (x - mean) * float(1 / sqrt(var + eps)) and the chain
 *                (gamma, beta, SiLU).
 * Layouts are ggml's: w [K, N] FP16 (rows of K), x [K, M], y [N, M]; images
 * [W, H, C, N]; attention q [D, LQ, H] token-major rows of H * D.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { KC = 256, MR = 6, NR = 16 };

static float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            exp = 127 - 15 + 1;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                --exp;
            }
            man &= 0x3ffu;
            bits = sign | (exp << 23) | (man << 13);
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

int rf_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void rf_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* A 6 x 16 tile: c[i][j] (+)= sum over kc of a[k][i] b[k][j] (microkernel.cc:51-69). */
static void tile_6x16(int kc, const float *a, const float *b, float *c, long ldc, int rows, int cols, int add) {
    float acc[MR][NR];
    memset(acc, 0, sizeof acc);
    for (int k = 0; k < kc; ++k) {
        const float *ak = a + (long)k * MR;
        const float *bk = b + (long)k * NR;
        for (int i = 0; i < MR; ++i)
            for (int j = 0; j < NR; ++j) acc[i][j] = fmaf(ak[i], bk[j], acc[i][j]);
    }
    for (int i = 0; i < rows; ++i)
        for (int j = 0; j < cols; ++j) c[i * ldc + j] = add ? c[i * ldc + j] + acc[i][j] : acc[i][j];
}

/* y[m][n] = sum_k x[m][k] w16[n][k], m in [0, M), the reference's form. */
void rf_mul_mat(const uint16_t *w16, int N, int K, const float *x, int M, float *y) {
    const int npanels = (N + NR - 1) / NR;
    float *wp = (float *)malloc(sizeof(float) * (size_t)npanels * NR * K);
    /* The weights' panels over the whole of K: [panel][k][16], widened once. */
#pragma omp parallel for schedule(static)
    for (int p = 0; p < npanels; ++p)
        for (int k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int n = p * NR + j;
                wp[((size_t)p * K + k) * NR + j] = n < N ? half_to_float(w16[(size_t)n * K + k]) : 0.0f;
            }
    const int mblocks = (M + 47) / 48;
#pragma omp parallel
    {
        float *ap = (float *)malloc(sizeof(float) * 48 * KC);
#pragma omp for schedule(dynamic)
        for (int mb = 0; mb < mblocks; ++mb) {
            const int m0 = mb * 48, m1 = m0 + 48 < M ? m0 + 48 : M;
            for (int k0 = 0; k0 < K; k0 += KC) {
                const int kc = K - k0 < KC ? K - k0 : KC;
                /* Rows of x over the stretch into panels of 6: [panel][k][6]. */
                for (int i0 = m0; i0 < m1; i0 += MR)
                    for (int k = 0; k < kc; ++k)
                        for (int i = 0; i < MR; ++i) {
                            const int m = i0 + i;
                            ap[((i0 - m0) / MR * kc + k) * MR + i] = m < m1 ? x[(size_t)m * K + k0 + k] : 0.0f;
                        }
                for (int p = 0; p < npanels; ++p) {
                    const int cols = N - p * NR < NR ? N - p * NR : NR;
                    for (int i0 = m0; i0 < m1; i0 += MR) {
                        const int rows = m1 - i0 < MR ? m1 - i0 : MR;
                        tile_6x16(kc, ap + (size_t)(i0 - m0) / MR * kc * MR, wp + ((size_t)p * K + k0) * NR,
                                  y + (size_t)i0 * N + p * NR, N, rows, cols, k0 > 0);
                    }
                }
            }
        }
        free(ap);
    }
    free(wp);
}

/* out[n][oc][oy][ox] for output channels [oc0, oc1): the direct convolution
 * of x [N][IC][H][W] by w16 [OC][IC][KH][KW], stride/pad/dilation as ggml's. */
void rf_conv2d(const uint16_t *w16, int OC, int IC, int KH, int KW, const float *x, int NI, int H, int W, int s0,
               int s1, int p0, int p1, int d0, int d1, float *out, int oc0, int oc1) {
    const int OH = (H + 2 * p1 - d1 * (KH - 1) - 1) / s1 + 1;
    const int OW = (W + 2 * p0 - d0 * (KW - 1) - 1) / s0 + 1;
    const int K = IC * KH * KW;
    const int noc = oc1 - oc0;
    const int npanels = (noc + NR - 1) / NR;
    float *wp = (float *)malloc(sizeof(float) * (size_t)npanels * NR * K);
#pragma omp parallel for schedule(static)
    for (int p = 0; p < npanels; ++p)
        for (int k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int oc = oc0 + p * NR + j;
                wp[((size_t)p * K + k) * NR + j] = oc < oc1 ? half_to_float(w16[(size_t)oc * K + k]) : 0.0f;
            }
    const long P = (long)NI * OH * OW;
    const long pblocks = (P + 47) / 48;
#pragma omp parallel
    {
        float *ap = (float *)malloc(sizeof(float) * 48 * KC);
        float *tmp = (float *)malloc(sizeof(float) * 48 * NR * npanels);
#pragma omp for schedule(dynamic)
        for (long pb = 0; pb < pblocks; ++pb) {
            const long q0 = pb * 48, q1 = q0 + 48 < P ? q0 + 48 : P;
            for (int k0 = 0; k0 < K; k0 += KC) {
                const int kc = K - k0 < KC ? K - k0 : KC;
                /* The columns of the image for these positions (conv2d.cc:231-316). */
                for (long i0 = q0; i0 < q1; i0 += MR)
                    for (int k = 0; k < kc; ++k) {
                        const int kk = k0 + k;
                        const int ic = kk / (KH * KW), ky = kk / KW % KH, kx = kk % KW;
                        for (int i = 0; i < MR; ++i) {
                            const long q = i0 + i;
                            float v = 0.0f;
                            if (q < q1) {
                                const int ox = (int)(q % OW), oy = (int)(q / OW % OH), n = (int)(q / ((long)OW * OH));
                                const int iy = oy * s1 + ky * d1 - p1, ix = ox * s0 + kx * d0 - p0;
                                if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                                    v = x[(((size_t)n * IC + ic) * H + iy) * W + ix];
                            }
                            ap[((i0 - q0) / MR * kc + k) * MR + i] = v;
                        }
                    }
                for (int p = 0; p < npanels; ++p)
                    for (long i0 = q0; i0 < q1; i0 += MR) {
                        const int rows = q1 - i0 < MR ? (int)(q1 - i0) : MR;
                        tile_6x16(kc, ap + (size_t)(i0 - q0) / MR * kc * MR, wp + ((size_t)p * K + k0) * NR,
                                  tmp + (size_t)(i0 - q0) * NR * npanels + p * NR, (long)NR * npanels, rows, NR,
                                  k0 > 0);
                    }
            }
            for (long q = q0; q < q1; ++q) {
                const int ox = (int)(q % OW), oy = (int)(q / OW % OH), n = (int)(q / ((long)OW * OH));
                for (int j = 0; j < noc; ++j)
                    out[(((size_t)n * OC + oc0 + j) * OH + oy) * OW + ox] = tmp[(size_t)(q - q0) * NR * npanels + j];
            }
        }
        free(ap);
        free(tmp);
    }
    free(wp);
}

/* scalar_math.h:34-51: the Cephes-form exponential. */
static float rf_exp(float x) {
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
    memcpy(&zi, &z, sizeof zi);
    const uint32_t e = (uint32_t)(zi - 0x4b400000 + 127) << 23;
    float s;
    memcpy(&s, &e, sizeof s);
    return p * s;
}

/* Attention of queries [q0, q1) of every head: q [B][LQ][H*D], k/v [B][LK][HK*D], out [B][LQ][H*DV]. */
void rf_attention(const float *q, const float *k, const float *v, float *out, int B, int LQ, int LK, int H, int HK,
                  int D, int DV, float scale, int q0, int q1) {
    const int group = H / HK;
    const int nq = q1 - q0;
    const int qblocks = (nq + 31) / 32;
#pragma omp parallel
    {
        float *s = (float *)malloc(sizeof(float) * 32 * (size_t)LK);
        float *o = (float *)malloc(sizeof(float) * 32 * (size_t)DV);
#pragma omp for collapse(3) schedule(dynamic)
        for (int b = 0; b < B; ++b)
            for (int h = 0; h < H; ++h)
                for (int qb = 0; qb < qblocks; ++qb) {
                    const int hk = h / group;
                    const int i0 = q0 + qb * 32, i1 = i0 + 32 < q1 ? i0 + 32 : q1;
                    for (int i = i0; i < i1; ++i) {
                        const float *qi = q + ((size_t)b * LQ + i) * H * D + (size_t)h * D;
                        float mx = -INFINITY;
                        float *si = s + (size_t)(i - i0) * LK;
                        for (int j = 0; j < LK; ++j) {
                            const float *kj = k + ((size_t)b * LK + j) * HK * D + (size_t)hk * D;
                            float acc = 0.0f;
                            for (int e = 0; e < D; ++e) acc = fmaf(qi[e], kj[e], acc);
                            si[j] = acc * scale;
                            mx = fmaxf(mx, si[j]);
                        }
                        double total = 0.0;
                        for (int j = 0; j < LK; ++j) {
                            si[j] = rf_exp(si[j] - mx);
                            total += (double)si[j];
                        }
                        float *oi = o + (size_t)(i - i0) * DV;
                        for (int e = 0; e < DV; ++e) oi[e] = 0.0f;
                        for (int j = 0; j < LK; ++j) {
                            const float *vj = v + ((size_t)b * LK + j) * HK * DV + (size_t)hk * DV;
                            const float w = si[j];
                            for (int e = 0; e < DV; ++e) oi[e] = fmaf(w, vj[e], oi[e]);
                        }
                        const float recip = (float)(1.0 / total);
                        float *dst = out + ((size_t)b * LQ + i) * H * DV + (size_t)h * DV;
                        for (int e = 0; e < DV; ++e) dst[e] = oi[e] * recip;
                    }
                }
        free(s);
        free(o);
    }
}

/* Group normalisation of x [N][C][HW] with gamma, beta per channel and SiLU (when silu). */
void rf_group_norm(const float *x, float *y, int N, int C, long HW, int groups, float eps, const float *gamma,
                   const float *beta, int silu) {
    const int per = (C + groups - 1) / groups;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int n = 0; n < N; ++n)
        for (int g = 0; g < groups; ++g) {
            const int c0 = g * per, c1 = c0 + per < C ? c0 + per : C;
            if (c0 >= c1) continue;
            const float *xs = x + ((size_t)n * C + c0) * HW;
            const long count = (long)(c1 - c0) * HW;
            double sum = 0.0;
            for (long i = 0; i < count; ++i) sum += (double)xs[i];
            const float mean = (float)(sum / (double)count);
            double sq = 0.0;
            for (long i = 0; i < count; ++i) {
                const float d = xs[i] - mean;
                sq += (double)(d * d);
            }
            const float var = (float)(sq / (double)count);
            const float scale = 1.0f / sqrtf(var + eps);
            for (int c = c0; c < c1; ++c) {
                const float *xr = x + ((size_t)n * C + c) * HW;
                float *yr = y + ((size_t)n * C + c) * HW;
                for (long i = 0; i < HW; ++i) {
                    float v = (xr[i] - mean) * scale;
                    if (gamma) v = v * gamma[c];
                    if (beta) v = v + beta[c];
                    if (silu) v = v / (1.0f + rf_exp(-v));
                    yr[i] = v;
                }
            }
        }
}

/* Layer normalisation of rows of C numbers (norm.cc:148-175): mean and variance
 * summed in double, then gamma and beta per column (when given). */
void rf_norm(const float *x, float *y, long rows, int C, float eps, const float *gamma, const float *beta) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; ++r) {
        const float *xr = x + (size_t)r * C;
        float *yr = y + (size_t)r * C;
        double sum = 0.0;
        for (int i = 0; i < C; ++i) sum += (double)xr[i];
        const float mean = (float)(sum / (double)C);
        double sq = 0.0;
        for (int i = 0; i < C; ++i) {
            const float d = xr[i] - mean;
            sq += (double)(d * d);
        }
        const float scale = 1.0f / sqrtf((float)(sq / (double)C) + eps);
        for (int i = 0; i < C; ++i) {
            float v = (xr[i] - mean) * scale;
            if (gamma) v = v * gamma[i];
            if (beta) v = v + beta[i];
            yr[i] = v;
        }
    }
}

/* ---- the quantized linear layer (bits = 8), quant.h / quant.cc ---------------
 * The inputs: per row, per group of `group` numbers of k (the last group
 * short, its missing numbers standing for zeros): the least and the greatest
 * with 0 between them, s = (hi - lo) / levels, inverse = s > 0 ? 1 / s : 0,
 * zero = rint(-lo * inverse), q = clamp(rint(x * inverse) + zero, 0, levels),
 * the group's scale s and offset s * zero (quant.cc quantize_input_row).
 * The weights: per row of k (an output feature), per group or the whole row,
 * m = max |w|, s = m / wmax, inverse = s > 0 ? 1 / s : 0,
 * q = clamp(rint(w * inverse), -wmax, wmax), scale s, offset s * sum(q)
 * (quant.cc quantize_weights).  The product: per tile element, from 0 (or the
 * output's value, with accumulate), group by group in order,
 * t = fma(sa * sb, sum(qa qb), t); t = fma(-oa, ob, t) (quant.cc qgemm).
 * rint rounds to the nearest and to even on a tie, as nearbyint does in the
 * default mode. */
static void quantize_input_group(const float *x, int n, int group, int levels, uint8_t *q, float *scale,
                                 float *offset) {
    float lo = 0.0f, hi = 0.0f;
    for (int e = 0; e < n; ++e) {
        lo = x[e] < lo ? x[e] : lo;
        hi = x[e] > hi ? x[e] : hi;
    }
    const float s = (hi - lo) / (float)levels;
    const float inverse = s > 0.0f ? 1.0f / s : 0.0f;
    const float zero = rintf(-lo * inverse);
    for (int e = 0; e < group; ++e) {
        float v;
        if (e < n) {
            const float r = rintf(x[e] * inverse);
            v = r + zero;
        } else {
            v = zero;
        }
        v = v < 0.0f ? 0.0f : (v > (float)levels ? (float)levels : v);
        q[e] = (uint8_t)v;
    }
    *scale = s;
    *offset = s * zero;
}

/* Weights (N, K) -> q [N][groups * group] int8, scale and offset [N][groups]. */
void rf_quantize_weights(const float *w, int N, int K, int group, int wmax, int weight_groups, int8_t *qw, float *sw,
                         float *ow) {
    const int groups = (K + group - 1) / group;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        float row_max = 0.0f;
        if (!weight_groups)
            for (int k = 0; k < K; ++k) {
                const float a = fabsf(w[(size_t)n * K + k]);
                row_max = a > row_max ? a : row_max;
            }
        for (int g = 0; g < groups; ++g) {
            const int cnt = K - g * group < group ? K - g * group : group;
            float m = row_max;
            if (weight_groups)
                for (int e = 0; e < cnt; ++e) {
                    const float a = fabsf(w[(size_t)n * K + g * group + e]);
                    m = a > m ? a : m;
                }
            const float s = m / (float)wmax;
            const float inverse = s > 0.0f ? 1.0f / s : 0.0f;
            int sum = 0;
            for (int e = 0; e < group; ++e) {
                const float we = e < cnt ? w[(size_t)n * K + g * group + e] : 0.0f;
                float r = rintf(we * inverse);
                r = r < (float)-wmax ? (float)-wmax : (r > (float)wmax ? (float)wmax : r);
                qw[((size_t)n * groups + g) * group + e] = (int8_t)r;
                sum += (int)r;
            }
            sw[(size_t)n * groups + g] = s;
            ow[(size_t)n * groups + g] = s * (float)sum;
        }
    }
}

/* Inputs (M, K) -> q [M][groups * group] uint8, scale and offset [M][groups]. */
void rf_quantize_inputs(const float *x, int M, int K, int group, int levels, uint8_t *qx, float *sx, float *ox) {
    const int groups = (K + group - 1) / group;
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m)
        for (int g = 0; g < groups; ++g) {
            const int cnt = K - g * group < group ? K - g * group : group;
            quantize_input_group(x + (size_t)m * K + g * group, cnt, group, levels, qx + ((size_t)m * groups + g) * group,
                                 &sx[(size_t)m * groups + g], &ox[(size_t)m * groups + g]);
        }
}

/* The fold of quantized operands: y (M, N), from 0 or (accumulate) y's values. */
void rf_qfold(const uint8_t *qx, const float *sx, const float *ox, int M, const int8_t *qw, const float *sw,
              const float *ow, int N, int groups, int group, float *y, int accumulate) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float t = accumulate ? y[(size_t)m * N + n] : 0.0f;
            for (int g = 0; g < groups; ++g) {
                const uint8_t *a = qx + ((size_t)m * groups + g) * group;
                const int8_t *b = qw + ((size_t)n * groups + g) * group;
                int32_t acc = 0;
                for (int e = 0; e < group; ++e) acc += (int32_t)a[e] * (int32_t)b[e];
                const float sab = sx[(size_t)m * groups + g] * sw[(size_t)n * groups + g];
                t = fmaf(sab, (float)acc, t);
                t = fmaf(-ox[(size_t)m * groups + g], ow[(size_t)n * groups + g], t);
            }
            y[(size_t)m * N + n] = t;
        }
}

void rf_qmul_mat(const float *w, int N, int K, const float *x, int M, float *y, int group, int levels, int wmax,
                 int weight_groups, int accumulate) {
    const int groups = (K + group - 1) / group;
    int8_t *qw = (int8_t *)malloc((size_t)N * groups * group);
    float *sw = (float *)malloc(sizeof(float) * (size_t)N * groups), *ow = (float *)malloc(sizeof(float) * (size_t)N * groups);
    uint8_t *qx = (uint8_t *)malloc((size_t)M * groups * group);
    float *sx = (float *)malloc(sizeof(float) * (size_t)M * groups), *ox = (float *)malloc(sizeof(float) * (size_t)M * groups);
    rf_quantize_weights(w, N, K, group, wmax, weight_groups, qw, sw, ow);
    rf_quantize_inputs(x, M, K, group, levels, qx, sx, ox);
    rf_qfold(qx, sx, ox, M, qw, sw, ow, N, groups, group, y, accumulate);
    free(qw);
    free(sw);
    free(ow);
    free(qx);
    free(sx);
    free(ox);
}

/* The C library's single-precision exp, element by element: the reference's
 * std::exp(float) for the keys past its vector kernel's last eight
 * (attention.cc:287-301). */
void rf_expf(const float *x, float *y, long n) {
    for (long i = 0; i < n; ++i) y[i] = expf(x[i]);
}
