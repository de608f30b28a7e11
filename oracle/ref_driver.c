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
void sdasm_gemm_6x16_avx512(int64_t kc, const float *a, const float *b, float *c, int64_t ldc, int64_t accumulate);
void sdasm_gemm_6x32_avx512(int64_t kc, const float *a, const float *b, int64_t b_next, float *c, int64_t ldc,
                            int64_t accumulate);
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

/* ---- the CPU baseline: the reference's micro-kernel on all host threads --------
 * The reference splits a product's row tiles over its thread pool with a
 * work queue (gemm.cc:142-186); here OpenMP hands out blocks of 48 rows the
 * same way (dynamic schedule), each thread packing its own rows.  The
 * weights are widened into panels once, by all threads. */
#ifdef _OPENMP
#include <omp.h>
#endif

int refk_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* The threads the products use: the caller names them (the host's cores), so
 * that a launcher's OMP_NUM_THREADS does not decide it. */
void refk_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* The micro-kernel the reference picks for the host (cpu.cc:302, Tuning::wide):
 * on AVX-512 the tile of 6 x 32 columns from two adjacent panels
 * (sdasm_gemm_6x32_avx512, gemm_avx512.S) and 6 x 16 at an odd last panel;
 * else AVX2's 6 x 16.  refk_set_isa(0) forces AVX2 (for the golden fixtures). */
static int use_avx512 = -1;

void refk_set_isa(int avx512) { use_avx512 = avx512; }

int refk_isa(void) {
    if (use_avx512 < 0) {
        __builtin_cpu_init();
        use_avx512 = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512vl") &&
                     __builtin_cpu_supports("avx512bw") && __builtin_cpu_supports("avx512dq");
    }
    return use_avx512;
}

static int refk_threads_internal(void) { return refk_threads(); }

/* Widened weight panels are kept between calls, keyed by the weights' address
 * and shape, as the reference's store keeps packed weights (store.cc:202-266):
 * its products never repack a weight they have seen. */
typedef struct {
    const void *w;
    int n, k, layout;
    float *panels;
} packed_entry;
static packed_entry packed_cache[256];
static int packed_next;

static float *cached_panels(const void *w, int n, int k, int layout) {
    for (int i = 0; i < 256; ++i)
        if (packed_cache[i].w == w && packed_cache[i].n == n && packed_cache[i].k == k &&
            packed_cache[i].layout == layout)
            return packed_cache[i].panels;
    return NULL;
}

static void keep_panels(const void *w, int n, int k, int layout, float *panels) {
    packed_entry *e = &packed_cache[packed_next];
    packed_next = (packed_next + 1) % 256;
    free(e->panels);
    e->w = w;
    e->n = n;
    e->k = k;
    e->layout = layout;
    e->panels = panels;
}

/* Forgets every kept panel set (the weights' memory is about to be reused). */
void refk_forget(void) {
    for (int i = 0; i < 256; ++i) {
        free(packed_cache[i].panels);
        packed_cache[i].panels = NULL;
        packed_cache[i].w = NULL;
    }
}

static float *widen_panels(const uint16_t *w16, int N, int K) {
    const int npanels = (N + NR - 1) / NR;
    float *wp = aligned(sizeof(float) * (size_t)npanels * NR * K);
    if (!wp) return NULL;
#pragma omp parallel for schedule(static)
    for (int p = 0; p < npanels; ++p)
        for (int k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int n = p * NR + j;
                wp[((size_t)p * K + k) * NR + j] = n < N ? half_to_float(w16[(size_t)n * K + k]) : 0.0f;
            }
    return wp;
}

/* One block of up to 48 rows whose A panels for stretch k0 are in ap, column
 * panels [p0, p1) (all when p1 <= 0). */
static void block_product_cols(const float *ap, const float *wp, int N, int K, int k0, int kc, int rows_total,
                               float *y, float *tile, int p0, int p1) {
    const int wide = refk_isa();
    void (*tile16)(int64_t, const float *, const float *, float *, int64_t, int64_t) =
        wide ? sdasm_gemm_6x16_avx512 : sdasm_gemm_6x16_avx2;
    for (int p = p0; p < p1; ++p) {
        const float *b = wp + ((size_t)p * K + k0) * NR;
        const int cols = N - p * NR < NR ? N - p * NR : NR;
        /* Two full panels: the 6 x 32 tile over both, rows of whole tiles. */
        if (wide && p + 1 < p1 && N - (p + 1) * NR >= NR) {
            const int64_t b_next = (int64_t)K * NR * 4;
            int i0 = 0;
            for (; i0 + MR <= rows_total; i0 += MR)
                sdasm_gemm_6x32_avx512(kc, ap + (size_t)(i0 / MR) * kc * MR, b, b_next, y + (size_t)i0 * N + p * NR,
                                       (int64_t)N * 4, k0 > 0);
            for (int q = p; q <= p + 1 && i0 < rows_total; ++q) {
                const float *bq = wp + ((size_t)q * K + k0) * NR;
                const int rows = rows_total - i0;
                float *c = y + (size_t)i0 * N + q * NR;
                tile16(kc, ap + (size_t)(i0 / MR) * kc * MR, bq, tile, NR * 4, 0);
                for (int i = 0; i < rows; ++i)
                    for (int j = 0; j < NR; ++j)
                        c[(size_t)i * N + j] = k0 > 0 ? c[(size_t)i * N + j] + tile[i * NR + j] : tile[i * NR + j];
            }
            ++p;
            continue;
        }
        for (int i0 = 0; i0 < rows_total; i0 += MR) {
            const float *a = ap + (size_t)(i0 / MR) * kc * MR;
            const int rows = rows_total - i0 < MR ? rows_total - i0 : MR;
            float *c = y + (size_t)i0 * N + p * NR;
            if (rows == MR && cols == NR) {
                tile16(kc, a, b, c, (int64_t)N * 4, k0 > 0);
            } else {
                tile16(kc, a, b, tile, NR * 4, 0);
                for (int i = 0; i < rows; ++i)
                    for (int j = 0; j < cols; ++j)
                        c[(size_t)i * N + j] = k0 > 0 ? c[(size_t)i * N + j] + tile[i * NR + j] : tile[i * NR + j];
            }
        }
    }
}

static void block_product(const float *ap, const float *wp, int N, int K, int k0, int kc, int rows_total, float *y,
                          float *tile) {
    block_product_cols(ap, wp, N, K, k0, kc, rows_total, y, tile, 0, (N + NR - 1) / NR);
}

/* Work items: blocks of 48 rows, each split over column-panel chunks when the
 * rows alone would leave threads idle (the reference's queue hands out tiles). */
static int column_chunks(int mblocks, int npanels) {
    const int pairs = (npanels + 1) / 2;
    const int want = (4 * refk_threads_internal() + mblocks - 1) / mblocks;
    return want < 1 ? 1 : (want > pairs ? pairs : want);
}

/* Panels per chunk, even, so that a chunk's 6 x 32 tiles pair its own panels. */
static int chunk_panels(int npanels, int chunks) {
    const int per = (npanels + chunks - 1) / chunks;
    return (per + 1) / 2 * 2;
}

/* y (M, N) = x (M, K) w16 (N, K)^T on all threads. */
int refk_mul_mat_mt(const uint16_t *w16, int N, int K, const float *x, int M, float *y) {
    float *wp = cached_panels(w16, N, K, 0);
    if (!wp) {
        wp = widen_panels(w16, N, K);
        if (!wp) return 1;
        keep_panels(w16, N, K, 0, wp);
    }
    const int mblocks = (M + 47) / 48, npanels = (N + NR - 1) / NR;
    const int chunks = column_chunks(mblocks, npanels), per = chunk_panels(npanels, chunks);
    int bad = 0;
#pragma omp parallel
    {
        float *ap = aligned(sizeof(float) * 48 * KC);
        float tile[MR * NR] __attribute__((aligned(64)));
        if (!ap) bad = 1;
#pragma omp for schedule(dynamic)
        for (int w = 0; w < mblocks * chunks; ++w) {
            if (!ap) continue;
            const int mb = w / chunks, p0 = (w % chunks) * per, p1 = p0 + per < npanels ? p0 + per : npanels;
            const int m0 = mb * 48, rows = M - m0 < 48 ? M - m0 : 48;
            for (int k0 = 0; k0 < K; k0 += KC) {
                const int kc = K - k0 < KC ? K - k0 : KC;
                for (int i0 = 0; i0 < rows; i0 += MR)
                    for (int k = 0; k < kc; ++k)
                        for (int i = 0; i < MR; ++i) {
                            const int m = i0 + i;
                            ap[((size_t)(i0 / MR) * kc + k) * MR + i] =
                                m < rows ? x[(size_t)(m0 + m) * K + k0 + k] : 0.0f;
                        }
                block_product_cols(ap, wp, N, K, k0, kc, rows, y + (size_t)m0 * N, tile, p0, p1);
            }
        }
        free(ap);
    }
    return bad;
}

/* The direct convolution as the same product (conv2d.cc:231-316): rows are
 * output positions, columns the output channels, k runs over the taps and, in
 * each tap, the input channels -- the image is first laid channels-last so
 * that a row's k-stretch packs from contiguous channels, and the weights
 * [OC][IC][KH][KW] are widened in that k order.  x [N][IC][H][W], y
 * [position][OC]. */
int refk_conv2d_mt(const uint16_t *w16, int OC, int IC, int KH, int KW, const float *x, int NI, int H, int W,
                   int stride, int pad, int OH, int OW, float *y) {
    const int K = IC * KH * KW;
    const int M = NI * OH * OW;
    const int npanels = (OC + NR - 1) / NR;
    float *wp = cached_panels(w16, OC, K, 1 + KH * 16 + KW);
    const int fresh = wp == NULL;
    if (fresh) wp = aligned(sizeof(float) * (size_t)npanels * NR * K);
    float *xl = aligned(sizeof(float) * (size_t)NI * H * W * IC);
    if (!wp || !xl) return 1;
    if (fresh) keep_panels(w16, OC, K, 1 + KH * 16 + KW, wp);
#pragma omp parallel for schedule(static) if (fresh)
    for (int p = 0; p < (fresh ? npanels : 0); ++p)
        for (int k = 0; k < K; ++k) {
            const int tap = k / IC, ic = k % IC, ky = tap / KW, kx = tap % KW;
            for (int j = 0; j < NR; ++j) {
                const int n = p * NR + j;
                wp[((size_t)p * K + k) * NR + j] =
                    n < OC ? half_to_float(w16[(((size_t)n * IC + ic) * KH + ky) * KW + kx]) : 0.0f;
            }
        }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < NI * H; ++r) {
        const int n = r / H, iy = r % H;
        for (int ix = 0; ix < W; ++ix)
            for (int ic = 0; ic < IC; ++ic)
                xl[(((size_t)n * H + iy) * W + ix) * IC + ic] = x[(((size_t)n * IC + ic) * H + iy) * W + ix];
    }
    const int mblocks = (M + 47) / 48;
    const int chunks = column_chunks(mblocks, npanels), per = chunk_panels(npanels, chunks);
    int bad = 0;
#pragma omp parallel
    {
        float *ap = aligned(sizeof(float) * 48 * KC);
        float tile[MR * NR] __attribute__((aligned(64)));
        if (!ap) bad = 1;
#pragma omp for schedule(dynamic)
        for (int w = 0; w < mblocks * chunks; ++w) {
            if (!ap) continue;
            const int mb = w / chunks, p0 = (w % chunks) * per, p1 = p0 + per < npanels ? p0 + per : npanels;
            const int m0 = mb * 48, rows = M - m0 < 48 ? M - m0 : 48;
            for (int k0 = 0; k0 < K; k0 += KC) {
                const int kc = K - k0 < KC ? K - k0 : KC;
                for (int i0 = 0; i0 < rows; i0 += MR) {
                    float *dst = ap + (size_t)(i0 / MR) * kc * MR;
                    for (int i = 0; i < MR; ++i) {
                        const int live = i0 + i < rows, m = live ? m0 + i0 + i : m0;
                        const int n = m / (OH * OW), pos = m % (OH * OW);
                        const int iy0 = (pos / OW) * stride - pad, ix0 = (pos % OW) * stride - pad;
                        int k = 0;
                        while (k < kc) {
                            const int kk = k0 + k, tap = kk / IC, ic0 = kk % IC, ky = tap / KW, kx = tap % KW;
                            const int run = IC - ic0 < kc - k ? IC - ic0 : kc - k;
                            const int iy = iy0 + ky, ix = ix0 + kx;
                            if (live && iy >= 0 && iy < H && ix >= 0 && ix < W) {
                                const float *src = xl + (((size_t)n * H + iy) * W + ix) * IC + ic0;
                                for (int t = 0; t < run; ++t) dst[(size_t)(k + t) * MR + i] = src[t];
                            } else {
                                for (int t = 0; t < run; ++t) dst[(size_t)(k + t) * MR + i] = 0.0f;
                            }
                            k += run;
                        }
                    }
                }
                block_product_cols(ap, wp, OC, K, k0, kc, rows, y + (size_t)m0 * OC, tile, p0, p1);
            }
        }
        free(ap);
    }
    free(xl);
    return bad;
}

/* Attention as the reference computes it (attention.cc:858-1064), products on
 * its micro-kernel: per head and block of 48 queries, the scores S = scale Q K^T
 * (the keys as a panel matrix of 16 keys x D), per query the maximum, the
 * exponentials (the C++ form's exponential, scalar_math.h:34-51) summed in
 * double, then O = P V (V^T as panels of 16 value dims x LK) and one
 * reciprocal per query.  q [B][LQ][H*D], k [B][LK][H*D], v [B][LK][H*DV],
 * out [B][LQ][H*DV]; queries [0, nq) of each head. */
static float *panels_rows(const float *src, long stride, int N, int K) {
    /* rows n of src (stride floats apart), K floats each, into [panel][k][16]. */
    const int np = (N + NR - 1) / NR;
    float *wp = aligned(sizeof(float) * (size_t)np * NR * K);
    if (!wp) return NULL;
    for (int p = 0; p < np; ++p)
        for (int k = 0; k < K; ++k)
            for (int j = 0; j < NR; ++j) {
                const int n = p * NR + j;
                wp[((size_t)p * K + k) * NR + j] = n < N ? src[(size_t)n * stride + k] : 0.0f;
            }
    return wp;
}

int refk_attention_mt(const float *q, const float *k, const float *v, float *out, int B, int H, int LQ, int LK, int D,
                      int DV, float scale, int nq) {
    const int heads = B * H;
    float **kp = calloc((size_t)heads, sizeof(float *)), **vp = calloc((size_t)heads, sizeof(float *));
    int bad = 0;
    if (!kp || !vp) return 1;
#pragma omp parallel for schedule(dynamic)
    for (int bh = 0; bh < heads; ++bh) {
        const int b = bh / H, h = bh % H;
        kp[bh] = panels_rows(k + ((size_t)b * LK * H + h) * D, (long)H * D, LK, D);
        /* V^T: value dim j's row is v[.][key][h*DV + j] over the keys. */
        float *vt = aligned(sizeof(float) * (size_t)DV * LK);
        if (vt) {
            for (int key = 0; key < LK; ++key)
                for (int j = 0; j < DV; ++j) vt[(size_t)j * LK + key] = v[((size_t)b * LK + key) * H * DV + h * DV + j];
            vp[bh] = panels_rows(vt, LK, DV, LK);
            free(vt);
        }
        if (!kp[bh] || !vp[bh]) bad = 1;
    }
    const int qblocks = (nq + 47) / 48;
    if (!bad) {
#pragma omp parallel
        {
            float *s = aligned(sizeof(float) * 48 * (size_t)((LK + NR - 1) / NR * NR));
            float *ap = aligned(sizeof(float) * 48 * (size_t)(D > KC ? D : KC));
            float *o = aligned(sizeof(float) * 48 * (size_t)((DV + NR - 1) / NR * NR));
            double *sum = malloc(sizeof(double) * 48);
            float tile[MR * NR] __attribute__((aligned(64)));
#pragma omp for schedule(dynamic)
            for (int w = 0; w < heads * qblocks; ++w) {
                if (!s || !ap || !o || !sum) continue;
                const int bh = w / qblocks, qb = w % qblocks, b = bh / H, h = bh % H;
                const int q0 = qb * 48, rows = nq - q0 < 48 ? nq - q0 : 48;
                /* S = Q K^T over K = D (one stretch when D <= 256). */
                for (int k0 = 0; k0 < D; k0 += KC) {
                    const int kc = D - k0 < KC ? D - k0 : KC;
                    for (int i0 = 0; i0 < rows; i0 += MR)
                        for (int kk = 0; kk < kc; ++kk)
                            for (int i = 0; i < MR; ++i)
                                ap[((size_t)(i0 / MR) * kc + kk) * MR + i] =
                                    i0 + i < rows ? q[((size_t)b * LQ + q0 + i0 + i) * H * D + h * D + k0 + kk] : 0.0f;
                    block_product(ap, kp[bh], LK, D, k0, kc, rows, s, tile);
                }
                for (int i = 0; i < rows; ++i) {
                    float *row = s + (size_t)i * LK;
                    float mx = -INFINITY;
                    for (int key = 0; key < LK; ++key) {
                        row[key] *= scale;
                        mx = row[key] > mx ? row[key] : mx;
                    }
                    /* The exponentials in one loop the compiler vectorises (the reference's own are
                     * sdasm_exponentials_*, vector code too), their sum in double in another. */
                    for (int key = 0; key < LK; ++key) row[key] = c_exponential(row[key] - mx);
                    double t = 0.0;
                    for (int key = 0; key < LK; ++key) t += row[key];
                    sum[i] = t;
                }
                /* O = P V over K = LK, stretch by stretch. */
                for (int k0 = 0; k0 < LK; k0 += KC) {
                    const int kc = LK - k0 < KC ? LK - k0 : KC;
                    for (int i0 = 0; i0 < rows; i0 += MR)
                        for (int kk = 0; kk < kc; ++kk)
                            for (int i = 0; i < MR; ++i)
                                ap[((size_t)(i0 / MR) * kc + kk) * MR + i] =
                                    i0 + i < rows ? s[(size_t)(i0 + i) * LK + k0 + kk] : 0.0f;
                    block_product(ap, vp[bh], DV, LK, k0, kc, rows, o, tile);
                }
                for (int i = 0; i < rows; ++i) {
                    const float r = (float)(1.0 / sum[i]);
                    for (int j = 0; j < DV; ++j)
                        out[((size_t)b * LQ + q0 + i) * H * DV + h * DV + j] = o[(size_t)i * DV + j] * r;
                }
            }
            free(s);
            free(ap);
            free(o);
            free(sum);
        }
    }
    for (int bh = 0; bh < heads; ++bh) {
        free(kp[bh]);
        free(vp[bh]);
    }
    free(kp);
    free(vp);
    return bad;
}

/* ------------------------------------------------------------------ Winograd
 * The reference sends a 3x3 stride-1 convolution to Winograd when an image has
 * at least winograd_positions (1024) outputs or all images together few tiles
 * (winograd.cc:194-196, 2107-2123), as F(4x4, 3x3) from winograd4_positions
 * (256) outputs an image with FP16 weights, else F(2x2, 3x3)
 * (winograd.cc:1204-1206, 2230-2272).  Its transforms are hand-written
 * (winograd4_avx512.S); here they are C over channels-last rows (the compiler
 * vectorises the channel loops), with the published transform matrices of
 * Lavin and Gray (F(2x2): points 0, +-1; F(4x4): 0, +-1, +-2), and each of the
 * (F+2)^2 products runs on the reference's micro-kernel as the linear layers'
 * do.  The transformed weights U are kept between calls as its store keeps
 * packed weights.  x [N][IC][H][W], y [position][OC]; padding `pad` on all
 * sides; the outputs OH x OW = H + 2 pad - 2 by W + 2 pad - 2.
 * TEST INFRASTRUCTURE (the CPU baseline's timing), not the product. */

static void bt_f4(const float *d, float *t, int n, size_t step, size_t ostep) {
    /* t_i = sum_j BT[i][j] d_j for the 6 x 6 BT of F(4x4), n lanes, element j at d + j*step. */
    for (int c = 0; c < n; ++c) {
        const float d0 = d[c], d1 = d[step + c], d2 = d[2 * step + c], d3 = d[3 * step + c], d4 = d[4 * step + c],
                    d5 = d[5 * step + c];
        t[c] = 4 * d0 - 5 * d2 + d4;
        t[ostep + c] = -4 * d1 - 4 * d2 + d3 + d4;
        t[2 * ostep + c] = 4 * d1 - 4 * d2 - d3 + d4;
        t[3 * ostep + c] = -2 * d1 - d2 + 2 * d3 + d4;
        t[4 * ostep + c] = 2 * d1 - d2 - 2 * d3 + d4;
        t[5 * ostep + c] = 4 * d1 - 5 * d3 + d5;
    }
}

static void bt_f2(const float *d, float *t, int n, size_t step, size_t ostep) {
    for (int c = 0; c < n; ++c) {
        const float d0 = d[c], d1 = d[step + c], d2 = d[2 * step + c], d3 = d[3 * step + c];
        t[c] = d0 - d2;
        t[ostep + c] = d1 + d2;
        t[2 * ostep + c] = d2 - d1;
        t[3 * ostep + c] = d1 - d3;
    }
}

static void at_f4(const float *m, float *o, int n, size_t step, size_t ostep) {
    for (int c = 0; c < n; ++c) {
        const float m0 = m[c], m1 = m[step + c], m2 = m[2 * step + c], m3 = m[3 * step + c], m4 = m[4 * step + c],
                    m5 = m[5 * step + c];
        o[c] = m0 + m1 + m2 + m3 + m4;
        o[ostep + c] = m1 - m2 + 2 * m3 - 2 * m4;
        o[2 * ostep + c] = m1 + m2 + 4 * m3 + 4 * m4;
        o[3 * ostep + c] = m1 - m2 + 8 * m3 - 8 * m4 + m5;
    }
}

static void at_f2(const float *m, float *o, int n, size_t step, size_t ostep) {
    for (int c = 0; c < n; ++c) {
        const float m0 = m[c], m1 = m[step + c], m2 = m[2 * step + c], m3 = m[3 * step + c];
        o[c] = m0 + m1 + m2;
        o[ostep + c] = m1 - m2 - m3;
    }
}

/* U[xi] = G g G^T of each (oc, ic) kernel, as [xi][panel][ic][16] panels. */
static float *winograd_weights(const uint16_t *w16, int OC, int IC, int F) {
    const int T = F + 2, np = (OC + NR - 1) / NR;
    static const float g4[6][3] = {{0.25f, 0, 0},
                                   {-1.0f / 6, -1.0f / 6, -1.0f / 6},
                                   {-1.0f / 6, 1.0f / 6, -1.0f / 6},
                                   {1.0f / 24, 1.0f / 12, 1.0f / 6},
                                   {1.0f / 24, -1.0f / 12, 1.0f / 6},
                                   {0, 0, 1}};
    static const float g2[4][3] = {{1, 0, 0}, {0.5f, 0.5f, 0.5f}, {0.5f, -0.5f, 0.5f}, {0, 0, 1}};
    float *u = aligned(sizeof(float) * (size_t)T * T * np * NR * IC);
    if (!u) return NULL;
#pragma omp parallel for schedule(static)
    for (int oc = 0; oc < np * NR; ++oc)
        for (int ic = 0; ic < IC; ++ic) {
            float g[3][3], t[6][3], r[6][6];
            for (int a = 0; a < 3; ++a)
                for (int b = 0; b < 3; ++b)
                    g[a][b] = oc < OC ? half_to_float(w16[(((size_t)oc * IC + ic) * 3 + a) * 3 + b]) : 0.0f;
            for (int i = 0; i < T; ++i)
                for (int b = 0; b < 3; ++b) {
                    float s = 0;
                    for (int a = 0; a < 3; ++a) s += (F == 4 ? g4[i][a] : g2[i][a]) * g[a][b];
                    t[i][b] = s;
                }
            for (int i = 0; i < T; ++i)
                for (int j = 0; j < T; ++j) {
                    float s = 0;
                    for (int b = 0; b < 3; ++b) s += t[i][b] * (F == 4 ? g4[j][b] : g2[j][b]);
                    r[i][j] = s;
                }
            const int p = oc / NR, lane = oc % NR;
            for (int xi = 0; xi < T * T; ++xi)
                u[(((size_t)xi * np + p) * IC + ic) * NR + lane] = r[xi / T][xi % T];
        }
    return u;
}

int refk_winograd_mt(const uint16_t *w16, int OC, int IC, const float *x, int NI, int H, int W, int pad, int F,
                     float *y) {
    const int T = F + 2, XI = T * T;
    const int OH = H + 2 * pad - 2, OW = W + 2 * pad - 2;
    const int TH = (OH + F - 1) / F, TW = (OW + F - 1) / F, tiles = NI * TH * TW;
    const int np = (OC + NR - 1) / NR;
    float *u = cached_panels(w16, OC, IC, 100 + F);
    if (!u) {
        u = winograd_weights(w16, OC, IC, F);
        if (!u) return 1;
        keep_panels(w16, OC, IC, 100 + F, u);
    }
    /* Channels-last padded image, V [xi][tile][IC], M [xi][tile][OC]. */
    const int PH = TH * F + 2, PW = TW * F + 2;
    float *xp = aligned(sizeof(float) * (size_t)NI * PH * PW * IC);
    float *v = aligned(sizeof(float) * (size_t)XI * tiles * IC);
    float *m = aligned(sizeof(float) * (size_t)XI * tiles * OC);
    if (!xp || !v || !m) return 1;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < NI * PH; ++r) {
        const int n = r / PH, iy = r % PH - pad;
        for (int ix = 0; ix < PW; ++ix) {
            float *dst = xp + ((size_t)r * PW + ix) * IC;
            const int sx = ix - pad;
            if (iy < 0 || iy >= H || sx < 0 || sx >= W) {
                memset(dst, 0, sizeof(float) * IC);
                continue;
            }
            for (int ic = 0; ic < IC; ++ic) dst[ic] = x[(((size_t)n * IC + ic) * H + iy) * W + sx];
        }
    }
    /* Inputs: V = B^T d B per tile, the channels as lanes. */
#pragma omp parallel
    {
        float *rows = aligned(sizeof(float) * 36 * (size_t)IC), *vt = aligned(sizeof(float) * 36 * (size_t)IC);
#pragma omp for schedule(static)
        for (int t = 0; t < tiles; ++t) {
            const int n = t / (TH * TW), ty = (t / TW) % TH, tx = t % TW;
            const float *patch = xp + (((size_t)n * PH + ty * F) * PW + tx * F) * IC;
            for (int i = 0; i < T; ++i) /* columns of each row of the patch */
                (F == 4 ? bt_f4 : bt_f2)(patch + (size_t)i * PW * IC, rows + (size_t)i * T * IC, IC, IC, IC);
            for (int j = 0; j < T; ++j) /* then down the columns */
                (F == 4 ? bt_f4 : bt_f2)(rows + (size_t)j * IC, vt + (size_t)j * IC, IC, (size_t)T * IC,
                                         (size_t)T * IC);
            for (int xi = 0; xi < XI; ++xi)
                memcpy(v + ((size_t)xi * tiles + t) * IC, vt + (size_t)xi * IC, sizeof(float) * IC);
        }
        free(rows);
        free(vt);
    }
    /* The products M[xi] = V[xi] U[xi]^T: blocks of 48 tiles of one xi. */
    const int mblocks = (tiles + 47) / 48;
    const int chunks = column_chunks(mblocks * XI, np), per = chunk_panels(np, chunks);
    int bad = 0;
#pragma omp parallel
    {
        float *ap = aligned(sizeof(float) * 48 * KC);
        float tile[MR * NR] __attribute__((aligned(64)));
        if (!ap) bad = 1;
#pragma omp for schedule(dynamic)
        for (int w = 0; w < XI * mblocks * chunks; ++w) {
            if (!ap) continue;
            const int xi = w / (mblocks * chunks), rest = w % (mblocks * chunks);
            const int mb = rest / chunks, p0 = (rest % chunks) * per, p1 = p0 + per < np ? p0 + per : np;
            const int m0 = mb * 48, rowsn = tiles - m0 < 48 ? tiles - m0 : 48;
            const float *vx = v + (size_t)xi * tiles * IC;
            const float *ux = u + (size_t)xi * np * NR * IC;
            for (int k0 = 0; k0 < IC; k0 += KC) {
                const int kc = IC - k0 < KC ? IC - k0 : KC;
                for (int i0 = 0; i0 < rowsn; i0 += MR)
                    for (int k = 0; k < kc; ++k)
                        for (int i = 0; i < MR; ++i)
                            ap[((size_t)(i0 / MR) * kc + k) * MR + i] =
                                i0 + i < rowsn ? vx[(size_t)(m0 + i0 + i) * IC + k0 + k] : 0.0f;
                block_product_cols(ap, ux, OC, IC, k0, kc, rowsn, m + ((size_t)xi * tiles + m0) * OC, tile, p0, p1);
            }
        }
        free(ap);
    }
    /* Outputs: Y = A^T M A per tile, the output channels as lanes. */
#pragma omp parallel
    {
        float *mt = aligned(sizeof(float) * 36 * (size_t)OC), *half = aligned(sizeof(float) * 24 * (size_t)OC);
        float *out = aligned(sizeof(float) * 16 * (size_t)OC);
#pragma omp for schedule(static)
        for (int t = 0; t < tiles; ++t) {
            const int n = t / (TH * TW), ty = (t / TW) % TH, tx = t % TW;
            for (int xi = 0; xi < XI; ++xi)
                memcpy(mt + (size_t)xi * OC, m + ((size_t)xi * tiles + t) * OC, sizeof(float) * OC);
            for (int i = 0; i < T; ++i) /* along each row of M */
                (F == 4 ? at_f4 : at_f2)(mt + (size_t)i * T * OC, half + (size_t)i * F * OC, OC, OC, OC);
            for (int j = 0; j < F; ++j) /* then down its columns */
                (F == 4 ? at_f4 : at_f2)(half + (size_t)j * OC, out + (size_t)j * OC, OC, (size_t)F * OC,
                                         (size_t)F * OC);
            for (int a = 0; a < F; ++a)
                for (int b = 0; b < F; ++b) {
                    const int oy = ty * F + a, ox = tx * F + b;
                    if (oy < OH && ox < OW)
                        memcpy(y + (((size_t)n * OH + oy) * OW + ox) * OC, out + ((size_t)a * F + b) * OC,
                               sizeof(float) * OC);
                }
        }
        free(mt);
        free(half);
        free(out);
    }
    free(xp);
    free(v);
    free(m);
    return bad;
}
