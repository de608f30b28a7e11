/*
 * sdb.h -- the C ABI of the B200 (sm_100a) kernels that stand in for
 * stable-diffusion.assembly's CPU operations.
 *
 * The reference's op layer (sources/ops.h:26-62) hands each operation a ggml
 * node: its sources, its output and the chain of element-wise nodes fused after
 * it (sources/fusion.h:51-91).  These entry points take the same things as
 * plain structs -- sdb_tensor mirrors the fields of ggml_tensor an operation
 * reads (type, ne, nb, data), sdb_chain mirrors sdasm::Epilogue -- with DEVICE
 * addresses, and enqueue the work on a CUDA stream.  Every entry point returns
 * an sdb_status; none aborts the process.  "Not supported" is the reference's
 * "not taken" (hooks.cc:29-55): the caller computes the node some other way.
 *
 * Threading: the entry points may be called from any host thread; the weight
 * store is shared and locked.  Work is stream-ordered; results are ready when
 * the stream is.
 */
#ifndef SDB_H
#define SDB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types, numbered as ggml's (GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1). */
enum { SDB_TYPE_F32 = 0, SDB_TYPE_F16 = 1 };

/* A tensor as ggml describes one: ne[k] elements along dimension k (0 is the
 * fastest), nb[k] bytes between neighbours along it, data a device address. */
typedef struct sdb_tensor {
    int32_t type;
    int64_t ne[4];
    int64_t nb[4];
    void *data;
} sdb_tensor;

/* One step of an epilogue chain (sdasm::Epilogue_step, fusion.h:51-59): an
 * in-place addition or multiplication by an FP32 operand whose element for the
 * output element (i0, i1, i2, i3) is operand[i0*nb[0] + i1*nb[1] + i2*nb[2] +
 * i3*nb[3]] (nb in ELEMENTS, 0 along a broadcast dimension), or SiLU. */
enum { SDB_STEP_ADD = 0, SDB_STEP_MUL = 1, SDB_STEP_SILU = 2 };
#define SDB_MAX_STEPS 6
typedef struct sdb_step {
    int32_t kind;
    const float *operand;
    int64_t nb[4];
} sdb_step;

/* The chain after an operation (sdasm::Epilogue, fusion.h:61-91).  With
 * redirect set, the operation writes its result there instead of into its own
 * output (same extents and strides), and with from_redirect the sum begins
 * from what redirect holds (the residual in its own memory); the steps before
 * are then additions only. */
typedef struct sdb_chain {
    int32_t count;
    sdb_step steps[SDB_MAX_STEPS];
    float *redirect;
    int32_t from_redirect;
} sdb_chain;

typedef enum sdb_status {
    SDB_OK = 0,
    SDB_NOT_SUPPORTED = 1, /* not taken: the caller computes it */
    SDB_INVALID = 2,       /* arguments that describe no valid operation */
    SDB_CUDA_ERROR = 3,    /* a CUDA call failed; sdb_last_error() says which */
    SDB_OUT_OF_MEMORY = 4,
    SDB_DEVICE_ERROR = 5   /* a kernel reported an error word (sdb_device_status) */
} sdb_status;

/* ---- linear layers: GGML_OP_MUL_MAT of a weight matrix ------------------
 * dst[m][n] = sum_k x[m][k] * w[n][k] (+ chain), for w FP16 or FP32 [K, N]
 * and x, dst FP32 with rows m over dimensions 1..3 (mul_mat.cc:9-18).
 * Replaces sdasm::mul_mat_supported / mul_mat_compute (ops.h:40-42,
 * mul_mat.cc:181-194, 1175-1196). */
int sdb_mul_mat_supported(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst);
int sdb_mul_mat(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const sdb_chain *chain,
                void *stream);

/* The same product for a first operand the graph itself writes between calls
 * -- the k of k.q and the v of v.softmax(k.q) when stable-diffusion.cpp builds
 * attention from MUL_MAT and SOFT_MAX (its VAE's 512-dim head, which
 * FLASH_ATTN_EXT does not take): w is packed into the workspace on every call
 * and never kept by the weight store.  The reference packs every operand per
 * call by default (its store budget is none, store.h:22-30, and a node's write
 * forgets what was kept, store.h:17-20). */
int sdb_mul_mat_transient(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const sdb_chain *chain,
                          void *stream);
/* The linear layer with the gated GELU after it (GEGLU): out[m][j] =
 * y[m][j] * GELU(y[m][half + j]), y the product with its chain, half = N/2.
 * Replaces sdasm::mul_mat_gated_supported / mul_mat_compute_gated (ops.h:43-47,
 * fusion.h:110-129, mul_mat.cc:934-1058). */
int sdb_mul_mat_gated_supported(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *out);
int sdb_mul_mat_gated(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *out, const sdb_chain *chain,
                      void *stream);

/* ---- convolutions: GGML_OP_CONV_2D (direct) ------------------------------
 * w [KW, KH, IC, OC] FP16 or FP32, x [W, H, IC, N] FP32, dst [OW, OH, OC, N]
 * FP32; params = {s0, s1, p0, p1, d0, d1} as ggml_conv_2d_direct's op_params.
 * 3x3 stride-1 cases go to Winograd when the tuning allows.  Replaces
 * sdasm::conv2d_* and winograd_* (ops.h:26-36, conv2d.cc:837-858,
 * winograd.cc:2107-2272). */
int sdb_conv2d_supported(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const int32_t params[6]);
int sdb_conv2d(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const int32_t params[6],
               const sdb_chain *chain, void *stream);

/* ---- attention: GGML_OP_FLASH_ATTN_EXT without a mask --------------------
 * q [D, LQ, H, B], k [D, LK, HK, B], v [DV, LK, HK, B] (FP32, or FP16 k/v),
 * dst [DV, H, LQ, B] FP32: softmax(scale q k^T) v per head, H % HK == 0.
 * Replaces sdasm::attention_supported / attention_compute (ops.h:49-54,
 * attention.cc:828-1064).  With a chain (residual add: an extension of the
 * reference, which fuses nothing into attention) the chain is applied to dst. */
int sdb_attention_supported(const sdb_tensor *q, const sdb_tensor *k, const sdb_tensor *v, const sdb_tensor *dst);
int sdb_attention(const sdb_tensor *q, const sdb_tensor *k, const sdb_tensor *v, const sdb_tensor *dst, float scale,
                  const sdb_chain *chain, void *stream);

/* ---- normalisation: GGML_OP_GROUP_NORM and GGML_OP_NORM -----------------
 * Mean and variance in double precision, two passes, then the chain
 * (norm.cc:100-175).  Replaces sdasm::group_norm_* / norm_* (ops.h:56-62). */
int sdb_group_norm(const sdb_tensor *x, const sdb_tensor *dst, int32_t groups, float eps, const sdb_chain *chain,
                   void *stream);
/* (x and dst may also be channels-last images -- [W, H, C, N] with nb[2] = 4 --
 * when C % groups == 0 and every chain step is one value per channel.) */
int sdb_norm(const sdb_tensor *x, const sdb_tensor *dst, float eps, const sdb_chain *chain, void *stream);
/* GroupNorm that allocates nothing, for callers that may not call cudaMalloc
 * (memory owned by another allocator, code running under stream capture, loops
 * that may not take the driver's allocation lock).  No counterpart in the
 * reference, whose CPU ops allocate from the host.  The arguments and result of
 * sdb_group_norm, for the contiguous (channel-major [W, H, C, N]) layout only:
 * channels-last images return SDB_NOT_SUPPORTED.  Its partial sums live in a
 * fixed 512 KiB device array that every GPU loading this library holds until
 * exit, so images x groups must be <= 32768 (else SDB_INVALID).  The first call
 * on a device looks the array up (make it before any stream capture).  Calls
 * share the array: calls that overlap on the GPU race. */
int sdb_group_norm_no_alloc(const sdb_tensor *x, const sdb_tensor *dst, int32_t groups, float eps,
                            const sdb_chain *chain, void *stream);

/* ---- GroupNorm fused into the operation that reads its output -----------
 * An extension of the reference, which computes GROUP_NORM as a node of its
 * own (norm.cc:100-140) between a convolution and the next: here the group
 * statistics are computed once (sdb_group_norm_stats: warp-shuffle and
 * cross-CTA reductions in double, the image's last CTA folding them) and the
 * normalisation (x - mean) * scale * gamma + beta, then SiLU, is applied as
 * the next operation reads its input -- in the Winograd input transform or
 * the split of the activations -- so the normalised tensor is never written.
 * The numbers the operation sees are those sdb_group_norm would have written
 * for a channels-last image with the chain (gamma, beta[, SiLU]).
 *
 * stats: [N][groups][2] FP32 -- mean, 1 / sqrt(variance + eps) per image and
 * group of C / groups consecutive channels (C % groups == 0). */
typedef struct sdb_norm_in {
    const float *stats;
    const float *gamma;  /* [C] and beta [C], or both NULL */
    const float *beta;
    int32_t groups;
    int32_t silu;
} sdb_norm_in;
/* The statistics of x, a channels-last image [W, H, C, N] (nb[2] = 4), into
 * stats (device memory of N * groups * 2 floats). */
int sdb_group_norm_stats(const sdb_tensor *x, int32_t groups, float eps, float *stats, void *stream);
/* sdb_conv2d of the normalised x (channels-last, or any layout on the Winograd
 * path), then the chain. */
int sdb_conv2d_normed(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const int32_t params[6],
                      const sdb_norm_in *norm, const sdb_chain *chain, void *stream);
/* sdb_mul_mat of the normalised x: x [C, P, N] -- P positions (rows) of each of
 * N images, C channels along a row. */
int sdb_mul_mat_normed(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, const sdb_norm_in *norm,
                       const sdb_chain *chain, void *stream);

/* LayerNorm fused into the linear layer that reads it (an extension of the
 * reference, whose NORM node writes its output, norm.cc:148-175): each row of
 * x is normalised -- mean and variance in double -- with the LayerNorm's chain
 * (norm_chain: its gamma and beta) as sdb_norm computes it, inside the split
 * of the linear layer's rows, and never written.  The result equals sdb_norm
 * followed by sdb_mul_mat (or sdb_mul_mat_gated) bit for bit.  Rows of at most
 * 1280 numbers. */
int sdb_mul_mat_layer_normed(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *dst, float eps,
                             const sdb_chain *norm_chain, const sdb_chain *chain, void *stream);
int sdb_mul_mat_gated_layer_normed(const sdb_tensor *w, const sdb_tensor *x, const sdb_tensor *out, float eps,
                                   const sdb_chain *norm_chain, const sdb_chain *chain, void *stream);

/* ---- the graph's data-movement nodes (device-resident runner) -----------
 * The reference takes only CONV_2D, MUL_MAT, FLASH_ATTN_EXT, GROUP_NORM and
 * NORM and leaves every other node of stable-diffusion.cpp's UNet graph to
 * ggml's CPU kernels ("the rest go by", hooks.cc:29-55).  With activations
 * resident on the GPU these nodes run here too:
 * sdb_concat: GGML_OP_CONCAT of a and b along ggml dim `dim` into dst; the three
 * tensors dense in one memory order (e.g. channels-last images along C). */
int sdb_concat(const sdb_tensor *a, const sdb_tensor *b, const sdb_tensor *dst, int32_t dim, void *stream);
/* GGML_OP_UPSCALE, nearest, by integer factors of W and H; channels-last images
 * [W, H, C, N] with C % 4 == 0. */
int sdb_upscale_nearest(const sdb_tensor *src, const sdb_tensor *dst, void *stream);
/* ToDo's coarser grid of an image's tokens (stable-diffusion.cpp patch 0004,
 * sdasm_coarser_tokens: a VIEW of every factor-th token of every factor-th row,
 * made contiguous): src [C, W, H, N] with contiguous channels -> dst
 * [C, ceil(W / factor), ceil(H / factor), N] dense, dst[c, i, j, n] =
 * src[c, factor i, factor j, n].  The keys' and values' projections of a
 * self-attention take these tokens when sdb_token_downsampling() > 1. */
int sdb_coarser_tokens(const sdb_tensor *src, const sdb_tensor *dst, int32_t factor, void *stream);
/* GGML_OP_TIMESTEP_EMBEDDING: timesteps [N] FP32 -> dst [>= dim, N]:
 * cos(t f_j) for j < dim/2, then sin(t f_j), f_j = max_period^(-j / (dim/2)). */
int sdb_timestep_embedding(const sdb_tensor *timesteps, const sdb_tensor *dst, int32_t dim, int32_t max_period,
                           void *stream);
/* GGML_OP_SOFT_MAX without a mask (ggml_soft_max_ext(x, NULL, scale, 0.0f)):
 * each row of ne0 softmax(scale * x), the sum of the exponentials in double and
 * one reciprocal per row, as ggml's CPU kernel computes it.  x and dst FP32 of
 * one shape (they may be the same memory). */
int sdb_soft_max(const sdb_tensor *x, const sdb_tensor *dst, float scale, void *stream);
/* One Euler step of the sampler with classifier-free guidance, in place:
 * e = eps[i] + cfg (eps[n + i] - eps[i]) (unconditional half first),
 * x[i] += (sigma_next - sigma) e, and, when x_in is given, both halves of the
 * next model input x_in[i] = x_in[n + i] = x[i] * c_in_next. */
int sdb_euler_cfg_step(const float *eps, float *x, float *x_in, int64_t n, float cfg, float sigma, float sigma_next,
                       float c_in_next, void *stream);
/* The ancestral Euler step (k-diffusion's sample_euler_ancestral, eta 1, the
 * sampler stable-diffusion.cpp runs as euler_a): with the guidance e as above,
 * sigma_up = min(sigma_next, sqrt(sigma_next^2 (sigma^2 - sigma_next^2) / sigma^2)),
 * sigma_down = sqrt(sigma_next^2 - sigma_up^2), x[i] += (sigma_down - sigma) e
 * + sigma_up noise[i] (no noise at sigma_next = 0); x_in as above.  noise [n]
 * is the step's fresh N(0, 1) draw. */
int sdb_euler_ancestral_cfg_step(const float *eps, float *x, float *x_in, const float *noise, int64_t n, float cfg,
                                 float sigma, float sigma_next, float c_in_next, void *stream);

/* ---- the weight store (store.h:58-120, store.cc:202-266) ----------------
 * Weights are repacked once into the layout the kernels read and kept on the
 * device, keyed by address, shape, strides and layout.  sdb_forget() drops
 * every entry packed from memory overlapping [begin, begin + size): call it
 * before changing weights in place (ggml patch 0004 calls sdasm_forget on
 * every buffer write).  Replaces sdasm_forget (sdasm.h:56-59). */
void sdb_forget(const void *begin, size_t size);
/* Entries and bytes the store holds on the current device. */
void sdb_store_stats(int64_t *entries, int64_t *bytes);

/* ToDo K/V downsampling factor of a token grid (sdasm.h:61-67, hooks.cc:166-172). */
int sdb_token_downsampling(int64_t width, int64_t height);

/* ---- tuning and diagnostics ----------------------------------------------
 * sdb_set_tuning parses "name=value,..." as SDASM_TUNE does (cpu.cc:166-220):
 * fuse, fuse_residual, winograd (0 direct, 1 F(2x2), 2 F(4x4)), store (0 repack
 * every call), todo, todo_tokens, bits (0, or 2..8: the linear layers of 256
 * rows or more as integer products, quant.cc), input_bits (2..8), group (32,
 * 64, 128 or 256), weight_group (1 per group, 0 per row), quantize (bit 1:
 * linear layers), block_n (the GEMM tile width: 0 automatic, 128, 160, 192 or
 * 256), gemm_fused (the linear layers' FP32 activations split inside the GEMM:
 * 1 where that is faster, 2 always, 0 never).  Returns SDB_INVALID on an
 * unknown name or value. */
int sdb_set_tuning(const char *spec);
int sdb_get_tuning(const char *name, int64_t *value);
/* The device error word of the current device (kernel-reported: bit 0 a
 * bounded wait ran out, bit 1 an activation beyond the FP16 range of the
 * split, bit 2 an index out of bounds); with clear != 0 it is reset.  Waits
 * for the device first. */
unsigned sdb_device_status(int clear);
/* The last host-side error of this thread, as text. */
const char *sdb_last_error(void);
/* Kernel launches this library made on this process (for accounting). */
uint64_t sdb_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif
