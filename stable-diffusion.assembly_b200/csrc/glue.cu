// The graph's data-movement nodes between the hot operations, for the
// device-resident UNet runner: GGML_OP_CONCAT, GGML_OP_UPSCALE (nearest),
// GGML_OP_TIMESTEP_EMBEDDING, and the sampler's classifier-free-guidance
// Euler update.  In the reference these stay with ggml's own CPU kernels
// (stable-diffusion.cpp builds them into the UNet graph); here they keep the
// runner's activations on the device.  All are HBM-bound copies: one thread
// moves four floats, and the index arithmetic is one 32-bit division per four
// elements where the sizes allow.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "runtime.cuh"

namespace sdb {

namespace {

bool f32t(const sdb_tensor* t) { return t && t->type == SDB_TYPE_F32 && t->data; }

// Contiguous in memory with the dims in order `order` (fastest first).
bool dense(const sdb_tensor* t, const int (&order)[4]) {
    int64_t expect = 4;
    for (int k = 0; k < 4; ++k) {
        const int d = order[k];
        if (t->ne[d] <= 0) return false;
        if (t->ne[d] > 1 && t->nb[d] != expect) return false;
        expect *= t->ne[d];
    }
    return true;
}

// Rows of a (ua floats) and b (ub floats) side by side into rows of ua + ub.
__global__ void concat_rows_kernel(const float* a, const float* b, float* d, long long rows, int ua, int ub,
                                   int vec) {
    const int w = ua + ub;
    if (vec) {
        const int w4 = w / 4, ua4 = ua / 4, ub4 = ub / 4;
        const long long total = rows * w4;
        for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
             i += static_cast<long long>(gridDim.x) * blockDim.x) {
            const long long r = i / w4;
            const int j = static_cast<int>(i - r * w4);
            const float4 v = j < ua4 ? __ldg(reinterpret_cast<const float4*>(a) + r * ua4 + j)
                                     : __ldg(reinterpret_cast<const float4*>(b) + r * ub4 + (j - ua4));
            reinterpret_cast<float4*>(d)[i] = v;
        }
    } else {
        const long long total = rows * w;
        for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
             i += static_cast<long long>(gridDim.x) * blockDim.x) {
            const long long r = i / w;
            const int j = static_cast<int>(i - r * w);
            d[i] = j < ua ? __ldg(a + r * ua + j) : __ldg(b + r * ub + (j - ua));
        }
    }
}

// Channels-last nearest upscale by integer factors: dst position (x, y) of
// image n takes source position (x / fx, y / fy); c floats a position.
// ToDo's coarser grid of tokens (the reference's stable-diffusion.cpp patch
// 0004, sdasm_coarser_tokens): dst[c, i, j, n] = src[c, f i, f j, n], the
// token nearest each point of the coarser grid; VEC consecutive channels a
// thread (cv of them a token), strides in floats.
template <int VEC>
__global__ void coarser_tokens_kernel(const float* __restrict__ src, float* __restrict__ dst, long long snb1,
                                      long long snb2, long long snb3, int cv, int w2, int h2, int f,
                                      long long total) {
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(idx % cv);
        long long rest = idx / cv;
        const int i = static_cast<int>(rest % w2);
        rest /= w2;
        const int j = static_cast<int>(rest % h2);
        const long long n = rest / h2;
        const float* s = src + n * snb3 + static_cast<long long>(j) * f * snb2 + static_cast<long long>(i) * f * snb1;
        if (VEC == 4) reinterpret_cast<float4*>(dst)[idx] = __ldg(reinterpret_cast<const float4*>(s + 4 * c));
        else dst[idx] = __ldg(s + c);
    }
}

__global__ void upscale_cl_kernel(const float* s, float* d, int c4, int dw, int dh, int fx, int fy, long long total4) {
    const int sw = dw / fx, sh = dh / fy;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pos = i / c4;
        const int ch = static_cast<int>(i - pos * c4);
        const long long img = pos / (static_cast<long long>(dw) * dh);
        const int rest = static_cast<int>(pos - img * dw * dh);
        const int y = rest / dw, x = rest - y * dw;
        const long long spos = (img * sh + y / fy) * sw + x / fx;
        reinterpret_cast<float4*>(d)[i] = __ldg(reinterpret_cast<const float4*>(s) + spos * c4 + ch);
    }
}

// [cos(t f_j) | sin(t f_j)], f_j = max_period^(-j / half), as ggml's
// timestep embedding writes it; an odd dim leaves its last element 0.
__global__ void timestep_kernel(const float* t, float* d, int dim, int n, float log_max_period, long long dnb1) {
    const int half = dim / 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * half; i += gridDim.x * blockDim.x) {
        const int img = i / half, j = i - img * half;
        const float freq = expf(-log_max_period * static_cast<float>(j) / static_cast<float>(half));
        const float arg = t[img] * freq;
        d[img * dnb1 + j] = cosf(arg);
        d[img * dnb1 + j + half] = sinf(arg);
        if ((dim & 1) && j == 0) d[img * dnb1 + dim - 1] = 0.0f;
    }
}

// noise (may be null): the ancestral sampler's fresh noise, added times s_up.
__global__ void euler_cfg_kernel(const float* eps, float* x, float* x_in, long long n, float cfg, float dt,
                                 float c_in, const float* noise, float s_up) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float u = eps[i], c = eps[n + i];
        const float e = u + cfg * (c - u);
        float xn = x[i] + dt * e;
        if (noise) xn += s_up * noise[i];
        x[i] = xn;
        if (x_in) {
            x_in[i] = xn * c_in;
            x_in[n + i] = xn * c_in;
        }
    }
}

int grid_for(long long work) {
    return static_cast<int>(std::max<long long>(1, std::min<long long>((work + 255) / 256, 148LL * 16)));
}

// GGML_OP_SOFT_MAX without a mask (ggml_soft_max_ext(x, NULL, scale, 0)),
// row by row as ggml's CPU kernel computes it: m = max of scale x, e_j =
// exp(scale x_j - m) summed in double, y_j = e_j * (float)(1 / sum).  The
// exponential is the epilogues' (scalar_math.h's method).  One CTA a row;
// with VPT > 0 a thread keeps its VPT numbers of the row in registers (rows
// of at most 256 VPT), else the row is read three times.
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) v = fmaxf(v, red[w]);
    __syncthreads();
    return v;
}

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    v = red[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) v += red[w];
    __syncthreads();
    return v;
}

struct SoftMaxArgs {
    const float* x;
    float* y;
    int ne0;
    long long rows, ne1, ne2;
    long long xnb[4], ynb[4];  // element strides
    float scale;
};

template <int VPT>
__global__ void __launch_bounds__(256) soft_max_kernel(const SoftMaxArgs a) {
    __shared__ float red_f[8];
    __shared__ double red_d[8];
    for (long long r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const long long i1 = r % a.ne1, rest = r / a.ne1, i2 = rest % a.ne2, i3 = rest / a.ne2;
        const float* xr = a.x + i1 * a.xnb[1] + i2 * a.xnb[2] + i3 * a.xnb[3];
        float* yr = a.y + i1 * a.ynb[1] + i2 * a.ynb[2] + i3 * a.ynb[3];
        float m = -INFINITY;
        if (VPT > 0) {
            float v[VPT > 0 ? VPT : 1];
#pragma unroll
            for (int e = 0; e < VPT; ++e) {
                const int j = threadIdx.x + e * 256;
                v[e] = j < a.ne0 ? __ldg(xr + j * a.xnb[0]) * a.scale : -INFINITY;
                m = fmaxf(m, v[e]);
            }
            m = block_max(m, red_f);
            double sum = 0.0;
#pragma unroll
            for (int e = 0; e < VPT; ++e) {
                const int j = threadIdx.x + e * 256;
                v[e] = j < a.ne0 ? exponential(v[e] - m) : 0.0f;
                sum += v[e];
            }
            sum = block_sum(sum, red_d);
            const float inv = static_cast<float>(1.0 / sum);
#pragma unroll
            for (int e = 0; e < VPT; ++e) {
                const int j = threadIdx.x + e * 256;
                if (j < a.ne0) yr[j * a.ynb[0]] = v[e] * inv;
            }
        } else {
            for (int j = threadIdx.x; j < a.ne0; j += blockDim.x) m = fmaxf(m, __ldg(xr + j * a.xnb[0]) * a.scale);
            m = block_max(m, red_f);
            double sum = 0.0;
            for (int j = threadIdx.x; j < a.ne0; j += blockDim.x)
                sum += exponential(__ldg(xr + j * a.xnb[0]) * a.scale - m);
            sum = block_sum(sum, red_d);
            const float inv = static_cast<float>(1.0 / sum);
            for (int j = threadIdx.x; j < a.ne0; j += blockDim.x)
                yr[j * a.ynb[0]] = exponential(__ldg(xr + j * a.xnb[0]) * a.scale - m) * inv;
        }
    }
}

}  // namespace

}  // namespace sdb

using namespace sdb;

extern "C" {

int sdb_concat(const sdb_tensor* a, const sdb_tensor* b, const sdb_tensor* dst, int32_t dim, void* stream) {
    if (!f32t(a) || !f32t(b) || !f32t(dst) || dim < 0 || dim > 3)
        return fail(SDB_NOT_SUPPORTED, "sdb_concat: FP32 tensors and dim 0..3");
    for (int d = 0; d < 4; ++d) {
        const int64_t want = d == dim ? a->ne[d] + b->ne[d] : a->ne[d];
        if (dst->ne[d] != want || (d != dim && b->ne[d] != a->ne[d]))
            return fail(SDB_INVALID, "sdb_concat: shapes do not concatenate");
    }
    // The memory order of dst (by stride), which a and b must share.
    int order[4] = {0, 1, 2, 3};
    for (int i = 0; i < 4; ++i)
        for (int j = i + 1; j < 4; ++j)
            if (dst->nb[order[j]] < dst->nb[order[i]] || (dst->nb[order[j]] == dst->nb[order[i]] && order[j] < order[i])) {
                const int t = order[i];
                order[i] = order[j];
                order[j] = t;
            }
    if (!dense(a, order) || !dense(b, order) || !dense(dst, order))
        return fail(SDB_NOT_SUPPORTED, "sdb_concat: tensors not dense in one memory order");
    // Rows: the dims slower than dim; a row holds dim and the dims faster than it.
    long long inner = 1, rows = 1;
    bool slower = false;
    for (int k = 0; k < 4; ++k) {
        const int d = order[k];
        if (d == dim) { slower = true; continue; }
        (slower ? rows : inner) *= a->ne[d];
    }
    const long long ua = a->ne[dim] * inner, ub = b->ne[dim] * inner;
    if (ua + ub > (1LL << 30)) return fail(SDB_NOT_SUPPORTED, "sdb_concat: rows too long");
    const int vec = (ua % 4 == 0) && (ub % 4 == 0) &&
                    ((reinterpret_cast<uintptr_t>(a->data) | reinterpret_cast<uintptr_t>(b->data) |
                      reinterpret_cast<uintptr_t>(dst->data)) & 15) == 0;
    const long long work = rows * (ua + ub) / (vec ? 4 : 1);
    concat_rows_kernel<<<grid_for(work), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(a->data), static_cast<const float*>(b->data), static_cast<float*>(dst->data), rows,
        static_cast<int>(ua), static_cast<int>(ub), vec);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_coarser_tokens(const sdb_tensor* src, const sdb_tensor* dst, int32_t factor, void* stream) {
    if (!f32t(src) || !f32t(dst) || factor < 1) return fail(SDB_NOT_SUPPORTED, "sdb_coarser_tokens: FP32 tensors");
    const int64_t c = src->ne[0], w = src->ne[1], h = src->ne[2], n = src->ne[3];
    const int64_t w2 = (w + factor - 1) / factor, h2 = (h + factor - 1) / factor;
    if (dst->ne[0] != c || dst->ne[1] != w2 || dst->ne[2] != h2 || dst->ne[3] != n)
        return fail(SDB_INVALID, "sdb_coarser_tokens: dst must be [C, ceil(W / f), ceil(H / f), N]");
    const int order[4] = {0, 1, 2, 3};
    if (src->nb[0] != 4 || !dense(dst, order)) return fail(SDB_NOT_SUPPORTED, "sdb_coarser_tokens: contiguous channels");
    for (int d = 1; d < 4; ++d)
        if (src->nb[d] % 4 != 0) return fail(SDB_NOT_SUPPORTED, "sdb_coarser_tokens: strides of whole floats");
    const bool vec = c % 4 == 0 && src->nb[1] % 16 == 0 && src->nb[2] % 16 == 0 && src->nb[3] % 16 == 0 &&
                     ((reinterpret_cast<uintptr_t>(src->data) | reinterpret_cast<uintptr_t>(dst->data)) & 15) == 0;
    const int cv = static_cast<int>(vec ? c / 4 : c);
    const long long total = static_cast<long long>(cv) * w2 * h2 * n;
    const auto st = static_cast<cudaStream_t>(stream);
    const long long e = 4;
    if (vec)
        coarser_tokens_kernel<4><<<grid_for(total), 256, 0, st>>>(
            static_cast<const float*>(src->data), static_cast<float*>(dst->data), src->nb[1] / e, src->nb[2] / e,
            src->nb[3] / e, cv, static_cast<int>(w2), static_cast<int>(h2), factor, total);
    else
        coarser_tokens_kernel<1><<<grid_for(total), 256, 0, st>>>(
            static_cast<const float*>(src->data), static_cast<float*>(dst->data), src->nb[1] / e, src->nb[2] / e,
            src->nb[3] / e, cv, static_cast<int>(w2), static_cast<int>(h2), factor, total);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_upscale_nearest(const sdb_tensor* src, const sdb_tensor* dst, void* stream) {
    if (!f32t(src) || !f32t(dst)) return fail(SDB_NOT_SUPPORTED, "sdb_upscale_nearest: FP32 tensors");
    if (dst->ne[2] != src->ne[2] || dst->ne[3] != src->ne[3] || dst->ne[0] % src->ne[0] || dst->ne[1] % src->ne[1])
        return fail(SDB_INVALID, "sdb_upscale_nearest: integer factors of W and H only");
    const int order[4] = {2, 0, 1, 3};  // channels-last
    const int64_t c = src->ne[2];
    if (!dense(src, order) || !dense(dst, order) || c % 4 ||
        ((reinterpret_cast<uintptr_t>(src->data) | reinterpret_cast<uintptr_t>(dst->data)) & 15))
        return fail(SDB_NOT_SUPPORTED, "sdb_upscale_nearest: channels-last images with C % 4 == 0");
    const long long total4 = dst->ne[0] * dst->ne[1] * dst->ne[3] * (c / 4);
    if (dst->ne[0] * dst->ne[1] > (1LL << 30)) return fail(SDB_NOT_SUPPORTED, "sdb_upscale_nearest: too large");
    upscale_cl_kernel<<<grid_for(total4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(src->data), static_cast<float*>(dst->data), static_cast<int>(c / 4),
        static_cast<int>(dst->ne[0]), static_cast<int>(dst->ne[1]), static_cast<int>(dst->ne[0] / src->ne[0]),
        static_cast<int>(dst->ne[1] / src->ne[1]), total4);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_timestep_embedding(const sdb_tensor* timesteps, const sdb_tensor* dst, int32_t dim, int32_t max_period,
                           void* stream) {
    if (!f32t(timesteps) || !f32t(dst) || dim <= 1 || max_period <= 0)
        return fail(SDB_NOT_SUPPORTED, "sdb_timestep_embedding: FP32 tensors, dim > 1");
    const int64_t n = timesteps->ne[0];
    if (timesteps->nb[0] != 4 || dst->nb[0] != 4 || dst->ne[0] < dim || dst->ne[1] != n || n > (1 << 20))
        return fail(SDB_INVALID, "sdb_timestep_embedding: dst must be [dim, N] with contiguous rows");
    timestep_kernel<<<grid_for(n * (dim / 2)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(timesteps->data), static_cast<float*>(dst->data), dim, static_cast<int>(n),
        logf(static_cast<float>(max_period)), dst->nb[1] / 4);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_euler_cfg_step(const float* eps, float* x, float* x_in, int64_t n, float cfg, float sigma, float sigma_next,
                       float c_in_next, void* stream) {
    if (!eps || !x || n <= 0) return fail(SDB_INVALID, "sdb_euler_cfg_step: null buffers");
    euler_cfg_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(eps, x, x_in, n, cfg,
                                                                                  sigma_next - sigma, c_in_next,
                                                                                  nullptr, 0.0f);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_euler_ancestral_cfg_step(const float* eps, float* x, float* x_in, const float* noise, int64_t n, float cfg,
                                 float sigma, float sigma_next, float c_in_next, void* stream) {
    if (!eps || !x || !noise || n <= 0) return fail(SDB_INVALID, "sdb_euler_ancestral_cfg_step: null buffers");
    if (!(sigma > 0.0f) || sigma_next < 0.0f || sigma_next > sigma)
        return fail(SDB_INVALID, "sdb_euler_ancestral_cfg_step: 0 <= sigma_next <= sigma, sigma > 0");
    // get_ancestral_step with eta 1 (k-diffusion, as stable-diffusion.cpp's euler_a samples).
    const double s = sigma, sn = sigma_next;
    const double up = std::min(sn, std::sqrt(sn * sn * (s * s - sn * sn) / (s * s)));
    const double down = std::sqrt(sn * sn - up * up);
    euler_cfg_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        eps, x, x_in, n, cfg, static_cast<float>(down - s), c_in_next, sn > 0.0 ? noise : nullptr,
        static_cast<float>(up));
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int sdb_soft_max(const sdb_tensor* x, const sdb_tensor* dst, float scale, void* stream) {
    if (!f32t(x) || !f32t(dst)) return fail(SDB_NOT_SUPPORTED, "sdb_soft_max: FP32 tensors only");
    for (int d = 0; d < 4; ++d) {
        if (x->ne[d] != dst->ne[d] || x->ne[d] <= 0) return fail(SDB_INVALID, "sdb_soft_max: shapes differ");
        if (x->nb[d] % 4 || dst->nb[d] % 4 || x->nb[d] < 0 || dst->nb[d] < 0)
            return fail(SDB_NOT_SUPPORTED, "sdb_soft_max: misaligned strides");
    }
    if (x->ne[0] > (1 << 30)) return fail(SDB_NOT_SUPPORTED, "sdb_soft_max: rows too long");
    SoftMaxArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.y = static_cast<float*>(dst->data);
    a.ne0 = static_cast<int>(x->ne[0]);
    a.ne1 = x->ne[1];
    a.ne2 = x->ne[2];
    a.rows = x->ne[1] * x->ne[2] * x->ne[3];
    for (int d = 0; d < 4; ++d) {
        a.xnb[d] = x->nb[d] / 4;
        a.ynb[d] = dst->nb[d] / 4;
    }
    a.scale = scale;
    const auto st = static_cast<cudaStream_t>(stream);
    const int blocks = static_cast<int>(std::min<long long>(a.rows, 148LL * 64));
    if (a.ne0 <= 1024) soft_max_kernel<4><<<blocks, 256, 0, st>>>(a);
    else if (a.ne0 <= 4096) soft_max_kernel<16><<<blocks, 256, 0, st>>>(a);
    else soft_max_kernel<0><<<blocks, 256, 0, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // extern "C"
