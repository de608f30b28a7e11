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

__global__ void euler_cfg_kernel(const float* eps, float* x, float* x_in, long long n, float cfg, float dt,
                                 float c_in) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float u = eps[i], c = eps[n + i];
        const float e = u + cfg * (c - u);
        const float xn = x[i] + dt * e;
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
                                                                                  sigma_next - sigma, c_in_next);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // extern "C"
