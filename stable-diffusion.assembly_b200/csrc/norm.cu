// GGML_OP_GROUP_NORM and GGML_OP_NORM with the chain after them.
//
// The reference (norm.cc:100-175) reads the tensor three times -- for the
// mean, for the variance, for the output -- sums in double precision, and
// applies the chain (scale, shift, SiLU) to each row as it writes it:
//   mean = float(sum(x) / n), var = float(sum(float(x - mean)^2) / n),
//   y = (x - mean) * float(1 / sqrt(var + eps)), then the chain.
// Here one CTA (or a cluster of CTAs for large groups) owns one (image,
// group) or a block of rows; the sums are double, reduced by warp shuffles
// and across warps in shared memory; the mean and variance are rounded to
// float exactly as the reference rounds them.  A group larger than what one
// CTA should stream alone is split over several CTAs that combine their
// double partial sums through global memory: the first pass writes per-CTA
// partials, the second kernel finishes the statistics and normalises.  No CTA
// waits on another (two launches instead of a grid barrier).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "ptx.cuh"
#include "runtime.cuh"

namespace sdb {

namespace {

constexpr int kNormThreads = 512;

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the CTA; every thread gets the total.
__device__ double block_sum(double v, double* scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    double t = 0.0;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) t += scratch[i];
    return t;
}

struct GroupArgs {
    const float* x;
    float* y;
    long long ne0, ne1, ne2, ne3;
    long long xnb[4], ynb[4];   // element strides
    int groups, per_group;
    float eps;
    int split;                  // CTAs per (image, group)
    double* partial;            // [items][split][2]
    int uniform;                // every chain operand is constant over (i0, i1): one value per channel
    Chain chain;
};

// The chain's operand values for channel c of image i3 (uniform chains).
__device__ __forceinline__ void channel_operands(const Chain& ch, long long c, long long i3, float (&op)[SDB_MAX_STEPS]) {
#pragma unroll
    for (int s = 0; s < SDB_MAX_STEPS; ++s)
        op[s] = (s < ch.count && ch.kind[s] != SDB_STEP_SILU) ? __ldg(ch.operand[s] + c * ch.nb[s][2] + i3 * ch.nb[s][3])
                                                              : 0.0f;
}

__device__ __forceinline__ float apply_uniform(const Chain& ch, const float (&op)[SDB_MAX_STEPS], float v) {
#pragma unroll
    for (int s = 0; s < SDB_MAX_STEPS; ++s) {
        if (s >= ch.count) break;
        v = ch.kind[s] == SDB_STEP_SILU ? silu(v) : ch.kind[s] == SDB_STEP_ADD ? v + op[s] : v * op[s];
    }
    return v;
}

// Normalises elements [e0, e1) of a group (channels c0.. contiguous, element
// e of the group in channel c0 + e / plane) from src into the output, with
// the chain.  A thread takes four elements (or four float4s) at a time and
// issues their operand loads before any of their stores, so the loads'
// latency is paid once per batch rather than once per element.
template <bool kSmem>
__device__ __forceinline__ void apply_range(const GroupArgs& a, const float* src, long long c0, long long i3,
                                            float mean, float scale, long long e0, long long e1) {
    const int ne0 = static_cast<int>(a.ne0);
    const int plane = static_cast<int>(a.ne0 * a.ne1);
    float* ybase = a.y + i3 * a.ynb[3];
    const bool flat = a.ynb[0] == 1 && a.ynb[1] == a.ne0 && a.ynb[2] == a.ne0 * a.ne1;
    if (a.uniform && flat && (plane & 3) == 0 && ((e0 | e1) & 3) == 0 &&
        ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(ybase + c0 * a.ynb[2])) & 15) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(ybase + c0 * a.ynb[2]);
        const int plane4 = plane / 4;
        const int b4 = static_cast<int>(e0 / 4), n4 = static_cast<int>(e1 / 4);
        for (int base = b4 + threadIdx.x; base < n4; base += 4 * blockDim.x) {
            float4 v[4];
            float op[4][SDB_MAX_STEPS];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int e = min(base + k * static_cast<int>(blockDim.x), n4 - 1);
                v[k] = kSmem ? s4[e] : __ldg(s4 + e);
                channel_operands(a.chain, c0 + e / plane4, i3, op[k]);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[k].x = apply_uniform(a.chain, op[k], (v[k].x - mean) * scale);
                v[k].y = apply_uniform(a.chain, op[k], (v[k].y - mean) * scale);
                v[k].z = apply_uniform(a.chain, op[k], (v[k].z - mean) * scale);
                v[k].w = apply_uniform(a.chain, op[k], (v[k].w - mean) * scale);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int e = base + k * static_cast<int>(blockDim.x);
                if (e < n4) d4[e] = v[k];
            }
        }
        return;
    }
    // General layouts and chains: batches of four elements.
    for (long long b = e0 + threadIdx.x; b < e1; b += 4 * blockDim.x) {
        float v[4];
        int i0[4], i1[4];
        long long c[4];
        bool live[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const long long e = b + k * static_cast<long long>(blockDim.x);
            live[k] = e < e1;
            const long long ec = live[k] ? e : e0;
            const int cc = static_cast<int>(ec / plane);
            const int pe = static_cast<int>(ec - static_cast<long long>(cc) * plane);
            c[k] = c0 + cc;
            i1[k] = pe / ne0;
            i0[k] = pe - i1[k] * ne0;
            v[k] = ((kSmem ? src[ec] : __ldg(src + ec)) - mean) * scale;
        }
#pragma unroll
        for (int s = 0; s < SDB_MAX_STEPS; ++s) {
            if (s >= a.chain.count) break;
            if (a.chain.kind[s] == SDB_STEP_SILU) {
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = silu(v[k]);
            } else {
                float o[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    o[k] = __ldg(a.chain.operand[s] + i0[k] * a.chain.nb[s][0] + i1[k] * a.chain.nb[s][1] +
                                 c[k] * a.chain.nb[s][2] + i3 * a.chain.nb[s][3]);
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = a.chain.kind[s] == SDB_STEP_ADD ? v[k] + o[k] : v[k] * o[k];
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (live[k]) ybase[i0[k] * a.ynb[0] + i1[k] * a.ynb[1] + c[k] * a.ynb[2]] = v[k];
    }
}

// Element e of the group's contiguous run (channels c0.. are contiguous: the
// tensor is contiguous, as group_norm_supported requires).
__device__ __forceinline__ float load_group(const GroupArgs& a, const float* base, long long e) {
    return __ldg(base + e);
}

// Pass 1 of a split group: this CTA's slice sums (of x), then (x - mean)^2
// after the mean is known -- done in two kernels, see group_stats_kernel.
__global__ void __launch_bounds__(kNormThreads) group_sum_kernel(const GroupArgs a, int phase) {
    __shared__ double scratch[32];
    __shared__ float mean_s;
    const int item = blockIdx.x / a.split;
    const int part = blockIdx.x % a.split;
    const int i3 = item / a.groups, g = item % a.groups;
    const long long c0 = static_cast<long long>(g) * a.per_group;
    const long long c1 = min(a.ne2, c0 + a.per_group);
    if (c0 >= c1) return;
    const long long count = a.ne0 * a.ne1 * (c1 - c0);
    const float* base = a.x + i3 * a.xnb[3] + c0 * a.xnb[2];
    const long long per = (count + 4 * a.split - 1) / (4 * a.split) * 4;
    const long long e0 = part * per, e1 = min(count, e0 + per);
    double s = 0.0;
    if (phase == 0) {
        for (long long e = e0 + threadIdx.x; e < e1; e += blockDim.x) s += static_cast<double>(load_group(a, base, e));
    } else {
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int p = 0; p < a.split; ++p) t += a.partial[(static_cast<long long>(item) * a.split + p) * 2];
            mean_s = static_cast<float>(t / static_cast<double>(count));
        }
        __syncthreads();
        const float mean = mean_s;
        for (long long e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
            const float v = load_group(a, base, e) - mean;
            s += static_cast<double>(v * v);
        }
    }
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) a.partial[(static_cast<long long>(item) * a.split + part) * 2 + phase] = s;
}

__global__ void __launch_bounds__(kNormThreads) group_apply_kernel(const GroupArgs a) {
    __shared__ float stats[2];
    const int item = blockIdx.x / a.split;
    const int part = blockIdx.x % a.split;
    const int i3 = item / a.groups, g = item % a.groups;
    const long long c0 = static_cast<long long>(g) * a.per_group;
    const long long c1 = min(a.ne2, c0 + a.per_group);
    if (c0 >= c1) return;
    const long long count = a.ne0 * a.ne1 * (c1 - c0);
    if (threadIdx.x == 0) {
        double s = 0.0, q = 0.0;
        for (int p = 0; p < a.split; ++p) {
            s += a.partial[(static_cast<long long>(item) * a.split + p) * 2];
            q += a.partial[(static_cast<long long>(item) * a.split + p) * 2 + 1];
        }
        const float mean = static_cast<float>(s / static_cast<double>(count));
        const float var = static_cast<float>(q / static_cast<double>(count));
        stats[0] = mean;
        stats[1] = 1.0f / sqrtf(var + a.eps);
    }
    __syncthreads();
    const float mean = stats[0], scale = stats[1];
    const float* xb = a.x + i3 * a.xnb[3] + c0 * a.xnb[2];
    const long long per = (count + 4 * a.split - 1) / (4 * a.split) * 4;
    const long long e0 = part * per, e1 = min(count, e0 + per);
    apply_range<false>(a, xb, c0, i3, mean, scale, e0, e1);
}

// The whole (image, group) in shared memory: read once from HBM, the two
// passes of the statistics and the normalisation from shared memory, written
// once.  One CTA per (image, group); for groups of up to kResident floats.
constexpr int kResidentThreads = 1024;
constexpr long long kResident = 50 * 1024;  // floats: 200 KB

__global__ void __launch_bounds__(kResidentThreads) group_resident_kernel(const GroupArgs a) {
    extern __shared__ float xs[];
    __shared__ double scratch[32];
    __shared__ float stats[2];
    const int item = blockIdx.x;
    const int i3 = item / a.groups, g = item % a.groups;
    const long long c0 = static_cast<long long>(g) * a.per_group;
    const long long c1 = min(a.ne2, c0 + a.per_group);
    if (c0 >= c1) return;
    const long long count = a.ne0 * a.ne1 * (c1 - c0);
    const float* xb = a.x + i3 * a.xnb[3] + c0 * a.xnb[2];
    double s = 0.0;
    if ((reinterpret_cast<uintptr_t>(xb) & 15) == 0 && (count & 3) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xb);
        float4* s4 = reinterpret_cast<float4*>(xs);
        // Unrolled: the loads of eight iterations are in flight together.
#pragma unroll 8
        for (long long e = threadIdx.x; e < count / 4; e += blockDim.x) {
            const float4 v = __ldg(x4 + e);
            s4[e] = v;
            s += static_cast<double>(v.x) + static_cast<double>(v.y) + static_cast<double>(v.z) +
                 static_cast<double>(v.w);
        }
    } else {
#pragma unroll 8
        for (long long e = threadIdx.x; e < count; e += blockDim.x) {
            const float v = __ldg(xb + e);
            xs[e] = v;
            s += static_cast<double>(v);
        }
    }
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) stats[0] = static_cast<float>(s / static_cast<double>(count));
    __syncthreads();
    const float mean = stats[0];
    double q = 0.0;
    for (long long e = threadIdx.x; e < count; e += blockDim.x) {
        const float v = xs[e] - mean;
        q += static_cast<double>(v * v);
    }
    q = block_sum(q, scratch);
    if (threadIdx.x == 0) stats[1] = 1.0f / sqrtf(static_cast<float>(q / static_cast<double>(count)) + a.eps);
    __syncthreads();
    const float scale = stats[1];
    apply_range<true>(a, xs, c0, i3, mean, scale, 0, count);
}

// ---- channels-last (NHWC) images -----------------------------------------
//
// x and y are [N][P positions][C], C % groups == 0 and C % 4 == 0: a group is
// cpg contiguous channels of every position.  Two launches, no grid-wide wait:
//
//   nhwc_gn_stats_kernel  every CTA takes a chunk of one image's positions
//       (float4 loads, a thread's rows a float4 column of channels) and sums,
//       in double, d = x - K and d^2 per group, K the group's first number
//       (x at position 0, the group's first channel) -- a shift that keeps
//       the one-pass variance free of cancellation for data of any offset;
//       the CTA's sums go to global memory, and the last CTA of the image to
//       finish (an atomic count, reset by that CTA) folds them in chunk order
//       into the group's float mean and 1 / sqrt(variance + eps);
//   nhwc_gn_apply_kernel  (x - mean) * scale, then the chain, float4 in and
//       out.
//
// The reference makes two passes of double sums, the mean and then the
// squares about the float mean (norm.cc:121-129); the shifted one-pass sums
// give the same mean and a variance within a relative (mean - K)^2 / var
// 2^-52 of it.  x is read twice (the second time mostly from L2) and y
// written once.
constexpr int kClThreads = 256;
constexpr int kClMaxCols = 3;     // float4 columns a thread may own: C <= 3 * 4 * 256
constexpr int kClMaxGroups = 128;
constexpr int kClMaxChannels = 3072;
constexpr int kClMaxCsum = kClMaxChannels;   // channel sums of the CTA's row phases (rpp * C <= 4 * threads)

struct NhwcArgs {
    const float* x;
    float* y;
    int positions;              // H * W
    int c, c4;                  // channels, channels / 4
    int groups, cpg;
    int cpi;                    // CTAs per image
    int per;                    // positions per CTA
    int rpp;                    // rows (positions) a pass of the CTA covers
    float eps;
    double* partial;            // [images][cpi][groups][2]: the CTAs' shifted sums
    float* stats;               // [images][groups][2]: mean, scale
    unsigned* count;            // [images]: CTAs of the image done (zero between launches)
    Chain chain;
};

// This thread's float4 columns and first row of a pass.
__device__ __forceinline__ int cl_columns(const NhwcArgs& a, int (&col)[kClMaxCols], int& r0) {
    int n = 0;
    if (a.c4 <= kClThreads) {
        r0 = threadIdx.x / a.c4;
        col[0] = threadIdx.x - r0 * a.c4;
        n = r0 < a.rpp ? 1 : 0;
    } else {
        r0 = 0;
        for (int j = threadIdx.x; j < a.c4 && n < kClMaxCols; j += kClThreads) col[n++] = j;
    }
    return n;
}

__global__ void __launch_bounds__(kClThreads) nhwc_gn_stats_kernel(const NhwcArgs a) {
    // [sum, squares][row phase * C + channel]: 2 * csum_len doubles of dynamic shared memory.
    extern __shared__ double csum_dyn[];
    const int csum_len = a.c4 <= kClThreads ? a.rpp * a.c : a.c;
    double* csum[2] = {csum_dyn, csum_dyn + csum_len};
    __shared__ float shift[kClMaxGroups];
    __shared__ int last;
    const int i3 = blockIdx.x / a.cpi, chunk = blockIdx.x - i3 * a.cpi;
    const long long p0 = static_cast<long long>(chunk) * a.per;
    const long long p1 = min(static_cast<long long>(a.positions), p0 + a.per);
    const long long base = static_cast<long long>(i3) * a.positions * a.c4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x) + base;
    for (int g = threadIdx.x; g < a.groups; g += blockDim.x) shift[g] = __ldg(a.x + base * 4 + g * a.cpg);
    __syncthreads();
    int col[kClMaxCols], r0;
    const int ncols = cl_columns(a, col, r0);
    for (int k = 0; k < ncols; ++k) {
        const int j = col[k];
        const float k0 = shift[4 * j / a.cpg], k1 = shift[(4 * j + 1) / a.cpg];
        const float k2 = shift[(4 * j + 2) / a.cpg], k3 = shift[(4 * j + 3) / a.cpg];
        double s[4] = {0.0, 0.0, 0.0, 0.0}, q[4] = {0.0, 0.0, 0.0, 0.0};
        const float4* src = x4 + j;
        const int rows = static_cast<int>((p1 - p0 - r0 + a.rpp - 1) / a.rpp);
        const long long step = static_cast<long long>(a.rpp) * a.c4;
        src += (p0 + r0) * a.c4;
        for (int r = 0; r < rows; r += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = r + u < rows ? __ldg(src + (r + u) * step) : make_float4(k0, k1, k2, k3);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const double d0 = static_cast<double>(v[u].x) - k0, d1 = static_cast<double>(v[u].y) - k1;
                const double d2 = static_cast<double>(v[u].z) - k2, d3 = static_cast<double>(v[u].w) - k3;
                s[0] += d0; s[1] += d1; s[2] += d2; s[3] += d3;
                q[0] = fma(d0, d0, q[0]); q[1] = fma(d1, d1, q[1]);
                q[2] = fma(d2, d2, q[2]); q[3] = fma(d3, d3, q[3]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            csum[0][r0 * a.c + 4 * j + e] = s[e];
            csum[1][r0 * a.c + 4 * j + e] = q[e];
        }
    }
    __syncthreads();
    // Each group's channels over the row phases, eight threads a group, into this CTA's partial.
    const int phases = a.c4 <= kClThreads ? a.rpp : 1;
    const int span = phases * a.cpg;
    double* part = a.partial + ((static_cast<long long>(i3) * a.cpi + chunk) * a.groups) * 2;
    for (int b0 = 0; b0 < a.groups * 8; b0 += blockDim.x) {
        const int t = b0 + threadIdx.x;
        const int g = t / 8, k = t % 8;
        double sv = 0.0, qv = 0.0;
        if (g < a.groups)
            for (int e = k; e < span; e += 8) {
                const int ph = e / a.cpg, ch = g * a.cpg + (e - ph * a.cpg);
                sv += csum[0][ph * a.c + ch];
                qv += csum[1][ph * a.c + ch];
            }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            sv += __shfl_xor_sync(0xffffffffu, sv, o);
            qv += __shfl_xor_sync(0xffffffffu, qv, o);
        }
        if (g < a.groups && k == 0) {
            part[2 * g] = sv;
            part[2 * g + 1] = qv;
        }
    }
    // The image's last CTA to finish folds every CTA's sums, in chunk order.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(a.count + i3, 1u) == static_cast<unsigned>(a.cpi - 1) ? 1 : 0;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const double n = static_cast<double>(a.positions) * a.cpg;
    const double2* img = reinterpret_cast<const double2*>(a.partial) + static_cast<long long>(i3) * a.cpi * a.groups;
    // lanes threads a group (a power of two within a warp), each folding every lanes-th CTA's
    // sums with eight loads in flight, then the lanes in a fixed order.
    int lanes = 32;
    while (lanes > 1 && lanes * a.groups > static_cast<int>(blockDim.x)) lanes >>= 1;
    for (int b0 = 0; b0 < a.groups * lanes; b0 += blockDim.x) {
        const int t = b0 + threadIdx.x;
        const int g = t / lanes, k = t % lanes;
        double sv = 0.0, qv = 0.0;
        if (g < a.groups) {
            int ch = k;
            for (; ch + 7 * lanes < a.cpi; ch += 8 * lanes) {
                double2 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(img + static_cast<long long>(ch + u * lanes) * a.groups + g);
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    sv += v[u].x;
                    qv += v[u].y;
                }
            }
            for (; ch < a.cpi; ch += lanes) {
                const double2 v = __ldcg(img + static_cast<long long>(ch) * a.groups + g);
                sv += v.x;
                qv += v.y;
            }
        }
        for (int o = lanes / 2; o > 0; o >>= 1) {
            sv += __shfl_xor_sync(0xffffffffu, sv, o);
            qv += __shfl_xor_sync(0xffffffffu, qv, o);
        }
        if (g < a.groups && k == 0) {
            const double dm = sv / n;
            const double var = fmax(qv / n - dm * dm, 0.0);
            float* st = a.stats + (static_cast<long long>(i3) * a.groups + g) * 2;
            st[0] = static_cast<float>(static_cast<double>(shift[g]) + dm);
            st[1] = 1.0f / sqrtf(static_cast<float>(var) + a.eps);
        }
    }
    if (threadIdx.x == 0) a.count[i3] = 0u;
}

// Chain patterns the apply pass compiles on their own: the GroupNorm's scale
// and shift (per channel), with or without the SiLU after them.
enum : int { kChainGeneral = 0, kChainAffine = 1, kChainAffineSilu = 2, kChainNone = 3 };

template <int PATTERN>
__device__ __forceinline__ float chain_pattern(const Chain& ch, const float (&op)[SDB_MAX_STEPS], float v) {
    if (PATTERN == kChainNone) return v;
    if (PATTERN == kChainAffine) return fmaf(v, op[0], op[1]);
    if (PATTERN == kChainAffineSilu) return silu_apply(fmaf(v, op[0], op[1]));
    return apply_uniform(ch, op, v);
}

template <int PATTERN>
__global__ void __launch_bounds__(kClThreads) nhwc_gn_apply_kernel(const NhwcArgs a) {
    const int i3 = blockIdx.x / a.cpi, chunk = blockIdx.x - i3 * a.cpi;
    const long long p0 = static_cast<long long>(chunk) * a.per;
    const long long p1 = min(static_cast<long long>(a.positions), p0 + a.per);
    const long long base = static_cast<long long>(i3) * a.positions * a.c4;
    const float4* x4 = reinterpret_cast<const float4*>(a.x) + base;
    float4* y4 = reinterpret_cast<float4*>(a.y) + base;
    const float* st = a.stats + static_cast<long long>(i3) * a.groups * 2;
    int col[kClMaxCols], r0;
    const int ncols = cl_columns(a, col, r0);
    for (int k = 0; k < ncols; ++k) {
        const int j = col[k];
        float mu[4], sc[4], op[4][SDB_MAX_STEPS];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int g = (4 * j + e) / a.cpg;
            mu[e] = __ldg(st + 2 * g);
            sc[e] = __ldg(st + 2 * g + 1);
            channel_operands(a.chain, 4 * j + e, i3, op[e]);
        }
        const int rows = static_cast<int>((p1 - p0 - r0 + a.rpp - 1) / a.rpp);
        const long long step = static_cast<long long>(a.rpp) * a.c4;
        const float4* src = x4 + (p0 + r0) * a.c4 + j;
        float4* dst = y4 + (p0 + r0) * a.c4 + j;
        for (int r = 0; r < rows; r += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(src + min(r + u, rows - 1) * step);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                v[u].x = chain_pattern<PATTERN>(a.chain, op[0], (v[u].x - mu[0]) * sc[0]);
                v[u].y = chain_pattern<PATTERN>(a.chain, op[1], (v[u].y - mu[1]) * sc[1]);
                v[u].z = chain_pattern<PATTERN>(a.chain, op[2], (v[u].z - mu[2]) * sc[2]);
                v[u].w = chain_pattern<PATTERN>(a.chain, op[3], (v[u].w - mu[3]) * sc[3]);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (r + u < rows) dst[(r + u) * step] = v[u];
        }
    }
}

struct RowArgs {
    const float* x;
    float* y;
    long long ne0, ne1, ne2;
    long long rows;
    long long xnb[4], ynb[4];
    float eps;
    Chain chain;
};

// One warp per row (rows of up to a few thousand elements: LayerNorm over
// channels); each row is read three times from L1/L2, written once.
__global__ void __launch_bounds__(256) norm_rows_kernel(const RowArgs a) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= a.rows) return;
    const long long i1 = row % a.ne1;
    const long long i2 = (row / a.ne1) % a.ne2;
    const long long i3 = row / (a.ne1 * a.ne2);
    const float* xr = a.x + i1 * a.xnb[1] + i2 * a.xnb[2] + i3 * a.xnb[3];
    float* yr = a.y + i1 * a.ynb[1] + i2 * a.ynb[2] + i3 * a.ynb[3];
    double s = 0.0;
    for (long long i = lane; i < a.ne0; i += 32) s += static_cast<double>(__ldg(xr + i * a.xnb[0]));
    s = warp_sum(s);
    const float mean = static_cast<float>(s / static_cast<double>(a.ne0));
    double q = 0.0;
    for (long long i = lane; i < a.ne0; i += 32) {
        const float v = __ldg(xr + i * a.xnb[0]) - mean;
        q += static_cast<double>(v * v);
    }
    q = warp_sum(q);
    const float var = static_cast<float>(q / static_cast<double>(a.ne0));
    const float scale = 1.0f / sqrtf(var + a.eps);
    // Four elements per lane at a time, each chain step's loads together.
    ChainRow cr;
    row_offsets(a.chain, cr, 0, i1, i2, i3);
    for (long long i0 = lane; i0 < a.ne0; i0 += 128) {
        float v[4];
        long long col[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            col[k] = min(i0 + 32 * k, a.ne0 - 1);
            v[k] = (__ldg(xr + col[k] * a.xnb[0]) - mean) * scale;
        }
#pragma unroll
        for (int s = 0; s < SDB_MAX_STEPS; ++s) {
            if (s >= a.chain.count) break;
            if (a.chain.kind[s] == SDB_STEP_SILU) {
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = silu(v[k]);
            } else {
                float o[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) o[k] = __ldg(a.chain.operand[s] + cr.off[s] + col[k] * a.chain.nb[s][0]);
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = a.chain.kind[s] == SDB_STEP_ADD ? v[k] + o[k] : v[k] * o[k];
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (i0 + 32 * k < a.ne0) yr[(i0 + 32 * k) * a.ynb[0]] = v[k];
    }
}

// One warp per R rows with the rows in registers (rows of up to 32 * kLnPer
// elements, contiguous): x is read from memory once, both statistics and the
// normalisation come from the registers.  The R rows' dependent chains (double
// sums, warp reductions) interleave, which hides their latency where a row is
// short; each row's arithmetic is the same, in the same order, for any R.
constexpr int kLnPer = 40;   // the widest row kept in registers: 32 x 40 elements

template <int PER, int R>
__global__ void __launch_bounds__(256) norm_rows_reg_kernel(const RowArgs a) {
    const long long row0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * R;
    const int lane = threadIdx.x & 31;
    if (row0 >= a.rows) return;
    const int n = static_cast<int>(a.ne0);
    bool live[R];
    long long i1[R], i2[R], i3[R];
    float v[R][PER];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        live[r] = row0 + r < a.rows;
        const long long row = live[r] ? row0 + r : row0;
        i1[r] = row % a.ne1;
        i2[r] = (row / a.ne1) % a.ne2;
        i3[r] = row / (a.ne1 * a.ne2);
        const float* xr = a.x + i1[r] * a.xnb[1] + i2[r] * a.xnb[2] + i3[r] * a.xnb[3];
#pragma unroll
        for (int k = 0; k < PER; ++k) v[r][k] = live[r] && lane + 32 * k < n ? __ldg(xr + lane + 32 * k) : 0.0f;
    }
    double s[R];
#pragma unroll
    for (int r = 0; r < R; ++r) s[r] = 0.0;
#pragma unroll
    for (int k = 0; k < PER; ++k)
#pragma unroll
        for (int r = 0; r < R; ++r) s[r] += static_cast<double>(v[r][k]);
    float mean[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        s[r] = warp_sum(s[r]);
        mean[r] = static_cast<float>(s[r] / static_cast<double>(n));
    }
    double q[R];
#pragma unroll
    for (int r = 0; r < R; ++r) q[r] = 0.0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        if (lane + 32 * k < n) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float d = v[r][k] - mean[r];
                q[r] += static_cast<double>(d * d);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        q[r] = warp_sum(q[r]);
        const float scale = 1.0f / sqrtf(static_cast<float>(q[r] / static_cast<double>(n)) + a.eps);
#pragma unroll
        for (int k = 0; k < PER; ++k) v[r][k] = (v[r][k] - mean[r]) * scale;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        ChainRow cr;
        row_offsets(a.chain, cr, 0, i1[r], i2[r], i3[r]);
#pragma unroll
        for (int st = 0; st < SDB_MAX_STEPS; ++st) {
            if (st >= a.chain.count) break;
            if (a.chain.kind[st] == SDB_STEP_SILU) {
#pragma unroll
                for (int k = 0; k < PER; ++k) v[r][k] = silu(v[r][k]);
            } else {
                float o[PER];
#pragma unroll
                for (int k = 0; k < PER; ++k)
                    o[k] = __ldg(a.chain.operand[st] + cr.off[st] + min(lane + 32 * k, n - 1) * a.chain.nb[st][0]);
#pragma unroll
                for (int k = 0; k < PER; ++k)
                    v[r][k] = a.chain.kind[st] == SDB_STEP_ADD ? v[r][k] + o[k] : v[r][k] * o[k];
            }
        }
        if (!live[r]) continue;
        float* yr = a.y + i1[r] * a.ynb[1] + i2[r] * a.ynb[2] + i3[r] * a.ynb[3];
#pragma unroll
        for (int k = 0; k < PER; ++k)
            if (lane + 32 * k < n) yr[(lane + 32 * k) * a.ynb[0]] = v[r][k];
    }
}

bool f32(const sdb_tensor* t) { return t && t->type == SDB_TYPE_F32 && t->data; }

bool contiguous(const sdb_tensor* t) {
    int64_t expect = 4;
    for (int d = 0; d < 4; ++d) {
        if (t->ne[d] <= 0) return false;
        if (t->ne[d] > 1 && t->nb[d] != expect) return false;
        expect *= t->ne[d];
    }
    return true;
}

bool same_shape(const sdb_tensor* a, const sdb_tensor* b) {
    for (int d = 0; d < 4; ++d)
        if (a->ne[d] != b->ne[d]) return false;
    return true;
}

// Double partial sums of split groups (2 per CTA slice), grown on demand.
double* partial_buffer(size_t count) {
    static thread_local double* buf = nullptr;
    static thread_local size_t cap = 0;
    static thread_local int dev = -1;
    int d = 0;
    cudaGetDevice(&d);
    if (count > cap || d != dev) {
        if (buf && d == dev) cudaFree(buf);
        buf = nullptr;
        cap = 0;
        if (cudaMalloc(&buf, count * sizeof(double)) != cudaSuccess) return nullptr;
        cap = count;
        dev = d;
    }
    return buf;
}

}  // namespace

}  // namespace sdb

using namespace sdb;

namespace sdb {
namespace {

bool channels_last(const sdb_tensor* t) {
    const int64_t c = t->ne[2], w = t->ne[0], h = t->ne[1];
    return t->nb[2] == 4 && t->nb[0] == 4 * c && t->nb[1] == 4 * c * w && t->nb[3] == 4 * c * w * h;
}

bool uniform_chain(const sdb_chain* c) {
    if (!c) return true;
    for (int s = 0; s < c->count; ++s)
        if (c->steps[s].kind != SDB_STEP_SILU && (c->steps[s].nb[0] != 0 || c->steps[s].nb[1] != 0)) return false;
    return true;
}

// Scratch of the channels-last path: the CTAs' partial sums, the groups'
// statistics and the per-image counts (zeroed when allocated; the last CTA of
// an image resets its count), grown on demand per thread and device, outside
// stream capture only.
struct ClScratch {
    double* partial;
    float* stats;
    unsigned* count;
};

bool cl_scratch(size_t partials, size_t stats, size_t images, cudaStream_t st, ClScratch* out) {
    static thread_local uint8_t* buf = nullptr;
    static thread_local size_t cap_p = 0, cap_s = 0, cap_i = 0;
    static thread_local int dev = -1;
    int d = 0;
    cudaGetDevice(&d);
    if (partials > cap_p || stats > cap_s || images > cap_i || d != dev) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
        if (buf && d == dev) {
            cudaStreamSynchronize(st);
            cudaFree(buf);
        }
        buf = nullptr;
        cap_p = std::max(partials, cap_p);
        cap_s = std::max(stats, cap_s);
        cap_i = std::max(images, cap_i);
        const size_t bytes = cap_p * sizeof(double) + cap_s * sizeof(float) + cap_i * sizeof(unsigned);
        if (cudaMalloc(&buf, bytes) != cudaSuccess) {
            cap_p = cap_s = cap_i = 0;
            return false;
        }
        if (cudaMemsetAsync(buf, 0, bytes, st) != cudaSuccess) return false;
        dev = d;
    }
    out->partial = reinterpret_cast<double*>(buf);
    out->stats = reinterpret_cast<float*>(buf + cap_p * sizeof(double));
    out->count = reinterpret_cast<unsigned*>(buf + cap_p * sizeof(double) + cap_s * sizeof(float));
    return true;
}

template <int PATTERN>
int launch_nhwc_apply(const NhwcArgs& a, int grid, cudaStream_t st) {
    nhwc_gn_apply_kernel<PATTERN><<<grid, kClThreads, 0, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

// The statistics pass alone, into `stats` (the caller's [N][groups][2]) or, with stats null, the scratch's.
int nhwc_stats(NhwcArgs& a, const sdb_tensor* x, int32_t groups, float eps, float* stats, cudaStream_t st,
               int* grid_out) {
    a.x = static_cast<const float*>(x->data);
    a.positions = static_cast<int>(x->ne[0] * x->ne[1]);
    a.c = static_cast<int>(x->ne[2]);
    a.c4 = a.c / 4;
    a.groups = groups;
    a.cpg = a.c / groups;
    a.eps = eps;
    a.rpp = a.c4 <= kClThreads ? kClThreads / a.c4 : 1;
    const int images = static_cast<int>(x->ne[3]);
    const int sms = current_sm_count();
    // CTAs: up to four per SM over all images, each thread at least eight rows (its fixed costs --
    // the group of each channel, the chain's operands, the CTA's reduction -- spread over them).
    const int most = std::max(1, a.positions / (8 * a.rpp));
    a.cpi = std::max(1, std::min(most, (4 * sms + images - 1) / images));
    a.per = (a.positions + a.cpi - 1) / a.cpi;
    a.cpi = (a.positions + a.per - 1) / a.per;
    const int grid = images * a.cpi;
    ClScratch sc{};
    if (!cl_scratch(2 * static_cast<size_t>(grid) * groups, 2 * static_cast<size_t>(images) * groups,
                    static_cast<size_t>(images), st, &sc))
        return fail(SDB_OUT_OF_MEMORY, "sdb_group_norm: scratch (first use of a size under stream capture?)");
    a.partial = sc.partial;
    a.stats = stats ? stats : sc.stats;
    a.count = sc.count;
    const int csum_len = a.c4 <= kClThreads ? a.rpp * a.c : a.c;
    const size_t smem = 2 * static_cast<size_t>(csum_len) * sizeof(double);
    SDB_CUDA(cudaFuncSetAttribute(nhwc_gn_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  2 * kClMaxCsum * static_cast<int>(sizeof(double))));
    nhwc_gn_stats_kernel<<<grid, kClThreads, smem, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    *grid_out = grid;
    return SDB_OK;
}

int group_norm_nhwc(const sdb_tensor* x, const sdb_tensor* dst, int32_t groups, float eps, const sdb_chain* chain,
                    cudaStream_t st) {
    NhwcArgs a{};
    a.y = static_cast<float*>(dst->data);
    a.chain = make_chain(chain);
    int grid = 0;
    if (int s = nhwc_stats(a, x, groups, eps, nullptr, st, &grid); s != SDB_OK) return s;
    // The chain's pattern: mul then add (then SiLU) -- the GroupNorm's affine -- compiles alone.
    const Chain& c = a.chain;
    if (c.count == 0) return launch_nhwc_apply<kChainNone>(a, grid, st);
    if (c.count >= 2 && c.kind[0] == SDB_STEP_MUL && c.kind[1] == SDB_STEP_ADD &&
        (c.count == 2 || (c.count == 3 && c.kind[2] == SDB_STEP_SILU)))
        return c.count == 2 ? launch_nhwc_apply<kChainAffine>(a, grid, st)
                            : launch_nhwc_apply<kChainAffineSilu>(a, grid, st);
    return launch_nhwc_apply<kChainGeneral>(a, grid, st);
}

}  // namespace
}  // namespace sdb

namespace sdb {
namespace {

// ---- LayerNorm fused into the split of a linear layer's rows ----------------
//
// A transformer's LayerNorm feeds a linear layer, whose pre-pass splits every
// FP32 row into FP16 hi and lo rows (split.cuh split_rows).  One warp a row
// does both: the row in registers (element lane + 32 k, as norm_rows_reg_kernel
// holds it), its mean and variance in double in the same order, (x - mean) *
// scale, the LayerNorm's chain (its gamma and beta) step by step as the
// LayerNorm kernel applies it -- the very numbers sdb_norm writes -- then
// split into the hi and lo rows the GEMM reads.  The normalised row is never
// written.
template <int PER>
__global__ void __launch_bounds__(256) norm_split_kernel(const RowArgs a, long long ld, uint16_t* __restrict__ out,
                                                         unsigned* err) {
    const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= a.rows) return;
    const int n = static_cast<int>(a.ne0);
    const long long i1 = row % a.ne1, i2 = (row / a.ne1) % a.ne2, i3 = row / (a.ne1 * a.ne2);
    const float* xr = a.x + i1 * a.xnb[1] + i2 * a.xnb[2] + i3 * a.xnb[3];
    float v[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) v[k] = lane + 32 * k < n ? __ldg(xr + (lane + 32 * k) * a.xnb[0]) : 0.0f;
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < PER; ++k) s += static_cast<double>(v[k]);
    s = warp_sum(s);
    const float mean = static_cast<float>(s / static_cast<double>(n));
    double q = 0.0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        if (lane + 32 * k < n) {
            const float d = v[k] - mean;
            q += static_cast<double>(d * d);
        }
    }
    q = warp_sum(q);
    const float scale = 1.0f / sqrtf(static_cast<float>(q / static_cast<double>(n)) + a.eps);
#pragma unroll
    for (int k = 0; k < PER; ++k) v[k] = (v[k] - mean) * scale;
    ChainRow cr;
    row_offsets(a.chain, cr, 0, i1, i2, i3);
#pragma unroll
    for (int st = 0; st < SDB_MAX_STEPS; ++st) {
        if (st >= a.chain.count) break;
        if (a.chain.kind[st] == SDB_STEP_SILU) {
#pragma unroll
            for (int k = 0; k < PER; ++k) v[k] = silu(v[k]);
        } else {
            float o[PER];
#pragma unroll
            for (int k = 0; k < PER; ++k)
                o[k] = __ldg(a.chain.operand[st] + cr.off[st] + min(lane + 32 * k, n - 1) * a.chain.nb[st][0]);
#pragma unroll
            for (int k = 0; k < PER; ++k) v[k] = a.chain.kind[st] == SDB_STEP_ADD ? v[k] + o[k] : v[k] * o[k];
        }
    }
    bool over = false;
    __half* hi = reinterpret_cast<__half*>(out) + row * ld;
    __half* lo = reinterpret_cast<__half*>(out) + (a.rows + row) * ld;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
        const int e = lane + 32 * k;
        if (e < n) {
            __half h, l;
            split_half(v[k], h, l);
            over |= !(fabsf(v[k]) <= kHalfLimit);
            hi[e] = h;
            lo[e] = l;
        } else if (e < ld) {
            hi[e] = __float2half_rn(0.0f);
            lo[e] = __float2half_rn(0.0f);
        }
    }
    for (int e = 32 * PER + lane; e < ld; e += 32) {
        hi[e] = __float2half_rn(0.0f);
        lo[e] = __float2half_rn(0.0f);
    }
    if (over) atomicOr(err, kErrRange);
}

}  // namespace

// LayerNorm of x's rows with its chain, split into out: hi rows [0, R), lo rows [R, 2R) of ld FP16.
int layer_norm_split(const sdb_tensor* x, float eps, const sdb_chain* chain, long long ld, uint16_t* out,
                     unsigned* err, cudaStream_t st) {
    if (!f32(x) || x->nb[0] % 4 || x->nb[1] % 4 || x->nb[2] % 4 || x->nb[3] % 4 || ld < x->ne[0])
        return fail(SDB_NOT_SUPPORTED, "LayerNorm prologue: not supported");
    if (chain && (chain->count > SDB_MAX_STEPS || chain->redirect || chain->from_redirect))
        return fail(SDB_INVALID, "LayerNorm prologue: invalid chain");
    RowArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.ne0 = x->ne[0]; a.ne1 = x->ne[1]; a.ne2 = x->ne[2];
    a.rows = x->ne[1] * x->ne[2] * x->ne[3];
    for (int d = 0; d < 4; ++d) a.xnb[d] = x->nb[d] / 4;
    a.eps = eps;
    a.chain = make_chain(chain);
    const unsigned blocks = static_cast<unsigned>((a.rows * 32 + 255) / 256);
    const int per = static_cast<int>((a.ne0 + 31) / 32);
    if (per <= 10) norm_split_kernel<10><<<blocks, 256, 0, st>>>(a, ld, out, err);
    else if (per <= 20) norm_split_kernel<20><<<blocks, 256, 0, st>>>(a, ld, out, err);
    else if (per <= 40) norm_split_kernel<40><<<blocks, 256, 0, st>>>(a, ld, out, err);
    else return fail(SDB_NOT_SUPPORTED, "LayerNorm prologue: rows of at most 1280");
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}
}  // namespace sdb

extern "C" int sdb_group_norm_stats(const sdb_tensor* x, int32_t groups, float eps, float* stats, void* stream) {
    if (!f32(x) || !channels_last(x) || groups <= 0 || x->ne[2] % groups != 0 || x->ne[2] % 4 != 0 ||
        x->ne[2] > kClMaxChannels || groups > kClMaxGroups || x->ne[0] * x->ne[1] > (1LL << 30) || x->ne[3] > 4096 ||
        (reinterpret_cast<uintptr_t>(x->data) & 15) || stats == nullptr)
        return fail(SDB_NOT_SUPPORTED,
                    "sdb_group_norm_stats: a channels-last image with C % groups == 0, C % 4 == 0, C <= 3072, "
                    "aligned, and a stats buffer");
    NhwcArgs a{};
    int grid = 0;
    return nhwc_stats(a, x, groups, eps, stats, static_cast<cudaStream_t>(stream), &grid);
}

extern "C" int sdb_group_norm(const sdb_tensor* x, const sdb_tensor* dst, int32_t groups, float eps,
                              const sdb_chain* chain, void* stream) {
    if (f32(x) && f32(dst) && same_shape(x, dst) && groups > 0 && channels_last(x) && channels_last(dst)) {
        if (x->ne[2] % groups != 0 || x->ne[2] % 4 != 0 || x->ne[2] > kClMaxChannels ||
            x->ne[0] * x->ne[1] > (1LL << 30) || x->ne[3] > 4096 || groups > kClMaxGroups || !uniform_chain(chain) ||
            (reinterpret_cast<uintptr_t>(x->data) & 15) || (reinterpret_cast<uintptr_t>(dst->data) & 15))
            return fail(SDB_NOT_SUPPORTED,
                        "sdb_group_norm: channels-last needs C % groups == 0, C % 4 == 0, C <= 3072, aligned "
                        "images and a per-channel chain");
        if (chain && (chain->count > SDB_MAX_STEPS || chain->redirect))
            return fail(SDB_INVALID, "sdb_group_norm: invalid chain");
        return group_norm_nhwc(x, dst, groups, eps, chain, static_cast<cudaStream_t>(stream));
    }
    if (!f32(x) || !f32(dst) || !contiguous(x) || !same_shape(x, dst) || groups <= 0)
        return fail(SDB_NOT_SUPPORTED, "sdb_group_norm: not supported");
    if (chain && (chain->count > SDB_MAX_STEPS || chain->redirect))
        return fail(SDB_INVALID, "sdb_group_norm: invalid chain");
    for (int d = 0; d < 4; ++d)
        if (dst->nb[d] % 4) return fail(SDB_NOT_SUPPORTED, "sdb_group_norm: misaligned output");
    const auto st = static_cast<cudaStream_t>(stream);
    GroupArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.y = static_cast<float*>(dst->data);
    a.ne0 = x->ne[0]; a.ne1 = x->ne[1]; a.ne2 = x->ne[2]; a.ne3 = x->ne[3];
    for (int d = 0; d < 4; ++d) { a.xnb[d] = x->nb[d] / 4; a.ynb[d] = dst->nb[d] / 4; }
    a.groups = groups;
    a.per_group = static_cast<int>((a.ne2 + groups - 1) / groups);
    a.eps = eps;
    a.chain = make_chain(chain);
    a.uniform = 1;
    for (int s = 0; s < a.chain.count; ++s)
        if (a.chain.kind[s] != SDB_STEP_SILU && (a.chain.nb[s][0] != 0 || a.chain.nb[s][1] != 0)) a.uniform = 0;
    const long long items = static_cast<long long>(groups) * a.ne3;
    const long long group_elems = a.ne0 * a.ne1 * a.per_group;
    if (group_elems <= kResident && items <= 0x7fffffffLL) {
        const int smem = static_cast<int>(group_elems * 4);
        SDB_CUDA(cudaFuncSetAttribute(group_resident_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kResident * 4)));
        group_resident_kernel<<<static_cast<unsigned>(items), kResidentThreads, smem, st>>>(a);
        count_launch();
        SDB_CUDA(cudaGetLastError());
        return SDB_OK;
    }
    // Enough CTAs for every SM several times over, each slice at least 8K elements.
    const long long want = std::max<long long>(1, (4LL * current_sm_count() + items - 1) / items);
    a.split = static_cast<int>(std::min<long long>(want, std::max<long long>(1, group_elems / 8192)));
    a.partial = partial_buffer(static_cast<size_t>(items * a.split * 2));
    if (!a.partial) return fail(SDB_OUT_OF_MEMORY, "sdb_group_norm: partial sums");
    const unsigned grid = static_cast<unsigned>(items * a.split);
    group_sum_kernel<<<grid, kNormThreads, 0, st>>>(a, 0);
    group_sum_kernel<<<grid, kNormThreads, 0, st>>>(a, 1);
    group_apply_kernel<<<grid, kNormThreads, 0, st>>>(a);
    count_launch(3);
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

extern "C" int sdb_norm(const sdb_tensor* x, const sdb_tensor* dst, float eps, const sdb_chain* chain, void* stream) {
    if (!f32(x) || !f32(dst) || !same_shape(x, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_norm: not supported");
    if (chain && (chain->count > SDB_MAX_STEPS || chain->redirect))
        return fail(SDB_INVALID, "sdb_norm: invalid chain");
    for (int d = 0; d < 4; ++d)
        if (x->nb[d] % 4 || dst->nb[d] % 4) return fail(SDB_NOT_SUPPORTED, "sdb_norm: misaligned");
    const auto st = static_cast<cudaStream_t>(stream);
    RowArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.y = static_cast<float*>(dst->data);
    a.ne0 = x->ne[0]; a.ne1 = x->ne[1]; a.ne2 = x->ne[2];
    a.rows = x->ne[1] * x->ne[2] * x->ne[3];
    for (int d = 0; d < 4; ++d) { a.xnb[d] = x->nb[d] / 4; a.ynb[d] = dst->nb[d] / 4; }
    a.eps = eps;
    a.chain = make_chain(chain);
    const long long threads = a.rows * 32;
    const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
    const unsigned blocks2 = static_cast<unsigned>(((a.rows + 1) / 2 * 32 + 255) / 256);   // two rows a warp
    const int per = static_cast<int>((a.ne0 + 31) / 32);
    if (a.xnb[0] == 1 && per <= 8)
        norm_rows_reg_kernel<8, 2><<<blocks2, 256, 0, st>>>(a);
    else if (a.xnb[0] == 1 && per <= 12)
        norm_rows_reg_kernel<12, 2><<<blocks2, 256, 0, st>>>(a);
    else if (a.xnb[0] == 1 && per <= 20)
        norm_rows_reg_kernel<20, 1><<<blocks, 256, 0, st>>>(a);
    else if (a.xnb[0] == 1 && per <= kLnPer)
        norm_rows_reg_kernel<kLnPer, 1><<<blocks, 256, 0, st>>>(a);
    else
        norm_rows_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

// ---- GroupNorm for callers that cannot allocate device memory ---------------
//
// Some callers may not call cudaMalloc at all: a host whose device memory is
// owned by another allocator (a memory pool or arena that must account for
// every byte), code running while a CUDA graph is being captured, or a
// real-time loop that may not take the driver's allocation lock.
// sdb_group_norm_no_alloc is sdb_group_norm for them: it takes the split path
// (sum pass, centred-sum pass, apply) and keeps the per-slice double partial
// sums in the fixed array below, which the module reserves when it loads on a
// device and holds until the process exits (512 KiB on every GPU that loads
// this library).  That bounds the work it takes: at most kStaticSlices slices,
// i.e. (images x groups) <= 32768.  Larger inputs are rejected.
//
// Every slot a call reads is written earlier in the same call (pass one writes
// the sums, pass two the centred sums, the apply pass reads both), so nothing
// has to be cleared between calls.  All calls share the array: two calls whose
// kernels overlap on the GPU (different streams, no ordering between them)
// race on it and give wrong results.

namespace sdb {
namespace {

constexpr long long kStaticSlices = 32768;                   // slices of (image, group)
static __device__ __align__(256) double g_static_partials[kStaticSlices * 2];

// The device address of g_static_partials on the current device, looked up
// once per device (the first call on a device does this; make that call
// before any stream capture begins).
double* static_partials(int* status) {
    static std::mutex lock;
    static std::unordered_map<int, double*> addresses;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { *status = cuda_fail(e, "cudaGetDevice"); return nullptr; }
    std::lock_guard<std::mutex> guard(lock);
    auto it = addresses.find(dev);
    if (it != addresses.end()) return it->second;
    double* p = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_static_partials);
    if (e != cudaSuccess) { *status = cuda_fail(e, "cudaGetSymbolAddress(g_static_partials)"); return nullptr; }
    addresses.emplace(dev, p);
    return p;
}

}  // namespace
}  // namespace sdb

extern "C" int sdb_group_norm_no_alloc(const sdb_tensor* x, const sdb_tensor* dst, int32_t groups, float eps,
                                       const sdb_chain* chain, void* stream) {
    if (!f32(x) || !f32(dst) || !contiguous(x) || !same_shape(x, dst) || groups <= 0)
        return fail(SDB_NOT_SUPPORTED, "sdb_group_norm_no_alloc: not supported");
    if (chain && (chain->count > SDB_MAX_STEPS || chain->redirect))
        return fail(SDB_INVALID, "sdb_group_norm_no_alloc: invalid chain");
    for (int d = 0; d < 4; ++d)
        if (dst->nb[d] % 4) return fail(SDB_NOT_SUPPORTED, "sdb_group_norm_no_alloc: misaligned output");
    const long long items = static_cast<long long>(groups) * x->ne[3];
    if (items > kStaticSlices)
        return fail(SDB_INVALID, "sdb_group_norm_no_alloc: images x groups = " + std::to_string(items) +
                                     " exceeds the static scratch limit of " + std::to_string(kStaticSlices));
    int status = SDB_OK;
    double* partials = static_partials(&status);
    if (!partials) return status;
    GroupArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.y = static_cast<float*>(dst->data);
    a.ne0 = x->ne[0]; a.ne1 = x->ne[1]; a.ne2 = x->ne[2]; a.ne3 = x->ne[3];
    for (int d = 0; d < 4; ++d) { a.xnb[d] = x->nb[d] / 4; a.ynb[d] = dst->nb[d] / 4; }
    a.groups = groups;
    a.per_group = static_cast<int>((a.ne2 + groups - 1) / groups);
    a.eps = eps;
    a.chain = make_chain(chain);
    a.uniform = 1;
    for (int s = 0; s < a.chain.count; ++s)
        if (a.chain.kind[s] != SDB_STEP_SILU && (a.chain.nb[s][0] != 0 || a.chain.nb[s][1] != 0)) a.uniform = 0;
    const long long group_elems = a.ne0 * a.ne1 * a.per_group;
    // As sdb_group_norm's split path, but no more slices than the array holds.
    const long long want = std::max<long long>(1, (4LL * current_sm_count() + items - 1) / items);
    const long long split = std::min({want, std::max<long long>(1, group_elems / 8192), kStaticSlices / items});
    a.split = static_cast<int>(split);
    a.partial = partials;
    const auto st = static_cast<cudaStream_t>(stream);
    const unsigned grid = static_cast<unsigned>(items * a.split);
    group_sum_kernel<<<grid, kNormThreads, 0, st>>>(a, 0);
    group_sum_kernel<<<grid, kNormThreads, 0, st>>>(a, 1);
    group_apply_kernel<<<grid, kNormThreads, 0, st>>>(a);
    count_launch(3);
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}
