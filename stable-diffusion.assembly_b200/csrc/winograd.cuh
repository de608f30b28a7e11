// Winograd's minimal filtering for 3x3 convolutions at stride 1: F(2x2, 3x3)
// and F(4x4, 3x3) (Lavin and Gray, 2016), as the reference computes them
// (winograd.cc:9-31 for F(2x2), winograd.cc:1148-1190 for F(4x4)):
//
//     Y = A^T [ sum over ic of (G g G^T) (.) (B^T d B) ] A
//
// for each tile of F x F outputs, d the (F+2) x (F+2) inputs around it, g a
// channel's kernel.  On the GPU the sum over the channels is XI = (F+2)^2
// matrix products, one per element xi of a tile -- tiles x IC times IC x OC --
// batched in one launch of the tcgen05 GEMM (gemm.cuh):
//
//   winograd_inputs_kernel   the image -> V = B^T d B of every tile and channel,
//                            split into FP16 pairs v = hi + lo 2^-11, written
//                            [plane][xi][tile][channel] (the GEMM's A rows);
//   winograd_weights_kernel  the kernels -> U = G g G^T, split the same way,
//                            [plane][xi][oc][channel] (the GEMM's B rows; once,
//                            kept by the weight store);
//   the GEMM                 M[xi][tile][oc] = sum_ic V U by three FP16
//                            products (hi hi, lo hi, hi lo), FP32 out;
//   winograd_outputs_kernel  Y = A^T M A of every tile and channel, then the
//                            chain, into the output.
//
// Both operands are FP32 after their transforms (G holds thirds and
// fifteenths), hence the three products.  The transforms are computed in
// single precision as the reference's are; F(4x4)'s larger transforms round
// about seven times as much as F(2x2)'s (winograd.cc:1165-1168), and that, not
// the split, sets its error.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "ptx.cuh"

namespace sdb {

template <int F>
struct Wino;

// F(2x2, 3x3): winograd.cc:14-22.
template <>
struct Wino<2> {
    static constexpr int kA = 4;  // inputs of a tile along a side
    static constexpr int kXi = 16;
    __host__ __device__ static constexpr float bt(int i, int j) {
        constexpr float m[4][4] = {{1, 0, -1, 0}, {0, 1, 1, 0}, {0, -1, 1, 0}, {0, 1, 0, -1}};
        return m[i][j];
    }
    __host__ __device__ static constexpr float g(int i, int j) {
        constexpr float m[4][3] = {{1, 0, 0}, {0.5f, 0.5f, 0.5f}, {0.5f, -0.5f, 0.5f}, {0, 0, 1}};
        return m[i][j];
    }
    __host__ __device__ static constexpr float at(int i, int j) {
        constexpr float m[2][4] = {{1, 1, 1, 0}, {0, 1, -1, -1}};
        return m[i][j];
    }
};

// F(4x4, 3x3), points 0, 1, -1, 2, -1/2 and infinity: winograd.cc:1155-1190, 1259-1264.
template <>
struct Wino<4> {
    static constexpr int kA = 6;
    static constexpr int kXi = 36;
    __host__ __device__ static constexpr float bt(int i, int j) {
        constexpr float m[6][6] = {{1.0f, 1.5f, -2.0f, -1.5f, 1.0f, 0.0f},  {0.0f, -1.0f, -2.5f, -0.5f, 1.0f, 0.0f},
                                   {0.0f, 1.0f, 0.5f, -2.5f, 1.0f, 0.0f},   {0.0f, -0.5f, -1.0f, 0.5f, 1.0f, 0.0f},
                                   {0.0f, 2.0f, -1.0f, -2.0f, 1.0f, 0.0f},  {0.0f, 1.0f, 1.5f, -2.0f, -1.5f, 1.0f}};
        return m[i][j];
    }
    __host__ __device__ static constexpr float g(int i, int j) {
        constexpr float m[6][3] = {{1.0f, 0.0f, 0.0f},
                                   {-1.0f / 3, -1.0f / 3, -1.0f / 3},
                                   {1.0f / 3, -1.0f / 3, 1.0f / 3},
                                   {1.0f / 15, 2.0f / 15, 4.0f / 15},
                                   {-16.0f / 15, 8.0f / 15, -4.0f / 15},
                                   {0.0f, 0.0f, 1.0f}};
        return m[i][j];
    }
    __host__ __device__ static constexpr float at(int i, int j) {
        constexpr float m[4][6] = {{1.0f, 1.0f, 1.0f, 1.0f, 1.0f, 0.0f},
                                   {0.0f, 1.0f, -1.0f, 2.0f, -0.5f, 0.0f},
                                   {0.0f, 1.0f, 1.0f, 4.0f, 0.25f, 0.0f},
                                   {0.0f, 1.0f, -1.0f, 8.0f, -0.125f, 1.0f}};
        return m[i][j];
    }
};

// The arguments of the transform kernels.  Tiles t = (img * th + ty) * tw + tx
// cover the output in F x F blocks; their rows in V and M are padded per xi
// to tiles_pad (a multiple of the GEMM's 128-row tile).
struct WinoArgs {
    const float* x;          // input [W, H, IC, N], element strides xnb
    long long xnb[4];
    int iw, ih, ic, n;
    int ow, oh, oc;
    int p0, p1;              // padding (left, top)
    int tw, th;              // tiles across and down an image
    long long tiles;         // n * th * tw
    long long tiles_pad;
    int icp8;                // channels of a V row (IC rounded up to 8; the rest zero)
    __half* v;               // V [2][XI][tiles_pad][icp8]
    const float* m;          // M [XI][tiles_pad][ldm]
    long long ldm;
    float* y;                // output (the redirect when the chain has one), element strides ynb
    long long ynb[4];
    Chain chain;
    unsigned* err;
    GnIn gn;                 // the inputs read through a GroupNorm prologue (gn.stats not null)
};

// The kernels' transform U = G g G^T of output channel o and input channel c,
// split, into [plane][xi][ocp][kpad] FP16 (winograd.cc:1266-1300: G g a
// column at a time, then (G g) G^T a row at a time, in single precision).
template <int F>
__global__ void winograd_weights_kernel(const uint8_t* __restrict__ src, int type, long long nb0, long long nb1,
                                        long long nb2, long long nb3, int ic, int oc, long long ocp, long long kpad,
                                        __half* __restrict__ out, unsigned* err) {
    using W = Wino<F>;
    constexpr int A = W::kA;
    const long long total = static_cast<long long>(oc) * ic;
    const long long plane = static_cast<long long>(W::kXi) * ocp * kpad;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long o = idx / ic;
        const long long c = idx - o * ic;
        float g[3][3];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const uint8_t* p = src + j * nb0 + r * nb1 + c * nb2 + o * nb3;
                g[r][j] = type == SDB_TYPE_F16 ? __half2float(*reinterpret_cast<const __half*>(p))
                                               : *reinterpret_cast<const float*>(p);
            }
        float t[A][3];
#pragma unroll
        for (int i = 0; i < A; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) t[i][j] = W::g(i, 0) * g[0][j] + W::g(i, 1) * g[1][j] + W::g(i, 2) * g[2][j];
        bool over = false;
#pragma unroll
        for (int i = 0; i < A; ++i)
#pragma unroll
            for (int j = 0; j < A; ++j) {
                const float u = t[i][0] * W::g(j, 0) + t[i][1] * W::g(j, 1) + t[i][2] * W::g(j, 2);
                __half hi, lo;
                split_half(u, hi, lo);
                over |= !(fabsf(u) <= kHalfLimit);
                const long long at = (static_cast<long long>(i * A + j) * ocp + o) * kpad + c;
                out[at] = hi;
                out[plane + at] = lo;
            }
        if (over) atomicOr(err, kErrRange);
    }
}

// V = B^T d B of tile t and channels c, c + 1 (VEC = 2: a channels-last
// image, whose channel pairs are one 8-byte load; VEC = 1 any strides),
// split; rows of padded tiles and channels past IC are zeros.  Consecutive
// threads take consecutive channels.  B^T d is formed a column of d at a
// time, then each row of (B^T d) B is split and stored as it is made.
// GN: the image read through the GroupNorm prologue (gn_in) -- inside the
// image only; the padding stays zero, as the normalised image's would.
template <int F, int VEC, bool GN = false>
__global__ void __launch_bounds__(256, GN ? 2 : 1) winograd_inputs_kernel(const WinoArgs a) {
    using W = Wino<F>;
    constexpr int A = W::kA;
    const int groups = a.icp8 / VEC;  // channel groups of a tile row
    const int total = static_cast<int>(a.tiles_pad) * groups;
    const long long xi_stride = a.tiles_pad * a.icp8;
    const long long plane = W::kXi * xi_stride;
    const int tiles = static_cast<int>(a.tiles);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const int t = idx / groups;
        const int c = (idx - t * groups) * VEC;
        const bool live = t < tiles && c < a.ic;
        int x0 = 0, y0 = 0, img = 0;
        const float* base = a.x;
        if (live) {
            const int tx = t % a.tw;
            const int rest = t / a.tw;
            const int ty = rest % a.th;
            img = rest / a.th;
            x0 = tx * F - a.p0;
            y0 = ty * F - a.p1;
            base = a.x + c * a.xnb[2] + img * a.xnb[3];
        }
        GnCoef gk[VEC];
        if (GN && live) {
#pragma unroll
            for (int e = 0; e < VEC; ++e) gk[e] = gn_coef(a.gn, c + e, img);
        }
        float s[VEC][A][A];  // B^T d
#pragma unroll
        for (int j = 0; j < A; ++j) {
            float d[VEC][A];
            const int xx = x0 + j;
            const bool col_ok = live && xx >= 0 && xx < a.iw;
#pragma unroll
            for (int k = 0; k < A; ++k) {
                const int yy = y0 + k;
                const bool ok = col_ok && yy >= 0 && yy < a.ih;
                const float* p = base + xx * a.xnb[0] + yy * a.xnb[1];
                if (VEC == 2) {
                    float2 v = ok ? __ldg(reinterpret_cast<const float2*>(p)) : make_float2(0.0f, 0.0f);
                    if (GN && ok) {
                        v.x = gn_in(a.gn, v.x, gk[0]);
                        v.y = gn_in(a.gn, v.y, gk[VEC - 1]);
                    }
                    d[0][k] = v.x;
                    d[VEC - 1][k] = v.y;
                } else {
                    d[0][k] = ok ? (GN ? gn_in(a.gn, __ldg(p), gk[0]) : __ldg(p)) : 0.0f;
                }
            }
#pragma unroll
            for (int e = 0; e < VEC; ++e)
#pragma unroll
                for (int i = 0; i < A; ++i) {
                    float acc = 0.0f;
#pragma unroll
                    for (int k = 0; k < A; ++k)
                        if (W::bt(i, k) != 0.0f) acc += W::bt(i, k) * d[e][k];
                    s[e][i][j] = acc;
                }
        }
        bool over = false;
        __half* out = a.v + static_cast<long long>(t) * a.icp8 + c;
#pragma unroll
        for (int i = 0; i < A; ++i)
#pragma unroll
            for (int j = 0; j < A; ++j) {
                __half hi[VEC], lo[VEC];
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    float acc = 0.0f;
#pragma unroll
                    for (int k = 0; k < A; ++k)
                        if (W::bt(j, k) != 0.0f) acc += s[e][i][k] * W::bt(j, k);
                    split_half(acc, hi[e], lo[e]);
                    over |= !(fabsf(acc) <= kHalfLimit);
                }
                __half* o = out + (i * A + j) * xi_stride;
                if (VEC == 2) {
                    *reinterpret_cast<__half2*>(o) = __halves2half2(hi[0], hi[VEC - 1]);
                    *reinterpret_cast<__half2*>(o + plane) = __halves2half2(lo[0], lo[VEC - 1]);
                } else {
                    o[0] = hi[0];
                    o[plane] = lo[0];
                }
            }
        if (over) atomicOr(a.err, kErrRange);
    }
}

// Y = A^T M A of tile t and output channels o, o + 1 (VEC = 2: an output
// whose channel pairs are adjacent and OC even), then the chain, into the
// output.  Consecutive threads take consecutive channels.  All of a thread's
// XI loads are issued before any is used; the chain is applied a step at a
// time over the tile's outputs, its operand offsets for the thread's channel
// and image formed once.
template <int F, int VEC>
__global__ void __launch_bounds__(256) winograd_outputs_kernel(const WinoArgs a) {
    using W = Wino<F>;
    constexpr int A = W::kA;
    const int groups = (a.oc + VEC - 1) / VEC;
    const int total = static_cast<int>(a.tiles) * groups;
    const long long xi_stride = a.tiles_pad * a.ldm;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
        const int t = idx / groups;
        const int o = (idx - t * groups) * VEC;
        const float* mp = a.m + static_cast<long long>(t) * a.ldm + o;
        float m[VEC][A * A];
#pragma unroll
        for (int x = 0; x < A * A; ++x) {
            if (VEC == 2) {
                const float2 v = __ldg(reinterpret_cast<const float2*>(mp + x * xi_stride));
                m[0][x] = v.x;
                m[VEC - 1][x] = v.y;
            } else {
                m[0][x] = __ldg(mp + x * xi_stride);
            }
        }
        float y[VEC][F * F];
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            float s[F][A];  // A^T M
#pragma unroll
            for (int i = 0; i < F; ++i)
#pragma unroll
                for (int j = 0; j < A; ++j) {
                    float acc = 0.0f;
#pragma unroll
                    for (int k = 0; k < A; ++k)
                        if (W::at(i, k) != 0.0f) acc += W::at(i, k) * m[e][k * A + j];
                    s[i][j] = acc;
                }
#pragma unroll
            for (int i = 0; i < F; ++i)
#pragma unroll
                for (int j = 0; j < F; ++j) {
                    float acc = 0.0f;
#pragma unroll
                    for (int k = 0; k < A; ++k)
                        if (W::at(j, k) != 0.0f) acc += s[i][k] * W::at(j, k);
                    y[e][i * F + j] = acc;
                }
        }
        const int tx = t % a.tw;
        const int rest = t / a.tw;
        const int ty = rest % a.th;
        const int img = rest / a.th;
        const int ox0 = tx * F, oy0 = ty * F;
        float* ybase = a.y + o * a.ynb[2] + static_cast<long long>(img) * a.ynb[3];
        auto at_out = [&](int i, int j) { return (ox0 + j) * a.ynb[0] + static_cast<long long>(oy0 + i) * a.ynb[1]; };
        auto inside = [&](int i, int j) { return oy0 + i < a.oh && ox0 + j < a.ow; };
        if (a.chain.from_redirect) {
#pragma unroll
            for (int i = 0; i < F; ++i)
#pragma unroll
                for (int j = 0; j < F; ++j)
                    if (inside(i, j))
#pragma unroll
                        for (int e = 0; e < VEC; ++e) y[e][i * F + j] += ybase[at_out(i, j) + e * a.ynb[2]];
        }
#pragma unroll
        for (int st = 0; st < SDB_MAX_STEPS; ++st) {
            if (st >= a.chain.count) break;
            if (a.chain.kind[st] == SDB_STEP_SILU) {
#pragma unroll
                for (int e = 0; e < VEC; ++e)
#pragma unroll
                    for (int q = 0; q < F * F; ++q) y[e][q] = silu(y[e][q]);
                continue;
            }
            const long long* nb = a.chain.nb[st];
            const float* op = a.chain.operand[st] + o * nb[2] + static_cast<long long>(img) * nb[3];
            const bool add = a.chain.kind[st] == SDB_STEP_ADD;
#pragma unroll
            for (int i = 0; i < F; ++i)
#pragma unroll
                for (int j = 0; j < F; ++j) {
                    if (!inside(i, j)) continue;
                    const float* p = op + (ox0 + j) * nb[0] + static_cast<long long>(oy0 + i) * nb[1];
#pragma unroll
                    for (int e = 0; e < VEC; ++e) {
                        const float v = __ldg(p + e * nb[2]);
                        y[e][i * F + j] = add ? y[e][i * F + j] + v : y[e][i * F + j] * v;
                    }
                }
        }
#pragma unroll
        for (int i = 0; i < F; ++i)
#pragma unroll
            for (int j = 0; j < F; ++j) {
                if (!inside(i, j)) continue;
                float* out = ybase + at_out(i, j);
                if (VEC == 2) *reinterpret_cast<float2*>(out) = make_float2(y[0][i * F + j], y[VEC - 1][i * F + j]);
                else *out = y[0][i * F + j];
            }
    }
}

// ---------------------------------------------------------------- quantized
//
// F(2x2, 3x3) with integer products (winograd.cc:1826-2100): the transforms in
// single precision, each xi's product quantized -- the transformed kernels a
// scale per output channel per group of input channels, the transformed inputs
// a scale and zero point per tile per group of input channels.  The quantized
// bytes depend on every bit of the transforms, so both follow the reference's
// C++ order of operations exactly.

// U = G g G^T in FP32 as transform_weights computes it (winograd.cc:681-729):
// G g a column of g at a time, then (G g) G^T a row at a time, each sum of
// three left to right and halved after.  Out: [16 xi][oc][ic], xi = 4 i + j
// (i the row of the transformed kernel).
static __global__ void winograd2_weights_f32_kernel(const uint8_t* __restrict__ src, int type, long long nb0, long long nb1,
                                                    long long nb2, long long nb3, int ic, int oc, float* __restrict__ out) {
    const long long total = static_cast<long long>(oc) * ic;
    const long long plane = total;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long o = idx / ic;
        const long long c = idx - o * ic;
        float g[3][3];  // g[row][column]
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
                const uint8_t* ptr = src + q * nb0 + r * nb1 + c * nb2 + o * nb3;
                g[r][q] = type == SDB_TYPE_F16 ? __half2float(*reinterpret_cast<const __half*>(ptr))
                                               : *reinterpret_cast<const float*>(ptr);
            }
        float t[4][3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const float g0 = g[0][j], g1 = g[1][j], g2 = g[2][j];
            t[0][j] = g0;
            t[1][j] = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(g0, g1), g2));
            t[2][j] = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(g0, g1), g2));
            t[3][j] = g2;
        }
        float* dst = out + o * ic + c;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = t[i][0], b = t[i][1], d = t[i][2];
            dst[(i * 4 + 0) * plane] = a;
            dst[(i * 4 + 1) * plane] = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(a, b), d));
            dst[(i * 4 + 2) * plane] = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(a, b), d));
            dst[(i * 4 + 3) * plane] = d;
        }
    }
}

// Where the quantized F(2x2) finds its inputs (quant.cu wino2_quantize_kernel):
// the image, its element strides, padding and tiles; the transformed inputs
// of tile t are rows xi * tiles_pad + t, tiles past the last zeros.
struct Wino2QuantLoader {
    const float* x;
    long long xnb[4];
    int iw, ih, p0, p1, tw, th;
    long long tiles, tiles_pad;
};

}  // namespace sdb
