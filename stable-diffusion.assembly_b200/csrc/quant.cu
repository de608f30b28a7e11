// The quantized linear layers (tuning bits = 2..8): the inputs quantized by a
// pre-pass, the weights by the store, the product by qgemm_kernel
// (quant.cuh).  Taken, as the reference takes its quantized path
// (mul_mat.cc:96-105), for products of 256 rows or more.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/sdb.h"
#include "quant.cuh"
#include "runtime.cuh"
#include "split.cuh"
#include "store.cuh"
#include "winograd.cuh"

namespace sdb {

namespace {

// The reference's quantization of a row's group of inputs (quant.cc:282-313):
// lo, hi the least and greatest of the group's numbers and 0,
// s = (hi - lo) / levels, inverse = s > 0 ? 1 / s : 0, zero = rint(-lo * inverse),
// q = clamp(rint(x * inverse) + zero, 0, levels); the numbers past k the zero
// point; the group's scale s and offset s * zero.  One warp a (row, group),
// EPL numbers a lane.  Output in the GEMM's tiles: the bytes of row
// 128 tm + r, k-byte 64 ls + b at q[(tm * nstages + ls) * 8192 +
// quant_tile_offset(r, b)]; its group g's scale and offset at
// scales[((tm * groups + g) * 2 + {0, 1}) * 128 + r].  The rows come from a
// loader: a linear layer's input rows, or a convolution's columns.
struct RowLoader {
    const float* x;
    long long k;
    __device__ __forceinline__ float operator()(long long row, long long kk) const { return __ldg(x + row * k + kk); }
};

// A convolution's column of output position `row` (image n, output row oh,
// column ow; rows run ow fastest) at k = (ic, kh, kw), kw fastest -- the order
// of the kernel's own elements, in which the reference packs its columns and
// groups them (conv2d.cc:231-316); taps outside the image are zeros.
struct ColumnLoader {
    const float* x;
    long long xnb[4];   // elements, ggml order (w, h, c, n)
    int iw, ih, ow, oh, kw, taps;
    int s0, s1, p0, p1, d0, d1;
    __device__ __forceinline__ float operator()(long long row, long long kk) const {
        const long long img = row / (static_cast<long long>(oh) * ow);
        const int pos = static_cast<int>(row - img * oh * ow);
        const int y0 = pos / ow, x0 = pos - y0 * ow;
        const int c = static_cast<int>(kk / taps);
        const int tap = static_cast<int>(kk - static_cast<long long>(c) * taps);
        const int ky = tap / kw, kx = tap - ky * kw;
        const int y = y0 * s1 + ky * d1 - p1, xx = x0 * s0 + kx * d0 - p0;
        if (y < 0 || y >= ih || xx < 0 || xx >= iw) return 0.0f;
        return __ldg(x + img * xnb[3] + c * xnb[2] + y * xnb[1] + xx * xnb[0]);
    }
};

// The bytes of row r, k-bytes k0.. of a lane: one store when they are a
// naturally aligned run of 1, 2, 4 or 8 (they then stay in one 16-byte
// chunk), else byte by byte.
template <int EPL>
__device__ __forceinline__ void store_quant_bytes(uint8_t* q, long long tm, int nstages, int r, long long k0,
                                                  uint64_t bytes) {
    if (EPL == 1 || EPL == 2 || EPL == 4 || EPL == 8) {
        uint8_t* dst = q + (tm * nstages + (k0 >> 6)) * 8192 + quant_tile_offset(r, static_cast<int>(k0 & 63));
        if (EPL == 8) *reinterpret_cast<uint64_t*>(dst) = bytes;
        else if (EPL == 4) *reinterpret_cast<uint32_t*>(dst) = static_cast<uint32_t>(bytes);
        else if (EPL == 2) *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(bytes);
        else *dst = static_cast<uint8_t>(bytes);
    } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const long long kk = k0 + e;
            q[(tm * nstages + (kk >> 6)) * 8192 + quant_tile_offset(r, static_cast<int>(kk & 63))] =
                static_cast<uint8_t>(bytes >> (8 * e));
        }
    }
}

// post multiplies each group's scale and offset after they are made (the
// scale of attention's softmax, folded into the queries' as the reference
// folds it, attention.cc:748-757); 1 elsewhere, which changes nothing.
// One warp's group of a row: v[EPL] a lane (numbers at k0 + e >= k are past
// the row's end), quantized and stored with the group's scale and offset.
template <int EPL>
__device__ __forceinline__ void quantize_group(const float (&v)[EPL], long long k0, long long k, int levels, float post,
                                               long long row, int g, int groups, int nstages, uint8_t* q,
                                               float* scales, int lane) {
    float lo = 0.0f, hi = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        lo = fminf(lo, v[e]);
        hi = fmaxf(hi, v[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    const float top = static_cast<float>(levels);
    const float s = __fdiv_rn(__fsub_rn(hi, lo), top);
    const float inverse = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
    const float zero = rintf(__fmul_rn(-lo, inverse));
    uint64_t bytes = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const float qv = k0 + e < k ? fminf(fmaxf(__fadd_rn(rintf(__fmul_rn(v[e], inverse)), zero), 0.0f), top)
                                    : zero;
        bytes |= static_cast<uint64_t>(static_cast<uint8_t>(qv)) << (8 * e);
    }
    const long long tm = row >> 7;
    const int r = static_cast<int>(row & 127);
    store_quant_bytes<EPL>(q, tm, nstages, r, k0, bytes);
    if (lane == 0) {
        float* sc = scales + (tm * groups + g) * 256;
        sc[r] = __fmul_rn(s, post);
        sc[128 + r] = __fmul_rn(__fmul_rn(s, zero), post);
    }
}

template <int EPL, class Loader>
__global__ void quantize_inputs_kernel(Loader load, long long m, long long k, int group, int groups,
                                       int nstages, int levels, float post, uint8_t* __restrict__ q,
                                       float* __restrict__ scales) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const long long total = m * groups;
    for (long long w = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
         w += warps) {
        const long long row = w / groups;
        const int g = static_cast<int>(w - row * groups);
        const long long k0 = static_cast<long long>(g) * group + lane * EPL;
        float v[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = k0 + e < k ? load(row, k0 + e) : 0.0f;
        quantize_group<EPL>(v, k0, k, levels, post, row, g, groups, nstages, q, scales, lane);
    }
}

// Quantizes m rows of k numbers from `load` into the GEMM's tiles, groups of
// `group` numbers (32 to 256, a multiple of 32).
template <class Loader>
void launch_quantize(const Loader& load, long long m, long long k, int group, int groups, int nstages, int levels,
                     uint8_t* q, float* scales, cudaStream_t st, float post = 1.0f) {
    const long long warps = m * groups;
    const int blocks = static_cast<int>(std::min<long long>((warps + 7) / 8, 148LL * 16));
#define SDB_QUANTIZE(E) quantize_inputs_kernel<E><<<blocks, 256, 0, st>>>(load, m, k, group, groups, nstages, levels, \
                                                                          post, q, scales)
    switch (group / 32) {
        case 1: SDB_QUANTIZE(1); break;
        case 2: SDB_QUANTIZE(2); break;
        case 3: SDB_QUANTIZE(3); break;
        case 4: SDB_QUANTIZE(4); break;
        case 5: SDB_QUANTIZE(5); break;
        default: SDB_QUANTIZE(8); break;
    }
#undef SDB_QUANTIZE
    count_launch();
}

// F(2x2)'s transformed inputs quantized: one warp a (tile, group of input
// channels), EPL channels a lane.  Each channel's 4 x 4 inputs are read once
// and all sixteen B^T d B made from them as the reference packs them
// (winograd.cc:440-500, 640-665): the tile's rows by row s of B^T (bt(),
// winograd.cc:321-333) first, then combined by row r, xi = 4 r + s; then each
// xi's group quantized as row xi * tiles_pad + tile.  Tiles past the last are
// zeros.
template <int EPL>
__global__ void wino2_quantize_kernel(const Wino2QuantLoader a, int ic, int group, int groups, int nstages, int levels,
                                      uint8_t* __restrict__ q, float* __restrict__ scales) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const long long total = a.tiles_pad * groups;
    for (long long w = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
         w += warps) {
        const long long t = w / groups;
        const int g = static_cast<int>(w - t * groups);
        const long long k0 = static_cast<long long>(g) * group + lane * EPL;
        float v[16][EPL];
        const bool live = t < a.tiles;
        const int tx = live ? static_cast<int>(t % a.tw) : 0;
        const long long rest = live ? t / a.tw : 0;
        const int ty = static_cast<int>(rest % a.th);
        const long long img = rest / a.th;
        const int y0 = 2 * ty - a.p1, x0 = 2 * tx - a.p0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const long long c = k0 + e;
            float d[4][4];
            const float* plane = a.x + img * a.xnb[3] + c * a.xnb[2];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int y = y0 + i, xx = x0 + j;
                    d[i][j] = (live && c < ic && y >= 0 && y < a.ih && xx >= 0 && xx < a.iw)
                                  ? __ldg(plane + y * a.xnb[1] + xx * a.xnb[0])
                                  : 0.0f;
                }
            float tr[4][4];  // tr[i][s]: row i by row s of B^T
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                tr[i][0] = __fsub_rn(d[i][0], d[i][2]);
                tr[i][1] = __fadd_rn(d[i][1], d[i][2]);
                tr[i][2] = __fsub_rn(d[i][2], d[i][1]);
                tr[i][3] = __fsub_rn(d[i][1], d[i][3]);
            }
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
                v[0 * 4 + s4][e] = __fsub_rn(tr[0][s4], tr[2][s4]);
                v[1 * 4 + s4][e] = __fadd_rn(tr[1][s4], tr[2][s4]);
                v[2 * 4 + s4][e] = __fsub_rn(tr[2][s4], tr[1][s4]);
                v[3 * 4 + s4][e] = __fsub_rn(tr[1][s4], tr[3][s4]);
            }
        }
#pragma unroll
        for (int x = 0; x < 16; ++x)
            quantize_group<EPL>(v[x], k0, ic, levels, 1.0f, x * a.tiles_pad + t, g, groups, nstages, q, scales, lane);
    }
}

// Attention's queries (b, h, query), each head's rows padded to lq_pad (a
// multiple of 128): row (b H + h) lq_pad + i, number kk of the head's d.
struct QueryLoader {
    const float* q;
    long long qnb[4];   // elements, ggml order (d, query, head, image)
    int h, lq;
    long long lq_pad;
    __device__ __forceinline__ float operator()(long long row, long long kk) const {
        const long long bh = row / lq_pad;
        const long long i = row - bh * lq_pad;
        if (i >= lq) return 0.0f;
        const long long b = bh / h, hh = bh - b * h;
        return __ldg(q + b * qnb[3] + hh * qnb[2] + i * qnb[1] + kk * qnb[0]);
    }
};

// A query's exponentials of its scores less its greatest (attention.cc:287-301,
// 767-800): the keys before `tail0` by the reference's exponential (its
// vector kernel's, eight keys at a time), those after by the C library's exp;
// summed in double, the reciprocal of the sum rounded once (838-841); and
// quantized, unsigned, in groups of keys.  One warp a row: the row's greatest
// score first, then each group's exponentials made once, summed and
// quantized.
template <int EPL>
__global__ void softmax_quantize_kernel(const float* __restrict__ s, long long rows, long long lds, int lk, int tail0,
                                        int group, int groups, int nstages, int levels, uint8_t* __restrict__ q,
                                        float* __restrict__ scales, float* __restrict__ rec) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    for (long long row = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows;
         row += warps) {
        const float* sr = s + row * lds;
        float mx = -INFINITY;
        if ((lds & 3) == 0) {
            const int l4 = lk >> 2;
            for (int j = lane; j < l4; j += 32) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(sr) + j);
                mx = fmaxf(fmaxf(mx, t.x), fmaxf(t.y, fmaxf(t.z, t.w)));
            }
            for (int j = 4 * l4 + lane; j < lk; j += 32) mx = fmaxf(mx, __ldg(sr + j));
        } else {
            for (int j = lane; j < lk; j += 32) mx = fmaxf(mx, __ldg(sr + j));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        double sum = 0.0;
        for (int g = 0; g < groups; ++g) {
            const long long k0 = static_cast<long long>(g) * group + lane * EPL;
            float v[EPL];
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
                const long long j = k0 + e;
                if (j < lk) {
                    const float x = __fsub_rn(__ldg(sr + j), mx);
                    v[e] = j >= tail0 ? expf(x) : exponential(x);
                    sum += static_cast<double>(v[e]);
                } else {
                    v[e] = 0.0f;
                }
            }
            quantize_group<EPL>(v, k0, lk, levels, 1.0f, row, g, groups, nstages, q, scales, lane);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) rec[row] = static_cast<float>(1.0 / sum);
    }
}

// out[b, h, i, c] = o[row][c] * rec[row] (attention.cc:838-844), then the chain
// (an extension: the reference's quantized attention has none), the element at
// ggml coordinates (c, h, i, b).
__global__ void attention_finish_kernel(const float* __restrict__ o, long long ldo, const float* __restrict__ rec,
                                        long long lq_pad, int lq, int h, int b, int dv, float* __restrict__ out,
                                        long long onb0, long long onb1, long long onb2, long long onb3,
                                        const Chain chain) {
    const long long total = static_cast<long long>(b) * h * lq * dv;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(idx % dv);
        long long rest = idx / dv;
        const int i = static_cast<int>(rest % lq);
        rest /= lq;
        const int hh = static_cast<int>(rest % h);
        const int bb = static_cast<int>(rest / h);
        const long long row = (static_cast<long long>(bb) * h + hh) * lq_pad + i;
        float v = __fmul_rn(__ldg(o + row * ldo + c), __ldg(rec + row));
        v = apply_chain(chain, v, c, hh, i, bb);
        out[c * onb0 + hh * onb1 + i * onb2 + bb * onb3] = v;
    }
}

template <bool GATED>
int launch_qgemm(const CUtensorMap& ymap, QGemmArgs a, cudaStream_t st) {
    auto kern = qgemm_kernel<GATED>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kQSmemBytes));
    const int grid = std::min(a.items, current_sm_count());
    kern<<<grid, kQThreads, kQSmemBytes, st>>>(ymap, a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // namespace

// The rows and the tuning's quantization as the reference reads them
// (quant.cc:54-66): quantized when bits is 2..8 and `quantize` has the linear
// layers' bit, for 256 rows or more.
bool quantized_linear(int64_t rows) {
    const Tuning& t = tuning();
    return t.bits >= 2 && t.bits <= 8 && (t.quantize & 1) != 0 && rows >= 256;
}

QuantSpec current_quant() {
    const Tuning& t = tuning();
    QuantSpec q;
    q.group = static_cast<int>(t.group);
    q.wmax = (1 << (std::clamp<int64_t>(t.bits, 2, 8) - 1)) - 1;
    q.weight_groups = t.weight_group != 0;
    return q;
}

int run_quantized_linear(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                         cudaStream_t st, bool gated) {
    const int64_t k = w->ne[0];
    const int64_t n = gated ? w->ne[1] / 2 : w->ne[1];
    const int64_t m = x->ne[1] * x->ne[2] * x->ne[3];
    const QuantSpec spec = current_quant();
    const int levels = (1 << std::clamp<int64_t>(tuning().input_bits, 2, 8)) - 1;
    if (gated && chain && chain->from_redirect)
        return fail(SDB_NOT_SUPPORTED, "quantized gated product: no residual in place");
    std::shared_ptr<Packed> p;
    if (int s = quantized_weights(w, gated, gated ? 2 * n : n, k, gated ? n : 0, spec, st, &p); s != SDB_OK)
        return s;
    const int groups = p->groups;
    const int cpg = spec.group / 32;
    const int nstages = (groups * cpg + 1) / 2;
    const int64_t tiles_m = (m + kQRows - 1) / kQRows;
    const size_t q_bytes = static_cast<size_t>(tiles_m * nstages * kQABytes);
    const size_t s_bytes = static_cast<size_t>(tiles_m * groups * 1024);
    void* ws = nullptr;
    if (int s = workspace(st, q_bytes + s_bytes, &ws); s != SDB_OK) return s;
    uint8_t* qa = static_cast<uint8_t*>(ws);
    float* sa = reinterpret_cast<float*>(qa + q_bytes);

    launch_quantize(RowLoader{static_cast<const float*>(x->data), k}, m, k, spec.group, groups, nstages, levels, qa,
                    sa, st);
    SDB_CUDA(cudaGetLastError());

    QGemmArgs a{};
    a.a = qa;
    a.as = sa;
    a.w = static_cast<const uint8_t*>(p->data);
    a.ws = static_cast<const float*>(p->qscales);
    a.m = static_cast<int>(m);
    a.n = static_cast<int>(n);
    a.groups = groups;
    a.cpg = cpg;
    a.kchunks = groups * a.cpg;
    a.tiles_m = static_cast<int>(tiles_m);
    a.tiles_n = static_cast<int>(gated ? (n + 63) / 64 : (n + 127) / 128);
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "quantized product: too many tiles");
    a.items = static_cast<int>(items);
    a.magic = static_cast<long long>(spec.group) * levels * spec.wmax < (1LL << 22) ? 1 : 0;
    a.y = static_cast<float*>(chain && chain->redirect ? chain->redirect : dst->data);
    for (int d = 0; d < 4; ++d) a.ynb[d] = dst->nb[d] / 4;
    a.rne1 = dst->ne[1];
    a.rne2 = dst->ne[2];
    a.chain = make_chain(chain);
    a.err = device_error_word();
    // The output by TMA stores when its rows are 16-byte aligned runs.
    CUtensorMap ymap{};
    a.store = kStoreDirect;
    if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ynb[0] == 1 && a.ynb[1] == n &&
        store_map(&ymap, a.y, n, m, n, 16))
        a.store = kStoreTma;
    if (p->tiles != a.tiles_n) return fail(SDB_INVALID, "quantized weights: tile count mismatch");
    return gated ? launch_qgemm<true>(ymap, a, st) : launch_qgemm<false>(ymap, a, st);
}

// The quantized convolution (conv2d.cc:338-470): the kernel as a (K, OC)
// matrix of K = (ic, kh, kw) rows quantized by the store, the columns of
// every output position quantized straight from the image, and the product
// by qgemm_kernel with the positions as its rows and the output channels as
// its columns.  The reference folds a stretch of K at a time into the output,
// each stretch a whole number of groups, starting each from the last one's
// FP32 result: the same fold, group after group, as one pass over all of K.
bool quantized_conv() {
    const Tuning& t = tuning();
    return t.bits >= 2 && t.bits <= 8 && (t.quantize & 2) != 0;
}

int run_quantized_conv(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                       const sdb_chain* chain, cudaStream_t st) {
    const int64_t kw = w->ne[0], kh = w->ne[1], ic = w->ne[2], oc = w->ne[3];
    const int64_t taps = kw * kh, k = taps * ic;
    const int64_t es = w->type == SDB_TYPE_F16 ? 2 : 4;
    if (w->nb[0] != es || w->nb[1] != es * kw || w->nb[2] != es * taps)
        return fail(SDB_NOT_SUPPORTED, "quantized convolution: each output channel's kernel must be contiguous");
    const int64_t ow = dst->ne[0], oh = dst->ne[1], n = dst->ne[3];
    const int64_t m = n * oh * ow;
    if (m >= (1LL << 31) - kQRows || k >= (1LL << 31) || taps >= (1LL << 24))
        return fail(SDB_NOT_SUPPORTED, "quantized convolution: too large");
    const QuantSpec spec = current_quant();
    const int levels = (1 << std::clamp<int64_t>(tuning().input_bits, 2, 8)) - 1;
    sdb_tensor wk = *w;
    wk.ne[0] = k;
    wk.ne[1] = oc;
    wk.ne[2] = wk.ne[3] = 1;
    wk.nb[0] = es;
    wk.nb[1] = w->nb[3];
    wk.nb[2] = wk.nb[3] = w->nb[3] * oc;
    std::shared_ptr<Packed> p;
    if (int s = quantized_weights(&wk, false, oc, k, 0, spec, st, &p); s != SDB_OK) return s;
    const int groups = p->groups;
    const int cpg = spec.group / 32;
    const int nstages = (groups * cpg + 1) / 2;
    const int64_t tiles_m = (m + kQRows - 1) / kQRows;
    const size_t q_bytes = static_cast<size_t>(tiles_m * nstages * kQABytes);
    const size_t s_bytes = static_cast<size_t>(tiles_m * groups * 1024);
    void* ws = nullptr;
    if (int s = workspace(st, q_bytes + s_bytes, &ws); s != SDB_OK) return s;
    uint8_t* qa = static_cast<uint8_t*>(ws);
    float* sa = reinterpret_cast<float*>(qa + q_bytes);

    ColumnLoader load{};
    load.x = static_cast<const float*>(x->data);
    for (int d = 0; d < 4; ++d) load.xnb[d] = x->nb[d] / 4;
    load.iw = static_cast<int>(x->ne[0]);
    load.ih = static_cast<int>(x->ne[1]);
    load.ow = static_cast<int>(ow);
    load.oh = static_cast<int>(oh);
    load.kw = static_cast<int>(kw);
    load.taps = static_cast<int>(taps);
    load.s0 = params[0];
    load.s1 = params[1];
    load.p0 = params[2];
    load.p1 = params[3];
    load.d0 = params[4];
    load.d1 = params[5];
    launch_quantize(load, m, k, spec.group, groups, nstages, levels, qa, sa, st);
    SDB_CUDA(cudaGetLastError());

    QGemmArgs a{};
    a.a = qa;
    a.as = sa;
    a.w = static_cast<const uint8_t*>(p->data);
    a.ws = static_cast<const float*>(p->qscales);
    a.m = static_cast<int>(m);
    a.n = static_cast<int>(oc);
    a.groups = groups;
    a.cpg = cpg;
    a.kchunks = groups * cpg;
    a.tiles_m = static_cast<int>(tiles_m);
    a.tiles_n = static_cast<int>((oc + 127) / 128);
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "quantized convolution: too many tiles");
    a.items = static_cast<int>(items);
    a.magic = static_cast<long long>(spec.group) * levels * spec.wmax < (1LL << 22) ? 1 : 0;
    a.y = static_cast<float*>(chain && chain->redirect ? chain->redirect : dst->data);
    // The product's columns are the output channels (ggml dimension 2), its
    // rows the positions (ow fastest, then oh, then the image).
    a.ynb[0] = dst->nb[2] / 4;
    a.ynb[1] = dst->nb[0] / 4;
    a.ynb[2] = dst->nb[1] / 4;
    a.ynb[3] = dst->nb[3] / 4;
    a.rne1 = ow;
    a.rne2 = oh;
    a.chain = make_chain(chain);
    for (int s = 0; s < a.chain.count; ++s) {
        const long long nb[4] = {a.chain.nb[s][2], a.chain.nb[s][0], a.chain.nb[s][1], a.chain.nb[s][3]};
        for (int d = 0; d < 4; ++d) a.chain.nb[s][d] = nb[d];
    }
    a.err = device_error_word();
    CUtensorMap ymap{};
    a.store = kStoreDirect;
    if (oc % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ynb[0] == 1 && a.ynb[1] == oc &&
        a.ynb[2] == ow * oc && a.ynb[3] == oh * ow * oc && store_map(&ymap, a.y, oc, m, oc, 16))
        a.store = kStoreTma;
    if (p->tiles != a.tiles_n) return fail(SDB_INVALID, "quantized weights: tile count mismatch");
    return launch_qgemm<false>(ymap, a, st);
}

// Whether the reference computes a quantized convolution by Winograd's
// F(2x2, 3x3) (winograd.cc:2107-2123, 2237-2244): 3x3 kernels at stride 1,
// dilation 1 and padding 0..2 with tuning winograd != 0, for images of at
// least winograd_positions outputs or of at most winograd_small_tiles tiles
// in all.  Quantized, F(4x4) is never taken.
bool quantized_winograd(const sdb_tensor* w, const sdb_tensor* dst, const int32_t params[6]) {
    const Tuning& t = tuning();
    if (t.winograd == 0 || w->ne[0] != 3 || w->ne[1] != 3) return false;
    if (params[0] != 1 || params[1] != 1 || params[4] != 1 || params[5] != 1) return false;
    if (params[2] < 0 || params[2] > 2 || params[3] < 0 || params[3] > 2) return false;
    const int64_t tiles = dst->ne[3] * ((dst->ne[0] + 1) / 2) * ((dst->ne[1] + 1) / 2);
    return dst->ne[0] * dst->ne[1] >= t.winograd_positions || tiles <= t.winograd_small_tiles;
}

// F(2x2, 3x3) quantized (winograd.cc:1826-2100): the transformed kernels
// quantized by the store; the transformed inputs of every tile made and
// quantized in one pass (wino2_quantize_kernel), rows xi * tiles_pad + tile; the
// sixteen products as one batched qgemm into M [16][tiles_pad][ldm]; then
// Y = A^T M A and the chain (winograd_outputs_kernel).  The reference folds a
// stretch of input channels at a time into its FP32 products, each a whole
// number of groups: the same fold, group after group, as one pass.
int run_quantized_winograd(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                           const sdb_chain* chain, cudaStream_t st) {
    constexpr int xi = 16;
    const Tuning& t = tuning();
    const QuantSpec spec = current_quant();
    const int levels = (1 << std::clamp<int64_t>(t.input_bits, 2, 8)) - 1;
    const int64_t ic = w->ne[2], oc = w->ne[3];
    WinoArgs wa{};
    wa.x = static_cast<const float*>(x->data);
    for (int d = 0; d < 4; ++d) wa.xnb[d] = x->nb[d] / 4;
    wa.iw = static_cast<int>(x->ne[0]);
    wa.ih = static_cast<int>(x->ne[1]);
    wa.ic = static_cast<int>(ic);
    wa.n = static_cast<int>(x->ne[3]);
    wa.ow = static_cast<int>(dst->ne[0]);
    wa.oh = static_cast<int>(dst->ne[1]);
    wa.oc = static_cast<int>(oc);
    wa.p0 = params[2];
    wa.p1 = params[3];
    wa.tw = (wa.ow + 1) / 2;
    wa.th = (wa.oh + 1) / 2;
    wa.tiles = static_cast<long long>(wa.n) * wa.th * wa.tw;
    wa.tiles_pad = (wa.tiles + kQRows - 1) / kQRows * kQRows;
    wa.ldm = (oc + 3) / 4 * 4;
    const long long m = xi * wa.tiles_pad;
    if (m >= (1LL << 31) - kQRows || m * wa.ldm >= (1LL << 40))
        return fail(SDB_NOT_SUPPORTED, "quantized Winograd: too many tiles");
    // Per-row scales span the reference's stretch of input channels: of its
    // plan for few tiles (winograd.cc:238-246) or for many (248-268), a whole
    // number of groups.
    const bool small = wa.tiles <= t.winograd_small_tiles;
    const int64_t base_kc = small ? std::min<int64_t>(ic, std::max<int64_t>(8, t.winograd_small_kc))
                                  : std::min<int64_t>(ic, t.winograd_kc);
    const int64_t span = std::max<int64_t>(spec.group, base_kc / spec.group * spec.group);
    std::shared_ptr<Packed> p;
    if (int s = quantized_winograd_weights(w, spec, span, st, &p); s != SDB_OK) return s;
    const int groups = p->groups;
    const int cpg = spec.group / 32;
    const int nstages = (groups * cpg + 1) / 2;
    const int64_t tiles_m = m / kQRows;
    const size_t q_bytes = static_cast<size_t>(tiles_m * nstages * kQABytes);
    const size_t s_bytes = static_cast<size_t>(tiles_m * groups * 1024);
    const size_t m_bytes = static_cast<size_t>(m * wa.ldm * 4);
    void* ws = nullptr;
    if (int s = workspace(st, q_bytes + s_bytes + m_bytes, &ws); s != SDB_OK) return s;
    uint8_t* qa = static_cast<uint8_t*>(ws);
    float* sa = reinterpret_cast<float*>(qa + q_bytes);
    float* mbuf = reinterpret_cast<float*>(qa + q_bytes + s_bytes);

    Wino2QuantLoader load{};
    load.x = wa.x;
    for (int d = 0; d < 4; ++d) load.xnb[d] = wa.xnb[d];
    load.iw = wa.iw;
    load.ih = wa.ih;
    load.p0 = wa.p0;
    load.p1 = wa.p1;
    load.tw = wa.tw;
    load.th = wa.th;
    load.tiles = wa.tiles;
    load.tiles_pad = wa.tiles_pad;
    {
        const long long warps = wa.tiles_pad * groups;
        const int blocks = static_cast<int>(std::min<long long>((warps + 7) / 8, 148LL * 16));
#define SDB_WINO_Q(E) wino2_quantize_kernel<E><<<blocks, 256, 0, st>>>(load, static_cast<int>(ic), spec.group, groups, \
                                                                       nstages, levels, qa, sa)
        switch (spec.group / 32) {
            case 1: SDB_WINO_Q(1); break;
            case 2: SDB_WINO_Q(2); break;
            case 4: SDB_WINO_Q(4); break;
            default: SDB_WINO_Q(8); break;
        }
#undef SDB_WINO_Q
        count_launch();
    }
    SDB_CUDA(cudaGetLastError());

    QGemmArgs a{};
    a.a = qa;
    a.as = sa;
    a.w = static_cast<const uint8_t*>(p->data);
    a.ws = static_cast<const float*>(p->qscales);
    a.m = static_cast<int>(m);
    a.n = static_cast<int>(oc);
    a.groups = groups;
    a.cpg = cpg;
    a.kchunks = groups * cpg;
    a.tiles_m = static_cast<int>(tiles_m);
    a.tiles_n = p->tiles;
    a.batch_tiles = static_cast<int>(wa.tiles_pad / kQRows);
    a.batch_rep = 1;
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "quantized Winograd: too many tiles");
    a.items = static_cast<int>(items);
    a.magic = static_cast<long long>(spec.group) * levels * spec.wmax < (1LL << 22) ? 1 : 0;
    a.y = mbuf;
    a.ynb[0] = 1;
    a.ynb[1] = wa.ldm;
    a.ynb[2] = a.ynb[3] = wa.ldm * m;
    a.rne1 = m;
    a.rne2 = 1;
    a.err = device_error_word();
    CUtensorMap ymap{};
    a.store = kStoreDirect;
    if (store_map(&ymap, mbuf, oc, m, wa.ldm, 16)) a.store = kStoreTma;
    if (int s = launch_qgemm<false>(ymap, a, st); s != SDB_OK) return s;

    wa.m = mbuf;
    wa.y = static_cast<float*>(chain && chain->redirect ? chain->redirect : dst->data);
    for (int d = 0; d < 4; ++d) wa.ynb[d] = dst->nb[d] / 4;
    wa.chain = make_chain(chain);
    wa.err = a.err;
    const bool out_pairs = wa.ynb[2] == 1 && wa.oc % 2 == 0 && (reinterpret_cast<uintptr_t>(wa.y) & 7) == 0 &&
                           wa.ynb[0] % 2 == 0 && wa.ynb[1] % 2 == 0 && wa.ynb[3] % 2 == 0;
    const long long out_total = wa.tiles * wa.oc / (out_pairs ? 2 : 1);
    const int out_blocks = static_cast<int>(std::min<long long>((out_total + 255) / 256, 148LL * 32));
    if (out_pairs) winograd_outputs_kernel<2, 2><<<out_blocks, 256, 0, st>>>(wa);
    else winograd_outputs_kernel<2, 1><<<out_blocks, 256, 0, st>>>(wa);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

// Self-attention over 256 keys or more with integer products
// (attention.cc:596-860): quantized when bits is 2..8 and `quantize` has
// attention's bit.
bool quantized_attention(int64_t lk) {
    const Tuning& t = tuning();
    return t.bits >= 2 && t.bits <= 8 && (t.quantize & 4) != 0 && lk >= 256;
}

// Attention with integer products, as the reference computes it
// (attention.cc:596-844):
//   * keys signed, a scale each over the head's d dimensions; queries
//     unsigned with a zero point, likewise, the softmax's scale multiplied
//     into their scales and offsets;
//   * the scores, a fold of one group, into S [rows][lds] FP32 -- rows
//     (image, head, query), each head's queries padded to a multiple of 128;
//   * each query's greatest score, its exponentials quantized unsigned in
//     groups of keys and the reciprocal of their sum (softmax_quantize_kernel,
//     one pass over the exponentials); the values signed, a scale each dimension
//     per group of keys; their fold into O [rows][ldo];
//   * out = O * reciprocal, and the chain (attention_finish_kernel).
// A group covering d dimensions is laid out as round_up(d, 32) bytes: the
// queries' missing numbers are their zero point and the keys' zeros, which
// add nothing to the integer sums or the keys' offsets.
int run_quantized_attention(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, const sdb_tensor* dst,
                            float scale, const sdb_chain* chain, cudaStream_t st) {
    const Tuning& t = tuning();
    const QuantSpec spec = current_quant();
    const int levels = (1 << std::clamp<int64_t>(t.input_bits, 2, 8)) - 1;
    const int64_t d = q->ne[0], lq = q->ne[1], h = q->ne[2], b = q->ne[3];
    const int64_t lk = k->ne[1], hk = k->ne[2], dv = v->ne[0];
    const int gd = static_cast<int>((d + 31) / 32 * 32);     // the group over d, as laid out
    const int gk = spec.group;                               // the groups over keys
    if (gd > 256) return fail(SDB_NOT_SUPPORTED, "quantized attention: heads of more than 256 dimensions");
    const int64_t lq_pad = (lq + kQRows - 1) / kQRows * kQRows;
    const int64_t rows = b * h * lq_pad;
    const int64_t tiles_m = rows / kQRows;
    const int64_t lk_tiles = (lk + 127) / 128, dv_tiles = (dv + 127) / 128;
    const int64_t kgroups = (lk + gk - 1) / gk;
    const int st_d = (gd / 32 + 1) / 2;                       // stages of one group over d
    const int st_k = static_cast<int>((kgroups * (gk / 32) + 1) / 2);
    const int64_t lds = (lk + 3) / 4 * 4, ldo = (dv + 3) / 4 * 4;
    if (rows >= (1LL << 31) - kQRows || tiles_m * std::max(lk_tiles, dv_tiles) >= (1LL << 31))
        return fail(SDB_NOT_SUPPORTED, "quantized attention: too large");
    // Workspace, 256-byte aligned parts.
    auto part = [](int64_t bytes) { return static_cast<size_t>((bytes + 255) / 256 * 256); };
    const size_t b_qq = part(tiles_m * st_d * kQABytes), b_qs = part(tiles_m * 1024);
    const size_t b_kq = part(b * hk * lk_tiles * st_d * kQBBytes), b_ks = part(b * hk * lk_tiles * 1024);
    const size_t b_s = part(rows * lds * 4), b_rec = part(rows * 4);
    const size_t b_pq = part(tiles_m * st_k * kQABytes), b_ps = part(tiles_m * kgroups * 1024);
    const size_t b_vq = part(b * hk * dv_tiles * st_k * kQBBytes), b_vs = part(b * hk * dv_tiles * kgroups * 1024);
    const size_t b_o = part(rows * ldo * 4);
    void* ws = nullptr;
    if (int s = workspace(st, b_qq + b_qs + b_kq + b_ks + b_s + b_rec + b_pq + b_ps + b_vq + b_vs + b_o, &ws);
        s != SDB_OK)
        return s;
    uint8_t* at = static_cast<uint8_t*>(ws);
    auto take = [&](size_t bytes) { uint8_t* r = at; at += bytes; return r; };
    uint8_t* qq = take(b_qq);
    float* qs = reinterpret_cast<float*>(take(b_qs));
    int8_t* kq = reinterpret_cast<int8_t*>(take(b_kq));
    float* ks = reinterpret_cast<float*>(take(b_ks));
    float* sbuf = reinterpret_cast<float*>(take(b_s));
    float* rec = reinterpret_cast<float*>(take(b_rec));
    uint8_t* pq = take(b_pq);
    float* ps = reinterpret_cast<float*>(take(b_ps));
    int8_t* vq = reinterpret_cast<int8_t*>(take(b_vq));
    float* vs = reinterpret_cast<float*>(take(b_vs));
    float* obuf = reinterpret_cast<float*>(take(b_o));
    // The keys' tiles and the values' are written whole only where rows and k
    // reach; the rest must be zeros.
    SDB_CUDA(cudaMemsetAsync(kq, 0, b_kq, st));
    SDB_CUDA(cudaMemsetAsync(vq, 0, b_vq, st));

    // Queries.
    QueryLoader ql{};
    ql.q = static_cast<const float*>(q->data);
    for (int i = 0; i < 4; ++i) ql.qnb[i] = q->nb[i] / 4;
    ql.h = static_cast<int>(h);
    ql.lq = static_cast<int>(lq);
    ql.lq_pad = lq_pad;
    launch_quantize(ql, rows, d, gd, 1, st_d, levels, qq, qs, st, scale);
    SDB_CUDA(cudaGetLastError());

    // Keys: (image, key head) matrices of lk rows of d.
    QPackArgs ka{};
    ka.src = static_cast<const uint8_t*>(k->data);
    ka.type = k->type;
    ka.nb0 = k->nb[0];
    ka.nb1 = k->nb[1];
    ka.n = lk;
    ka.k = d;
    ka.rows = b * hk * lk_tiles * 128;
    ka.group = gd;
    ka.groups = 1;
    ka.nstages = st_d;
    ka.wmax = spec.wmax;
    ka.weight_groups = 1;
    ka.span = gd;
    ka.batches = static_cast<int>(b * hk);
    ka.bdiv = static_cast<int>(hk);
    ka.bnb_hi = k->nb[3];
    ka.bnb_lo = k->nb[2];
    ka.q = kq;
    ka.scales = ks;
    launch_quantize_weights(ka, st);
    SDB_CUDA(cudaGetLastError());

    // Scores.
    QGemmArgs a{};
    a.a = qq;
    a.as = qs;
    a.w = reinterpret_cast<const uint8_t*>(kq);
    a.ws = ks;
    a.m = static_cast<int>(rows);
    a.n = static_cast<int>(lk);
    a.groups = 1;
    a.cpg = gd / 32;
    a.kchunks = a.cpg;
    a.tiles_m = static_cast<int>(tiles_m);
    a.tiles_n = static_cast<int>(lk_tiles);
    a.batch_tiles = static_cast<int>(lq_pad / kQRows);
    a.batch_rep = static_cast<int>(h / hk);
    a.items = static_cast<int>(tiles_m * lk_tiles);
    a.magic = d * levels * spec.wmax < (1LL << 22) ? 1 : 0;
    a.y = sbuf;
    a.ynb[0] = 1;
    a.ynb[1] = lds;
    a.ynb[2] = a.ynb[3] = lds * rows;
    a.rne1 = rows;
    a.rne2 = 1;
    a.err = device_error_word();
    CUtensorMap smap{};
    a.store = store_map(&smap, sbuf, lk, rows, lds, 16) ? kStoreTma : kStoreDirect;
    if (int s = launch_qgemm<false>(smap, a, st); s != SDB_OK) return s;

    // The softmax and its quantized exponentials.  The reference's vector
    // kernel takes the keys of each stretch eight at a time and the C
    // library's exp the rest: with stretches of a multiple of eight keys, the
    // last lk % 8 keys.
    const int tail0 = static_cast<int>(lk - lk % 8);
    const int sblocks = static_cast<int>(std::min<long long>((rows + 7) / 8, 148LL * 16));
#define SDB_SOFTMAX_Q(E) softmax_quantize_kernel<E><<<sblocks, 256, 0, st>>>(sbuf, rows, lds, static_cast<int>(lk), \
        tail0, gk, static_cast<int>(kgroups), st_k, levels, pq, ps, rec)
    switch (gk / 32) {
        case 1: SDB_SOFTMAX_Q(1); break;
        case 2: SDB_SOFTMAX_Q(2); break;
        case 4: SDB_SOFTMAX_Q(4); break;
        default: SDB_SOFTMAX_Q(8); break;
    }
#undef SDB_SOFTMAX_Q
    count_launch();
    SDB_CUDA(cudaGetLastError());

    // Values: (image, key head) matrices of dv rows (dimensions) of lk keys.
    QPackArgs va{};
    va.src = static_cast<const uint8_t*>(v->data);
    va.type = v->type;
    va.nb0 = v->nb[1];
    va.nb1 = v->nb[0];
    va.n = dv;
    va.k = lk;
    va.rows = b * hk * dv_tiles * 128;
    va.group = gk;
    va.groups = static_cast<int>(kgroups);
    va.nstages = st_k;
    va.wmax = spec.wmax;
    va.weight_groups = 1;
    va.span = kgroups * gk;
    va.batches = static_cast<int>(b * hk);
    va.bdiv = static_cast<int>(hk);
    va.bnb_hi = v->nb[3];
    va.bnb_lo = v->nb[2];
    va.q = vq;
    va.scales = vs;
    launch_quantize_weights(va, st);
    SDB_CUDA(cudaGetLastError());

    // The values by the exponentials.
    QGemmArgs o{};
    o.a = pq;
    o.as = ps;
    o.w = reinterpret_cast<const uint8_t*>(vq);
    o.ws = vs;
    o.m = static_cast<int>(rows);
    o.n = static_cast<int>(dv);
    o.groups = static_cast<int>(kgroups);
    o.cpg = gk / 32;
    o.kchunks = o.groups * o.cpg;
    o.tiles_m = static_cast<int>(tiles_m);
    o.tiles_n = static_cast<int>(dv_tiles);
    o.batch_tiles = static_cast<int>(lq_pad / kQRows);
    o.batch_rep = static_cast<int>(h / hk);
    o.items = static_cast<int>(tiles_m * dv_tiles);
    o.magic = static_cast<long long>(gk) * levels * spec.wmax < (1LL << 22) ? 1 : 0;
    o.y = obuf;
    o.ynb[0] = 1;
    o.ynb[1] = ldo;
    o.ynb[2] = o.ynb[3] = ldo * rows;
    o.rne1 = rows;
    o.rne2 = 1;
    o.err = a.err;
    CUtensorMap omap{};
    o.store = store_map(&omap, obuf, dv, rows, ldo, 16) ? kStoreTma : kStoreDirect;
    if (int s = launch_qgemm<false>(omap, o, st); s != SDB_OK) return s;

    const long long total = b * h * lq * dv;
    const int fblocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
    attention_finish_kernel<<<fblocks, 256, 0, st>>>(obuf, ldo, rec, lq_pad, static_cast<int>(lq), static_cast<int>(h),
                                                     static_cast<int>(b), static_cast<int>(dv),
                                                     static_cast<float*>(dst->data), dst->nb[0] / 4, dst->nb[1] / 4,
                                                     dst->nb[2] / 4, dst->nb[3] / 4, make_chain(chain));
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // namespace sdb
