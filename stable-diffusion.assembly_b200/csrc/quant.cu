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
// scales[((tm * groups + g) * 2 + {0, 1}) * 128 + r].
template <int EPL>
__global__ void quantize_inputs_kernel(const float* __restrict__ x, long long m, long long k, int group, int groups,
                                       int nstages, int levels, uint8_t* __restrict__ q,
                                       float* __restrict__ scales) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const long long total = m * groups;
    for (long long w = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
         w += warps) {
        const long long row = w / groups;
        const int g = static_cast<int>(w - row * groups);
        const long long k0 = static_cast<long long>(g) * group + lane * EPL;
        const float* src = x + row * k;
        float v[EPL];
        float lo = 0.0f, hi = 0.0f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            v[e] = k0 + e < k ? __ldg(src + k0 + e) : 0.0f;
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
        uint8_t* dst = q + (tm * nstages + (k0 >> 6)) * 8192 + quant_tile_offset(r, static_cast<int>(k0 & 63));
        if (EPL == 8) *reinterpret_cast<uint64_t*>(dst) = bytes;
        else if (EPL == 4) *reinterpret_cast<uint32_t*>(dst) = static_cast<uint32_t>(bytes);
        else if (EPL == 2) *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(bytes);
        else *dst = static_cast<uint8_t>(bytes);
        if (lane == 0) {
            float* sc = scales + (tm * groups + g) * 256;
            sc[r] = s;
            sc[128 + r] = __fmul_rn(s, zero);
        }
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

    const long long warps = m * groups;
    const int blocks = static_cast<int>(std::min<long long>((warps + 7) / 8, 148LL * 16));
    const float* xs = static_cast<const float*>(x->data);
    switch (cpg) {
        case 1: quantize_inputs_kernel<1><<<blocks, 256, 0, st>>>(xs, m, k, spec.group, groups, nstages, levels, qa, sa); break;
        case 2: quantize_inputs_kernel<2><<<blocks, 256, 0, st>>>(xs, m, k, spec.group, groups, nstages, levels, qa, sa); break;
        case 4: quantize_inputs_kernel<4><<<blocks, 256, 0, st>>>(xs, m, k, spec.group, groups, nstages, levels, qa, sa); break;
        default: quantize_inputs_kernel<8><<<blocks, 256, 0, st>>>(xs, m, k, spec.group, groups, nstages, levels, qa, sa); break;
    }
    count_launch();
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

}  // namespace sdb
