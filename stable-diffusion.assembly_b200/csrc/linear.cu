// Entry points of the GEMM-backed operations: MUL_MAT (with and without the
// gated GELU) and the direct convolution.  Each splits its activation once
// into the workspace (split.cuh), takes the packed weights from the store
// (store.cuh) and runs the TMA-fed tcgen05 GEMM (gemm.cuh), with K split over
// several CTAs when the output has too few tiles to fill the GPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "../../include/sdb.h"
#include "gemm.cuh"
#include "gemm_fused.cuh"
#include "gemm_wide.cuh"
#include "quant.cuh"
#include "runtime.cuh"
#include "split.cuh"
#include "store.cuh"
#include "winograd.cuh"

namespace sdb {

namespace {

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// The partial sums' map: [ksplit * tiles_m * 128 rows][part_ld] FP32, stored in 32 x 32 boxes.
int partial_map(const GemmArgs& a, CUtensorMap* map) {
    const uint64_t dims[2] = {static_cast<uint64_t>(a.part_ld),
                              static_cast<uint64_t>(a.ksplit) * static_cast<uint64_t>(a.tiles_m) * kBM};
    const uint64_t strides[1] = {static_cast<uint64_t>(a.part_ld) * 4};
    const uint32_t box[2] = {32, 32};
    if (encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.part, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the partial sums");
    return SDB_OK;
}

// The split-K reduction: four columns a thread where the output's columns
// are contiguous and aligned, else one.
template <int MODE>
int launch_reduce(const GemmArgs& a, cudaStream_t st) {
    const bool cols = MODE == kModeLinear ? a.ynb[0] == 1 && a.ynb[1] % 4 == 0
                                          : a.ynb[2] == 1 && a.ynb[0] % 4 == 0 && a.ynb[1] % 4 == 0;
    const bool vec = cols && a.n % 4 == 0 && a.part_ld % 4 == 0 && a.ynb[3] % 4 == 0 &&
                     (MODE != kModeLinear || a.ynb[2] % 4 == 0) && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
    const long long total = static_cast<long long>(a.tiles_m) * kBM * a.n / (vec ? 4 : 1);
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    if (vec) splitk_reduce4_kernel<MODE><<<blocks, 256, 0, st>>>(a, a.tiles_m);
    else splitk_reduce_kernel<MODE><<<blocks, 256, 0, st>>>(a, a.tiles_m);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

template <int MODE, int WMODE>
int launch_gemm(const CUtensorMap& amap, const CUtensorMap& wmap, const CUtensorMap& ymap, GemmArgs a,
                cudaStream_t st) {
    using S = GemmShape<WMODE>;
    auto kern = gemm_split_kernel<MODE, WMODE>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes));
    a.tiles_n = (a.n + S::BN - 1) / S::BN;
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n * a.ksplit;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "gemm: too many tiles");
    a.items = static_cast<int>(items);
    const int grid = static_cast<int>(std::min<long long>(items, current_sm_count()));
    CUtensorMap pmap;
    if (a.ksplit > 1)
        if (int s = partial_map(a, &pmap); s != SDB_OK) return s;
    kern<<<grid, kGemmThreads, S::kSmemBytes, st>>>(amap, wmap, a.ksplit > 1 ? pmap : ymap, a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    if (a.ksplit > 1) return launch_reduce<MODE>(a, st);
    return SDB_OK;
}

template <int MODE>
int dispatch(const CUtensorMap& amap, const Packed& p, int wmode, const CUtensorMap& ymap, const GemmArgs& a,
             cudaStream_t st) {
    if (wmode == kWeightGated) return launch_gemm<MODE, kWeightGated>(amap, p.map64, ymap, a, st);
    return wmode == kWeightSplit ? launch_gemm<MODE, kWeightSplit>(amap, p.map128, ymap, a, st)
                                 : launch_gemm<MODE, kWeightHalf>(amap, p.map128, ymap, a, st);
}

// K is split when the output tiles leave most SMs idle: enough parts to fill
// the GPU once, at least 8 k-blocks each, none empty.
void choose_ksplit(GemmArgs& a, int tiles, int wmode) {
    a.ksplit = 1;
    a.per_split = a.kblocks;
    if (wmode == kWeightGated) return;
    const int sms = current_sm_count();
    if (tiles >= sms / 2 || a.kblocks < 16) return;
    const int want = std::max(1, std::min((sms + tiles - 1) / tiles, a.kblocks / 8));
    a.per_split = (a.kblocks + want - 1) / want;
    a.ksplit = (a.kblocks + a.per_split - 1) / a.per_split;
}

// The wide kernel's plan for an M x N x K product (gated: N of the output, 2N
// of the product): the tile width and the K split that minimise
//   waves x (k-blocks of an item) x (a k-block's shared-memory bytes)
// + the split's partial sums (written and read back by the reduction),
// where waves = ceil(items / SMs) -- a wave with fewer items than SMs costs
// as much as a full one.  A k-block moves 2 (A + B) for the MMA operand
// reads of the hi and lo products plus A (both planes) + B for the TMA
// writes; B = BN x 128 bytes.  Returns the width (0: run the 128-wide
// kernel) and sets ksplit / per_split.
int plan_wide(GemmArgs& a, int64_t n, int tiles_m, int64_t m, bool gated) {
    const int64_t forced = tuning().block_n;
    a.ksplit = 1;
    a.per_split = a.kblocks;
    if (forced == 128 && !gated) return 0;
    const int64_t cols = gated ? 2 * n : n;
    const int sms = current_sm_count();
    int best_bn = 0, best_split = 1;
    double best_cost = 0.0;
    for (int bn : {256, 192, 128}) {
        if (gated && bn == 192) continue;
        if (forced == 256 && bn != 256) continue;
        const int64_t tiles = tiles_m * ((cols + bn - 1) / bn);
        const double kb_bytes = 2.0 * (16384 + bn * 128) + 32768 + bn * 128;
        const int max_split = gated ? 1 : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(32, a.kblocks / 4)));
        for (int split = 1; split <= max_split; ++split) {
            const int per = (a.kblocks + split - 1) / split;
            const int parts = (a.kblocks + per - 1) / per;
            if (parts != split) continue;
            const int64_t items = tiles * parts;
            const int64_t waves = (items + sms - 1) / sms;
            double cost = static_cast<double>(waves) * per * kb_bytes;
            // The reduction: partial sums written, read back, the output written -- over all SMs,
            // about 48 bytes a clock each, in the units of one SM's shared-memory bytes above.
            if (parts > 1) cost += (2.0 * parts + 1.0) * static_cast<double>(m) * n * 4 / sms / 48.0 * 128.0;
            if (best_bn == 0 || cost < best_cost * 0.98) {
                best_bn = bn;
                best_split = parts;
                best_cost = cost;
            }
        }
    }
    a.per_split = (a.kblocks + best_split - 1) / best_split;
    a.ksplit = best_split;
    return best_bn;
}

template <int MODE, bool GATED, int BN>
int launch_wide_bn(const CUtensorMap& amap, const CUtensorMap& wmap, const CUtensorMap& ymap, GemmArgs a,
                   cudaStream_t st) {
    using S = WideShape<BN>;
    auto kern = gemm_wide_kernel<MODE, GATED, BN>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes));
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n * a.ksplit;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "gemm: too many tiles");
    a.items = static_cast<int>(items);
    const int grid = static_cast<int>(std::min<long long>(items, current_sm_count()));
    CUtensorMap pmap;
    if (a.ksplit > 1) {
        const long long rows = static_cast<long long>(a.ksplit) * a.tiles_m * kBM;
        if (!store_map(&pmap, a.part, a.part_ld, rows, a.part_ld, 16))
            return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the partial sums");
    }
    kern<<<grid, kWideThreads, S::kSmemBytes, st>>>(amap, wmap, a.ksplit > 1 ? pmap : ymap, a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    if (a.ksplit > 1) return launch_reduce<MODE>(a, st);
    return SDB_OK;
}

template <int MODE>
int launch_wide(const CUtensorMap& amap, const Packed& p, bool gated, int bn, const CUtensorMap& ymap,
                const GemmArgs& a, cudaStream_t st) {
    if (gated)
        return bn == 256 ? launch_wide_bn<MODE, true, 256>(amap, p.map128, ymap, a, st)
                         : launch_wide_bn<MODE, true, 128>(amap, p.map64, ymap, a, st);
    if (bn == 256) return launch_wide_bn<MODE, false, 256>(amap, p.map256, ymap, a, st);
    if (bn == 192) return launch_wide_bn<MODE, false, 192>(amap, p.map192, ymap, a, st);
    return launch_wide_bn<MODE, false, 128>(amap, p.map128, ymap, a, st);
}

// Bytes of split-K partial sums: [ksplit][tiles * 128][npad].
size_t partial_bytes(int ksplit, int tiles, int64_t n, int bn) {
    if (ksplit <= 1) return 0;
    return static_cast<size_t>(ksplit) * tiles * kBM * round_up(n, bn) * 4;
}

void set_partials(GemmArgs& a, void* ws, size_t offset, int tiles, int bn) {
    if (a.ksplit <= 1) return;
    const long long ld = round_up(a.n, bn);
    a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + offset);
    a.part_ld = ld;
    a.part_split = static_cast<long long>(tiles) * kBM * ld;
}

bool is_type(const sdb_tensor* t, int type) { return t != nullptr && t->type == type && t->data != nullptr; }

bool contiguous_f32(const sdb_tensor* t) {
    if (!is_type(t, SDB_TYPE_F32)) return false;
    int64_t expect = 4;
    for (int d = 0; d < 4; ++d) {
        if (t->ne[d] <= 0) return false;
        if (t->ne[d] > 1 && t->nb[d] != expect) return false;
        expect *= t->ne[d];
    }
    return true;
}

// A channels-last (NHWC) image described in ggml order [W, H, C, N]: channels
// contiguous, then positions, rows, images.
bool channels_last(const sdb_tensor* t) {
    const int64_t c = t->ne[2], w = t->ne[0], h = t->ne[1];
    return t->nb[2] == 4 && t->nb[0] == 4 * c && t->nb[1] == 4 * c * w && t->nb[3] == 4 * c * w * h;
}

bool valid_chain(const sdb_chain* c) {
    if (c == nullptr) return true;
    if (c->count < 0 || c->count > SDB_MAX_STEPS) return false;
    for (int s = 0; s < c->count; ++s) {
        const int k = c->steps[s].kind;
        if (k != SDB_STEP_ADD && k != SDB_STEP_MUL && k != SDB_STEP_SILU) return false;
        if (k != SDB_STEP_SILU && c->steps[s].operand == nullptr) return false;
    }
    if (c->from_redirect) {
        if (c->redirect == nullptr) return false;
        for (int s = 0; s < c->count; ++s)
            if (c->steps[s].kind != SDB_STEP_ADD) return false;
    }
    return true;
}

void set_out(GemmArgs& a, const sdb_tensor* dst, const sdb_chain* chain) {
    a.y = static_cast<float*>(chain && chain->redirect ? chain->redirect : dst->data);
    for (int d = 0; d < 4; ++d) a.ynb[d] = dst->nb[d] / 4;
    a.chain = make_chain(chain);
    a.err = device_error_word();
}

bool mul_mat_shapes(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst) {
    if (w == nullptr || x == nullptr || dst == nullptr) return false;
    if (!(is_type(w, SDB_TYPE_F16) || is_type(w, SDB_TYPE_F32))) return false;
    const int64_t es = w->type == SDB_TYPE_F16 ? 2 : 4;
    if (w->ne[2] != 1 || w->ne[3] != 1 || w->nb[0] != es || w->ne[0] <= 0 || w->ne[1] <= 0) return false;
    if (!contiguous_f32(x) || !contiguous_f32(dst)) return false;
    if (x->ne[0] != w->ne[0]) return false;
    return true;
}

// ---- the fused-split linear GEMM (gemm_fused.cuh)

// GroupNorm prologue for the fused path: the rows of x (an image's positions,
// channels along the row) normalised into `out`, the same values the split
// pre-pass reads through chain.cuh gn_in.  Four channels a thread.
__global__ void gn_rows_kernel(const float* __restrict__ x, long long rows, int k, float* __restrict__ out,
                               GnIn gn) {
    const int q4 = k / 4;
    const long long total = rows * q4;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = idx / q4;
        const int c0 = static_cast<int>(idx - r * q4) * 4;
        const long long img = r / gn.positions;
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + r * k + c0));
        float4 o;
        o.x = gn_in(gn, v.x, gn_coef(gn, c0, img));
        o.y = gn_in(gn, v.y, gn_coef(gn, c0 + 1, img));
        o.z = gn_in(gn, v.z, gn_coef(gn, c0 + 2, img));
        o.w = gn_in(gn, v.w, gn_coef(gn, c0 + 3, img));
        *reinterpret_cast<float4*>(out + r * k + c0) = o;
    }
}

// The fused kernel's plan: the tile width (the product's columns a tile: 128,
// 160 or 192) and the K split that minimise
//   waves x (k-blocks of an item x a k-block's cost + an item's epilogue),
// a k-block costing its operand bytes from L2 (x 32 KB, W 128 BN bytes) at
// ~48 bytes a clock an SM, plus the split's partial sums.  Gated products are
// not split.
int plan_fused(GemmArgs& a, int64_t n, int tiles_m, int64_t m, bool gated) {
    const int64_t cols = gated ? 2 * n : n;
    const int sms = current_sm_count();
    const int64_t forced = tuning().block_n;
    int best_bn = 0, best_split = 1;
    double best_cost = 0.0;
    for (int bn : {192, 160, 128}) {
        if ((forced == 128 || forced == 160 || forced == 192) && bn != forced) continue;
        const int64_t tiles = tiles_m * ((cols + bn - 1) / bn);
        const double kb_cost = (32768.0 + 128.0 * bn) / 48.0;
        const int max_split = gated ? 1 : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(32, a.kblocks / 4)));
        for (int split = 1; split <= max_split; ++split) {
            const int per = (a.kblocks + split - 1) / split;
            const int parts = (a.kblocks + per - 1) / per;
            if (parts != split) continue;
            const int64_t items = tiles * parts;
            const int64_t waves = (items + sms - 1) / sms;
            double cost = static_cast<double>(waves) * (per * kb_cost + 600.0);
            if (parts > 1) cost += (2.0 * parts + 1.0) * static_cast<double>(m) * n * 4 / sms / 48.0;
            if (best_bn == 0 || cost < best_cost * 0.98) {
                best_bn = bn;
                best_split = parts;
                best_cost = cost;
            }
        }
    }
    a.per_split = (a.kblocks + best_split - 1) / best_split;
    a.ksplit = best_split;
    return best_bn;
}

template <bool GATED, int BN>
int launch_fused_bn(const CUtensorMap& xmap, const CUtensorMap& wmap, const CUtensorMap& ymap, GemmArgs a,
                    cudaStream_t st) {
    using S = FusedShape<BN>;
    auto kern = gemm_fused_kernel<GATED, BN>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes));
    const long long items = static_cast<long long>(a.tiles_m) * a.tiles_n * a.ksplit;
    if (items >= (1LL << 31)) return fail(SDB_NOT_SUPPORTED, "gemm: too many tiles");
    a.items = static_cast<int>(items);
    const int grid = static_cast<int>(std::min<long long>(items, current_sm_count()));
    CUtensorMap pmap;
    if (a.ksplit > 1) {
        const long long rows = static_cast<long long>(a.ksplit) * a.tiles_m * kBM;
        if (!store_map(&pmap, a.part, a.part_ld, rows, a.part_ld, 16))
            return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the partial sums");
    }
    kern<<<grid, kFusedThreads, S::kSmemBytes, st>>>(xmap, wmap, a.ksplit > 1 ? pmap : ymap, a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    if (a.ksplit > 1) return launch_reduce<kModeLinear>(a, st);
    return SDB_OK;
}

int launch_fused(const CUtensorMap& xmap, const Packed& p, bool gated, int bn, const CUtensorMap& ymap,
                 const GemmArgs& a, cudaStream_t st) {
    if (gated) {
        if (bn == 192) return launch_fused_bn<true, 192>(xmap, p.map96, ymap, a, st);
        if (bn == 160) return launch_fused_bn<true, 160>(xmap, p.map80, ymap, a, st);
        return launch_fused_bn<true, 128>(xmap, p.map64, ymap, a, st);
    }
    if (bn == 192) return launch_fused_bn<false, 192>(xmap, p.map192, ymap, a, st);
    if (bn == 160) return launch_fused_bn<false, 160>(xmap, p.map160, ymap, a, st);
    return launch_fused_bn<false, 128>(xmap, p.map128, ymap, a, st);
}

// Whether the fused kernel takes x: FP32 rows of K % 4 == 0 (TMA's 16-byte
// row pitch), 16-byte aligned, at most 2^31 rows; with gemm_fused = 1 only
// where it measured faster than the split pre-pass (plain products: the gated
// ones keep the wide kernel's 256-column tiles), with 2 always.
bool fused_rows(const sdb_tensor* x, int64_t k, int64_t m, bool gated) {
    const int64_t mode = tuning().gemm_fused;
    if (mode == 0 || (mode == 1 && gated)) return false;
    return k % 4 == 0 && (reinterpret_cast<uintptr_t>(x->data) & 15) == 0 && m < (1LL << 31) && k < (1LL << 31);
}

// run_linear's body on the fused kernel: x (or, with a normalisation
// prologue, x normalised into the workspace by the same kernels as the
// separate GroupNorm / LayerNorm nodes) read as FP32 rows straight by TMA.
int run_linear_fused(std::shared_ptr<Packed> p, size_t w_bytes, bool transient, const sdb_tensor* w,
                     const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain, cudaStream_t st, bool gated,
                     const GnIn* gn, const LnIn* ln, int64_t m, int64_t n, int64_t k) {
    const int tiles = static_cast<int>((m + kBM - 1) / kBM);
    GemmArgs a{};
    a.m = static_cast<int>(m);
    a.kblocks = static_cast<int>(p->kpad / kBK);
    a.n = static_cast<int>(n);
    a.b1_row = static_cast<int>(p->b1_row);
    a.tiles_m = tiles;
    a.rne1 = dst->ne[1];
    a.rne2 = dst->ne[2];
    set_out(a, dst, chain);
    const int bn = plan_fused(a, n, tiles, m, gated);

    // Workspace: a transient operand's packing, the normalised x (with a prologue), partial sums.
    const size_t xn_bytes = (gn || ln) ? static_cast<size_t>(round_up(m * k * 4, 256)) : 0;
    void* ws0 = nullptr;
    if (int s = workspace(st, w_bytes + xn_bytes + partial_bytes(a.ksplit, tiles, gated ? 2 * n : n, bn), &ws0);
        s != SDB_OK)
        return s;
    if (transient)
        if (int s = pack_transient(w, n, k, ws0, st, p.get()); s != SDB_OK) return s;
    uint8_t* ws = static_cast<uint8_t*>(ws0) + w_bytes;
    set_partials(a, ws, xn_bytes, tiles, bn);
    const float* xrows = static_cast<const float*>(x->data);
    if (ln) {
        sdb_tensor xn = *x;
        xn.data = ws;
        if (int s = sdb_norm(x, &xn, ln->eps, ln->chain, st); s != SDB_OK) return s;
        xrows = reinterpret_cast<const float*>(ws);
    } else if (gn) {
        const long long total = m * (k / 4);
        const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
        gn_rows_kernel<<<blocks, 256, 0, st>>>(xrows, m, static_cast<int>(k), reinterpret_cast<float*>(ws), *gn);
        count_launch();
        SDB_CUDA(cudaGetLastError());
        xrows = reinterpret_cast<const float*>(ws);
    }
    CUtensorMap xmap;
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k) * 4};
    const uint32_t box[2] = {32, 128};
    if (encode_tensor_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(xrows), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the activation rows");
    CUtensorMap ymap{};
    a.store = kStoreDirect;
    if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ynb[0] == 1 && a.ynb[1] == n &&
        store_map(&ymap, a.y, n, m, n, 16))
        a.store = kStoreTma;
    a.tiles_n = static_cast<int>(((gated ? 2 * n : n) + bn - 1) / bn);
    return launch_fused(xmap, *p, gated, bn, ymap, a, st);
}

// transient: w is packed into the workspace on every call instead of being
// kept by the store (an operand the graph writes between calls).
int run_linear(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
               cudaStream_t st, bool gated, bool transient = false, const GnIn* gn = nullptr,
               const LnIn* ln = nullptr) {
    const int64_t k = w->ne[0];
    const int64_t n = gated ? w->ne[1] / 2 : w->ne[1];
    const int64_t m = x->ne[1] * x->ne[2] * x->ne[3];
    if (m > (1LL << 30) || k > (1 << 24)) return fail(SDB_NOT_SUPPORTED, "mul_mat: too large");
    if (!transient && quantized_linear(m)) {
        if (gn || ln) return fail(SDB_NOT_SUPPORTED, "mul_mat: no normalisation prologue on integer products");
        return run_quantized_linear(w, x, dst, chain, st, gated);
    }
    std::shared_ptr<Packed> p;
    size_t w_bytes = 0;
    if (transient) {
        // The fields the plan reads; pack_transient fills the same ones once the workspace is known.
        p = std::make_shared<Packed>();
        p->borrowed = true;
        p->split = w->type == SDB_TYPE_F32;
        p->kpad = round_up(std::max<int64_t>(k, 1), 64);
        p->npad = round_up(n, kRowPad);
        p->b1_row = p->split ? p->npad : 0;
        w_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(transient_bytes(w, n, k)), 256));
    } else {
        const int rc = gated ? packed_weights(w, Layout::gated, 2 * n, k, 0, n, st, &p)
                             : packed_weights(w, Layout::linear, n, k, 0, 0, st, &p);
        if (rc != SDB_OK) return rc;
    }
    const int wmode = gated ? kWeightGated : p->split ? kWeightSplit : kWeightHalf;
    const int tiles = static_cast<int>((m + kBM - 1) / kBM);
    if (wmode != kWeightSplit && fused_rows(x, k, m, gated))
        return run_linear_fused(p, w_bytes, transient, w, x, dst, chain, st, gated, gn, ln, m, n, k);
    const int kblocks = static_cast<int>(p->kpad / kBK);

    GemmArgs a{};
    a.m = static_cast<int>(m);
    a.kblocks = static_cast<int>(p->kpad / kBK);
    a.n = static_cast<int>(n);
    a.b1_row = static_cast<int>(p->b1_row);
    a.a_tx = kBM * kBK * 2;
    a.a_planes = 2;
    a.tiles_m = tiles;
    a.rne1 = dst->ne[1];
    a.rne2 = dst->ne[2];
    set_out(a, dst, chain);
    // FP16 weights take the wide kernel (tile width and K split by plan_wide); FP32 weights the 128-wide one.
    a.kblocks = kblocks;
    const int wide_bn = wmode == kWeightSplit ? 0 : plan_wide(a, n, tiles, m, gated);
    const int bn = wide_bn ? (gated ? wide_bn / 2 : wide_bn) : (wmode == kWeightGated ? 64 : 128);
    if (!wide_bn) choose_ksplit(a, tiles * static_cast<int>((n + bn - 1) / bn), wmode);

    // Workspace: a transient operand's packing, the split rows [0, M) hi, [M, 2M) lo of kp8
    // FP16, then any partial sums.
    const int64_t kp8 = round_up(k, 8);
    const size_t a_bytes = static_cast<size_t>(round_up(2 * m * kp8 * 2, 256));
    void* ws0 = nullptr;
    if (int s = workspace(st, w_bytes + a_bytes + partial_bytes(a.ksplit, tiles, n, bn), &ws0); s != SDB_OK)
        return s;
    if (transient)
        if (int s = pack_transient(w, n, k, ws0, st, p.get()); s != SDB_OK) return s;
    void* ws = static_cast<uint8_t*>(ws0) + w_bytes;
    set_partials(a, ws, a_bytes, tiles, bn);
    const long long ne[4] = {x->ne[0], x->ne[1], x->ne[2], x->ne[3]};
    const long long nb[4] = {x->nb[0] / 4, x->nb[1] / 4, x->nb[2] / 4, x->nb[3] / 4};
    if (ln) {
        if (int s = layer_norm_split(x, ln->eps, ln->chain, kp8, static_cast<uint16_t*>(ws), a.err, st); s != SDB_OK)
            return s;
    } else if (int s = split_rows(static_cast<const float*>(x->data), ne, nb, kp8, static_cast<uint16_t*>(ws), a.err,
                                  st, gn);
               s != SDB_OK) {
        return s;
    }
    // A as [plane][row][k]: one box {64, 128, 2} brings a tile's hi and lo rows.
    CUtensorMap amap;
    const uint64_t dims[3] = {static_cast<uint64_t>(kp8), static_cast<uint64_t>(m), 2};
    const uint64_t strides[2] = {static_cast<uint64_t>(kp8) * 2, static_cast<uint64_t>(m * kp8) * 2};
    const uint32_t box[3] = {64, 128, 2};
    if (encode_tensor_map(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ws, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the activations");
    // The output by TMA stores when its rows are 16-byte aligned runs.
    CUtensorMap ymap{};
    a.store = kStoreDirect;
    if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 && a.ynb[0] == 1 && a.ynb[1] == n &&
        store_map(&ymap, a.y, n, m, n, wide_bn ? 16 : 32))
        a.store = kStoreTma;
    if (wide_bn) {
        a.tiles_n = static_cast<int>((n + bn - 1) / bn);
        return launch_wide<kModeLinear>(amap, *p, gated, wide_bn, ymap, a, st);
    }
    return dispatch<kModeLinear>(amap, *p, wmode, ymap, a, st);
}

// The output positions of a conv tile: OWt x OHt x NT <= 128 with the box's
// extents within TMA's 256 elements a dimension (with the stride as the
// element stride, a box spans OWt * s0 elements).
bool conv_tiles(ConvGeom& g) {
    g.owt = std::min(g.ow, 128);
    if (g.owt * g.s0 > 256) g.owt = 256 / g.s0;
    g.oht = std::max(1, std::min(g.oh, 128 / g.owt));
    if (g.oht * g.s1 > 256) g.oht = 256 / g.s1;
    g.nt = std::max(1, std::min(g.n, 128 / (g.owt * g.oht)));
    g.tw = (g.ow + g.owt - 1) / g.owt;
    g.th = (g.oh + g.oht - 1) / g.oht;
    g.tn = (g.n + g.nt - 1) / g.nt;
    return g.owt >= 1 && g.oht >= 1 && static_cast<long long>(g.tw) * g.th * g.tn < (1LL << 31);
}

// The form a convolution is computed in, by the reference's rule
// (winograd.cc:2107-2123, 1204-1206): Winograd for 3x3 kernels at stride 1,
// dilation 1 and padding 0..2 with tuning winograd != 0 and at least
// winograd_positions outputs an image; F(4x4, 3x3) with winograd = 2 for FP16
// kernels of at least winograd4_positions outputs an image, else F(2x2, 3x3).
// Two rules of this build's own: Winograd for at least winograd_channels
// input channels (fewer fill a fraction of the GEMM's 64-channel k-block),
// and F(4x4) for 16 input channels and more -- a sum of fewer channels does
// not average the split's rounding down, and F(4x4)'s output transform
// (coefficients up to 64) would carry it past 1e-6 of the magnitudes.
// Returns 0 (direct), 2 or 4.
int winograd_form(const sdb_tensor* w, const sdb_tensor* dst, const int32_t params[6]) {
    const Tuning& t = tuning();
    if (t.winograd == 0 || w->ne[0] != 3 || w->ne[1] != 3) return 0;
    if (params[0] != 1 || params[1] != 1 || params[4] != 1 || params[5] != 1) return 0;
    if (params[2] < 0 || params[2] > 2 || params[3] < 0 || params[3] > 2) return 0;
    const int64_t positions = dst->ne[0] * dst->ne[1];
    if (positions < t.winograd_positions || w->ne[2] < t.winograd_channels) return 0;
    return t.winograd == 2 && w->type == SDB_TYPE_F16 && positions >= t.winograd4_positions && w->ne[2] >= 16 ? 4
                                                                                                           : 2;
}

// Winograd's F(f x f, 3x3) (winograd.cuh): the inputs' transform into the
// workspace, the XI products as one batched launch of the split GEMM (three
// FP16 products of the split transforms), the outputs' transform with the
// chain.  Workspace: V [2][XI][Tp][icp8] FP16, M [XI][Tp][ldm] FP32, then any
// split-K partial sums.
int run_winograd(int f, const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                 const sdb_chain* chain, cudaStream_t st, const GnIn* gn = nullptr) {
    std::shared_ptr<Packed> p;
    if (int s = winograd_weights(w, f, st, &p); s != SDB_OK) return s;
    const int xi = f == 2 ? Wino<2>::kXi : Wino<4>::kXi;
    WinoArgs wa{};
    wa.x = static_cast<const float*>(x->data);
    for (int d = 0; d < 4; ++d) wa.xnb[d] = x->nb[d] / 4;
    wa.iw = static_cast<int>(x->ne[0]);
    wa.ih = static_cast<int>(x->ne[1]);
    wa.ic = static_cast<int>(x->ne[2]);
    wa.n = static_cast<int>(x->ne[3]);
    wa.ow = static_cast<int>(dst->ne[0]);
    wa.oh = static_cast<int>(dst->ne[1]);
    wa.oc = static_cast<int>(dst->ne[2]);
    wa.p0 = params[2];
    wa.p1 = params[3];
    wa.tw = (wa.ow + f - 1) / f;
    wa.th = (wa.oh + f - 1) / f;
    wa.tiles = static_cast<long long>(wa.n) * wa.th * wa.tw;
    wa.tiles_pad = round_up(wa.tiles, kBM);
    wa.icp8 = static_cast<int>(round_up(wa.ic, 8));
    wa.ldm = round_up(wa.oc, 4);
    if (wa.tiles_pad * xi >= (1LL << 30) || wa.tiles_pad * wa.icp8 >= (1LL << 31) ||
        wa.tiles_pad * wa.oc >= (1LL << 31))
        return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: too many Winograd tiles");

    GemmArgs a{};
    a.m = static_cast<int>(xi * wa.tiles_pad);
    a.kblocks = static_cast<int>(p->kpad / GemmShape<kWeightSplitK32>::kStageK);
    a.n = wa.oc;
    a.b1_row = static_cast<int>(p->b1_row);
    a.a_tx = GemmShape<kWeightSplitK32>::kABytes;
    a.a_planes = 2;
    a.tiles_m = a.m / kBM;
    a.batch_tiles = static_cast<int>(wa.tiles_pad / kBM);
    a.b_batch_rows = static_cast<int>(p->npad / xi);
    a.rne1 = a.m;
    a.rne2 = 1;
    a.ynb[0] = 1;
    a.ynb[1] = wa.ldm;
    a.ynb[2] = a.ynb[3] = wa.ldm * a.m;
    a.err = device_error_word();
    choose_ksplit(a, a.tiles_m * static_cast<int>((wa.oc + 127) / 128), kWeightSplit);

    const size_t v_bytes = static_cast<size_t>(round_up(2LL * xi * wa.tiles_pad * wa.icp8 * 2, 256));
    const size_t m_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(xi) * wa.tiles_pad * wa.ldm * 4, 256));
    void* ws = nullptr;
    if (int s = workspace(st, v_bytes + m_bytes + partial_bytes(a.ksplit, a.tiles_m, wa.oc, 128), &ws); s != SDB_OK)
        return s;
    wa.v = static_cast<__half*>(ws);
    float* mbuf = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + v_bytes);
    wa.m = mbuf;
    a.y = mbuf;
    set_partials(a, ws, v_bytes + m_bytes, a.tiles_m, 128);

    // Channel pairs as one load when the image's channels are adjacent (channels-last) and even in number.
    const bool in_pairs = wa.xnb[2] == 1 && wa.ic % 2 == 0 && (reinterpret_cast<uintptr_t>(wa.x) & 7) == 0 &&
                          wa.xnb[0] % 2 == 0 && wa.xnb[1] % 2 == 0 && wa.xnb[3] % 2 == 0;
    const long long in_total = wa.tiles_pad * wa.icp8 / (in_pairs ? 2 : 1);
    const int in_blocks = static_cast<int>(std::min<long long>((in_total + 255) / 256, 148LL * 32));
    if (gn) {
        wa.gn = *gn;
        if (f == 2) {
            if (in_pairs) winograd_inputs_kernel<2, 2, true><<<in_blocks, 256, 0, st>>>(wa);
            else winograd_inputs_kernel<2, 1, true><<<in_blocks, 256, 0, st>>>(wa);
        } else {
            if (in_pairs) winograd_inputs_kernel<4, 2, true><<<in_blocks, 256, 0, st>>>(wa);
            else winograd_inputs_kernel<4, 1, true><<<in_blocks, 256, 0, st>>>(wa);
        }
    } else if (f == 2) {
        if (in_pairs) winograd_inputs_kernel<2, 2><<<in_blocks, 256, 0, st>>>(wa);
        else winograd_inputs_kernel<2, 1><<<in_blocks, 256, 0, st>>>(wa);
    } else {
        if (in_pairs) winograd_inputs_kernel<4, 2><<<in_blocks, 256, 0, st>>>(wa);
        else winograd_inputs_kernel<4, 1><<<in_blocks, 256, 0, st>>>(wa);
    }
    count_launch();
    SDB_CUDA(cudaGetLastError());

    // A as [plane][xi * Tp rows][icp8]: one box {32, 128, 2} (64-byte swizzle) brings a
    // stage's hi and lo rows.
    CUtensorMap amap;
    const uint64_t dims[3] = {static_cast<uint64_t>(wa.icp8), static_cast<uint64_t>(a.m), 2};
    const uint64_t strides[2] = {static_cast<uint64_t>(wa.icp8) * 2, static_cast<uint64_t>(a.m) * wa.icp8 * 2};
    const uint32_t box[3] = {32, 128, 2};
    if (encode_tensor_map(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, wa.v, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_64B) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the transformed inputs");
    CUtensorMap ymap{};
    if (!store_map(&ymap, mbuf, wa.oc, a.m, wa.ldm, 32))
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the Winograd products");
    a.store = kStoreTma;
    if (int s = launch_gemm<kModeLinear, kWeightSplitK32>(amap, p->map128k32, ymap, a, st); s != SDB_OK) return s;

    wa.y = static_cast<float*>(chain && chain->redirect ? chain->redirect : dst->data);
    for (int d = 0; d < 4; ++d) wa.ynb[d] = dst->nb[d] / 4;
    wa.chain = make_chain(chain);
    wa.err = a.err;
    const bool out_pairs = wa.ynb[2] == 1 && wa.oc % 2 == 0 && (reinterpret_cast<uintptr_t>(wa.y) & 7) == 0 &&
                           wa.ynb[0] % 2 == 0 && wa.ynb[1] % 2 == 0 && wa.ynb[3] % 2 == 0;
    const long long out_total = wa.tiles * wa.oc / (out_pairs ? 2 : 1);
    const int out_blocks = static_cast<int>(std::min<long long>((out_total + 255) / 256, 148LL * 32));
    if (f == 2) {
        if (out_pairs) winograd_outputs_kernel<2, 2><<<out_blocks, 256, 0, st>>>(wa);
        else winograd_outputs_kernel<2, 1><<<out_blocks, 256, 0, st>>>(wa);
    } else {
        if (out_pairs) winograd_outputs_kernel<4, 2><<<out_blocks, 256, 0, st>>>(wa);
        else winograd_outputs_kernel<4, 1><<<out_blocks, 256, 0, st>>>(wa);
    }
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // namespace

}  // namespace sdb

using namespace sdb;

namespace sdb {
// sdb_conv2d's body, with an optional GroupNorm prologue on x (chain.cuh GnIn).
int conv2d_impl(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                const sdb_chain* chain, void* stream, const GnIn* gn);

// The prologue's parameters from the C ABI's sdb_norm_in, for an input of C channels and
// `positions` positions an image; SDB_OK or SDB_INVALID.
int make_gn_in(const sdb_norm_in* in, long long channels, long long positions, GnIn* out) {
    if (!in || !in->stats || in->groups <= 0 || channels % in->groups != 0 || positions <= 0 ||
        (in->gamma == nullptr) != (in->beta == nullptr))
        return fail(SDB_INVALID, "GroupNorm prologue: stats, groups dividing the channels, gamma with beta");
    out->stats = in->stats;
    out->gamma = in->gamma;
    out->beta = in->beta;
    out->groups = in->groups;
    out->cpg = static_cast<int>(channels / in->groups);
    out->silu = in->silu ? 1 : 0;
    out->positions = positions;
    return SDB_OK;
}
}  // namespace sdb

extern "C" {

int sdb_mul_mat_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst) {
    if (!mul_mat_shapes(w, x, dst)) return 0;
    return dst->ne[0] == w->ne[1] && dst->ne[1] == x->ne[1] && dst->ne[2] == x->ne[2] && dst->ne[3] == x->ne[3];
}

int sdb_mul_mat(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                void* stream) {
    if (!sdb_mul_mat_supported(w, x, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat: shapes not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_mul_mat: invalid chain");
    return run_linear(w, x, dst, chain, static_cast<cudaStream_t>(stream), false);
}

int sdb_mul_mat_transient(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                          void* stream) {
    if (!sdb_mul_mat_supported(w, x, dst))
        return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_transient: shapes not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_mul_mat_transient: invalid chain");
    return run_linear(w, x, dst, chain, static_cast<cudaStream_t>(stream), false, true);
}

int sdb_mul_mat_gated_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* out) {
    if (!mul_mat_shapes(w, x, out) || w->type != SDB_TYPE_F16 || w->ne[1] % 2 != 0) return 0;
    const int64_t half = w->ne[1] / 2;
    // Quantized, each half's columns begin a panel of 16 (mul_mat.cc:1130-1133).
    if (quantized_linear(x->ne[1] * x->ne[2] * x->ne[3]) && half % 16 != 0) return 0;
    return out->ne[0] == half && out->ne[1] == x->ne[1] && out->ne[2] == x->ne[2] && out->ne[3] == x->ne[3];
}

int sdb_mul_mat_gated(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* out, const sdb_chain* chain,
                      void* stream) {
    if (!sdb_mul_mat_gated_supported(w, x, out))
        return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_gated: shapes not supported");
    if (!valid_chain(chain) || (chain && (chain->redirect || chain->from_redirect)))
        return fail(SDB_INVALID, "sdb_mul_mat_gated: invalid chain");
    return run_linear(w, x, out, chain, static_cast<cudaStream_t>(stream), true);
}

int sdb_conv2d_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6]) {
    if (w == nullptr || x == nullptr || dst == nullptr || params == nullptr) return 0;
    if (!(is_type(w, SDB_TYPE_F16) || is_type(w, SDB_TYPE_F32)) || !is_type(x, SDB_TYPE_F32) ||
        !is_type(dst, SDB_TYPE_F32))
        return 0;
    const int s0 = params[0], s1 = params[1], p0 = params[2], p1 = params[3], d0 = params[4], d1 = params[5];
    if (s0 < 1 || s1 < 1 || d0 < 1 || d1 < 1 || p0 < 0 || p1 < 0 || s0 > 8 || s1 > 8) return 0;
    if (w->ne[2] != x->ne[2] || dst->ne[2] != w->ne[3] || dst->ne[3] != x->ne[3]) return 0;
    const int64_t ow = (x->ne[0] + 2 * p0 - d0 * (w->ne[0] - 1) - 1) / s0 + 1;
    const int64_t oh = (x->ne[1] + 2 * p1 - d1 * (w->ne[1] - 1) - 1) / s1 + 1;
    if (ow <= 0 || oh <= 0 || dst->ne[0] != ow || dst->ne[1] != oh) return 0;
    for (const sdb_tensor* t : {x, dst})
        for (int d = 0; d < 4; ++d)
            if (t->nb[d] % 4 != 0 || t->nb[d] < 0) return 0;
    const int64_t es = w->type == SDB_TYPE_F16 ? 2 : 4;
    for (int d = 0; d < 4; ++d)
        if (w->nb[d] % es != 0 || w->nb[d] < 0) return 0;
    // TMA coordinates are 32-bit and its images are at most 2^16 deep here.
    if (x->ne[0] > (1 << 24) || x->ne[1] > (1 << 24) || x->ne[2] > (1 << 20) || 2 * x->ne[3] > 65535) return 0;
    return w->ne[0] * w->ne[1] <= 64 * 64;
}

int sdb_conv2d(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
               const sdb_chain* chain, void* stream) {
    return conv2d_impl(w, x, dst, params, chain, stream, nullptr);
}

int sdb_conv2d_normed(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                      const sdb_norm_in* norm, const sdb_chain* chain, void* stream) {
    if (!sdb_conv2d_supported(w, x, dst, params)) return fail(SDB_NOT_SUPPORTED, "sdb_conv2d_normed: not supported");
    GnIn gn{};
    if (int s = make_gn_in(norm, x->ne[2], x->ne[0] * x->ne[1], &gn); s != SDB_OK) return s;
    return conv2d_impl(w, x, dst, params, chain, stream, &gn);
}

int sdb_mul_mat_layer_normed(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, float eps,
                             const sdb_chain* norm_chain, const sdb_chain* chain, void* stream) {
    if (!sdb_mul_mat_supported(w, x, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_layer_normed: not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_mul_mat_layer_normed: invalid chain");
    const LnIn ln{eps, norm_chain};
    return run_linear(w, x, dst, chain, static_cast<cudaStream_t>(stream), false, false, nullptr, &ln);
}

int sdb_mul_mat_gated_layer_normed(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* out, float eps,
                                   const sdb_chain* norm_chain, const sdb_chain* chain, void* stream) {
    if (!sdb_mul_mat_gated_supported(w, x, out))
        return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_gated_layer_normed: not supported");
    if (!valid_chain(chain) || (chain && (chain->redirect || chain->from_redirect)))
        return fail(SDB_INVALID, "sdb_mul_mat_gated_layer_normed: invalid chain");
    const LnIn ln{eps, norm_chain};
    return run_linear(w, x, out, chain, static_cast<cudaStream_t>(stream), true, false, nullptr, &ln);
}

int sdb_mul_mat_normed(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_norm_in* norm,
                       const sdb_chain* chain, void* stream) {
    if (!sdb_mul_mat_supported(w, x, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_normed: shapes not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_mul_mat_normed: invalid chain");
    GnIn gn{};
    if (int s = make_gn_in(norm, x->ne[0], x->ne[1], &gn); s != SDB_OK) return s;
    return run_linear(w, x, dst, chain, static_cast<cudaStream_t>(stream), false, false, &gn);
}

}  // extern "C"

namespace sdb {

int conv2d_impl(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                const sdb_chain* chain, void* stream, const GnIn* gn) {
    if (!sdb_conv2d_supported(w, x, dst, params)) return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_conv2d: invalid chain");
    const auto st = static_cast<cudaStream_t>(stream);
    if (quantized_conv()) {
        if (gn) return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: no GroupNorm prologue on integer products");
        // Integer products (conv2d.cc:843-844, winograd.cc:2237-2244): the reference's own choice of form.
        if (quantized_winograd(w, dst, params)) return run_quantized_winograd(w, x, dst, params, chain, st);
        return run_quantized_conv(w, x, dst, params, chain, st);
    }
    if (const int f = winograd_form(w, dst, params); f != 0) return run_winograd(f, w, x, dst, params, chain, st, gn);
    // A 1x1 convolution at stride 1 without padding, channels-last in and out, is a linear
    // layer over the image's positions (rows of IC channels in, rows of OC out, the same
    // memory): it takes the linear layers' path, whose GEMM splits the rows itself.  The
    // chain's operands are read in the output's (x, y, c, n) order; the linear view is
    // (c, x, y, n).
    const int64_t ic1 = x->ne[2], oc1 = w->ne[3];
    if (tuning().gemm_fused != 0 && w->type == SDB_TYPE_F16 && w->ne[0] == 1 && w->ne[1] == 1 && params[0] == 1 &&
        params[1] == 1 && params[2] == 0 && params[3] == 0 && w->nb[0] == 2 && w->nb[1] == 2 && w->nb[2] == 2 &&
        w->nb[3] == 2 * ic1 && channels_last(x) && channels_last(dst) && !(chain && chain->redirect)) {
        const int64_t W = x->ne[0], H = x->ne[1], N = x->ne[3];
        sdb_tensor wl = *w, xl = *x, dl = *dst;
        const int64_t wne[4] = {ic1, oc1, 1, 1}, wnb[4] = {2, 2 * ic1, 2 * ic1 * oc1, 2 * ic1 * oc1};
        const int64_t xne[4] = {ic1, W, H, N}, xnb[4] = {4, 4 * ic1, 4 * ic1 * W, 4 * ic1 * W * H};
        const int64_t dne[4] = {oc1, W, H, N}, dnb[4] = {4, 4 * oc1, 4 * oc1 * W, 4 * oc1 * W * H};
        for (int d = 0; d < 4; ++d) {
            wl.ne[d] = wne[d]; wl.nb[d] = wnb[d];
            xl.ne[d] = xne[d]; xl.nb[d] = xnb[d];
            dl.ne[d] = dne[d]; dl.nb[d] = dnb[d];
        }
        sdb_chain cl{};
        if (chain) {
            cl = *chain;
            for (int s = 0; s < cl.count; ++s) {
                const int64_t* nb = chain->steps[s].nb;
                const int64_t perm[4] = {nb[2], nb[0], nb[1], nb[3]};
                for (int d = 0; d < 4; ++d) cl.steps[s].nb[d] = perm[d];
            }
        }
        return run_linear(&wl, &xl, &dl, chain ? &cl : nullptr, st, false, false, gn);
    }
    if (gn && !channels_last(x))
        return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: a GroupNorm prologue needs a channels-last image");
    const int64_t ic = x->ne[2], oc = w->ne[3];
    const int icp = static_cast<int>(round_up(ic, 64));
    std::shared_ptr<Packed> p;
    if (int s = packed_weights(w, Layout::conv, oc, 0, icp, 0, st, &p); s != SDB_OK) return s;

    GemmArgs a{};
    ConvGeom& g = a.cg;
    g.ow = static_cast<int>(dst->ne[0]);
    g.oh = static_cast<int>(dst->ne[1]);
    g.n = static_cast<int>(x->ne[3]);
    g.kw = static_cast<int>(w->ne[0]);
    g.kh = static_cast<int>(w->ne[1]);
    g.s0 = params[0]; g.s1 = params[1]; g.p0 = params[2]; g.p1 = params[3]; g.d0 = params[4]; g.d1 = params[5];
    g.cblocks = icp / 64;
    if (!conv_tiles(g)) return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: tiling");
    const int tiles = g.tw * g.th * g.tn;
    const int wmode = p->split ? kWeightSplit : kWeightHalf;

    a.m = 0;
    a.kblocks = static_cast<int>(p->kpad / kBK);
    a.n = static_cast<int>(oc);
    a.b1_row = static_cast<int>(p->b1_row);
    a.a_tx = static_cast<uint32_t>(64 * 2 * g.owt * g.oht * g.nt);
    a.a_planes = g.owt * g.oht * g.nt == kBM ? 2 : 1;
    a.tiles_m = tiles;
    a.store = kStoreDirect;
    set_out(a, dst, chain);
    const int wide_bn =
        wmode == kWeightSplit ? 0 : plan_wide(a, oc, tiles, static_cast<int64_t>(tiles) * kBM, false);
    const int bn = wide_bn ? wide_bn : 128;
    if (!wide_bn) choose_ksplit(a, tiles * static_cast<int>((oc + bn - 1) / bn), wmode);

    // Workspace: the image split and channels-last, [2N][H][W][cp8] (hi images,
    // then lo), then any partial sums.
    const int64_t cp8 = round_up(ic, 8);
    const int64_t W = x->ne[0], H = x->ne[1], N = x->ne[3];
    const size_t a_bytes = static_cast<size_t>(round_up(2 * N * H * W * cp8 * 2, 256));
    void* ws = nullptr;
    if (int s = workspace(st, a_bytes + partial_bytes(a.ksplit, tiles, oc, bn), &ws); s != SDB_OK) return s;
    set_partials(a, ws, a_bytes, tiles, bn);
    if (channels_last(x)) {
        // Already channels-last: the split is a split of rows (positions).
        const long long ne[4] = {ic, W, H, N};
        const long long nb[4] = {1, ic, W * ic, H * W * ic};
        if (int s = split_rows(static_cast<const float*>(x->data), ne, nb, cp8, static_cast<uint16_t*>(ws), a.err, st,
                               gn);
            s != SDB_OK)
            return s;
    } else {
        const long long ne[4] = {W, H, ic, N};
        const long long nb[4] = {x->nb[0] / 4, x->nb[1] / 4, x->nb[2] / 4, x->nb[3] / 4};
        if (int s = split_nhwc(static_cast<const float*>(x->data), ne, nb, cp8, static_cast<uint16_t*>(ws), a.err, st);
            s != SDB_OK)
            return s;
    }
    // The split image as [plane][N][H][W][cp8]: a box {64 channels, OWt s0, OHt s1, NT, planes}.
    CUtensorMap amap;
    const uint64_t dims[5] = {static_cast<uint64_t>(cp8), static_cast<uint64_t>(W), static_cast<uint64_t>(H),
                              static_cast<uint64_t>(N), 2};
    const uint64_t strides[4] = {static_cast<uint64_t>(cp8 * 2), static_cast<uint64_t>(W * cp8 * 2),
                                 static_cast<uint64_t>(H * W * cp8 * 2), static_cast<uint64_t>(N * H * W * cp8 * 2)};
    const uint32_t box[5] = {64, static_cast<uint32_t>(g.owt * g.s0), static_cast<uint32_t>(g.oht * g.s1),
                             static_cast<uint32_t>(g.nt), static_cast<uint32_t>(a.a_planes)};
    const uint32_t estr[5] = {1, static_cast<uint32_t>(g.s0), static_cast<uint32_t>(g.s1), 1, 1};
    if (encode_tensor_map(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, ws, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B, estr) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for the image");
    // A channels-last output whose tiles are whole runs of 128 positions leaves by TMA stores.
    CUtensorMap ymap{};
    const bool whole_tiles = g.owt == g.ow && g.owt * g.oht * g.nt == kBM && g.oh % g.oht == 0 && g.n % g.nt == 0;
    if (channels_last(dst) && whole_tiles && oc % 4 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0 &&
        store_map(&ymap, a.y, oc, static_cast<long long>(g.n) * g.oh * g.ow, oc, wide_bn ? 16 : 32))
        a.store = kStoreTma;
    if (wide_bn) {
        a.tiles_n = static_cast<int>((oc + bn - 1) / bn);
        return launch_wide<kModeConv>(amap, *p, false, wide_bn, ymap, a, st);
    }
    return dispatch<kModeConv>(amap, *p, wmode, ymap, a, st);
}

}  // namespace sdb
