// Entry points of the GEMM-backed operations: MUL_MAT (with and without the
// gated GELU) and the direct convolution.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "../../include/sdb.h"
#include "gemm.cuh"
#include "runtime.cuh"
#include "store.cuh"

namespace sdb {

namespace {

template <int MODE, int WMODE>
int launch_gemm(const CUtensorMap& map, const GemmArgs& a, cudaStream_t st) {
    using S = GemmShape<WMODE>;
    auto kern = gemm_split_kernel<MODE, WMODE>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes));
    const dim3 grid(static_cast<unsigned>((a.m + kBM - 1) / kBM), static_cast<unsigned>((a.n + S::BN - 1) / S::BN));
    if (grid.y > 65535u) return fail(SDB_NOT_SUPPORTED, "gemm: too many column tiles");
    kern<<<grid, kGemmThreads, S::kSmemBytes, st>>>(map, a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

template <int MODE>
int dispatch(const Packed& p, int wmode, const GemmArgs& a, cudaStream_t st) {
    if (wmode == kWeightGated) return launch_gemm<MODE, kWeightGated>(p.map64, a, st);
    return wmode == kWeightSplit ? launch_gemm<MODE, kWeightSplit>(p.map128, a, st)
                                 : launch_gemm<MODE, kWeightHalf>(p.map128, a, st);
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

}  // namespace

}  // namespace sdb

using namespace sdb;

extern "C" {

int sdb_mul_mat_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst) {
    if (!mul_mat_shapes(w, x, dst)) return 0;
    return dst->ne[0] == w->ne[1] && dst->ne[1] == x->ne[1] && dst->ne[2] == x->ne[2] && dst->ne[3] == x->ne[3];
}

int sdb_mul_mat(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                void* stream) {
    if (!sdb_mul_mat_supported(w, x, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat: shapes not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_mul_mat: invalid chain");
    const auto st = static_cast<cudaStream_t>(stream);
    const int64_t k = w->ne[0], n = w->ne[1];
    const int64_t m = x->ne[1] * x->ne[2] * x->ne[3];
    if (m > (1LL << 31) - kBM || k > (1 << 24)) return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat: too large");
    std::shared_ptr<Packed> p;
    if (int s = packed_weights(w, Layout::linear, n, k, 0, 0, st, &p); s != SDB_OK) return s;
    GemmArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.xld = k;
    a.m = static_cast<int>(m);
    a.kpad = static_cast<int>(p->kpad);
    a.klog = static_cast<int>(k);
    a.n = static_cast<int>(n);
    a.b1_row = static_cast<int>(p->b1_row);
    a.rne1 = dst->ne[1];
    a.rne2 = dst->ne[2];
    a.vec = (reinterpret_cast<uintptr_t>(x->data) % 16 == 0) && (k % 4 == 0);
    set_out(a, dst, chain);
    const int wmode = p->split ? kWeightSplit : kWeightHalf;
    return dispatch<kModeLinear>(*p, wmode, a, st);
}

int sdb_mul_mat_gated_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* out) {
    if (!mul_mat_shapes(w, x, out) || w->type != SDB_TYPE_F16 || w->ne[1] % 2 != 0) return 0;
    const int64_t half = w->ne[1] / 2;
    return out->ne[0] == half && out->ne[1] == x->ne[1] && out->ne[2] == x->ne[2] && out->ne[3] == x->ne[3];
}

int sdb_mul_mat_gated(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* out, const sdb_chain* chain,
                      void* stream) {
    if (!sdb_mul_mat_gated_supported(w, x, out))
        return fail(SDB_NOT_SUPPORTED, "sdb_mul_mat_gated: shapes not supported");
    if (!valid_chain(chain) || (chain && (chain->redirect || chain->from_redirect)))
        return fail(SDB_INVALID, "sdb_mul_mat_gated: invalid chain");
    const auto st = static_cast<cudaStream_t>(stream);
    const int64_t k = w->ne[0], half = w->ne[1] / 2;
    const int64_t m = x->ne[1] * x->ne[2] * x->ne[3];
    std::shared_ptr<Packed> p;
    if (int s = packed_weights(w, Layout::gated, 2 * half, k, 0, half, st, &p); s != SDB_OK) return s;
    GemmArgs a{};
    a.x = static_cast<const float*>(x->data);
    a.xld = k;
    a.m = static_cast<int>(m);
    a.kpad = static_cast<int>(p->kpad);
    a.klog = static_cast<int>(k);
    a.n = static_cast<int>(half);
    a.b1_row = static_cast<int>(p->b1_row);
    a.rne1 = out->ne[1];
    a.rne2 = out->ne[2];
    a.vec = (reinterpret_cast<uintptr_t>(x->data) % 16 == 0) && (k % 4 == 0);
    set_out(a, out, chain);
    return dispatch<kModeLinear>(*p, kWeightGated, a, st);
}

// ---------------------------------------------------------------- conv2d

int sdb_conv2d_supported(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6]) {
    if (w == nullptr || x == nullptr || dst == nullptr || params == nullptr) return 0;
    if (!(is_type(w, SDB_TYPE_F16) || is_type(w, SDB_TYPE_F32)) || !is_type(x, SDB_TYPE_F32) ||
        !is_type(dst, SDB_TYPE_F32))
        return 0;
    const int s0 = params[0], s1 = params[1], p0 = params[2], p1 = params[3], d0 = params[4], d1 = params[5];
    if (s0 < 1 || s1 < 1 || d0 < 1 || d1 < 1 || p0 < 0 || p1 < 0) return 0;
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
    const int64_t m = ow * oh * x->ne[3];
    return m < (1LL << 31) - kBM && w->ne[0] * w->ne[1] <= 64 * 64;
}

int sdb_conv2d(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
               const sdb_chain* chain, void* stream) {
    if (!sdb_conv2d_supported(w, x, dst, params)) return fail(SDB_NOT_SUPPORTED, "sdb_conv2d: not supported");
    if (!valid_chain(chain)) return fail(SDB_INVALID, "sdb_conv2d: invalid chain");
    const auto st = static_cast<cudaStream_t>(stream);
    const int64_t ic = x->ne[2], oc = w->ne[3];
    const int icp = static_cast<int>((ic + 15) / 16 * 16);
    std::shared_ptr<Packed> p;
    if (int s = packed_weights(w, Layout::conv, oc, 0, icp, 0, st, &p); s != SDB_OK) return s;
    GemmArgs a{};
    a.x = static_cast<const float*>(x->data);
    ConvGeom& g = a.cg;
    g.iw = static_cast<int>(x->ne[0]);
    g.ih = static_cast<int>(x->ne[1]);
    g.ic = static_cast<int>(ic);
    g.n = static_cast<int>(x->ne[3]);
    g.ow = static_cast<int>(dst->ne[0]);
    g.oh = static_cast<int>(dst->ne[1]);
    g.kw = static_cast<int>(w->ne[0]);
    g.kh = static_cast<int>(w->ne[1]);
    g.s0 = params[0]; g.s1 = params[1]; g.p0 = params[2]; g.p1 = params[3]; g.d0 = params[4]; g.d1 = params[5];
    g.icp = icp;
    for (int d = 0; d < 4; ++d) g.xnb[d] = x->nb[d] / 4;
    a.m = g.ow * g.oh * g.n;
    a.kpad = static_cast<int>(p->kpad);
    a.klog = 0;
    a.n = static_cast<int>(oc);
    a.b1_row = static_cast<int>(p->b1_row);
    set_out(a, dst, chain);
    const int wmode = p->split ? kWeightSplit : kWeightHalf;
    return dispatch<kModeConv>(*p, wmode, a, st);
}

}  // extern "C"
