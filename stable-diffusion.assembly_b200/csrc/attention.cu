// GGML_OP_FLASH_ATTN_EXT without a mask: softmax(scale q k^T) v per head, the
// reference's attention_compute (attention.cc:858-1064) on tcgen05.
//
// One CTA takes a block of 128 queries of one head and walks the keys in
// blocks of BK.  Q, K and V arrive in FP32 (or FP16 K/V) and are split by
// four converter warps into FP16 pairs x = hi + lo 2^-11 (ptx.cuh); each
// product is taken as three tensor-core products (hi.hi into one FP32
// accumulator, hi.lo + lo.hi into a second, both in tensor memory):
//   S   = Q K^T  (M = 128 queries, N = BK keys, K = D)
//   O  += P V    (M = 128 queries, N = DV, K = BK keys; V read MN-major)
// Four softmax warps own one query row each: they read S from tensor memory,
// scale it, and take exponentials (the reference's exponential(), the
// Cephes-form polynomial of scalar_math.h) against a reference maximum that
// is raised -- and O rescaled -- only when a block's maximum exceeds it by
// more than 8 (so every weight stays below e^8 in FP16).  The row sums are
// kept in double precision and the output is divided once, by
// float(1 / sum), at the end (attention.cc:1052-1063).  Keys past LK get
// weight 0; queries past LQ are not written.
//
// The tensor core's FP32 accumulation rounds toward zero, so no sum is left
// to it for long: each key block's P V lands in a fresh tensor-memory
// accumulator that the softmax warps add into FP32 registers (where the
// rescale is a multiply), and the hi product of S is kept per 64 dims and
// summed in registers.  A CTA computes at most 80 output dims (DVC); wider
// value heads take several CTAs, each recomputing S.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "ptx.cuh"
#include "runtime.cuh"

namespace sdb {

namespace {

constexpr int kAttnQ = 128;
constexpr int kAttnThreads = 288;   // warps 0-3 softmax, 4-7 converters, 8 MMA
constexpr float kRescaleAbove = 8.0f;

struct AttnArgs {
    const void* q;
    const void* k;
    const void* v;
    float* out;
    long long qnb[4], knb[4], vnb[4], onb[4];  // element strides
    int k_half, v_half;                         // K / V stored as FP16
    int d, dv, lq, lk, h, hk, b;
    int dp, dvp;                                // padded to multiples of 16
    int dv_chunks;                              // CTAs along the value dims
    float scale;
    Chain chain;
    unsigned* err;
};

template <int BK>
struct AttnLayout {
    int q_hi, q_lo, stage0, stage_bytes, k_lo_off, v_hi_off, v_lo_off, p_hi, p_lo, bars, total;
    __host__ __device__ AttnLayout(int dp, int dvp) {
        const int qb = kAttnQ * dp * 2;
        q_hi = 0;
        q_lo = qb;
        stage0 = 2 * qb;
        const int kb = BK * dp * 2, vb = BK * dvp * 2;
        k_lo_off = kb;
        v_hi_off = 2 * kb;
        v_lo_off = 2 * kb + vb;
        stage_bytes = (2 * kb + 2 * vb + 127) / 128 * 128;
        p_hi = stage0 + 2 * stage_bytes;
        p_lo = p_hi + kAttnQ * BK * 2;
        bars = p_lo + kAttnQ * BK * 2;
        total = bars + 128;
    }
};

__device__ __forceinline__ float load_elem(const void* base, long long off, int half) {
    return half ? __half2float(__ldg(reinterpret_cast<const __half*>(base) + off))
                : __ldg(reinterpret_cast<const float*>(base) + off);
}

// 8 consecutive elements (dims) of one row; zero past `limit`.
__device__ __forceinline__ void load8(const void* base, long long row_off, long long nb0, int c0, int limit, int half,
                                      float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (c0 + i < limit) ? load_elem(base, row_off + (c0 + i) * nb0, half) : 0.0f;
}

// Converts rows [0, rows) x dims [0, dp) of a K-major operand into the
// no-swizzle core-matrix layout (rows of 16 B, 8-row groups `sbo` apart,
// 8-dim groups 128 B apart).  valid(r) gives the row's element offset or -1.
template <class RowOff>
__device__ __forceinline__ bool convert_kmajor(const void* src, int half, long long nb0, int d, int dp, int rows,
                                               uint32_t hi, uint32_t lo, int t, RowOff row_off) {
    const int chunks = dp / 8;
    bool over = false;
    for (int idx = t; idx < rows * chunks; idx += 128) {
        const int r = idx / chunks, c = idx - (idx / chunks) * chunks;
        const long long off = row_off(r);
        float v[8];
        if (off >= 0) load8(src, off, nb0, c * 8, d, half, v);
        else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        uint4 h4, l4;
        over |= split8(v, h4, l4);
        const uint32_t o = static_cast<uint32_t>((r >> 3) * (dp * 16) + c * 128 + (r & 7) * 16);
        st_shared_v4(hi + o, h4);
        st_shared_v4(lo + o, l4);
    }
    return over;
}

// V rows (keys) into the MN-major no-swizzle layout of the PV product's B:
// core matrices of 8 keys x 8 dims, key groups 128 B apart, dim groups
// BK * 16 B apart.
template <int BK, class RowOff>
__device__ __forceinline__ bool convert_v(const void* src, int half, long long nb0, int dv, int dvp, uint32_t hi,
                                          uint32_t lo, int t, RowOff row_off) {
    const int chunks = dvp / 8;
    bool over = false;
    for (int idx = t; idx < BK * chunks; idx += 128) {
        const int k = idx / chunks, c = idx - (idx / chunks) * chunks;
        const long long off = row_off(k);
        float v[8];
        if (off >= 0) load8(src, off, nb0, c * 8, dv, half, v);
        else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        uint4 h4, l4;
        over |= split8(v, h4, l4);
        const uint32_t o = static_cast<uint32_t>(c * (BK * 16) + (k >> 3) * 128 + (k & 7) * 16);
        st_shared_v4(hi + o, h4);
        st_shared_v4(lo + o, l4);
    }
    return over;
}

template <int BK, int DVC>
__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const AttnLayout<BK> L(a.dp, DVC);
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [2]
    uint64_t* kv_empty = kv_full + 2;                                // [2]
    uint64_t* q_full = kv_empty + 2;
    uint64_t* s_full = q_full + 1;
    uint64_t* p_full = s_full + 1;
    uint64_t* pv_done = p_full + 1;
    uint64_t* drain = pv_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kAttnQ;
    const int head = blockIdx.y / a.dv_chunks;
    const int dv0 = (blockIdx.y - head * a.dv_chunks) * DVC;
    const int batch = blockIdx.z;
    const int khead = head / (a.h / a.hk);
    const int nblk = (a.lk + BK - 1) / BK;
    const int nsc = (a.dp + 63) / 64;  // hi accumulators of S, one per 64 dims
    const uint32_t base = smem_u32(smem);
    const int need = (nsc + 1) * BK + 2 * DVC;
    const uint32_t tmem_cols = static_cast<uint32_t>(need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512);

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 4);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(q_full, 4);
        mbar_init(s_full, 1);
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 8) tmem_alloc(tmem_slot, tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s_lo = tmem + nsc * BK;
    const uint32_t t_o_hi = tmem + (nsc + 1) * BK, t_o_lo = t_o_hi + DVC;

    if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ converters
        const int t = threadIdx.x - 128;
        bool over = false;
        const long long qb = static_cast<long long>(head) * a.qnb[2] + static_cast<long long>(batch) * a.qnb[3];
        over |= convert_kmajor(a.q, 0, a.qnb[0], a.d, a.dp, kAttnQ, base + L.q_hi, base + L.q_lo, t, [&](int r) {
            const int i = q0 + r;
            return i < a.lq ? qb + static_cast<long long>(i) * a.qnb[1] : -1LL;
        });
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
        const long long kbase = static_cast<long long>(khead) * a.knb[2] + static_cast<long long>(batch) * a.knb[3];
        const long long vbase = static_cast<long long>(khead) * a.vnb[2] + static_cast<long long>(batch) * a.vnb[3] +
                                static_cast<long long>(dv0) * a.vnb[0];
        for (int j = 0; j < nblk; ++j) {
            const int s = j & 1;
            if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort, a.err)) break;
            const uint32_t st = base + L.stage0 + s * L.stage_bytes;
            const int key0 = j * BK;
            over |= convert_kmajor(a.k, a.k_half, a.knb[0], a.d, a.dp, BK, st, st + L.k_lo_off, t, [&](int r) {
                const int key = key0 + r;
                return key < a.lk ? kbase + static_cast<long long>(key) * a.knb[1] : -1LL;
            });
            over |= convert_v<BK>(a.v, a.v_half, a.vnb[0], a.dv - dv0, DVC, st + L.v_hi_off, st + L.v_lo_off, t,
                                  [&](int r) {
                                      const int key = key0 + r;
                                      return key < a.lk ? vbase + static_cast<long long>(key) * a.vnb[1] : -1LL;
                                  });
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&kv_full[s]);
        }
        if (over) atomicOr(a.err, kErrRange);
    } else if (warp == 8) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_f16_f32(kAttnQ, BK);
            const uint32_t id_pv = idesc_f16_f32_bmajor(kAttnQ, DVC, 1);
            const uint32_t sbo_q = static_cast<uint32_t>(a.dp * 16);
            const uint32_t sbo_p = BK * 16;
            bool ok = mbar_wait(q_full, 0, abort, a.err);
            for (int j = 0; j < nblk && ok; ++j) {
                const int s = j & 1;
                if (!mbar_wait(&kv_full[s], (j >> 1) & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t st = base + L.stage0 + s * L.stage_bytes;
                for (int kk = 0; kk < a.dp / 16; ++kk) {
                    const uint64_t qh = desc_noswizzle(base + L.q_hi + kk * 256, 128, sbo_q);
                    const uint64_t ql = desc_noswizzle(base + L.q_lo + kk * 256, 128, sbo_q);
                    const uint64_t kh = desc_noswizzle(st + kk * 256, 128, sbo_q);
                    const uint64_t kl = desc_noswizzle(st + L.k_lo_off + kk * 256, 128, sbo_q);
                    mma_f16(tmem + (kk >> 2) * BK, qh, kh, id_s, (kk & 3) ? 1u : 0u);
                    mma_f16(t_s_lo, qh, kl, id_s, kk > 0 ? 1u : 0u);
                    mma_f16(t_s_lo, ql, kh, id_s, 1u);
                }
                mma_commit(s_full);
                if (!mbar_wait(p_full, j & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ph = desc_noswizzle(base + L.p_hi + kk * 256, 128, sbo_p);
                    const uint64_t pl = desc_noswizzle(base + L.p_lo + kk * 256, 128, sbo_p);
                    const uint64_t vh = desc_noswizzle(st + L.v_hi_off + kk * 256, 128, sbo_p);
                    const uint64_t vl = desc_noswizzle(st + L.v_lo_off + kk * 256, 128, sbo_p);
                    const uint32_t acc = kk > 0 ? 1u : 0u;
                    mma_f16(t_o_hi, ph, vh, id_pv, acc);
                    mma_f16(t_o_lo, ph, vl, id_pv, acc);
                    mma_f16(t_o_lo, pl, vh, id_pv, 1u);
                }
                mma_commit(pv_done);
                mma_commit(&kv_empty[s]);
            }
            if (!ok) {
                // Wind down: every MMA issued completes before tensor memory is freed.
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------ softmax + epilogue (warps 0-3)
        const int r = warp * 32 + lane;
        const int qi = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
        float m_ref = -INFINITY;
        double l = 0.0;
        float o[DVC];
#pragma unroll
        for (int i = 0; i < DVC; ++i) o[i] = 0.0f;
        // o += the block product in tensor memory (hi + lo 2^-11).
        auto drain_o = [&]() {
#pragma unroll
            for (int c = 0; c < DVC; c += 16) {
                float oh[16], ol[16];
                tmem_ld16(t_o_hi + lane_off + c, oh);
                tmem_ld16(t_o_lo + lane_off + c, ol);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) o[c + i] += fmaf(ol[i], kLoUnscale, oh[i]);
            }
        };
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            if (!mbar_wait(s_full, j & 1, abort, a.err)) { ok = false; break; }
            tc_fence_after();
            float s[BK];
#pragma unroll
            for (int c = 0; c < BK; c += 32) {
                float part[32], lo[32];
                tmem_ld32(t_s_lo + lane_off + c, lo);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) s[c + i] = lo[i] * kLoUnscale;
                for (int sc = 0; sc < nsc; ++sc) {
                    tmem_ld32(tmem + sc * BK + lane_off + c, part);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[c + i] += part[i];
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) s[c + i] *= a.scale;
            }
            const int valid = min(BK, a.lk - j * BK);
            float bmax = -INFINITY;
#pragma unroll
            for (int i = 0; i < BK; ++i)
                if (i < valid) bmax = fmaxf(bmax, s[i]);
            // The previous block's product: into the registers (P's buffer is then free).
            if (j > 0) {
                if (!mbar_wait(pv_done, (j - 1) & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                drain_o();
            }
            if (j == 0) {
                m_ref = bmax;
            } else if (bmax > m_ref + kRescaleAbove) {
                const float factor = exponential(m_ref - bmax);
                m_ref = bmax;
#pragma unroll
                for (int i = 0; i < DVC; ++i) o[i] *= factor;
                l *= static_cast<double>(factor);
            }
            // Weights of this block into P (hi / lo), row r, K-major core matrices.
            double bsum = 0.0;
#pragma unroll
            for (int c = 0; c < BK / 8; ++c) {
                float p[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int key = c * 8 + i;
                    p[i] = key < valid ? exponential(s[key] - m_ref) : 0.0f;
                    bsum += static_cast<double>(p[i]);
                }
                uint4 h4, l4;
                split8(p, h4, l4);
                const uint32_t off = static_cast<uint32_t>((r >> 3) * (BK * 16) + c * 128 + (r & 7) * 16);
                st_shared_v4(base + L.p_hi + off, h4);
                st_shared_v4(base + L.p_lo + off, l4);
            }
            l += bsum;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && mbar_wait(pv_done, (nblk - 1) & 1, abort, a.err)) {
            tc_fence_after();
            drain_o();
            if (qi < a.lq) {
                const float recip = static_cast<float>(1.0 / l);
                const long long ob = static_cast<long long>(head) * a.onb[1] + static_cast<long long>(qi) * a.onb[2] +
                                     static_cast<long long>(batch) * a.onb[3];
#pragma unroll
                for (int i = 0; i < DVC; ++i) {
                    const int dcol = dv0 + i;
                    if (dcol < a.dv) {
                        const float v = apply_chain(a.chain, o[i] * recip, dcol, head, qi, batch);
                        a.out[ob + dcol * a.onb[0]] = v;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, tmem_cols);
    }
}

bool floaty(const sdb_tensor* t) {
    return t && t->data && (t->type == SDB_TYPE_F32 || t->type == SDB_TYPE_F16);
}

int esize(const sdb_tensor* t) { return t->type == SDB_TYPE_F16 ? 2 : 4; }

template <int BK, int DVC>
int launch_attention(const AttnArgs& a, cudaStream_t st) {
    const AttnLayout<BK> L(a.dp, DVC);
    const int smem = L.total + 1024;
    if (smem > 227 * 1024) return fail(SDB_NOT_SUPPORTED, "sdb_attention: head too wide");
    SDB_CUDA(cudaFuncSetAttribute(attention_kernel<BK, DVC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const dim3 grid(static_cast<unsigned>((a.lq + kAttnQ - 1) / kAttnQ), static_cast<unsigned>(a.h * a.dv_chunks),
                    static_cast<unsigned>(a.b));
    attention_kernel<BK, DVC><<<grid, kAttnThreads, smem, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

template <int BK>
int launch_dvc(AttnArgs& a, cudaStream_t st) {
    const int dvp = (a.dv + 15) / 16 * 16;
    const int chunks = (dvp + 79) / 80;
    const int dvc = ((dvp / 16 + chunks - 1) / chunks) * 16;
    a.dv_chunks = chunks;
    switch (dvc) {
    case 16: return launch_attention<BK, 16>(a, st);
    case 32: return launch_attention<BK, 32>(a, st);
    case 48: return launch_attention<BK, 48>(a, st);
    case 64: return launch_attention<BK, 64>(a, st);
    default: return launch_attention<BK, 80>(a, st);
    }
}

}  // namespace

}  // namespace sdb

using namespace sdb;

extern "C" int sdb_attention_supported(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v,
                                       const sdb_tensor* dst) {
    if (!q || !k || !v || !dst) return 0;
    if (q->type != SDB_TYPE_F32 || !q->data || !floaty(k) || !floaty(v) || dst->type != SDB_TYPE_F32 || !dst->data)
        return 0;
    const int64_t d = q->ne[0], lq = q->ne[1], h = q->ne[2], b = q->ne[3];
    const int64_t lk = k->ne[1], hk = k->ne[2], dv = v->ne[0];
    if (k->ne[0] != d || v->ne[1] != lk || v->ne[2] != hk || k->ne[3] != b || v->ne[3] != b) return 0;
    if (hk <= 0 || h % hk != 0 || d <= 0 || dv <= 0 || lq <= 0 || lk <= 0) return 0;
    if (dst->ne[0] != dv || dst->ne[1] != h || dst->ne[2] != lq || dst->ne[3] != b) return 0;
    if (d > 160 || dv > 512) return 0;
    for (const sdb_tensor* t : {q, k, v, dst})
        for (int i = 0; i < 4; ++i)
            if (t->nb[i] % esize(t) != 0 || t->nb[i] < 0) return 0;
    return h * ((dv + 79) / 80) <= 65535 && b <= 65535;
}

extern "C" int sdb_attention(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, const sdb_tensor* dst,
                             float scale, const sdb_chain* chain, void* stream) {
    if (!sdb_attention_supported(q, k, v, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_attention: not supported");
    if (chain && (chain->count < 0 || chain->count > SDB_MAX_STEPS || chain->redirect))
        return fail(SDB_INVALID, "sdb_attention: invalid chain");
    AttnArgs a{};
    a.q = q->data;
    a.k = k->data;
    a.v = v->data;
    a.out = static_cast<float*>(dst->data);
    for (int i = 0; i < 4; ++i) {
        a.qnb[i] = q->nb[i] / 4;
        a.knb[i] = k->nb[i] / esize(k);
        a.vnb[i] = v->nb[i] / esize(v);
        a.onb[i] = dst->nb[i] / 4;
    }
    a.k_half = k->type == SDB_TYPE_F16;
    a.v_half = v->type == SDB_TYPE_F16;
    a.d = static_cast<int>(q->ne[0]);
    a.lq = static_cast<int>(q->ne[1]);
    a.h = static_cast<int>(q->ne[2]);
    a.b = static_cast<int>(q->ne[3]);
    a.lk = static_cast<int>(k->ne[1]);
    a.hk = static_cast<int>(k->ne[2]);
    a.dv = static_cast<int>(v->ne[0]);
    a.dp = (a.d + 15) / 16 * 16;
    a.dvp = (a.dv + 15) / 16 * 16;
    a.scale = scale;
    a.chain = make_chain(chain);
    a.err = device_error_word();
    const auto st = static_cast<cudaStream_t>(stream);
    // Keys per block: 64 where the registers hold a block's scores beside a
    // CTA's output dims (<= 48), 32 otherwise.
    const int dvp = (a.dv + 15) / 16 * 16;
    const int dvc = ((dvp / 16 + (dvp + 79) / 80 - 1) / ((dvp + 79) / 80)) * 16;
    if (a.dp <= 96 && dvc <= 48) return launch_dvc<64>(a, st);
    return launch_dvc<32>(a, st);
}
