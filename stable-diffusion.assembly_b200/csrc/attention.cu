// GGML_OP_FLASH_ATTN_EXT without a mask: softmax(scale q k^T) v per head, the
// reference's attention_compute (attention.cc:858-1064) on tcgen05.
//
// Q, K and V are split once (split.cuh, split_tiles) into FP16 pairs
// x = hi + lo 2^-11, stored tile by tile in the UMMA no-swizzle core-matrix
// layout, so that each tile arrives in shared memory as one contiguous bulk
// copy.  One CTA takes a block of 128 queries of one
// head (and up to 80 of its value dims) and walks the keys in blocks of BK;
// each product is three tensor-core products (hi.hi into one FP32
// accumulator, hi.lo + lo.hi into a second):
//   S   = Q K^T  (M = 128 queries, N = BK keys, K = head dims)
//   O_j = P V    (M = 128 queries, N = value dims, K = BK keys; V MN-major)
// S is double-buffered in tensor memory, so the next block's Q K^T runs while
// the softmax warps work on this one.  Eight softmax warps, two per quarter of
// the tensor-memory lanes, own one query row per lane pair, each half of a
// block's keys: they read S, scale it by scale * log2(e) and take 2^(s - m)
// with the ex2 instruction against a reference maximum that is raised -- and
// the output rescaled -- only when a block's maximum exceeds it by 11.5 (e^8),
// so every weight stays a normal FP16 pair.  The row sums are kept in double
// precision, and the output is divided once, by float(1 / sum), at the end
// (attention.cc:1052-1063).  Keys past LK get weight 0; queries past LQ are
// not written.
//
// The tensor core's FP32 accumulation rounds toward zero, so no long sum is
// left to it: each block's P V lands in a fresh accumulator that the softmax
// warps add into FP32 registers, and the hi product of S is kept per 64 dims
// and summed in registers.  Value heads wider than 80 dims take several CTAs,
// each recomputing S.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "ptx.cuh"
#include "quant.cuh"
#include "runtime.cuh"
#include "split.cuh"

namespace sdb {

namespace {

constexpr int kAttnQ = 128;
constexpr int kAttnThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax
constexpr int kStagesKV = 3;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleAbove = 11.5f;  // log2 units: e^8

struct AttnArgs {
    const uint8_t* qs;   // split tiles of 128 queries x dp: hi plane, then lo plane
    const uint8_t* ks;   // split tiles of BK keys x dp
    const uint8_t* vs;   // split tiles of BK keys x dvs (value dims padded to the CTAs' chunks)
    long long q_plane, k_plane, v_plane;  // bytes of one (hi) plane
    int ntq, ntk;        // tiles of queries / keys per head
    int dvs;             // value dims of a stored row
    float* out;
    long long onb[4];  // element strides of dst [DV, H, LQ, B]
    int d, dv, lq, lk, h, hk, b;
    int dp, dvp, dv_chunks;
    int rq, rk;        // rows of the hi planes of Q and of K / V
    float scale2;      // scale * log2(e)
    Chain chain;
    unsigned* err;
};

struct AttnLayout {
    static __host__ __device__ int p_bytes(int bk) { return 2 * kAttnQ * bk * 2; }
    int q_hi, q_lo, stage0, stage_bytes, k_lo, v_hi, v_lo, p_hi, p_lo, xmax, xsum, bars, total;
    __host__ __device__ AttnLayout(int dp, int dvc, int bk) {
        const int qb = kAttnQ * dp * 2;
        q_hi = 0;
        q_lo = qb;
        stage0 = 2 * qb;
        const int kb = bk * dp * 2, vb = bk * dvc * 2;
        k_lo = kb;
        v_hi = 2 * kb;
        v_lo = 2 * kb + vb;
        stage_bytes = (2 * kb + 2 * vb + 127) / 128 * 128;
        p_hi = stage0 + kStagesKV * stage_bytes;   // [2] buffers, p_bytes apart
        p_lo = p_hi + kAttnQ * bk * 2;
        xmax = p_hi + 2 * p_bytes(bk);            // [2][128][2] floats
        xsum = xmax + 2 * kAttnQ * 2 * 4;  // [128][2] doubles
        bars = xsum + kAttnQ * 2 * 8;
        total = bars + 512;
    }
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


template <int BK, int DVC, int NO>
__global__ void __launch_bounds__(kAttnThreads, 1) attention_kernel(const AttnArgs a) {
    constexpr int KH = BK / 2;                  // keys of a block per softmax warp
    constexpr int OCH = DVC / 16;               // 16-column chunks of the output
    constexpr int OMINE = (OCH + 1) / 2;        // chunks per softmax warp (at most)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const AttnLayout L(a.dp, DVC, BK);
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [3]
    uint64_t* kv_empty = kv_full + kStagesKV;                        // [3]
    uint64_t* q_full = kv_empty + kStagesKV;
    uint64_t* s_full = q_full + 1;    // [2]
    uint64_t* p_full = s_full + 2;    // [2]
    uint64_t* pv_done = p_full + 2;   // [2]
    uint64_t* drain = pv_done + 2;
    uint64_t* pair = drain + 1;       // [4]: the two softmax warps of a lane quarter meet here
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair + 4);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xmax = reinterpret_cast<float*>(smem + L.xmax);
    double* xsum = reinterpret_cast<double*>(smem + L.xsum);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kAttnQ;
    const int head = blockIdx.y / a.dv_chunks;
    const int dv0 = (blockIdx.y - head * a.dv_chunks) * DVC;
    const int batch = blockIdx.z;
    const int khead = head / (a.h / a.hk);
    const int nblk = (a.lk + BK - 1) / BK;
    const int nsc = (a.dp + 63) / 64;                 // hi accumulators of S, one per 64 dims
    const int sbuf = (nsc + 1) * BK;                  // tensor-memory columns of one S buffer
    const uint32_t base = smem_u32(smem);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesKV; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(q_full, 1);
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&p_full[i], 8);
            mbar_init(&pv_done[i], 1);
        }
        mbar_init(drain, 1);
        for (int i = 0; i < 4; ++i) mbar_init(&pair[i], 2);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Output blocks: NO buffers of (hi, lo), the block in buffer j % NO.
    auto t_o_hi = [&](int ob) { return tmem + 2 * sbuf + ob * 2 * DVC; };
    auto t_o_lo = [&](int ob) { return tmem + 2 * sbuf + ob * 2 * DVC + DVC; };
    const int pbuf = AttnLayout::p_bytes(BK);

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint32_t qbytes = kAttnQ * a.dp * 2;
            const uint32_t kbytes = BK * a.dp * 2, vbytes = BK * DVC * 2;
            const uint8_t* qt = a.qs + (static_cast<long long>(batch * a.h + head) * a.ntq + blockIdx.x) * qbytes;
            mbar_arrive_expect_tx(q_full, 2 * qbytes);
            bulk_load(smem + L.q_hi, qt, qbytes, q_full);
            bulk_load(smem + L.q_lo, qt + a.q_plane, qbytes, q_full);
            const long long ktile0 = static_cast<long long>(batch * a.hk + khead) * a.ntk;
            int issued = 0;
            for (int j = 0; j < nblk; ++j) {
                const int s = j % kStagesKV;
                if (!mbar_wait(&kv_empty[s], ((j / kStagesKV) & 1) ^ 1, abort, a.err)) break;
                uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kbytes + 2 * vbytes);
                const uint8_t* kt = a.ks + (ktile0 + j) * kbytes;
                const uint8_t* vt = a.vs + (ktile0 + j) * static_cast<long long>(BK) * a.dvs * 2 +
                                    static_cast<long long>(dv0 / 8) * BK * 16;
                bulk_load(st, kt, kbytes, &kv_full[s]);
                bulk_load(st + L.k_lo, kt + a.k_plane, kbytes, &kv_full[s]);
                bulk_load(st + L.v_hi, vt, vbytes, &kv_full[s]);
                bulk_load(st + L.v_lo, vt + a.v_plane, vbytes, &kv_full[s]);
                ++issued;
            }
            if (*abort) {
                mbar_wait_quiet(q_full, 0, 100000000ull);
                for (int j = (issued > kStagesKV ? issued - kStagesKV : 0); j < issued; ++j)
                    mbar_wait_quiet(&kv_full[j % kStagesKV], (j / kStagesKV) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_f16_f32(kAttnQ, BK);
            const uint32_t id_pv = idesc_f16_f32_bmajor(kAttnQ, DVC, 1);
            const uint32_t q_lbo = kAttnQ * 16, k_lbo = BK * 16, kv_sbo = 128, p_sbo = BK * 16;
            auto issue_s = [&](int j) {
                const int s = j % kStagesKV;
                const uint32_t st = base + L.stage0 + s * L.stage_bytes;
                const uint32_t sb = tmem + (j & 1) * sbuf;
                for (int kk = 0; kk < a.dp / 16; ++kk) {
                    const uint64_t qh = desc_noswizzle(base + L.q_hi + kk * 2 * q_lbo, q_lbo, 128);
                    const uint64_t ql = desc_noswizzle(base + L.q_lo + kk * 2 * q_lbo, q_lbo, 128);
                    const uint64_t kh = desc_noswizzle(st + kk * 2 * k_lbo, k_lbo, kv_sbo);
                    const uint64_t kl = desc_noswizzle(st + L.k_lo + kk * 2 * k_lbo, k_lbo, kv_sbo);
                    mma_f16(sb + (kk >> 2) * BK, qh, kh, id_s, (kk & 3) ? 1u : 0u);
                    mma_f16(sb + nsc * BK, qh, kl, id_s, kk > 0 ? 1u : 0u);
                    mma_f16(sb + nsc * BK, ql, kh, id_s, 1u);
                }
                mma_commit(&s_full[j & 1]);
            };
            bool ok = mbar_wait(q_full, 0, abort, a.err);
            if (ok && nblk > 0) {
                ok = mbar_wait(&kv_full[0], 0, abort, a.err);
                if (ok) {
                    tc_fence_after();
                    issue_s(0);
                }
            }
            for (int j = 0; j < nblk && ok; ++j) {
                if (j + 1 < nblk) {
                    const int s1 = (j + 1) % kStagesKV;
                    if (!mbar_wait(&kv_full[s1], ((j + 1) / kStagesKV) & 1, abort, a.err)) { ok = false; break; }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                const int pb = j % NO;
                if (!mbar_wait(&p_full[pb], (j / NO) & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                const int s = j % kStagesKV;
                const uint32_t st = base + L.stage0 + s * L.stage_bytes;
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ph = desc_noswizzle(base + L.p_hi + pb * pbuf + kk * 256, 128, p_sbo);
                    const uint64_t pl = desc_noswizzle(base + L.p_lo + pb * pbuf + kk * 256, 128, p_sbo);
                    const uint64_t vh = desc_noswizzle(st + L.v_hi + kk * 256, 128, BK * 16);
                    const uint64_t vl = desc_noswizzle(st + L.v_lo + kk * 256, 128, BK * 16);
                    const uint32_t acc = kk > 0 ? 1u : 0u;
                    mma_f16(t_o_hi(pb), ph, vh, id_pv, acc);
                    mma_f16(t_o_lo(pb), ph, vl, id_pv, acc);
                    mma_f16(t_o_lo(pb), pl, vh, id_pv, 1u);
                }
                mma_commit(&pv_done[pb]);
                mma_commit(&kv_empty[s]);
            }
            if (!ok) {
                // Wind down: every MMA issued completes before tensor memory is freed.
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------ softmax + epilogue (warps 2-9)
        const int ew = warp - 2;
        const int q = warp & 3;          // lane quarter
        const int half = ew >> 2;        // which half of a block's keys, and of the output chunks
        const int r = q * 32 + lane;     // query row of the tile
        const int qi = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        // The pair's exchange through shared memory: each warp writes, arrives,
        // and waits (bounded) for the other's arrival.
        uint32_t pair_uses = 0;
        auto pair_sync = [&]() {
            __syncwarp();
            if (lane == 0) mbar_arrive(&pair[q]);
            const bool met = mbar_wait(&pair[q], pair_uses & 1, abort, a.err);
            ++pair_uses;
            return met;
        };
        float m_ref = -INFINITY;
        double l = 0.0;
        float o[OMINE * 16];
#pragma unroll
        for (int i = 0; i < OMINE * 16; ++i) o[i] = 0.0f;
        // Rescale factors applied since the weights of the block in each
        // output buffer were taken (that block's product still in flight).
        float pend[NO];
#pragma unroll
        for (int i = 0; i < NO; ++i) pend[i] = 1.0f;
        // o += pend * (the block product in output buffer ob).
        auto drain_o = [&](int ob) {
            const float f = pend[ob];
#pragma unroll
            for (int c = 0; c < OMINE; ++c) {
                const int ch = 2 * c + half;
                if (ch < OCH) {
                    float oh[16], ol[16];
                    tmem_ld16(t_o_hi(ob) + lane_off + ch * 16, oh);
                    tmem_ld16(t_o_lo(ob) + lane_off + ch * 16, ol);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[c * 16 + i] = fmaf(f, fmaf(ol[i], kLoUnscale, oh[i]), o[c * 16 + i]);
                }
            }
        };
        // Waits for block jb's product and adds it in.
        auto take = [&](int jb) {
            const int ob = jb % NO;
            if (!mbar_wait(&pv_done[ob], (jb / NO) & 1, abort, a.err)) return false;
            tc_fence_after();
            drain_o(ob);
            return true;
        };
        bool ok = true;
        for (int j = 0; j < nblk; ++j) {
            const int b = j & 1;
            if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort, a.err)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sb = tmem + b * sbuf + lane_off + half * KH;
            float s[KH];
            {
                float lo[KH];
                if constexpr (KH == 32) tmem_ld32(sb + nsc * BK, lo);
                else tmem_ld16(sb + nsc * BK, lo);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < KH; ++i) s[i] = lo[i] * kLoUnscale;
                for (int sc = 0; sc < nsc; ++sc) {
                    float part[KH];
                    if constexpr (KH == 32) tmem_ld32(sb + sc * BK, part);
                    else tmem_ld16(sb + sc * BK, part);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < KH; ++i) s[i] += part[i];
                }
#pragma unroll
                for (int i = 0; i < KH; ++i) s[i] *= a.scale2;
            }
            const int valid = min(BK, a.lk - j * BK) - half * KH;  // my keys that exist
            float mine = -INFINITY;
#pragma unroll
            for (int i = 0; i < KH; ++i)
                if (i < valid) mine = fmaxf(mine, s[i]);
            xmax[(b * kAttnQ + r) * 2 + half] = mine;
            if (!pair_sync()) { ok = false; break; }
            const float bmax = fmaxf(xmax[(b * kAttnQ + r) * 2], xmax[(b * kAttnQ + r) * 2 + 1]);
            // The product of the block that last used this P / output buffer
            // into the registers (the buffers are then free).
            const int pb = j % NO;
            if (j >= NO && !take(j - NO)) { ok = false; break; }
            if (j == 0) {
                m_ref = bmax;
            } else if (bmax > m_ref + kRescaleAbove) {
                const float factor = ex2(m_ref - bmax);
                m_ref = bmax;
#pragma unroll
                for (int i = 0; i < OMINE * 16; ++i) o[i] *= factor;
                l *= static_cast<double>(factor);
#pragma unroll
                for (int i = 0; i < NO; ++i)
                    if (i != pb) pend[i] *= factor;  // blocks still in flight
            }
            pend[pb] = 1.0f;
            // This warp's keys of the block into P (hi / lo), row r, K-major core matrices.
            // The block's weights summed in FP32 with compensation (Neumaier),
            // the block sum then added to the row's double total.
            float bsum = 0.0f, bcomp = 0.0f;
#pragma unroll
            for (int c = 0; c < KH / 8; ++c) {
                float p[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int key = c * 8 + i;
                    p[i] = key < valid ? ex2(s[key] - m_ref) : 0.0f;
                    const float t = bsum + p[i];
                    bcomp += fabsf(bsum) >= p[i] ? (bsum - t) + p[i] : (p[i] - t) + bsum;
                    bsum = t;
                }
                uint4 h4, l4;
                split8(p, h4, l4);
                const uint32_t off =
                    static_cast<uint32_t>((r >> 3) * (BK * 16) + (half * (KH / 8) + c) * 128 + (r & 7) * 16);
                st_shared_v4(base + L.p_hi + pb * pbuf + off, h4);
                st_shared_v4(base + L.p_lo + pb * pbuf + off, l4);
            }
            l += static_cast<double>(bsum) + static_cast<double>(bcomp);
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[pb]);
        }
        // The blocks still in flight.
        for (int jb = max(0, nblk - NO); ok && jb < nblk; ++jb) ok = take(jb);
        if (ok && nblk > 0) {
            xsum[r * 2 + half] = l;
            if (!pair_sync()) ok = false;
            const double total = xsum[r * 2] + xsum[r * 2 + 1];
            if (ok && qi < a.lq) {
                const float recip = static_cast<float>(1.0 / total);
                const long long ob = static_cast<long long>(head) * a.onb[1] + static_cast<long long>(qi) * a.onb[2] +
                                     static_cast<long long>(batch) * a.onb[3];
                // Whole 16-column chunks of a row with unit stride leave as four float4s.
                const bool vec = a.onb[0] == 1 && dv0 % 4 == 0 && (reinterpret_cast<uintptr_t>(a.out + ob) & 15) == 0;
#pragma unroll
                for (int c = 0; c < OMINE; ++c) {
                    const int ch = 2 * c + half;
                    if (ch < OCH) {
                        const int d0c = dv0 + ch * 16;
                        if (vec && d0c + 16 <= a.dv) {
                            float w[16];
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                w[i] = apply_chain(a.chain, o[c * 16 + i] * recip, d0c + i, head, qi, batch);
#pragma unroll
                            for (int i = 0; i < 16; i += 4)
                                *reinterpret_cast<float4*>(a.out + ob + d0c + i) = make_float4(w[i], w[i + 1], w[i + 2],
                                                                                                w[i + 3]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int dcol = d0c + i;
                                if (dcol < a.dv) {
                                    const float v = apply_chain(a.chain, o[c * 16 + i] * recip, dcol, head, qi, batch);
                                    a.out[ob + dcol * a.onb[0]] = v;
                                }
                            }
                        }
                    }
                }
            }
        }
    }

    // Single-lane roles rejoin their warps before the CTA-wide barrier.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---- two softmax warpgroups, one query row a thread ----------------------
//
// For heads up to 128 dims whose accumulators fit tensor memory twice over.
// Warps 2-5 (warpgroup 0) take the key blocks j = 0, 2, 4, ...; warps 6-9
// (warpgroup 1) j = 1, 3, 5, ...: each thread owns one query row of its
// warpgroup's blocks -- all BK keys of it, so a block's maximum needs no
// exchange -- and each warpgroup keeps its own online softmax (reference
// maximum, double row sum, output in registers) and its own output
// accumulator in tensor memory.  A block's product P V is taken into the
// registers at the warpgroup's next block, so it runs under that block's
// softmax.  The two streams merge once at the end: m = max(m0, m1),
// O = O0 2^(m0 - m) + O1 2^(m1 - m), l likewise, then O / l with the chain.
// A block's weights are summed in FP32 as a pairwise tree (at most log2(BK)
// roundings), blocks in double.
//
// Each product lands in ONE accumulator: its lo products (hi.lo and lo.hi,
// whose lo operands carry the split's 2^11) are issued first, then the first
// hi.hi product with tcgen05.mma's input scale 2^-11 (mma_f16_scale_lo), the
// others plain -- hi.hi + (hi.lo + lo.hi) 2^-11 with no second accumulator to
// read and no combining instruction.  S keeps one accumulator per 64 dims
// (the first also holding the lo sum), the output one per block.  Tensor
// memory: 2 NSC BK + 2 DVC columns (224 for 40-dim heads).
struct AttnWgLayout {
    int q_hi, q_lo, stage0, stage_bytes, k_lo, v_hi, v_lo, p0, p_bytes, merge_o, merge_m, merge_l, bars, total;
    __host__ __device__ AttnWgLayout(int dp, int dvc, int bk) {
        const int qb = kAttnQ * dp * 2;
        q_hi = 0;
        q_lo = qb;
        stage0 = 2 * qb;
        const int kb = bk * dp * 2, vb = bk * dvc * 2;
        k_lo = kb;
        v_hi = 2 * kb;
        v_lo = 2 * kb + vb;
        stage_bytes = (2 * kb + 2 * vb + 127) / 128 * 128;
        p_bytes = 2 * kAttnQ * bk * 2;                     // hi then lo plane of one warpgroup's P
        p0 = (stage0 + kStagesKV * stage_bytes + 1023) / 1024 * 1024;   // [2] buffers, 1024-aligned (swizzle)
        merge_o = p0 + 2 * p_bytes;                      // [128][dvc] floats of warpgroup 1
        merge_m = merge_o + kAttnQ * dvc * 4;            // [128] floats
        merge_l = merge_m + kAttnQ * 4;                  // [128] doubles
        bars = merge_l + kAttnQ * 8;
        total = bars + 512;
    }
};

// Tensor-memory columns an allocation takes: a power of two, at least 32.
__host__ __device__ constexpr int tmem_columns(int used) {
    return used <= 32 ? 32 : used <= 64 ? 64 : used <= 128 ? 128 : used <= 256 ? 256 : 512;
}

template <int BK, int NSC, int DVC>
__global__ void __launch_bounds__(kAttnThreads, 1) attention_wg_kernel(const AttnArgs a) {
    constexpr int OCH = DVC / 16;
    constexpr int kCols = tmem_columns(2 * NSC * BK + 2 * DVC);
    // P (the A operand of P V) in the 128-byte swizzle when a row of it is 128 bytes (64 keys): the
    // tensor core reads swizzled rows at full shared-memory width, no-swizzle core matrices slower.
    constexpr bool kPSwizzle = BK == 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const AttnWgLayout L(a.dp, DVC, BK);
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [3]
    uint64_t* kv_empty = kv_full + kStagesKV;                        // [3]
    uint64_t* q_full = kv_empty + kStagesKV;
    uint64_t* s_full = q_full + 1;    // [2] per S buffer (block parity)
    uint64_t* p_full = s_full + 2;    // [2] per warpgroup
    uint64_t* o_full = p_full + 2;    // [2] per warpgroup
    uint64_t* merged = o_full + 2;
    uint64_t* drain = merged + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* merge_o = reinterpret_cast<float*>(smem + L.merge_o);
    float* merge_m = reinterpret_cast<float*>(smem + L.merge_m);
    double* merge_l = reinterpret_cast<double*>(smem + L.merge_l);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kAttnQ;
    const int head = blockIdx.y / a.dv_chunks;
    const int dv0 = (blockIdx.y - head * a.dv_chunks) * DVC;
    const int batch = blockIdx.z;
    const int khead = head / (a.h / a.hk);
    const int nblk = (a.lk + BK - 1) / BK;
    constexpr int sbuf = NSC * BK;                    // tensor-memory columns of one S buffer
    const uint32_t base = smem_u32(smem);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesKV; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&o_full[i], 1);
        }
        mbar_init(merged, 4);
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto t_o = [&](int wg) { return tmem + 2 * sbuf + wg * DVC; };

    if (warp == 0) {
        // ------------------------------------------------ bulk-copy producer
        if (lane == 0) {
            const uint32_t qbytes = kAttnQ * a.dp * 2;
            const uint32_t kbytes = BK * a.dp * 2, vbytes = BK * DVC * 2;
            const uint8_t* qt = a.qs + (static_cast<long long>(batch * a.h + head) * a.ntq + blockIdx.x) * qbytes;
            mbar_arrive_expect_tx(q_full, 2 * qbytes);
            bulk_load(smem + L.q_hi, qt, qbytes, q_full);
            bulk_load(smem + L.q_lo, qt + a.q_plane, qbytes, q_full);
            const long long ktile0 = static_cast<long long>(batch * a.hk + khead) * a.ntk;
            int issued = 0;
            for (int j = 0; j < nblk; ++j) {
                const int s = j % kStagesKV;
                if (!mbar_wait(&kv_empty[s], ((j / kStagesKV) & 1) ^ 1, abort, a.err)) break;
                uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kbytes + 2 * vbytes);
                const uint8_t* kt = a.ks + (ktile0 + j) * kbytes;
                const uint8_t* vt = a.vs + (ktile0 + j) * static_cast<long long>(BK) * a.dvs * 2 +
                                    static_cast<long long>(dv0 / 8) * BK * 16;
                bulk_load(st, kt, kbytes, &kv_full[s]);
                bulk_load(st + L.k_lo, kt + a.k_plane, kbytes, &kv_full[s]);
                bulk_load(st + L.v_hi, vt, vbytes, &kv_full[s]);
                bulk_load(st + L.v_lo, vt + a.v_plane, vbytes, &kv_full[s]);
                ++issued;
            }
            if (*abort) {
                mbar_wait_quiet(q_full, 0, 100000000ull);
                for (int j = (issued > kStagesKV ? issued - kStagesKV : 0); j < issued; ++j)
                    mbar_wait_quiet(&kv_full[j % kStagesKV], (j / kStagesKV) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_f16_f32(kAttnQ, BK);
            const uint32_t id_pv = idesc_f16_f32_bmajor(kAttnQ, DVC, 1);
            const uint32_t q_lbo = kAttnQ * 16, k_lbo = BK * 16, kv_sbo = 128, p_sbo = BK * 16;
            auto issue_s = [&](int j) {
                const int s = j % kStagesKV;
                const uint32_t st = base + L.stage0 + s * L.stage_bytes;
                const uint32_t sb = tmem + (j & 1) * sbuf;
                // The lo products into the first accumulator, ...
                for (int kk = 0; kk < a.dp / 16; ++kk) {
                    const uint64_t qh = desc_noswizzle(base + L.q_hi + kk * 2 * q_lbo, q_lbo, 128);
                    const uint64_t ql = desc_noswizzle(base + L.q_lo + kk * 2 * q_lbo, q_lbo, 128);
                    const uint64_t kh = desc_noswizzle(st + kk * 2 * k_lbo, k_lbo, kv_sbo);
                    const uint64_t kl = desc_noswizzle(st + L.k_lo + kk * 2 * k_lbo, k_lbo, kv_sbo);
                    mma_f16(sb, qh, kl, id_s, kk > 0 ? 1u : 0u);
                    mma_f16(sb, ql, kh, id_s, 1u);
                }
                // ... then hi.hi, 64 dims an accumulator, the first scaling the lo sum by 2^-11.
                for (int kk = 0; kk < a.dp / 16; ++kk) {
                    const uint64_t qh = desc_noswizzle(base + L.q_hi + kk * 2 * q_lbo, q_lbo, 128);
                    const uint64_t kh = desc_noswizzle(st + kk * 2 * k_lbo, k_lbo, kv_sbo);
                    if (kk == 0) mma_f16_scale_lo(sb, qh, kh, id_s);
                    else mma_f16(sb + (kk >> 2) * BK, qh, kh, id_s, (kk & 3) ? 1u : 0u);
                }
                mma_commit(&s_full[j & 1]);
            };
            bool ok = mbar_wait(q_full, 0, abort, a.err);
            if (ok) ok = mbar_wait(&kv_full[0], 0, abort, a.err);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < nblk && ok; ++j) {
                // S of the next block into the other buffer (the warpgroup that read it last published P).
                if (j + 1 < nblk) {
                    const int s1 = (j + 1) % kStagesKV;
                    if (!mbar_wait(&kv_full[s1], ((j + 1) / kStagesKV) & 1, abort, a.err)) { ok = false; break; }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                // P V of this block once its warpgroup published P (it drained its output first).
                const int wg = j & 1;
                if (!mbar_wait(&p_full[wg], (j >> 1) & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                const int s = j % kStagesKV;
                const uint32_t st = base + L.stage0 + s * L.stage_bytes;
                const uint32_t pb = base + L.p0 + wg * L.p_bytes;
                // The block's P V into the warpgroup's fresh accumulator: lo products, then hi.hi.
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ph = kPSwizzle ? desc_kmajor_sw128(pb + kk * 32) : desc_noswizzle(pb + kk * 256, 128, p_sbo);
                    const uint64_t pl = kPSwizzle ? desc_kmajor_sw128(pb + kAttnQ * BK * 2 + kk * 32)
                                                  : desc_noswizzle(pb + kAttnQ * BK * 2 + kk * 256, 128, p_sbo);
                    const uint64_t vh = desc_noswizzle(st + L.v_hi + kk * 256, 128, BK * 16);
                    const uint64_t vl = desc_noswizzle(st + L.v_lo + kk * 256, 128, BK * 16);
                    mma_f16(t_o(wg), ph, vl, id_pv, kk > 0 ? 1u : 0u);
                    mma_f16(t_o(wg), pl, vh, id_pv, 1u);
                }
                for (int kk = 0; kk < BK / 16; ++kk) {
                    const uint64_t ph = kPSwizzle ? desc_kmajor_sw128(pb + kk * 32) : desc_noswizzle(pb + kk * 256, 128, p_sbo);
                    const uint64_t vh = desc_noswizzle(st + L.v_hi + kk * 256, 128, BK * 16);
                    if (kk == 0) mma_f16_scale_lo(t_o(wg), ph, vh, id_pv);
                    else mma_f16(t_o(wg), ph, vh, id_pv, 1u);
                }
                mma_commit(&o_full[wg]);
                mma_commit(&kv_empty[s]);
            }
            if (!ok) {
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------ softmax warpgroups
        const int wg = (warp - 2) >> 2;  // 0: blocks 0, 2, ...; 1: blocks 1, 3, ...
        const int q = warp & 3;          // lane quarter: the rows this warp owns
        const int r = q * 32 + lane;     // query row of the tile
        const int qi = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const uint32_t pbuf = base + L.p0 + wg * L.p_bytes;
        float m_ref = -INFINITY;
        double l = 0.0;
        float o[DVC];
#pragma unroll
        for (int i = 0; i < DVC; ++i) o[i] = 0.0f;
        // All lanes wait together; the warp's verdict is unanimous.
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.err) ? 1 : 0) != 0;
        };
        // o += (the warpgroup's last block product, normalised to m_ref).
        auto take = [&](int jb) {
            if (!warp_wait(&o_full[wg], (jb >> 1) & 1)) return false;
            tc_fence_after();
#pragma unroll
            for (int ch = 0; ch < OCH; ++ch) {
                float oh[16];
                tmem_ld16(t_o(wg) + lane_off + ch * 16, oh);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 16; ++i) o[ch * 16 + i] += oh[i];
            }
            return true;
        };
        bool ok = true;
        bool first = true;
        for (int j = wg; j < nblk; j += 2) {
            if (!warp_wait(&s_full[wg], (j >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sb = tmem + wg * sbuf + lane_off;
            float s[BK];
            // The block's scores, every 16 keys' load issued before the one wait.
#pragma unroll
            for (int c = 0; c < BK; c += 16) tmem_ld16(sb + c, *reinterpret_cast<float(*)[16]>(s + c));
            if (NSC > 1) {
                float h1[BK];
#pragma unroll
                for (int c = 0; c < BK; c += 16) tmem_ld16(sb + BK + c, *reinterpret_cast<float(*)[16]>(h1 + c));
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < BK; ++i) s[i] += h1[i];
            } else {
                tmem_ld_wait();
            }
            const int valid = min(BK, a.lk - j * BK);
            const bool full = valid == BK;
            float bmax = -INFINITY;
            if (full) {
#pragma unroll
                for (int i = 0; i < BK; ++i) bmax = fmaxf(bmax, s[i]);
            } else {
#pragma unroll
                for (int i = 0; i < BK; ++i)
                    if (i < valid) bmax = fmaxf(bmax, s[i]);
            }
            bmax *= a.scale2;
            // The block product of two blocks ago into the registers: its P buffer
            // and output accumulator are then free.
            if (j >= 2 && !take(j - 2)) { ok = false; break; }
            if (first) {
                m_ref = bmax;
                first = false;
            } else if (bmax > m_ref + kRescaleAbove) {
                const float factor = ex2(m_ref - bmax);
                m_ref = bmax;
#pragma unroll
                for (int i = 0; i < DVC; ++i) o[i] *= factor;
                l *= static_cast<double>(factor);
            }
            // The weights (0 past the last key), their pairwise sum, and P in
            // the UMMA no-swizzle K-major layout: row r, 8 keys per 16-byte chunk.
            if (full) {
#pragma unroll
                for (int i = 0; i < BK; ++i) s[i] = ex2(fmaf(s[i], a.scale2, -m_ref));
            } else {
#pragma unroll
                for (int i = 0; i < BK; ++i) s[i] = i < valid ? ex2(fmaf(s[i], a.scale2, -m_ref)) : 0.0f;
            }
#pragma unroll
            for (int c = 0; c < BK / 8; ++c) {
                float p8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) p8[i] = s[c * 8 + i];
                uint4 h4, l4;
                split8_inrange(p8, h4, l4);
                // Rows of 64 keys (128 bytes) in the 128-byte swizzle (16-byte chunk c of row r at
                // chunk c ^ (r mod 8)), else the no-swizzle core matrices of 8 rows x 16 bytes.
                const uint32_t off = kPSwizzle ? static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 +
                                                                       ((c ^ (r & 7)) * 16))
                                               : static_cast<uint32_t>((r >> 3) * (BK * 16) + c * 128 + (r & 7) * 16);
                st_shared_v4(pbuf + off, h4);
                st_shared_v4(pbuf + kAttnQ * BK * 2 + off, l4);
            }
#pragma unroll
            for (int w = BK / 2; w > 0; w >>= 1) {
#pragma unroll
                for (int i = 0; i < w; ++i) s[i] += s[i + w];
            }
            l += static_cast<double>(s[0]);
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[wg]);
        }
        // The warpgroup's last block product.
        if (ok) {
            const int last = nblk - 1 - ((nblk - 1 - wg) & 1);   // the last j with j % 2 == wg
            if (last >= wg && !take(last)) ok = false;
        }
        // Merge: warpgroup 1 hands its stream to warpgroup 0 through shared memory.
        if (wg == 1) {
            merge_m[r] = m_ref;
            merge_l[r] = l;
#pragma unroll
            for (int i = 0; i < DVC; ++i) merge_o[r * DVC + ((i + r) % DVC)] = o[i];
            __threadfence_block();
            __syncwarp();
            if (lane == 0) mbar_arrive(merged);
        } else if (ok && mbar_wait(merged, 0, abort, a.err)) {
            const float m1 = merge_m[r];
            const float m = fmaxf(m_ref, m1);
            const float f0 = m_ref == -INFINITY ? 0.0f : ex2(m_ref - m);
            const float f1 = m1 == -INFINITY ? 0.0f : ex2(m1 - m);
            const double total = l * static_cast<double>(f0) + merge_l[r] * static_cast<double>(f1);
#pragma unroll
            for (int i = 0; i < DVC; ++i) o[i] = o[i] * f0 + merge_o[r * DVC + ((i + r) % DVC)] * f1;
            if (qi < a.lq) {
                const float recip = static_cast<float>(1.0 / total);
#pragma unroll
                for (int i = 0; i < DVC; ++i) o[i] *= recip;
                ChainRow cr;
                row_offsets(a.chain, cr, 0, head, qi, batch);
                const int ncols = min(DVC, a.dv - dv0);
#pragma unroll
                for (int c = 0; c < DVC; c += 16) apply_chain_cols<0, 16>(a.chain, cr, o + c, dv0 + c, a.dv - 1);
                float* orow = a.out + static_cast<long long>(head) * a.onb[1] + static_cast<long long>(qi) * a.onb[2] +
                              static_cast<long long>(batch) * a.onb[3];
                if (a.onb[0] == 1 && ncols % 4 == 0 && ((reinterpret_cast<uintptr_t>(orow + dv0)) & 15) == 0) {
                    // Whole float4s up to the value dims the row holds (40 of a 48-wide chunk, say).
#pragma unroll
                    for (int i = 0; i < DVC; i += 4)
                        if (i < ncols)
                            *reinterpret_cast<float4*>(orow + dv0 + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
                } else {
#pragma unroll
                    for (int i = 0; i < DVC; ++i)
                        if (i < ncols) orow[static_cast<long long>(dv0 + i) * a.onb[0]] = o[i];
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
}

// ---- both A operands in tensor memory, two query tiles a CTA -------------------
//
// For heads up to 64 dims (value chunks up to 64).  Q and P, the A operands of
// the two products, live in tensor memory, so the tensor core reads only K and
// V from shared memory (A in shared memory would take most of its ~128 B/cycle
// at these widths).  A CTA holds two tiles of 128 queries of one head, which
// share every K/V stage, so each key block crosses L2 once per 256 queries.
// Products are issued by three threads: one for both tiles' S = Q K^T, one per
// tile for O = P V.  One issuing thread's products run back to back at ~47-65
// cycles each whatever their width up to N = 64, and products of different
// issuing threads overlap (measured, M = 128, K = 16, A in tensor memory: one
// issuer 3000-4000 FLOP/cycle, two 6000-8000, four 8100-8170 -- the tensor
// pipe's peak), so the S products of the next block run beside this block's
// P V products.
//
// Warp 0 loads the K/V stages; warp 1 issues both tiles' S products; warps 2
// and 3 issue tile 0's and tile 1's P V products; warps 4-7 and 8-11 are the
// softmax warpgroups of tiles 0 and 1 (one query row a thread): they write
// their Q rows into tensor memory, then per block of 64 keys read S, take the
// weights against the reference maximum (raised as in the kernels above),
// write P -- the FP16 pairs of split8_inrange, so the same products -- over S's
// columns, and add the previous block's P V into their registers before
// publishing P.  S(j + 2) reuses the buffer of P(j): its issue waits for that
// P V to complete.  (Buffers of their own for S and P, or two threads a row
// sharing a block's keys, measured slower: both made the softmax warps of an
// SM sub-partition reach their exponentials together.)
// Tensor memory (columns), tile t at 256 t: S / P buffers [0, 64) and [64, 128)
// (P hi in the first 32 columns of a buffer, lo in the next 32); O [128, 128 +
// DVC); Q hi then lo from 128 + DVC, DP / 2 columns each.
constexpr int kAttnTmThreads = 384;
constexpr int kAttnTmBK = 64;
constexpr int kAttnTmMaxStages = 8;

// Q in tensor memory when a tile's S / P buffers, O and Q fit its 256 columns;
// else (heads of 80 dims) in shared memory, the S products reading it there.
__host__ __device__ constexpr bool attention_tm_q_in_tmem(int dp, int dvc) { return 2 * kAttnTmBK + dvc + dp <= 256; }

struct AttnTmLayout {
    int q_plane = 0, stage0 = 0, stage_bytes = 0, k_lo = 0, v_hi = 0, v_lo = 0, stages = 0, bars = 0, total = 0;
    __host__ __device__ constexpr AttnTmLayout(int dp, int dvc) {
        q_plane = attention_tm_q_in_tmem(dp, dvc) ? 0 : kAttnQ * dp * 2;
        stage0 = 4 * q_plane;  // tile 0 hi, lo, tile 1 hi, lo
        const int kb = kAttnTmBK * dp * 2, vb = kAttnTmBK * dvc * 2;
        k_lo = kb;
        v_hi = 2 * kb;
        v_lo = 2 * kb + vb;
        stage_bytes = (2 * kb + 2 * vb + 127) / 128 * 128;
        const int fit = (200 * 1024 - stage0) / stage_bytes;
        stages = fit < kAttnTmMaxStages ? fit : kAttnTmMaxStages;
        bars = stage0 + stages * stage_bytes;
        total = bars + 512;
    }
};

__host__ __device__ constexpr bool attention_tm_fits(int dp, int dvc) {
    return dp == dvc && 2 * kAttnTmBK + dvc <= 256 && dp <= 80 && AttnTmLayout(dp, dvc).stages >= 2 &&
           AttnTmLayout(dp, dvc).total + 128 <= 227 * 1024;
}

// The barriers of one query tile.
struct AttnTmTile {
    uint64_t* q_full;   // its Q rows are in tensor memory (4 warp arrivals)
    uint64_t* s_full;   // [2] S(j) complete, per buffer
    uint64_t* p_full;   // P(j) written and the previous product taken (4 warp arrivals)
    uint64_t* o_full;   // P V (j) complete
    uint64_t* pv_done;  // [2] P V (j) complete, per buffer: S(j + 2) may overwrite P(j)
};

// max (scale >= 0) or min (scale < 0) of a block's scores: the one whose
// scaled value is the block's largest.
template <bool kMin>
__device__ __forceinline__ float extreme64(const float (&s)[kAttnTmBK]) {
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = s[i];
#pragma unroll
    for (int i = 4; i < kAttnTmBK; i += 8) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (i + 2 * t + 1 < kAttnTmBK)
                e[t] = kMin ? -fmax3(-e[t], -s[i + 2 * t], -s[i + 2 * t + 1]) : fmax3(e[t], s[i + 2 * t], s[i + 2 * t + 1]);
        }
    }
    return kMin ? fminf(fminf(e[0], e[1]), fminf(e[2], e[3])) : fmaxf(fmaxf(e[0], e[1]), fmaxf(e[2], e[3]));
}

// A softmax warpgroup of attention_tm_kernel (thread = query row of tile `qt`).
// `tb` is the tile's tensor memory; lane quarter from the warp index.
template <int DP, int DVC>
__device__ __forceinline__ void attention_tm_softmax(const AttnArgs& a, uint32_t tb, const AttnTmTile& T,
                                                     volatile int* abort, int qt, int head, int dv0, int batch,
                                                     int nblk) {
    constexpr int BK = kAttnTmBK;
    constexpr int OCH = DVC / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = warp & 3;  // lane quarter of tensor memory this warp may access
    const int r = q * 32 + lane;
    const int qi = qt * kAttnQ + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t t_o = tb + 2 * BK;
    const uint32_t t_qh = t_o + DVC;
    const uint32_t t_ql = t_qh + DP / 2;
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, a.err) ? 1 : 0) != 0;
    };

    // Row r of the Q tile (hi, then lo: 16-byte chunks of 8 dims, [chunk][row][8]) into tensor memory.
    if constexpr (attention_tm_q_in_tmem(DP, DVC)) {
        const uint8_t* qtile = a.qs + (static_cast<long long>(batch * a.h + head) * a.ntq + qt) * (kAttnQ * DP * 2);
#pragma unroll
        for (int plane = 0; plane < 2; ++plane) {
            const uint8_t* src = qtile + plane * a.q_plane;
            const uint32_t dst = (plane ? t_ql : t_qh) + lane_off;
#pragma unroll
            for (int c0 = 0; c0 < DP / 8; c0 += 2) {
                const uint4 h0 = __ldg(reinterpret_cast<const uint4*>(src + (c0 * kAttnQ + r) * 16));
                const uint4 h1 = __ldg(reinterpret_cast<const uint4*>(src + ((c0 + 1) * kAttnQ + r) * 16));
                const uint32_t w[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                tmem_st8_bits(dst + c0 * 4, w);
            }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(T.q_full);
    }

    const bool neg = a.scale2 < 0.0f;
    const float masked = neg ? INFINITY : -INFINITY;
    const uint64_t scale2 = pack2(a.scale2, a.scale2);
    float m_ref = -INFINITY;
    double l = 0.0;
    float o[DVC];
#pragma unroll
    for (int i = 0; i < DVC; ++i) o[i] = 0.0f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
        if (!warp_wait(&T.s_full[j & 1], (j >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sb = tb + (j & 1) * BK + lane_off;
        float s[BK];
        tmem_ld32(sb, *reinterpret_cast<float(*)[32]>(s));
        tmem_ld32(sb + 32, *reinterpret_cast<float(*)[32]>(s + 32));
        tmem_ld_wait();
        const int valid = a.lk - j * BK;
        if (valid < BK) {
#pragma unroll
            for (int i = 0; i < BK; ++i)
                if (i >= valid) s[i] = masked;
        }
        const float bmax = (neg ? extreme64<true>(s) : extreme64<false>(s)) * a.scale2;
        float factor = 1.0f;
        if (j == 0) {
            m_ref = bmax;
        } else if (bmax > m_ref + kRescaleAbove) {
            factor = ex2(m_ref - bmax);
            m_ref = bmax;
        }
        // The weights 2^(s scale2 - m), two keys a packed FMA.
        const uint64_t nm = pack2(-m_ref, -m_ref);
#pragma unroll
        for (int i = 0; i < BK; i += 2) {
            float x0, x1;
            unpack2(ffma2(pack2(s[i], s[i + 1]), scale2, nm), x0, x1);
            s[i] = ex2(x0);
            s[i + 1] = ex2(x1);
        }
        // P over S's columns: hi pairs in columns [0, 32), lo pairs in [32, 64).
#pragma unroll
        for (int c = 0; c < BK / 16; ++c) {
            uint32_t ph[8], pl[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) split_weights2(s[c * 16 + 2 * w], s[c * 16 + 2 * w + 1], ph[w], pl[w]);
            tmem_st8_bits(sb + c * 8, ph);
            tmem_st8_bits(sb + 32 + c * 8, pl);
        }
        // The block's weights summed pairwise, two lanes of pairs at a time.
        uint64_t sum2[BK / 4];
#pragma unroll
        for (int i = 0; i < BK / 4; ++i)
            sum2[i] = fadd2(pack2(s[2 * i], s[2 * i + 1]), pack2(s[BK / 2 + 2 * i], s[BK / 2 + 2 * i + 1]));
#pragma unroll
        for (int w = BK / 8; w > 0; w >>= 1) {
#pragma unroll
            for (int i = 0; i < w; ++i) sum2[i] = fadd2(sum2[i], sum2[i + w]);
        }
        float b0, b1;
        unpack2(sum2[0], b0, b1);
        l = l * static_cast<double>(factor) + static_cast<double>(b0 + b1);
        // The previous block's product (taken against the old maximum) into the registers: its
        // accumulator is then free for this block's.
        if (j >= 1) {
            if (!warp_wait(T.o_full, (j - 1) & 1)) { ok = false; break; }
            tc_fence_after();
            float oh[DVC];
#pragma unroll
            for (int ch = 0; ch < OCH; ++ch)
                tmem_ld16(t_o + lane_off + ch * 16, *reinterpret_cast<float(*)[16]>(oh + ch * 16));
            tmem_ld_wait();
            // Packed: two dims an instruction, each rounded as the scalar form.
            add_packed<DVC>(o, oh);
            if (factor != 1.0f) {
                const uint64_t f2 = pack2(factor, factor);
#pragma unroll
                for (int i = 0; i < DVC; i += 2) {
                    float x0, x1;
                    unpack2(fmul2(pack2(o[i], o[i + 1]), f2), x0, x1);
                    o[i] = x0;
                    o[i + 1] = x1;
                }
            }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(T.p_full);
    }
    if (!ok) return;
    if (!warp_wait(T.o_full, (nblk - 1) & 1)) return;
    tc_fence_after();
    {
        float oh[DVC];
#pragma unroll
        for (int ch = 0; ch < OCH; ++ch) tmem_ld16(t_o + lane_off + ch * 16, *reinterpret_cast<float(*)[16]>(oh + ch * 16));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < DVC; ++i) o[i] += oh[i];
    }
    if (qi >= a.lq) return;
    const float recip = static_cast<float>(1.0 / l);
#pragma unroll
    for (int i = 0; i < DVC; ++i) o[i] *= recip;
    ChainRow cr;
    row_offsets(a.chain, cr, 0, head, qi, batch);
#pragma unroll
    for (int c = 0; c < DVC; c += 16) apply_chain_cols<0, 16>(a.chain, cr, o + c, dv0 + c, a.dv - 1);
    const int ncols = min(DVC, a.dv - dv0);
    float* orow = a.out + static_cast<long long>(head) * a.onb[1] + static_cast<long long>(qi) * a.onb[2] +
                  static_cast<long long>(batch) * a.onb[3];
    if (a.onb[0] == 1 && ncols % 4 == 0 && ((reinterpret_cast<uintptr_t>(orow + dv0)) & 15) == 0) {
#pragma unroll
        for (int i = 0; i < DVC; i += 4)
            if (i < ncols) *reinterpret_cast<float4*>(orow + dv0 + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < DVC; ++i)
            if (i < ncols) orow[static_cast<long long>(dv0 + i) * a.onb[0]] = o[i];
    }
}

template <int DP, int DVC>
__global__ void __launch_bounds__(kAttnTmThreads, 1) attention_tm_kernel(const AttnArgs a) {
    constexpr int BK = kAttnTmBK;
    constexpr AttnTmLayout L(DP, DVC);
    constexpr int stages = L.stages;
    constexpr bool kQt = attention_tm_q_in_tmem(DP, DVC);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint64_t* kv_full = reinterpret_cast<uint64_t*>(smem + L.bars);  // [stages]
    uint64_t* kv_empty = kv_full + kAttnTmMaxStages;                 // [stages]
    uint64_t* tile_bars = kv_empty + kAttnTmMaxStages;               // [2][7]
    uint64_t* drain = tile_bars + 14;                                // [3] per issuing thread
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 3);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt0 = blockIdx.x * 2;                   // first query tile
    const int ntile = qt0 + 1 < a.ntq ? 2 : 1;        // the last CTA of a head may hold one
    const int head = blockIdx.y / a.dv_chunks;
    const int dv0 = (blockIdx.y - head * a.dv_chunks) * DVC;
    const int batch = blockIdx.z;
    const int khead = head / (a.h / a.hk);
    const int nblk = (a.lk + BK - 1) / BK;
    const uint32_t base = smem_u32(smem);
    AttnTmTile tiles[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        uint64_t* b = tile_bars + 7 * t;
        tiles[t] = AttnTmTile{b, b + 1, b + 3, b + 4, b + 5};
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], ntile);  // one release per tile's P V
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(tiles[t].q_full, kQt ? 4 : 1);  // the softmax warps' stores, or the producer's copies
            mbar_init(&tiles[t].s_full[0], 1);
            mbar_init(&tiles[t].s_full[1], 1);
            mbar_init(tiles[t].p_full, 4);
            mbar_init(tiles[t].o_full, 1);
            mbar_init(&tiles[t].pv_done[0], 1);
            mbar_init(&tiles[t].pv_done[1], 1);
        }
        for (int i = 0; i < 3; ++i) mbar_init(&drain[i], 1);
        *abort = 0;
        fence_barrier_init();
    }
    // The dims past the head's last 8-dim chunk are zero in every stage: written once here, never loaded.
    const int kch = (a.d + 7) / 8;
    const int vch = (min(DVC, a.dv - dv0) + 7) / 8;
    {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        constexpr int kpl = BK * DP * 2, vpl = BK * DVC * 2;  // bytes of a plane
        const int kpad = kpl - kch * BK * 16, vpad = vpl - vch * BK * 16;
        for (int s = 0; s < stages; ++s) {
            uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
            for (int o = threadIdx.x * 16; o < kpad; o += kAttnTmThreads * 16) {
                *reinterpret_cast<uint4*>(st + kch * BK * 16 + o) = z;
                *reinterpret_cast<uint4*>(st + L.k_lo + kch * BK * 16 + o) = z;
            }
            for (int o = threadIdx.x * 16; o < vpad; o += kAttnTmThreads * 16) {
                *reinterpret_cast<uint4*>(st + L.v_hi + vch * BK * 16 + o) = z;
                *reinterpret_cast<uint4*>(st + L.v_lo + vch * BK * 16 + o) = z;
            }
        }
        fence_proxy_async_smem();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t id_s = idesc_f16_f32(kAttnQ, BK);
    constexpr uint32_t id_pv = idesc_f16_f32_bmajor(kAttnQ, DVC, 1);

    if (warp == 0) {
        // ------------------------------------------------ bulk-copy producer
        if (lane == 0) {
            constexpr uint32_t kbytes = BK * DP * 2;                     // a stored K plane tile
            const uint32_t kload = kch * BK * 16, vload = vch * BK * 16;  // its dims that are loaded
            const long long ktile0 = static_cast<long long>(batch * a.hk + khead) * a.ntk;
            if constexpr (!kQt) {
                // Both tiles' Q planes into shared memory, completing on tile 0's barrier.
                mbar_arrive_expect_tx(tiles[0].q_full, ntile * 2 * L.q_plane);
                for (int t = 0; t < ntile; ++t) {
                    const uint8_t* qsrc = a.qs + (static_cast<long long>(batch * a.h + head) * a.ntq + qt0 + t) * L.q_plane;
                    bulk_load(smem + 2 * t * L.q_plane, qsrc, L.q_plane, tiles[0].q_full);
                    bulk_load(smem + (2 * t + 1) * L.q_plane, qsrc + a.q_plane, L.q_plane, tiles[0].q_full);
                }
            }
            int issued = 0;
            for (int j = 0; j < nblk; ++j) {
                const int s = j % stages;
                if (!mbar_wait(&kv_empty[s], ((j / stages) & 1) ^ 1, abort, a.err)) break;
                uint8_t* st = smem + L.stage0 + s * L.stage_bytes;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kload + 2 * vload);
                const uint8_t* kt = a.ks + (ktile0 + j) * kbytes;
                const uint8_t* vt = a.vs + (ktile0 + j) * static_cast<long long>(BK) * a.dvs * 2 +
                                    static_cast<long long>(dv0 / 8) * BK * 16;
                bulk_load(st, kt, kload, &kv_full[s]);
                bulk_load(st + L.k_lo, kt + a.k_plane, kload, &kv_full[s]);
                bulk_load(st + L.v_hi, vt, vload, &kv_full[s]);
                bulk_load(st + L.v_lo, vt + a.v_plane, vload, &kv_full[s]);
                ++issued;
            }
            if (*abort) {
                if (!kQt) mbar_wait_quiet(tiles[0].q_full, 0, 100000000ull);
                for (int j = (issued > stages ? issued - stages : 0); j < issued; ++j)
                    mbar_wait_quiet(&kv_full[j % stages], (j / stages) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ S = Q K^T of both tiles
        if (lane == 0) {
            constexpr uint32_t k_lbo = BK * 16;
            // Descriptors of stage 0; another stage's, and another k-step's, add their byte offset / 16 to
            // the start-address field (shared addresses stay below 256 KB, so the field does not carry).
            const uint64_t dk0 = desc_noswizzle(base + L.stage0, k_lbo, 128);
            constexpr uint32_t q_lbo = kAttnQ * 16;
            const uint64_t dq0 = desc_noswizzle(base, q_lbo, 128);   // Q in shared memory: tile 0 hi
            bool ok = true;
            for (int t = 0; t < (kQt ? ntile : 1) && ok; ++t) ok = mbar_wait(tiles[t].q_full, 0, abort, a.err);
            for (int j = 0; j < nblk && ok; ++j) {
                if (!mbar_wait(&kv_full[j % stages], (j / stages) & 1, abort, a.err)) { ok = false; break; }
                const uint64_t dk = dk0 + static_cast<uint64_t>(((j % stages) * L.stage_bytes) >> 4);
                for (int t = 0; t < ntile; ++t) {
                    // Buffer j & 1 holds P(j - 2) until that block's P V completes.
                    if (j >= 2 && !mbar_wait(&tiles[t].pv_done[j & 1], ((j - 2) >> 1) & 1, abort, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t tb = tmem + 256 * t;
                    const uint32_t sb = tb + (j & 1) * BK;
                    // The lo products (Q.K lo, Q lo.K, each carrying 2^11) first, then Q.K hi with the
                    // input scale 2^-11.
                    if constexpr (kQt) {
                        const uint32_t t_qh = tb + 2 * BK + DVC, t_ql = t_qh + DP / 2;
#pragma unroll
                        for (int kk = 0; kk < DP / 16; ++kk) {
                            mma_f16_ta(sb, t_qh + kk * 8, dk + ((L.k_lo + kk * 2 * k_lbo) >> 4), id_s, kk > 0 ? 1u : 0u);
                            mma_f16_ta(sb, t_ql + kk * 8, dk + ((kk * 2 * k_lbo) >> 4), id_s, 1u);
                        }
#pragma unroll
                        for (int kk = 0; kk < DP / 16; ++kk) {
                            if (kk == 0) mma_f16_ta_scale_lo(sb, t_qh, dk, id_s);
                            else mma_f16_ta(sb, t_qh + kk * 8, dk + ((kk * 2 * k_lbo) >> 4), id_s, 1u);
                        }
                    } else {
                        const uint64_t dqh = dq0 + ((2 * t * L.q_plane) >> 4), dql = dqh + (L.q_plane >> 4);
#pragma unroll
                        for (int kk = 0; kk < DP / 16; ++kk) {
                            mma_f16(sb, dqh + ((kk * 2 * q_lbo) >> 4), dk + ((L.k_lo + kk * 2 * k_lbo) >> 4), id_s,
                                    kk > 0 ? 1u : 0u);
                            mma_f16(sb, dql + ((kk * 2 * q_lbo) >> 4), dk + ((kk * 2 * k_lbo) >> 4), id_s, 1u);
                        }
#pragma unroll
                        for (int kk = 0; kk < DP / 16; ++kk) {
                            if (kk == 0) mma_f16_scale_lo(sb, dqh, dk, id_s);
                            else mma_f16(sb, dqh + ((kk * 2 * q_lbo) >> 4), dk + ((kk * 2 * k_lbo) >> 4), id_s, 1u);
                        }
                    }
                    mma_commit(&tiles[t].s_full[j & 1]);
                }
            }
            if (!ok) {
                mma_commit(&drain[0]);
                mbar_wait_quiet(&drain[0], 0, 100000000ull);
            }
        }
    } else if (warp < 4) {
        // ------------------------------------------------ O = P V of tile warp - 2
        const int t = warp - 2;
        if (lane == 0 && t < ntile) {
            const AttnTmTile& T = tiles[t];
            const uint32_t tb = tmem + 256 * t;
            const uint32_t t_o = tb + 2 * BK;
            const uint64_t dv0d = desc_noswizzle(base + L.stage0 + L.v_hi, 128, BK * 16);
            constexpr uint32_t vlo = (L.v_lo - L.v_hi) >> 4;
            bool ok = true;
            for (int j = 0; j < nblk; ++j) {
                if (!mbar_wait(T.p_full, j & 1, abort, a.err)) { ok = false; break; }
                tc_fence_after();
                const int s = j % stages;
                const uint64_t dvh = dv0d + static_cast<uint64_t>((s * L.stage_bytes) >> 4);
                const uint32_t pb = tb + (j & 1) * BK;
                // hi.V lo and lo.V hi (each carrying 2^11) first, then hi.V hi with the input scale 2^-11.
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    mma_f16_ta(t_o, pb + kk * 8, dvh + vlo + kk * 16, id_pv, kk > 0 ? 1u : 0u);
                    mma_f16_ta(t_o, pb + 32 + kk * 8, dvh + kk * 16, id_pv, 1u);
                }
#pragma unroll
                for (int kk = 0; kk < BK / 16; ++kk) {
                    if (kk == 0) mma_f16_ta_scale_lo(t_o, pb, dvh, id_pv);
                    else mma_f16_ta(t_o, pb + kk * 8, dvh + kk * 16, id_pv, 1u);
                }
                mma_commit(&kv_empty[s]);
                mma_commit(&T.pv_done[j & 1]);
                mma_commit(T.o_full);
            }
            if (!ok) {
                mma_commit(&drain[1 + t]);
                mbar_wait_quiet(&drain[1 + t], 0, 100000000ull);
            }
        }
    } else {
        const int t = (warp - 4) >> 2;
        if (t < ntile)
            attention_tm_softmax<DP, DVC>(a, tmem + 256 * t, tiles[t], abort, qt0 + t, head, dv0, batch, nblk);
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

bool floaty(const sdb_tensor* t) {
    return t && t->data && (t->type == SDB_TYPE_F32 || t->type == SDB_TYPE_F16);
}

int esize(const sdb_tensor* t) { return t->type == SDB_TYPE_F16 ? 2 : 4; }

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Splits Q, K and V into the workspace as tiles (128 queries, BK keys) and
// launches the kernel.
// Splits Q, K and V into the workspace as tiles of 128 queries / BK keys.
template <int BK, int DVC>
int prepare_tiles(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    auto dims = [](const sdb_tensor* t, long long (&ne)[4], long long (&nb)[4]) {
        const int es = t->type == SDB_TYPE_F16 ? 2 : 4;
        for (int i = 0; i < 4; ++i) {
            ne[i] = t->ne[i];
            nb[i] = t->nb[i] / es;
        }
    };
    long long qne[4], qnb[4], kne[4], knb[4], vne[4], vnb[4];
    dims(q, qne, qnb);
    dims(k, kne, knb);
    dims(v, vne, vnb);
    a.dvs = a.dv_chunks * DVC;
    a.ntq = static_cast<int>((a.lq + kAttnQ - 1) / kAttnQ);
    a.ntk = static_cast<int>((a.lk + BK - 1) / BK);
    a.q_plane = split_tiles_plane(qne, a.dp, kAttnQ);
    a.k_plane = split_tiles_plane(kne, a.dp, BK);
    a.v_plane = split_tiles_plane(vne, a.dvs, BK);
    void* ws = nullptr;
    const size_t bytes = static_cast<size_t>(2 * (a.q_plane + a.k_plane + a.v_plane) + 256);
    if (int s = workspace(st, bytes, &ws); s != SDB_OK) return s;
    uint8_t* base = static_cast<uint8_t*>(ws);
    a.qs = base;
    a.ks = base + 2 * a.q_plane;
    a.vs = base + 2 * (a.q_plane + a.k_plane);
    // Q, K and V split in one launch.
    const SplitTilesJob jobs[3] = {
        split_tiles_job(q->data, 0, qne, qnb, a.dp, kAttnQ, const_cast<uint16_t*>(reinterpret_cast<const uint16_t*>(a.qs))),
        split_tiles_job(k->data, k->type == SDB_TYPE_F16, kne, knb, a.dp, BK,
                        const_cast<uint16_t*>(reinterpret_cast<const uint16_t*>(a.ks))),
        split_tiles_job(v->data, v->type == SDB_TYPE_F16, vne, vnb, a.dvs, BK,
                        const_cast<uint16_t*>(reinterpret_cast<const uint16_t*>(a.vs)))};
    return split_tiles_many(jobs, 3, a.err, st);
}

template <int BK, int DVC, int NO>
int launch_attention(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    const AttnLayout L(a.dp, DVC, BK);
    const int smem = L.total + 1024;
    if (smem > 227 * 1024) return fail(SDB_NOT_SUPPORTED, "sdb_attention: head too wide");
    if (int s = prepare_tiles<BK, DVC>(a, q, k, v, st); s != SDB_OK) return s;
    SDB_CUDA(cudaFuncSetAttribute(attention_kernel<BK, DVC, NO>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const dim3 grid(static_cast<unsigned>((a.lq + kAttnQ - 1) / kAttnQ), static_cast<unsigned>(a.h * a.dv_chunks),
                    static_cast<unsigned>(a.b));
    attention_kernel<BK, DVC, NO><<<grid, kAttnThreads, smem, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

template <int BK, int NSC, int DVC>
int launch_attention_wg(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    const AttnWgLayout L(a.dp, DVC, BK);
    const int smem = L.total + 1024;
    if (int s = prepare_tiles<BK, DVC>(a, q, k, v, st); s != SDB_OK) return s;
    auto kern = attention_wg_kernel<BK, NSC, DVC>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const dim3 grid(static_cast<unsigned>((a.lq + kAttnQ - 1) / kAttnQ), static_cast<unsigned>(a.h * a.dv_chunks),
                    static_cast<unsigned>(a.b));
    kern<<<grid, kAttnThreads, smem, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

// Shared memory of more than half an SM's, so that no second CTA waits on an SM
// whose tensor memory the first holds.
template <int DP, int DVC>
int launch_attention_tm(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    constexpr AttnTmLayout L(DP, DVC);
    const int smem = std::max(L.total + 128, 120 * 1024);
    if (int s = prepare_tiles<kAttnTmBK, DVC>(a, q, k, v, st); s != SDB_OK) return s;
    auto kern = attention_tm_kernel<DP, DVC>;
    SDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const dim3 grid(static_cast<unsigned>((a.ntq + 1) / 2), static_cast<unsigned>(a.h * a.dv_chunks),
                    static_cast<unsigned>(a.b));
    kern<<<grid, kAttnTmThreads, smem, st>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

template <int DVC>
int launch_attention_tm(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    return launch_attention_tm<DVC, DVC>(a, q, k, v, st);
}

// The two-warpgroup kernel when its S buffers and two output accumulators fit
// tensor memory (heads up to 64 dims with 64-key blocks, up to 128 with 32).
template <int DVC>
int launch_wg(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st,
              bool* taken) {
    *taken = false;
    const int nsc = (a.dp + 63) / 64;
    auto fits = [&](int bk) {
        return 2 * nsc * bk + 2 * DVC <= 512 && AttnWgLayout(a.dp, DVC, bk).total + 1024 <= 227 * 1024;
    };
    if (nsc == 1 && fits(64)) {
        *taken = true;
        return launch_attention_wg<64, 1, DVC>(a, q, k, v, st);
    }
    if (nsc == 2 && fits(32)) {
        *taken = true;
        return launch_attention_wg<32, 2, DVC>(a, q, k, v, st);
    }
    return SDB_OK;
}

// Keys per block (64, else 32) and output buffers (two, so the softmax of a
// block overlaps the product of the one before; else one): the first choice
// whose S double buffer and output accumulators fit tensor memory.
template <int DVC>
int launch_bk(AttnArgs& a, const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, cudaStream_t st) {
    if constexpr (attention_tm_fits(DVC, DVC)) {
        if (tuning().attention_wg == 2 && a.dp == DVC) return launch_attention_tm<DVC>(a, q, k, v, st);
    }
    if (tuning().attention_wg) {
        bool taken = false;
        const int rc = launch_wg<DVC>(a, q, k, v, st, &taken);
        if (taken || rc != SDB_OK) return rc;
    }
    const int nsc = (a.dp + 63) / 64;
    auto fits = [&](int bk, int no) {
        return 2 * (nsc + 1) * bk + no * 2 * DVC <= 512 &&
               AttnLayout(a.dp, DVC, bk).total + 1024 <= 227 * 1024;
    };
    if (fits(64, 2)) return launch_attention<64, DVC, 2>(a, q, k, v, st);
    if (fits(32, 2)) return launch_attention<32, DVC, 2>(a, q, k, v, st);
    if (fits(64, 1)) return launch_attention<64, DVC, 1>(a, q, k, v, st);
    if (fits(32, 1)) return launch_attention<32, DVC, 1>(a, q, k, v, st);
    return fail(SDB_NOT_SUPPORTED, "sdb_attention: head too wide");
}

// ---------------------------------------------------------------- wide heads
// Heads of more than 160 dims (the VAE's one head of 512, attention.cc:828-845
// takes any width) do not fit the fused kernels' shared and tensor memory: a
// 128-query tile of Q alone, split, is 128 x 512 x 4 B = 256 KB.  They run per
// (image, head) as the product, the softmax and the product again, which is the
// reference's own two-pass order (attention.cc:9-27): S = Q K^T by the linear
// layers' split GEMM (three FP16 products of the FP32 operands), the rows of S
// through softmax(scale S) with its exponentials summed in double and one
// reciprocal a row (sdb_soft_max), and O = P V by the same GEMM.  The head's
// rows are gathered into dense matrices first (V transposed, so that keys run
// along the GEMM's K), and O is scattered into dst.

__global__ void gather2d_kernel(const void* src, int f16, long long s0, long long s1, long long n0, long long n1,
                                float* dst, long long d0, long long d1) {
    const long long total = n0 * n1;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long i = e / n1, j = e - i * n1;
        const long long at = i * s0 + j * s1;
        const float v = f16 ? __half2float(static_cast<const __half*>(src)[at]) : static_cast<const float*>(src)[at];
        dst[i * d0 + j * d1] = v;
    }
}

// Device memory of the wide path, per (device, stream), apart from the GEMM's
// workspace; grows outside stream capture only.
int wide_scratch(cudaStream_t st, size_t bytes, float** out) {
    static std::mutex lock;
    static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> spaces;
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> guard(lock);
    auto& s = spaces[{dev, st}];
    if (s.second < bytes) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        SDB_CUDA(cudaStreamIsCapturing(st, &cap));
        if (cap != cudaStreamCaptureStatusNone)
            return fail(SDB_INVALID, "sdb_attention: scratch must grow under stream capture: run it once before");
        if (s.first) {
            SDB_CUDA(cudaStreamSynchronize(st));
            SDB_CUDA(cudaFree(s.first));
            s = {nullptr, 0};
        }
        SDB_CUDA(cudaMalloc(&s.first, bytes));
        s.second = bytes;
    }
    *out = static_cast<float*>(s.first);
    return SDB_OK;
}

int gather2d(const void* src, bool f16, long long s0, long long s1, long long n0, long long n1, float* dst,
             long long d0, long long d1, cudaStream_t st) {
    const long long total = n0 * n1;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    gather2d_kernel<<<blocks, 256, 0, st>>>(src, f16 ? 1 : 0, s0, s1, n0, n1, dst, d0, d1);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

sdb_tensor dense(float* data, long long ne0, long long ne1) {
    sdb_tensor t{};
    t.type = SDB_TYPE_F32;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = 1; t.ne[3] = 1;
    t.nb[0] = 4; t.nb[1] = 4 * ne0; t.nb[2] = t.nb[1] * ne1; t.nb[3] = t.nb[2];
    t.data = data;
    return t;
}

int run_wide_attention(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, const sdb_tensor* dst,
                       float scale, cudaStream_t st) {
    const long long d = q->ne[0], lq = q->ne[1], h = q->ne[2], b = q->ne[3];
    const long long lk = k->ne[1], hk = k->ne[2], dv = v->ne[0];
    const int ke = esize(k), ve = esize(v);
    const long long qn = lq * d, kn = lk * d, vn = dv * lk, sn = lq * lk, on = lq * dv;
    float* base = nullptr;
    const auto pad = [](long long n) { return (n + 63) / 64 * 64; };
    const size_t bytes = 4 * static_cast<size_t>(pad(qn) + pad(kn) + pad(vn) + pad(sn) + pad(on));
    if (int s = wide_scratch(st, bytes, &base); s != SDB_OK) return s;
    float* qc = base;
    float* kc = qc + pad(qn);
    float* vt = kc + pad(kn);
    float* sc = vt + pad(vn);
    float* oc = sc + pad(sn);
    for (long long bi = 0; bi < b; ++bi) {
        for (long long hi = 0; hi < h; ++hi) {
            const long long khi = hi / (h / hk);
            const char* qh = static_cast<const char*>(q->data) + bi * q->nb[3] + hi * q->nb[2];
            const char* kh = static_cast<const char*>(k->data) + bi * k->nb[3] + khi * k->nb[2];
            const char* vh = static_cast<const char*>(v->data) + bi * v->nb[3] + khi * v->nb[2];
            if (int s = gather2d(qh, false, q->nb[1] / 4, q->nb[0] / 4, lq, d, qc, d, 1, st); s != SDB_OK) return s;
            if (int s = gather2d(kh, ke == 2, k->nb[1] / ke, k->nb[0] / ke, lk, d, kc, d, 1, st); s != SDB_OK)
                return s;
            if (int s = gather2d(vh, ve == 2, v->nb[0] / ve, v->nb[1] / ve, dv, lk, vt, lk, 1, st); s != SDB_OK)
                return s;
            const sdb_tensor tq = dense(qc, d, lq), tk = dense(kc, d, lk), ts = dense(sc, lk, lq),
                             tv = dense(vt, lk, dv), to = dense(oc, dv, lq);
            if (int s = sdb_mul_mat_transient(&tk, &tq, &ts, nullptr, st); s != SDB_OK) return s;
            if (int s = sdb_soft_max(&ts, &ts, scale, st); s != SDB_OK) return s;
            if (int s = sdb_mul_mat_transient(&tv, &ts, &to, nullptr, st); s != SDB_OK) return s;
            char* oh = static_cast<char*>(dst->data) + bi * dst->nb[3] + hi * dst->nb[1];
            if (int s = gather2d(oc, false, dv, 1, lq, dv, reinterpret_cast<float*>(oh), dst->nb[2] / 4,
                                 dst->nb[0] / 4, st);
                s != SDB_OK)
                return s;
        }
    }
    return SDB_OK;
}

}  // namespace

}  // namespace sdb

using namespace sdb;

extern "C" int sdb_attention_supported(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v,
                                       const sdb_tensor* dst) {
    if (!q || !k || !v || !dst) return 0;
    if (q->type != SDB_TYPE_F32 || !q->data || !floaty(k) || !floaty(v) || dst->type != SDB_TYPE_F32 || !dst->data)
        return 0;
    if (k->type != v->type) return 0;
    const int64_t d = q->ne[0], lq = q->ne[1], h = q->ne[2], b = q->ne[3];
    const int64_t lk = k->ne[1], hk = k->ne[2], dv = v->ne[0];
    if (k->ne[0] != d || v->ne[1] != lk || v->ne[2] != hk || k->ne[3] != b || v->ne[3] != b) return 0;
    if (hk <= 0 || h % hk != 0 || d <= 0 || dv <= 0 || lq <= 0 || lk <= 0) return 0;
    if (dst->ne[0] != dv || dst->ne[1] != h || dst->ne[2] != lq || dst->ne[3] != b) return 0;
    for (const sdb_tensor* t : {q, k, v, dst})
        for (int i = 0; i < 4; ++i)
            if (t->nb[i] % esize(t) != 0 || t->nb[i] < 0) return 0;
    // Heads wider than the fused kernels take: by the product, softmax, product path.
    if (d > 160 || dv > 512) return d <= (1 << 16) && dv <= (1 << 16) && lk <= (1 << 24) && lq <= (1 << 30);
    // TMA row coordinates are 32-bit (hi and lo planes).
    if (2 * b * h * lq >= (1LL << 31) || 2 * b * hk * lk >= (1LL << 31)) return 0;
    return h * ((dv + 79) / 80) <= 65535 && b <= 65535;
}

extern "C" int sdb_attention(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, const sdb_tensor* dst,
                             float scale, const sdb_chain* chain, void* stream) {
    if (!sdb_attention_supported(q, k, v, dst)) return fail(SDB_NOT_SUPPORTED, "sdb_attention: not supported");
    if (chain && (chain->count < 0 || chain->count > SDB_MAX_STEPS || chain->redirect))
        return fail(SDB_INVALID, "sdb_attention: invalid chain");
    const auto st = static_cast<cudaStream_t>(stream);
    // Integer products for self-attention over 256 keys or more (attention.cc:612-618, 858-862);
    // heads wider than 160 dims stay in single precision.
    const bool wide = q->ne[0] > 160 || v->ne[0] > 512;
    if (!wide && quantized_attention(k->ne[1])) return run_quantized_attention(q, k, v, dst, scale, chain, st);
    if (wide) {
        if (chain && (chain->count > 0 || chain->from_redirect))
            return fail(SDB_NOT_SUPPORTED, "sdb_attention: heads over 160 dims take no chain");
        return run_wide_attention(q, k, v, dst, scale, st);
    }
    AttnArgs a{};
    a.out = static_cast<float*>(dst->data);
    for (int i = 0; i < 4; ++i) a.onb[i] = dst->nb[i] / 4;
    a.d = static_cast<int>(q->ne[0]);
    a.lq = static_cast<int>(q->ne[1]);
    a.h = static_cast<int>(q->ne[2]);
    a.b = static_cast<int>(q->ne[3]);
    a.lk = static_cast<int>(k->ne[1]);
    a.hk = static_cast<int>(k->ne[2]);
    a.dv = static_cast<int>(v->ne[0]);
    a.dp = static_cast<int>(round_up(a.d, 16));
    a.dvp = static_cast<int>(round_up(a.dv, 16));
    a.rq = a.b * a.h * a.lq;
    a.rk = a.b * a.hk * a.lk;
    a.scale2 = scale * kLog2e;
    a.chain = make_chain(chain);
    a.err = device_error_word();
    const int chunks = (a.dvp + 79) / 80;
    const int dvc = ((a.dvp / 16 + chunks - 1) / chunks) * 16;
    a.dv_chunks = chunks;

    switch (dvc) {
    case 16: return launch_bk<16>(a, q, k, v, st);
    case 32: return launch_bk<32>(a, q, k, v, st);
    case 48: return launch_bk<48>(a, q, k, v, st);
    case 64: return launch_bk<64>(a, q, k, v, st);
    default: return launch_bk<80>(a, q, k, v, st);
    }
}
