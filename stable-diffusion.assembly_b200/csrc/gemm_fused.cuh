// The linear layers' GEMM with the activation split done inside the kernel.
//
// The arithmetic is the wide kernel's (gemm_wide.cuh): x = hi + lo 2^-11 in
// FP16 pairs against FP16 weights, two kind::f16 products, k-blocks of 64 of K
// added into FP32 registers with round-to-nearest.  What changes is where the
// split happens and how the work overlaps:
//
// * x arrives as FP32 rows by TMA (two 32-float boxes a k-block, 128-byte
//   swizzle).  Sixteen worker warps read their rows out of shared memory,
//   split them and write hi and lo into tensor memory as the A operand of
//   both products (tcgen05.mma with A in tensor memory).  No pre-pass writes
//   the split to HBM and reads it back, and the tensor core reads only the
//   weights from shared memory.
// * One accumulator a k-block holds hi W + (lo W) 2^-11: the lo products go
//   first into a fresh accumulator, the first hi product scales it by 2^-11
//   as it adds (tcgen05.mma's scale of the input D), the rest add plainly.
//   So a k-block needs BN columns, two of them fit beside two A buffers (64
//   columns each), and the products of k-block kb + 1 run while the workers
//   drain kb's accumulator.
// * x and the weights travel in rings of their own: an x stage is free again
//   once the workers have split it (a k-block ahead of its products), a
//   weight stage once its products completed; the x ring is the deeper one,
//   since x streams from HBM.
// * Warp roles (640 threads): warps 0-15 split, drain and store (warp w:
//   tensor-memory lanes 32 (w % 4) .. + 31, a quarter of each k-block's K and
//   the column groups w / 4 + 4 i); warp 16 lane 0 loads x, warp 18 lane 0
//   the weights; warp 17 lane 0 issues the products and owns the
//   tensor-memory allocation; warp 19 idles.
//
// Tensor memory (512 columns): accumulators at 0 and 192, A buffers at 384
// and 448 (hi at +0, lo at +32; k16 step j at +8 j).
#pragma once

#include "gemm_wide.cuh"

namespace sdb {

constexpr int kFusedWorkers = 16;
constexpr int kFusedThreads = (kFusedWorkers + 4) * 32;
constexpr int kFusedXWarp = kFusedWorkers;
constexpr int kFusedMmaWarp = kFusedWorkers + 1;
constexpr int kFusedWWarp = kFusedWorkers + 2;

template <int BN>
struct FusedShape {
    static_assert(BN == 128 || BN == 160 || BN == 192, "tile width (two accumulators and two A buffers in 512 columns)");
    static constexpr int kXBoxBytes = kBM * 32 * 4;           // 128 rows x 32 FP32
    static constexpr int kXBytes = 2 * kXBoxBytes;            // a k-block of x
    static constexpr int kBBytes = BN * kBK * 2;              // a k-block of the weights
    static constexpr int kBoxBytes = 32 * 64;                 // a 32-row x 16-column FP32 store box
    static constexpr int kStagingBytes = kFusedWorkers * kBoxBytes;
    static constexpr int kBarrierBytes = 512;
    static constexpr int kBudget = 227 * 1024 - kStagingBytes - 1024 - kBarrierBytes;
    static constexpr int kWStages = BN == 128 ? 4 : BN == 160 ? 3 : 2;
    static constexpr int kXStagesFit = (kBudget - kWStages * kBBytes) / kXBytes;
    static constexpr int kXStages = kXStagesFit > 6 ? 6 : kXStagesFit;
    static constexpr int kWOffset = kXStages * kXBytes;
    static constexpr int kStagingOffset = kWOffset + kWStages * kBBytes;
    static constexpr int kSmemBytes = kStagingOffset + kStagingBytes + 1024 + kBarrierBytes;
    static constexpr uint32_t kAccStride = 192;               // accumulator b at kAccStride b
    static constexpr uint32_t kACol = 384;                    // A buffer b at kACol + 64 b
    static_assert(kXStages >= 3 && kWStages >= 2, "too few stages");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kBBytes % 1024 == 0 && kXBytes % 1024 == 0, "swizzle atoms");
};

template <bool GATED, int BN>
__global__ void __launch_bounds__(kFusedThreads, 1)
gemm_fused_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap ymap, const GemmArgs args) {
    using S = FusedShape<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + S::kStagingOffset;
    uint64_t* xfull = reinterpret_cast<uint64_t*>(staging + S::kStagingBytes);
    uint64_t* xempty = xfull + S::kXStages;   // every worker read its part
    uint64_t* wfull = xempty + S::kXStages;
    uint64_t* wempty = wfull + S::kWStages;   // the products completed
    // The two buffers of A and of the accumulator need no "free again" barriers of their
    // own: a worker splits k-block it + 1 into A buffer (it + 1) % 2 after it drained
    // k-block it - 1, whose d_full says that the products that read that buffer are done;
    // and every worker drained accumulator it % 2 (k-block it - 2) before it split k-block
    // it, so a_full(it) also says that the accumulator is free.
    uint64_t* a_full = wempty + S::kWStages;  // [2] the workers wrote an A buffer
    uint64_t* d_full = a_full + 2;            // [2] an accumulator's products completed
    uint64_t* drain = d_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kXStages; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], kFusedWorkers);
        }
        for (int s = 0; s < S::kWStages; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&a_full[b], kFusedWorkers);
            mbar_init(&d_full[b], 1);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&xmap);
        tma_prefetch_desc(&wmap);
        if (args.store == kStoreTma || args.ksplit > 1) tma_prefetch_desc(&ymap);
    }
    if (warp == kFusedMmaWarp) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto item_range = [&](int item, int& tm, int& tn, int& split, int& kb0, int& kb1) {
        tn = item % args.tiles_n;
        const int rest = item / args.tiles_n;
        tm = rest % args.tiles_m;
        split = rest / args.tiles_m;
        kb0 = split * args.per_split;
        kb1 = min(args.kblocks, kb0 + args.per_split);
    };
    // Every role walks the same sequence of k-blocks: the CTA's items in turn.
    int total_kb = 0;
    for (int item = blockIdx.x; item < args.items; item += gridDim.x) {
        int tm, tn, split, kb0, kb1;
        item_range(item, tm, tn, split, kb0, kb1);
        total_kb += kb1 - kb0;
    }

    bool ok = true;
    if (warp == kFusedXWarp || warp == kFusedWWarp) {
        // ---- TMA producers: x (warp 16) and the weights (warp 18), each in its own ring
        if (lane == 0) {
            const bool is_x = warp == kFusedXWarp;
            const int stages = is_x ? S::kXStages : S::kWStages;
            uint64_t* fullb = is_x ? xfull : wfull;
            uint64_t* emptyb = is_x ? xempty : wempty;
            int it = 0;
            for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
                int tm, tn, split, kb0, kb1;
                item_range(item, tm, tn, split, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % stages;
                    if (!mbar_wait_sleep(&emptyb[s], ((it / stages) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                    if (is_x) {
                        mbar_arrive_expect_tx(&xfull[s], S::kXBytes);
                        uint8_t* st = smem + s * S::kXBytes;
                        tma_load_2d(st, &xmap, &xfull[s], kb * kBK, tm * kBM);
                        tma_load_2d(st + S::kXBoxBytes, &xmap, &xfull[s], kb * kBK + 32, tm * kBM);
                    } else {
                        mbar_arrive_expect_tx(&wfull[s], S::kBBytes);
                        uint8_t* st = smem + S::kWOffset + s * S::kBBytes;
                        if (GATED) {
                            tma_load_2d(st, &wmap, &wfull[s], kb * kBK, tn * (BN / 2));
                            tma_load_2d(st + S::kBBytes / 2, &wmap, &wfull[s], kb * kBK, args.b1_row + tn * (BN / 2));
                        } else {
                            tma_load_2d(st, &wmap, &wfull[s], kb * kBK, tn * BN);
                        }
                    }
                }
            }
            if (!ok) {   // wind down: the loads in flight land before the CTA leaves
                for (int i = (it > stages ? it - stages : 0); i < it; ++i)
                    mbar_wait_quiet(&fullb[i % stages], (i / stages) & 1, 100000000ull);
            }
        }
    } else if (warp == kFusedMmaWarp) {
        // ---- MMA issuer: per k-block, the lo products into a fresh accumulator, then the hi
        // products (the first one scaling the lo sum by 2^-11).
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
            for (int it = 0; it < total_kb; ++it) {
                const int s = it % S::kWStages, b = it & 1;
                const uint32_t use = static_cast<uint32_t>(it >> 1) & 1u;
                // Tested in a loop, not suspended: a woken thread would start the products
                // a few hundred clocks late.
                if (!mbar_wait(&wfull[s], (it / S::kWStages) & 1, abort, args.err) ||
                    !mbar_wait(&a_full[b], use, abort, args.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + S::kAccStride * b;
                const uint32_t a = tmem + S::kACol + 64u * b;
                const uint32_t b0 = smem_u32(smem + S::kWOffset + s * S::kBBytes);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    mma_f16_ta(d, a + 32 + 8 * kk, desc_kmajor_sw128(b0 + kk * 32), idesc, kk > 0 ? 1u : 0u);
                mma_f16_ta_scale_lo(d, a, desc_kmajor_sw128(b0), idesc);
#pragma unroll
                for (int kk = 1; kk < kBK / 16; ++kk)
                    mma_f16_ta(d, a + 8 * kk, desc_kmajor_sw128(b0 + kk * 32), idesc, 1u);
                mma_commit(&wempty[s]);
                mma_commit(&d_full[b]);
            }
            if (!ok) {
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else if (warp < kFusedWorkers) {
        // ---- workers
        const int q = warp & 3;           // tensor-memory lane quarter
        const int part = warp >> 2;       // k16 step of the split; column groups part, part + 4, ...
        const int row = q * 32 + lane;
        uint8_t* box = staging + warp * S::kBoxBytes;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        // The tile's columns in groups of 16 (gated: 16 output columns, i.e. 16 of the x half
        // and the matching 16 of the gate half); this warp sums groups part + 4 i.
        constexpr int G = GATED ? BN / 32 : BN / 16;
        constexpr int NG = (G + 3) / 4;
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait_sleep(bar, parity, abort, args.err) ? 1 : 0) != 0;
        };
        // The split of k-block number `it`: this thread's row, K 16 part .. + 15 of the block,
        // read from the stage's x boxes (128-byte swizzle: chunk c of row r at (c ^ r % 8) 16).
        float amax = 0.0f;   // the largest |x| split: 65520 or more rounds to an FP16 infinity
        auto split_block = [&](int it) -> bool {
            const int s = it % S::kXStages, b = it & 1;
            if (!warp_wait(&xfull[s], (it / S::kXStages) & 1)) return false;
            const uint32_t xb = smem_u32(smem + s * S::kXBytes + (part >> 1) * S::kXBoxBytes) + row * 128;
            uint4 hv[2], lv[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float e[8];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int c = (part & 1) * 4 + 2 * h + j;
                    const uint4 w = ld_shared_v4(xb + ((c ^ (row & 7)) << 4));
                    e[4 * j] = __uint_as_float(w.x);
                    e[4 * j + 1] = __uint_as_float(w.y);
                    e[4 * j + 2] = __uint_as_float(w.z);
                    e[4 * j + 3] = __uint_as_float(w.w);
                }
                split8_packed(e, hv[h], lv[h], amax);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[s]);
            const uint32_t a = lane_addr + S::kACol + 64u * b + 8u * part;
            tmem_st4_bits(a, hv[0]);
            tmem_st4_bits(a + 4, hv[1]);
            tmem_st4_bits(a + 32, lv[0]);
            tmem_st4_bits(a + 36, lv[1]);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
            return true;
        };
        // sum[i][..] += the accumulator's group part + 4 i (gated: [i][0..15] x, [i][16..31] gate).
        auto drain_groups = [&](uint32_t acc, float (*sum)[GATED ? 32 : 16]) {
            if (GATED) {
#pragma unroll
                for (int i = 0; i < NG; ++i) {
                    const int gidx = part + 4 * i;
                    if (i == NG - 1 && gidx >= G) break;
                    float a[16], g[16];
                    tmem_ld16(acc + 16 * gidx, a);
                    tmem_ld16(acc + BN / 2 + 16 * gidx, g);
                    tmem_ld_wait();
                    add16_packed(sum[i], a);
                    add16_packed(sum[i] + 16, g);
                }
            } else {
                // Two groups' loads in flight at a time.
#pragma unroll
                for (int i = 0; i < NG; i += 2) {
                    const int g0 = part + 4 * i, g1 = g0 + 4;
                    const bool has0 = i < NG - 1 || g0 < G;
                    const bool has1 = i + 1 < NG && (i + 1 < NG - 1 || g1 < G);
                    float a[16], c[16];
                    if (has0) tmem_ld16(acc + 16 * g0, a);
                    if (has1) tmem_ld16(acc + 16 * g1, c);
                    tmem_ld_wait();
                    if (has0) add16_packed(sum[i], a);
                    if (has1) add16_packed(sum[i + 1], c);
                }
            }
        };

        // Splits every k-block up to j not split yet.  A worker may split k-block j once it has
        // seen d_full(j - 2) (the products that read A buffer j % 2 are done).
        int next_split = 0;
        auto split_upto = [&](int j) -> bool {
            for (; next_split <= j && next_split < total_kb; ++next_split)
                if (!split_block(next_split)) return false;
            return true;
        };
        int it = 0;
        ok = split_upto(0);
        for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
            int tm, tn, split, kb0, kb1;
            item_range(item, tm, tn, split, kb0, kb1);
            float sum[NG][GATED ? 32 : 16];
#pragma unroll
            for (int i = 0; i < NG; ++i)
#pragma unroll
                for (int j = 0; j < (GATED ? 32 : 16); ++j) sum[i][j] = 0.0f;
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                if (!split_upto(it + 1)) { ok = false; break; }
                const int b = it & 1;
                if (!warp_wait(&d_full[b], (static_cast<uint32_t>(it) >> 1) & 1u)) { ok = false; break; }
                tc_fence_after();
                drain_groups(lane_addr + S::kAccStride * b, sum);
                tc_fence_before();
                __syncwarp();
            }
            if (!ok) break;
            // ---- the tile's epilogue (the next item's first products run meanwhile)
            if (args.ksplit > 1) {
                const int prow = (split * args.tiles_m + tm) * kBM + q * 32;
#pragma unroll
                for (int i = 0; i < NG; ++i) {
                    const int gidx = part + 4 * i;
                    if (i == NG - 1 && gidx >= G) break;
                    store_box16(&ymap, box, lane, sum[i], tn * BN + 16 * gidx, prow);
                }
            } else {
                const LinearRow r = linear_row(args, tm, row);
#pragma unroll
                for (int i = 0; i < NG; ++i) {
                    const int gidx = part + 4 * i;
                    if (i == NG - 1 && gidx >= G) break;
                    const long long cb = static_cast<long long>(tn) * (GATED ? BN / 2 : BN) + 16 * gidx;
                    store_linear_group<GATED>(args, &ymap, r, sum[i], GATED ? sum[i] + 16 : nullptr, cb, tm, q, lane,
                                              box);
                }
            }
        }
        if (amax >= 65520.0f) atomicOr(args.err, kErrRange);
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kFusedMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace sdb
