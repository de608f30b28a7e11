// The tcgen05 GEMM of the linear layers and the direct convolution.
//
// C[m][n] = sum_k A[m][k] B[n][k] with
//   A: the activations, split once by the pre-pass (split.cuh) into FP16
//      pairs x = hi + lo 2^-11: rows of K for a linear layer; for a
//      convolution the channels-last image, whose im2col rows TMA reads
//      straight from it -- one box of 64 channels x (OWt x OHt x NT output
//      positions) per (tap, channel block), at the tap's offset, with the
//      convolution's stride as TMA's element stride and the padding as its
//      out-of-bounds zero fill (conv2d.cc:231-316 packs the same columns on
//      the CPU);
//   B: the weights, repacked once by the weight store into FP16 [rows][Kpad]
//      (K-major, per-tap channels padded to 64 for a convolution).
// All three tiles arrive by TMA in the 128-byte swizzle; one thread issues
// tcgen05.mma kind::f16 for hi x W and lo x W.  FP32 weights are split the
// same way (w = whi + wlo 2^-11) and add hi x wlo to the lo product.  The
// gated variant computes the x and the gate halves of a GEGLU product side by
// side and writes x * GELU(gate) (fusion.cc:290-310, mul_mat.cc:934-1058).
//
// Precision of the sums.  The tensor core's FP32 accumulation rounds toward
// zero: one k-step's add loses up to an ulp of the running sum, always in the
// same direction, so over hundreds of k-steps the error grows linearly (about
// 2^-23 of the sum per k-step, measured).  The hi product, which carries the
// sum, is therefore accumulated over 64 of K (4 k-steps) at a time, into
// one of three tensor-memory buffers in turn, and the epilogue warps add each
// partial sum to FP32 registers with round-to-nearest while the next ones
// compute.  The lo product (2^-11 of the sum) accumulates over all of
// the CTA's K.  The chain (bias, scale, SiLU, residual; fusion.h:51-91) is
// applied to sum + lo 2^-11 before the store -- or, when K is split over
// several CTAs (few output tiles, long K), each CTA writes its sum to the
// workspace and a reduction adds the splits in order and applies the chain.
//
// Warp roles (320 threads): warp 0 TMA producer; warp 1 MMA issuer and the
// tensor-memory allocation; warps 2-9 epilogue, two per quarter of
// tensor-memory lanes (warp w reads lanes 32*(w%4)..+31), each taking half
// the tile's columns.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "chain.cuh"
#include "ptx.cuh"

namespace sdb {

enum : int { kModeLinear = 0, kModeConv = 1 };
// kWeightSplitK32: FP32 (split) weights with stages of 32 of K in the 64-byte
// swizzle -- half the bytes a stage, so six stages fit where three would of
// 64; used where K is short and the loads' latency is not hidden otherwise
// (Winograd's batched products).  Linear mode only.
enum : int { kWeightHalf = 0, kWeightSplit = 1, kWeightGated = 2, kWeightSplitK32 = 3 };

constexpr int kBM = 128;        // rows of A per tile (the MMA's M)
constexpr int kBK = 64;         // K per stage: one 128-byte swizzle row of FP16
constexpr int kGemmWarps = 10;
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kEpiWarp0 = 2;    // first epilogue warp

struct ConvGeom {
    int ow, oh, n;          // output positions [OW, OH, N]
    int kw, kh;
    int s0, s1, p0, p1, d0, d1;
    int cblocks;            // 64-channel blocks per tap
    int owt, oht, nt;       // output positions of a tile: OWt x OHt x NT
    int tw, th, tn;         // tiles along W, H, N
};

struct GemmArgs {
    int m;                  // rows of C (linear: tokens; conv: unused, see cg)
    int kblocks;            // K / kBK of the whole product
    int ksplit;             // parts K is split into (each at least one k-block)
    int per_split;          // k-blocks of a part
    int n;                  // columns of C (linear: output features; gated: the half)
    int b1_row;             // row offset in the packed weights of the second B operand
    int batch_tiles;        // batched products (Winograd's xi): row tiles of one batch; 0 = one product
    int b_batch_rows;       // packed weight rows of one batch (batch b's B rows start at b * b_batch_rows)
    uint32_t a_tx;          // bytes of one A tile (hi or lo) as TMA writes it
    int a_planes;           // 2: one TMA box brings hi and lo (a full 128-row tile); 1: one box each
    int tiles_m, tiles_n;   // output tiles along rows / columns
    int items;              // tiles_m * tiles_n * ksplit work items, taken round-robin by the CTAs
    int store;              // kStoreTma: the output through ymap in 32 x 32 boxes; kStoreDirect
    float* y;               // output (the redirect when the chain has one)
    float* part;            // split-K: partial sums [ksplit][tiles_m * 128][part_ld]
    long long part_ld;      // columns of a partial row
    long long part_split;   // elements between splits
    long long ynb[4];       // output strides in elements
    long long rne1, rne2;   // linear: row m -> (i1, i2, i3) = (m % rne1, m / rne1 % rne2, m / (rne1 rne2))
    ConvGeom cg;
    Chain chain;
    unsigned* err;
};

enum : int { kStoreDirect = 0, kStoreTma = 1 };

template <int WMODE>
struct GemmShape {
    static constexpr int BN = WMODE == kWeightGated ? 64 : 128;
    static constexpr bool kHasB1 = WMODE != kWeightHalf;
    static constexpr bool kSplitW = WMODE == kWeightSplit || WMODE == kWeightSplitK32;
    static constexpr int kStageK = WMODE == kWeightSplitK32 ? 32 : kBK;  // K of a stage
    static constexpr int kABytes = kBM * kStageK * 2;  // one of hi / lo
    static constexpr int kBBytes = BN * kStageK * 2;
    static constexpr int kStageBytes = 2 * kABytes + kBBytes * (kHasB1 ? 2 : 1);
    // Output staging for the TMA stores: a 32 x 32 FP32 box (4 KB) per epilogue warp.
    static constexpr int kStagingBytes = 8 * 32 * 128;
    static constexpr int kBudget = 227 * 1024 - kStagingBytes - 1024 /*align*/ - 256 /*barriers*/;
    static constexpr int kStages = kBudget / kStageBytes >= 6 ? 6 : kBudget / kStageBytes;
    // The hi product is drained every kDrainStages stages (64 of K) into one of
    // kNHi tensor-memory buffers in turn, so that the MMAs run up to two drains
    // ahead of the epilogue.
    static constexpr int kDrainStages = kBK / kStageK;
    static constexpr int kNHi = 3;
    // Tensor-memory columns: hi buffers (gated: x buffers, then gate buffers) then lo (gated: x, g).
    static constexpr int kHiCols = WMODE == kWeightGated ? 2 * kNHi * BN : kNHi * BN;
    static constexpr int kLoCol = kHiCols;
    static constexpr int kAccCols = kHiCols + (WMODE == kWeightGated ? 2 * BN : BN);
    static constexpr int kTmemCols = 512;
    static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 + 256;
    static_assert(kAccCols <= 512, "accumulators exceed tensor memory");
    static_assert(kStages >= 2, "too few stages");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// ---------------------------------------------------------------- tiles

// The output position of lane row r of conv tile `tile`: valid when inside
// the output.
struct ConvPos {
    int ox, oy, img;
    bool ok;
};

__device__ __forceinline__ ConvPos conv_pos(const ConvGeom& g, int tile, int r) {
    const int tx = tile % g.tw;
    const int ty = (tile / g.tw) % g.th;
    const int tz = tile / (g.tw * g.th);
    const int per = g.owt * g.oht;
    ConvPos p;
    p.ox = tx * g.owt + r % g.owt;
    p.oy = ty * g.oht + (r / g.owt) % g.oht;
    p.img = tz * g.nt + r / per;
    p.ok = r < per * g.nt && p.ox < g.ow && p.oy < g.oh && p.img < g.n;
    return p;
}

// ---------------------------------------------------------------- epilogue

// A linear layer's output rows are contiguous: each epilogue warp writes its
// 32 rows x 32 columns as one TMA store from a 4 KB staging box in the
// 128-byte swizzle (row r's 16-byte chunk k at r * 128 + ((k ^ r % 8) * 16),
// so the 32 lanes' vector stores hit every bank once per 8 lanes).
__device__ __forceinline__ void stage_row32(uint8_t* box, int lane, const float* v) {
    const uint32_t base = smem_u32(box) + lane * 128;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint4 q = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                   __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
        st_shared_v4(base + ((k ^ (lane & 7)) << 4), q);
    }
}

// ---------------------------------------------------------------- kernel
//
// Persistent: each CTA takes work items blockIdx.x, blockIdx.x + gridDim.x, ...
// (item = (row tile fastest, column tile, K part)).  The TMA warp streams the
// items' k-blocks through one ring of stages; the MMA warp fills the two hi
// buffers and the lo accumulator item after item; the epilogue warps read the
// lo accumulator at an item's end and release it at once, so the next item's
// products run while they apply the chain and store.

template <int MODE, int WMODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_split_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                  const __grid_constant__ CUtensorMap ymap, const GemmArgs args) {
    using S = GemmShape<WMODE>;
    constexpr int BN = S::BN;
    constexpr bool kGated = WMODE == kWeightGated;
    static_assert(MODE == kModeLinear || WMODE != kWeightSplitK32, "32-wide stages: linear mode only");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + S::kStages * S::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + S::kStagingBytes);
    uint64_t* empty = full + S::kStages;
    uint64_t* hi_full = empty + S::kStages;   // [kNHi]
    uint64_t* hi_empty = hi_full + S::kNHi;   // [kNHi]
    uint64_t* lo_full = hi_empty + S::kNHi;
    uint64_t* lo_empty = lo_full + 1;
    uint64_t* drain = lo_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1);   // TMA arrive.expect_tx
            mbar_init(&empty[s], 1);  // the MMA commit
        }
        for (int b = 0; b < S::kNHi; ++b) {
            mbar_init(&hi_full[b], 1);
            mbar_init(&hi_empty[b], 8);  // the eight epilogue warps
        }
        mbar_init(lo_full, 1);
        mbar_init(lo_empty, 8);
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&amap);
        tma_prefetch_desc(&wmap);
        if (args.store == kStoreTma || args.ksplit > 1) tma_prefetch_desc(&ymap);
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * S::kStageBytes; };            // hi, then lo at + kABytes
    auto stage_b0 = [&](int s) { return smem + s * S::kStageBytes + 2 * S::kABytes; };
    auto stage_b1 = [&](int s) { return smem + s * S::kStageBytes + 2 * S::kABytes + S::kBBytes; };
    // The k-block range of an item.
    auto item_range = [&](int item, int& tm, int& tn, int& split, int& kb0, int& kb1) {
        tm = item % args.tiles_m;
        const int rest = item / args.tiles_m;
        tn = rest % args.tiles_n;
        split = rest / args.tiles_n;
        kb0 = split * args.per_split;
        kb1 = min(args.kblocks, kb0 + args.per_split);
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const ConvGeom& g = args.cg;
            const uint32_t tx_bytes = 2 * args.a_tx + S::kBBytes * (S::kHasB1 ? 2 : 1);
            int it = 0;  // k-blocks issued
            bool ok = true;
            for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
                int tm, tn, split, kb0, kb1;
                item_range(item, tm, tn, split, kb0, kb1);
                int ax = 0, ay = 0, az = 0;
                if (MODE == kModeConv) {
                    const int tx = tm % g.tw, ty = (tm / g.tw) % g.th, tz = tm / (g.tw * g.th);
                    ax = tx * g.owt * g.s0 - g.p0;
                    ay = ty * g.oht * g.s1 - g.p1;
                    az = tz * g.nt;
                }
                // B rows of this item: its column tile, in its batch's block of weights.
                const int n0 = tn * BN + (args.batch_tiles ? (tm / args.batch_tiles) * args.b_batch_rows : 0);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S::kStages;
                    if (!mbar_wait(&empty[s], ((it / S::kStages) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], tx_bytes);
                    if (MODE == kModeLinear) {
                        tma_load_3d(stage_a(s), &amap, &full[s], kb * S::kStageK, tm * kBM, 0);
                    } else {
                        const int tap = kb / g.cblocks;
                        const int cx0 = (kb - tap * g.cblocks) * kBK;
                        const int ky = tap / g.kw, kx = tap - ky * g.kw;
                        const int x = ax + kx * g.d0, y = ay + ky * g.d1;
                        if (args.a_planes == 2) {
                            tma_load_5d(stage_a(s), &amap, &full[s], cx0, x, y, az, 0);
                        } else {
                            tma_load_5d(stage_a(s), &amap, &full[s], cx0, x, y, az, 0);
                            tma_load_5d(stage_a(s) + S::kABytes, &amap, &full[s], cx0, x, y, az, 1);
                        }
                    }
                    tma_load_2d(stage_b0(s), &wmap, &full[s], kb * S::kStageK, n0);
                    if (S::kHasB1) tma_load_2d(stage_b1(s), &wmap, &full[s], kb * S::kStageK, args.b1_row + n0);
                }
            }
            if (*abort) {
                // Let the loads this thread started land before the CTA exits.
                for (int i = (it > S::kStages ? it - S::kStages : 0); i < it; ++i)
                    mbar_wait_quiet(&full[i % S::kStages], (i / S::kStages) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
            bool ok = true;
            int it = 0, t = 0, g = 0;  // stages consumed, items done, hi drains
            // One k-step is 16 of K, 32 bytes along a swizzled row.
            auto desc = [](uint32_t addr) {
                return S::kStageK == 32 ? desc_kmajor_sw64(addr) : desc_kmajor_sw128(addr);
            };
            for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x, ++t) {
                int tm, tn, split, kb0, kb1;
                item_range(item, tm, tn, split, kb0, kb1);
                // The previous item's lo accumulator has been read.
                if (!mbar_wait(lo_empty, (t & 1) ^ 1, abort, args.err)) { ok = false; break; }
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S::kStages;
                    const int q = (kb - kb0) % S::kDrainStages;  // stage within its drain
                    const int b = g % S::kNHi;
                    if (!mbar_wait(&full[s], (it / S::kStages) & 1, abort, args.err)) { ok = false; break; }
                    if (q == 0 && !mbar_wait(&hi_empty[b], ((g / S::kNHi) & 1) ^ 1, abort, args.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t ahi = smem_u32(stage_a(s)), alo = ahi + S::kABytes;
                    const uint32_t b0 = smem_u32(stage_b0(s)), b1 = smem_u32(stage_b1(s));
                    const uint32_t d_hi = tmem + b * BN;
#pragma unroll
                    for (int kk = 0; kk < S::kStageK / 16; ++kk) {
                        const uint32_t fresh = (q > 0 || kk > 0) ? 1u : 0u;
                        const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
                        const uint64_t dah = desc(ahi + kk * 32), dal = desc(alo + kk * 32);
                        const uint64_t db0 = desc(b0 + kk * 32);
                        mma_f16(d_hi, dah, db0, idesc, fresh);
                        mma_f16(tmem + S::kLoCol, dal, db0, idesc, acc);
                        if (S::kSplitW) {
                            mma_f16(tmem + S::kLoCol, dah, desc(b1 + kk * 32), idesc, 1u);
                        } else if (kGated) {
                            const uint64_t db1 = desc(b1 + kk * 32);
                            mma_f16(tmem + S::kNHi * BN + b * BN, dah, db1, idesc, fresh);
                            mma_f16(tmem + S::kLoCol + BN, dal, db1, idesc, acc);
                        }
                    }
                    mma_commit(&empty[s]);
                    if (q == S::kDrainStages - 1 || kb == kb1 - 1) {
                        mma_commit(&hi_full[b]);
                        ++g;
                    }
                }
                if (ok) mma_commit(lo_full);
            }
            if (!ok) {
                // Wind down: every MMA issued completes before tensor memory is freed.
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const int ew = warp - kEpiWarp0;      // 0..7
        const int q = warp & 3;               // TMEM lane quarter this warp may read
        const int half = ew >> 2;             // which half of the tile's columns
        constexpr int NV = BN / 2;            // columns per warp
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        uint8_t* box = staging + ew * (32 * 128);
        bool ok = true;
        int g = 0, t = 0;  // hi drains, items done
        for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x, ++t) {
            int tm, tn, split, kb0, kb1;
            item_range(item, tm, tn, split, kb0, kb1);
            const int drains = (kb1 - kb0 + S::kDrainStages - 1) / S::kDrainStages;
            float sum[NV], gsum[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                sum[j] = 0.0f;
                gsum[j] = 0.0f;
            }
            // Drain the hi product 64 of K at a time.
            for (int d = 0; d < drains; ++d, ++g) {
                const int b = g % S::kNHi;
                if (!mbar_wait(&hi_full[b], (g / S::kNHi) & 1, abort, args.err)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < NV; c += 32) {
                    float part[32];
                    tmem_ld32(lane_addr + b * BN + half * NV + c, part);
                    if (kGated) {
                        float gpart[32];
                        tmem_ld32(lane_addr + S::kNHi * BN + b * BN + half * NV + c, gpart);
                        tmem_ld_wait();
                        add_packed<32>(gsum + c, gpart);
                    } else {
                        tmem_ld_wait();
                    }
                    add_packed<32>(sum + c, part);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&hi_empty[b]);
            }
            if (!ok || !mbar_wait(lo_full, t & 1, abort, args.err)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < NV; c += 32) {
                float lo[32];
                tmem_ld32(lane_addr + S::kLoCol + half * NV + c, lo);
                if (kGated) {
                    float glo[32];
                    tmem_ld32(lane_addr + S::kLoCol + BN + half * NV + c, glo);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) gsum[c + j] = fmaf(glo[j], kLoUnscale, gsum[c + j]);
                } else {
                    tmem_ld_wait();
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[c + j] = fmaf(lo[j], kLoUnscale, sum[c + j]);
            }
            // Tensor memory is free for the next item.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(lo_empty);

            const int row = q * 32 + lane;                  // row of the tile this thread owns
            const int col0 = tn * BN + half * NV;
            if (args.ksplit > 1) {
                // Raw sums into the workspace: rows (split, tile row), TMA-stored.
#pragma unroll
                for (int c = 0; c < NV; c += 32) {
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    stage_row32(box, lane, sum + c);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&ymap, box, col0 + c, (split * args.tiles_m + tm) * kBM + q * 32);
                        bulk_commit_group();
                    }
                }
            } else if (MODE == kModeLinear) {
                const long long m = static_cast<long long>(tm) * kBM + row;
                const bool live = m < args.m;
                // Rows past the end take the last row's operand offsets (their results are not stored).
                const long long mc = live ? m : args.m - 1;
                const long long i1 = mc % args.rne1, rest = mc / args.rne1;
                const long long i2 = rest % args.rne2, i3 = rest / args.rne2;
                ChainRow cr;
                row_offsets(args.chain, cr, 0, i1, i2, i3);
                float* yrow = args.y + i1 * args.ynb[1] + i2 * args.ynb[2] + i3 * args.ynb[3];
#pragma unroll
                for (int c = 0; c < NV; c += 32) {
                    float* v = sum + c;   // the chain's results replace the sums
                    const long long cb = col0 + c;
                    if (kGated) {
                        apply_chain_cols<0, 32>(args.chain, cr, v, cb, args.n - 1);
                        apply_chain_cols<0, 32>(args.chain, cr, gsum + c, args.n + cb, 2LL * args.n - 1);
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] *= gelu(gsum[c + j]);
                    } else {
                        if (args.chain.from_redirect) {
                            float old[32];
#pragma unroll
                            for (int j = 0; j < 32; ++j) old[j] = yrow[min(cb + j, args.n - 1LL) * args.ynb[0]];
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = old[j] + v[j];
                        }
                        apply_chain_cols<0, 32>(args.chain, cr, v, cb, args.n - 1);
                    }
                    if (args.store == kStoreTma) {
                        if (lane == 0) bulk_wait_read_all();
                        __syncwarp();
                        stage_row32(box, lane, v);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&ymap, box, static_cast<int>(cb), tm * kBM + q * 32);
                            bulk_commit_group();
                        }
                    } else if (live) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (cb + j < args.n) yrow[(cb + j) * args.ynb[0]] = v[j];
                    }
                }
            } else {
                // Convolution: a lane's row is an output position; the warp's 32
                // positions are neighbours, so each channel is written as one run.
                const ConvPos p = conv_pos(args.cg, tm, row);
                const int ox = p.ok ? p.ox : 0, oy = p.ok ? p.oy : 0, img = p.ok ? p.img : 0;
                ChainRow cr;
                row_offsets(args.chain, cr, 2, ox, oy, img);
                float* ybase = args.y + ox * args.ynb[0] + static_cast<long long>(oy) * args.ynb[1] + img * args.ynb[3];
#pragma unroll
                for (int c = 0; c < NV; c += 32) {
                    float* v = sum + c;
                    const long long cb = col0 + c;
                    if (args.chain.from_redirect) {
                        float old[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) old[j] = ybase[min(cb + j, args.n - 1LL) * args.ynb[2]];
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = old[j] + v[j];
                    }
                    apply_chain_cols<2, 32>(args.chain, cr, v, cb, args.n - 1);
                    if (args.store == kStoreTma) {
                        // Channels-last output whose tiles are runs of 128 consecutive positions.
                        const ConvGeom& g = args.cg;
                        const int ty = (tm / g.tw) % g.th, tz = tm / (g.tw * g.th);
                        const int row0 = (tz * g.nt * g.oh + ty * g.oht) * g.ow;
                        if (lane == 0) bulk_wait_read_all();
                        __syncwarp();
                        stage_row32(box, lane, v);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&ymap, box, static_cast<int>(cb), row0 + q * 32);
                            bulk_commit_group();
                        }
                    } else if (p.ok) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (cb + j < args.n) ybase[(cb + j) * args.ynb[2]] = v[j];
                    }
                }
            }
        }
        // Bulk stores read their staging before the CTA's shared memory goes away.
        if (lane == 0) bulk_wait_all();
    }

    // Single-lane roles rejoin their warps before the CTA-wide barrier.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

// Split-K reduction: output (row, col) = sum over the splits in order, then
// the chain; rows enumerate tiles as the GEMM's (conv positions via conv_pos).
template <int MODE>
__global__ void splitk_reduce_kernel(const GemmArgs a, int tiles) {
    // Rows a warp at a time, columns along the lanes (the host keeps
    // tiles * 128 * n below 2^31).
    const int rows = tiles * kBM;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int wr = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wr < rows * ((a.n + 31) / 32); wr += warps) {
        const int row = wr % rows;
        const int col = (wr / rows) * 32 + (threadIdx.x & 31);
        if (col >= a.n) continue;
        float v = 0.0f;
        for (int s = 0; s < a.ksplit; ++s) v += a.part[s * a.part_split + row * a.part_ld + col];
        if (MODE == kModeLinear) {
            const long long m = row;
            if (m >= a.m) continue;
            const long long i1 = m % a.rne1, t = m / a.rne1, i2 = t % a.rne2, i3 = t / a.rne2;
            float* out = a.y + i1 * a.ynb[1] + i2 * a.ynb[2] + i3 * a.ynb[3] + col * a.ynb[0];
            if (a.chain.from_redirect) v = *out + v;
            *out = apply_chain(a.chain, v, col, i1, i2, i3);
        } else {
            const ConvPos p = conv_pos(a.cg, static_cast<int>(row / kBM), static_cast<int>(row % kBM));
            if (!p.ok) continue;
            float* out = a.y + p.ox * a.ynb[0] + static_cast<long long>(p.oy) * a.ynb[1] + p.img * a.ynb[3] +
                         col * a.ynb[2];
            if (a.chain.from_redirect) v = *out + v;
            *out = apply_chain(a.chain, v, p.ox, p.oy, col, p.img);
        }
    }
}

// The same reduction four columns a thread, for outputs whose columns are
// contiguous and 16-byte aligned (linear: ynb[0] == 1; convolution:
// channels-last, ynb[2] == 1) with N % 4 == 0: one float4 of every split's
// partial row (part_ld is a multiple of 4) loaded four splits at a time, added
// in split order as the scalar kernel adds them, then the chain.
template <int MODE>
__global__ void __launch_bounds__(256) splitk_reduce4_kernel(const GemmArgs a, int tiles) {
    const long long rows = static_cast<long long>(tiles) * kBM;
    const int n4 = a.n / 4;
    const long long total = rows * n4;
    const long long step4 = a.part_split / 4;
    for (long long idx = blockIdx.x * 256LL + threadIdx.x; idx < total; idx += gridDim.x * 256LL) {
        const long long row = idx / n4;
        const int col = static_cast<int>(idx - row * n4) * 4;
        float* out;
        long long c0, c1, c2, c3;  // the chain's coordinates of the first column
        if (MODE == kModeLinear) {
            if (row >= a.m) continue;
            const long long i1 = row % a.rne1, t = row / a.rne1, i2 = t % a.rne2, i3 = t / a.rne2;
            out = a.y + i1 * a.ynb[1] + i2 * a.ynb[2] + i3 * a.ynb[3] + col;
            c0 = col; c1 = i1; c2 = i2; c3 = i3;
        } else {
            const ConvPos p = conv_pos(a.cg, static_cast<int>(row / kBM), static_cast<int>(row % kBM));
            if (!p.ok) continue;
            out = a.y + p.ox * a.ynb[0] + static_cast<long long>(p.oy) * a.ynb[1] + p.img * a.ynb[3] + col;
            c0 = p.ox; c1 = p.oy; c2 = col; c3 = p.img;
        }
        const float4* src = reinterpret_cast<const float4*>(a.part + row * a.part_ld + col);
        float4 acc = __ldg(src);
        int s = 1;
        for (; s + 3 < a.ksplit; s += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(src + (s + u) * step4);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc.x += v[u].x;
                acc.y += v[u].y;
                acc.z += v[u].z;
                acc.w += v[u].w;
            }
        }
        for (; s < a.ksplit; ++s) {
            const float4 v = __ldg(src + s * step4);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        float v[4] = {acc.x, acc.y, acc.z, acc.w};
        if (a.chain.from_redirect) {
            const float4 old = *reinterpret_cast<const float4*>(out);
            v[0] = old.x + v[0];
            v[1] = old.y + v[1];
            v[2] = old.z + v[2];
            v[3] = old.w + v[3];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
            v[e] = MODE == kModeLinear ? apply_chain(a.chain, v[e], c0 + e, c1, c2, c3)
                                       : apply_chain(a.chain, v[e], c0, c1, c2 + e, c3);
        *reinterpret_cast<float4*>(out) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

}  // namespace sdb
