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
// sum, is therefore accumulated over one k-block (4 k-steps) at a time, into
// one of two tensor-memory buffers in turn, and the epilogue warps add each
// block's partial sum to FP32 registers with round-to-nearest while the next
// block computes.  The lo product (2^-11 of the sum) accumulates over all of
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
enum : int { kWeightHalf = 0, kWeightSplit = 1, kWeightGated = 2 };

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
    int a_lo_row;           // row (linear) / image (conv) offset of the lo plane in A's map
    int kblocks;            // K / kBK of the whole product
    int ksplit;             // CTAs along K (grid.z)
    int n;                  // columns of C (linear: output features; gated: the half)
    int b1_row;             // row offset in the packed weights of the second B operand
    uint32_t a_tx;          // bytes of one A tile (hi or lo) as TMA writes it
    float* y;               // output (the redirect when the chain has one)
    float* part;            // split-K: partial sums [ksplit][rows][part_ld]
    long long part_ld;      // columns of a partial row
    long long part_split;   // elements between splits
    long long ynb[4];       // output strides in elements
    long long rne1, rne2;   // linear: row m -> (i1, i2, i3) = (m % rne1, m / rne1 % rne2, m / (rne1 rne2))
    ConvGeom cg;
    Chain chain;
    unsigned* err;
};

template <int WMODE>
struct GemmShape {
    static constexpr int BN = WMODE == kWeightGated ? 64 : 128;
    static constexpr bool kHasB1 = WMODE != kWeightHalf;
    static constexpr int kABytes = kBM * kBK * 2;  // one of hi / lo
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = 2 * kABytes + kBBytes * (kHasB1 ? 2 : 1);
    static constexpr int kStages = (200 * 1024) / kStageBytes >= 6 ? 6 : (200 * 1024) / kStageBytes;
    // Tensor-memory columns: hi buffers (two; gated: x0 x1 g0 g1) then lo (gated: x, g).
    static constexpr int kHiCols = WMODE == kWeightGated ? 4 * BN : 2 * BN;
    static constexpr int kLoCol = kHiCols;
    static constexpr int kAccCols = kHiCols + (WMODE == kWeightGated ? 2 * BN : BN);
    static constexpr int kTmemCols = 512;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(kAccCols <= 512, "accumulators exceed tensor memory");
    static_assert(kStages >= 2, "too few stages");
    static_assert(kStages * kStageBytes >= 2 * 8 * 32 * 33 * 4 + 8 * 32 * 32, "epilogue staging does not fit");
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

struct RowInfo {
    long long base, i1, i2, i3;
};

// A linear layer's rows are contiguous: the 32 x 32 values of a warp go
// through shared memory (the pipeline stages, idle once the lo accumulator is
// full) and the warp writes 32 rows as 128-byte runs.
template <int WMODE, int NV>
__device__ __forceinline__ void store_linear(const GemmArgs& a, uint8_t* smem, int ew, int q, int lane, int m0,
                                             int col0, const float (&v)[NV], const float (&gv)[NV]) {
    constexpr bool kGated = WMODE == kWeightGated;
    float* tile = reinterpret_cast<float*>(smem) + ew * (32 * 33);
    RowInfo* info = reinterpret_cast<RowInfo*>(smem + 8 * 32 * 33 * 4) + ew * 32;
    float* gtile = reinterpret_cast<float*>(smem + 8 * 32 * 33 * 4 + 8 * 32 * 32) + ew * (32 * 33);
    {
        const long long m = m0 + q * 32 + lane;
        RowInfo r;
        r.i1 = m % a.rne1;
        const long long t = m / a.rne1;
        r.i2 = t % a.rne2;
        r.i3 = t / a.rne2;
        r.base = r.i1 * a.ynb[1] + r.i2 * a.ynb[2] + r.i3 * a.ynb[3];
        info[lane] = r;
    }
    const int rows = min(32, a.m - (m0 + q * 32));
#pragma unroll
    for (int c = 0; c < NV / 32; ++c) {
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            tile[lane * 33 + j] = v[c * 32 + j];
            if (kGated) gtile[lane * 33 + j] = gv[c * 32 + j];
        }
        __syncwarp();
        const int col = col0 + c * 32 + lane;
        if (col < a.n) {
#pragma unroll 4
            for (int r = 0; r < rows; ++r) {
                const RowInfo ri = info[r];
                float* out = a.y + ri.base + col * a.ynb[0];
                float val = tile[r * 33 + lane];
                if (kGated) {
                    const float xv = apply_chain(a.chain, val, col, ri.i1, ri.i2, ri.i3);
                    const float g = apply_chain(a.chain, gtile[r * 33 + lane], a.n + col, ri.i1, ri.i2, ri.i3);
                    *out = xv * gelu(g);
                } else {
                    if (a.chain.from_redirect) val = *out + val;
                    *out = apply_chain(a.chain, val, col, ri.i1, ri.i2, ri.i3);
                }
            }
        }
    }
}

// A convolution's output is [OW, OH, OC, N]: a lane's row is an output
// position and neighbouring lanes are neighbouring positions, so each column
// (channel) is written by the warp as one run.
template <int NV>
__device__ __forceinline__ void store_conv(const GemmArgs& a, const ConvPos& p, int col0, const float (&v)[NV]) {
    if (!p.ok) return;
    const long long base = p.ox * a.ynb[0] + static_cast<long long>(p.oy) * a.ynb[1] + p.img * a.ynb[3];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = col0 + j;
        if (col < a.n) {
            float* out = a.y + base + col * a.ynb[2];
            float val = v[j];
            if (a.chain.from_redirect) val = *out + val;
            *out = apply_chain(a.chain, val, p.ox, p.oy, col, p.img);
        }
    }
}

// Split-K: the CTA's raw sums into its slice of the workspace, [row][col]
// with row = tile * 128 + lane row.
template <int NV>
__device__ __forceinline__ void store_partial(const GemmArgs& a, int split, int row, int col0, const float (&v)[NV]) {
    float* dst = a.part + split * a.part_split + static_cast<long long>(row) * a.part_ld + col0;
#pragma unroll
    for (int j = 0; j < NV; j += 4)
        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

// ---------------------------------------------------------------- kernel

template <int MODE, int WMODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_split_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                  const GemmArgs args) {
    using S = GemmShape<WMODE>;
    constexpr int BN = S::BN;
    constexpr bool kGated = WMODE == kWeightGated;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
    uint64_t* empty = full + S::kStages;
    uint64_t* hi_full = empty + S::kStages;   // [2]
    uint64_t* hi_empty = hi_full + 2;         // [2]
    uint64_t* lo_full = hi_empty + 2;
    uint64_t* drain = lo_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    const int n0 = blockIdx.y * BN;
    const int split = blockIdx.z;
    const int per_split = (args.kblocks + args.ksplit - 1) / args.ksplit;
    const int kb0 = split * per_split;
    const int kb1 = min(args.kblocks, kb0 + per_split);
    const int kblocks = max(0, kb1 - kb0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1);   // TMA arrive.expect_tx
            mbar_init(&empty[s], 1);  // the MMA commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&hi_full[b], 1);
            mbar_init(&hi_empty[b], 8);  // the eight epilogue warps
        }
        mbar_init(lo_full, 1);
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&amap);
        tma_prefetch_desc(&wmap);
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a_hi = [&](int s) { return smem + s * S::kStageBytes; };
    auto stage_a_lo = [&](int s) { return smem + s * S::kStageBytes + S::kABytes; };
    auto stage_b0 = [&](int s) { return smem + s * S::kStageBytes + 2 * S::kABytes; };
    auto stage_b1 = [&](int s) { return smem + s * S::kStageBytes + 2 * S::kABytes + S::kBBytes; };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            // This tile's A coordinates.
            int ax = 0, ay = 0, az = 0;
            const ConvGeom& g = args.cg;
            if (MODE == kModeConv) {
                const int tx = tile % g.tw, ty = (tile / g.tw) % g.th, tz = tile / (g.tw * g.th);
                ax = tx * g.owt * g.s0 - g.p0;
                ay = ty * g.oht * g.s1 - g.p1;
                az = tz * g.nt;
            }
            int issued = 0;
            const uint32_t tx_bytes = 2 * args.a_tx + S::kBBytes * (S::kHasB1 ? 2 : 1);
            for (int i = 0; i < kblocks; ++i) {
                const int kb = kb0 + i;
                const int s = i % S::kStages;
                const uint32_t parity = ((i / S::kStages) & 1) ^ 1;
                if (!mbar_wait(&empty[s], parity, abort, args.err)) break;
                mbar_arrive_expect_tx(&full[s], tx_bytes);
                if (MODE == kModeLinear) {
                    tma_load_2d(stage_a_hi(s), &amap, &full[s], kb * kBK, tile * kBM);
                    tma_load_2d(stage_a_lo(s), &amap, &full[s], kb * kBK, args.a_lo_row + tile * kBM);
                } else {
                    const int tap = kb / g.cblocks;
                    const int cx0 = (kb - tap * g.cblocks) * kBK;
                    const int ky = tap / g.kw, kx = tap - ky * g.kw;
                    const int x = ax + kx * g.d0, y = ay + ky * g.d1;
                    tma_load_4d(stage_a_hi(s), &amap, &full[s], cx0, x, y, az);
                    tma_load_4d(stage_a_lo(s), &amap, &full[s], cx0, x, y, args.a_lo_row + az);
                }
                tma_load_2d(stage_b0(s), &wmap, &full[s], kb * kBK, n0);
                if (S::kHasB1) tma_load_2d(stage_b1(s), &wmap, &full[s], kb * kBK, args.b1_row + n0);
                ++issued;
            }
            if (*abort) {
                // Let the loads this thread started land before the CTA exits.
                for (int i = (issued > S::kStages ? issued - S::kStages : 0); i < issued; ++i)
                    mbar_wait_quiet(&full[i % S::kStages], (i / S::kStages) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
            bool ok = true;
            for (int i = 0; i < kblocks && ok; ++i) {
                const int s = i % S::kStages;
                const int b = i & 1;
                if (!mbar_wait(&full[s], (i / S::kStages) & 1, abort, args.err)) { ok = false; break; }
                if (!mbar_wait(&hi_empty[b], ((i >> 1) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ahi = smem_u32(stage_a_hi(s)), alo = smem_u32(stage_a_lo(s));
                const uint32_t b0 = smem_u32(stage_b0(s)), b1 = smem_u32(stage_b1(s));
                const uint32_t d_hi = tmem + b * BN;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t fresh = kk > 0 ? 1u : 0u;
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    const uint64_t dah = desc_kmajor_sw128(ahi + kk * 32), dal = desc_kmajor_sw128(alo + kk * 32);
                    const uint64_t db0 = desc_kmajor_sw128(b0 + kk * 32);
                    mma_f16(d_hi, dah, db0, idesc, fresh);
                    mma_f16(tmem + S::kLoCol, dal, db0, idesc, acc);
                    if (WMODE == kWeightSplit) {
                        mma_f16(tmem + S::kLoCol, dah, desc_kmajor_sw128(b1 + kk * 32), idesc, 1u);
                    } else if (kGated) {
                        const uint64_t db1 = desc_kmajor_sw128(b1 + kk * 32);
                        mma_f16(tmem + 2 * BN + b * BN, dah, db1, idesc, fresh);
                        mma_f16(tmem + S::kLoCol + BN, dal, db1, idesc, acc);
                    }
                }
                mma_commit(&empty[s]);
                mma_commit(&hi_full[b]);
            }
            if (ok) {
                mma_commit(lo_full);
            } else {
                // Wind down: every MMA issued completes before tensor memory is freed.
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (drains hi per k-block)
        const int ew = warp - kEpiWarp0;      // 0..7
        const int q = warp & 3;               // TMEM lane quarter this warp may read
        const int half = ew >> 2;             // which half of the tile's columns
        constexpr int NV = BN / 2;            // columns per warp
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        float sum[NV], gsum[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            sum[j] = 0.0f;
            gsum[j] = 0.0f;
        }
        bool ok = true;
        for (int i = 0; i < kblocks; ++i) {
            const int b = i & 1;
            if (!mbar_wait(&hi_full[b], (i >> 1) & 1, abort, args.err)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < NV; c += 32) {
                float part[32];
                tmem_ld32(lane_addr + b * BN + half * NV + c, part);
                if (kGated) {
                    float gpart[32];
                    tmem_ld32(lane_addr + 2 * BN + b * BN + half * NV + c, gpart);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) gsum[c + j] += gpart[j];
                } else {
                    tmem_ld_wait();
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) sum[c + j] += part[j];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&hi_empty[b]);
        }
        if (ok && kblocks > 0 && mbar_wait(lo_full, 0, abort, args.err)) {
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
            const int col0 = n0 + half * NV;
            const int row = q * 32 + lane;
            if (args.ksplit > 1) {
                store_partial<NV>(args, split, tile * kBM + row, col0, sum);
            } else if (MODE == kModeLinear) {
                store_linear<WMODE, NV>(args, smem, ew, q, lane, tile * kBM, col0, sum, gsum);
            } else {
                store_conv<NV>(args, conv_pos(args.cg, tile, row), col0, sum);
            }
        } else if (ok && kblocks == 0 && args.ksplit > 1) {
            float zero[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) zero[j] = 0.0f;
            store_partial<NV>(args, split, tile * kBM + q * 32 + lane, n0 + half * NV, zero);
        }
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

}  // namespace sdb
