// The tcgen05 GEMM of the linear layers and the direct convolution.
//
// C[m][n] = sum_k A[m][k] B[n][k] with
//   A: the activations (FP32 in HBM), rows m = tokens (linear) or output
//      positions (convolution, the im2col rows gathered straight from the
//      image: conv2d.cc:231-316 packs the same columns on the CPU);
//   B: the weights, repacked once by the weight store into FP16 [rows][Kpad]
//      (K-major, zero padded) and loaded by TMA in the 128-byte swizzle.
// Each A element is split x = hi + lo 2^-11 (ptx.cuh split_half) by the
// converter warps, which write both halves into shared memory in the UMMA
// K-major 128B-swizzled layout; one thread issues tcgen05.mma kind::f16 for
// hi x W and lo x W.  FP32 weights are split the same way (w = whi + wlo 2^-11)
// and add hi x wlo to the lo product.  The gated variant computes the x and
// the gate halves of a GEGLU product side by side and writes x * GELU(gate)
// (fusion.cc:290-310, mul_mat.cc:934-1058).
//
// Precision of the sums.  The tensor core's FP32 accumulation rounds toward
// zero: one k-step's add loses up to an ulp of the running sum, always in the
// same direction, so over hundreds of k-steps the error grows linearly (about
// 2^-23 of the sum per k-step, measured).  The hi product, which carries the
// sum, is therefore accumulated over one k-block (4 k-steps) at a time, into
// one of two tensor-memory buffers in turn, and the epilogue warps add each
// block's partial sum to FP32 registers with round-to-nearest while the next
// block computes.  The lo product (2^-11 of the sum) accumulates over all of K.
// The chain (bias, scale, SiLU, residual; fusion.h:51-91) is applied to
// sum + lo 2^-11 before the store.
//
// Warp roles (448 threads): warp 0 TMA producer; warp 1 MMA issuer and the
// tensor-memory allocation; warps 2-5 converters, which issue the loads of
// the next k-block while they convert the current one; warps 6-13 epilogue,
// two per quarter of tensor-memory lanes (warp w reads lanes 32*(w%4)..+31),
// each taking half the tile's columns.
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
constexpr int kGemmWarps = 14;  // 4 per SM sub-partition at most: 128 registers a thread
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kConvWarp0 = 2;   // first converter warp
constexpr int kEpiWarp0 = 6;    // first epilogue warp

struct ConvGeom {
    int iw, ih, ic, n;      // input [IW, IH, IC, N]
    int ow, oh;             // output [OW, OH, OC, N]
    int kw, kh;
    int s0, s1, p0, p1, d0, d1;
    int icp;                // channels per tap in the packed K order (a multiple of 16)
    long long xnb[4];       // input strides in elements
};

struct GemmArgs {
    const float* x;         // A source
    long long xld;          // linear: elements between rows of x
    int m;                  // rows of C
    int kpad;               // K padded to a multiple of kBK (packed weights' row length)
    int klog;               // logical K of a linear layer (columns of x read)
    int n;                  // columns of C (linear: output features; gated: the half)
    int b1_row;             // row offset in the packed weights of the second B operand
    float* y;               // output (the redirect when the chain has one)
    long long ynb[4];       // output strides in elements
    long long rne1, rne2;   // linear: row m -> (i1, i2, i3) = (m % rne1, m / rne1 % rne2, m / (rne1 rne2))
    ConvGeom cg;
    Chain chain;
    int vec;                // linear: x rows 16-byte aligned
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

// ---------------------------------------------------------------- producers
//
// A k-block of A is 128 rows x 64 columns: 1024 chunks of 8 values, one
// 16-byte chunk of hi and one of lo in shared memory.  Each of the 128
// converter threads takes 8 chunks, in two halves of 4; the loads of a half
// go into 32 registers, which are converted and stored while the loads of the
// next half are in flight.

// Linear: chunk (r, c) of k-block kb is x[m0 + r][kb*64 + 8c .. +7]; the
// thread takes chunks it*128 + t, it = 4h .. 4h + 3 (8 threads share a row:
// a row's 256 bytes are read by neighbouring threads).
__device__ __forceinline__ void load_linear(const GemmArgs& a, int m0, int kb, int h, int t, float (&v)[32]) {
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
        const int chunk = (4 * h + i4) * 128 + t;
        const int r = chunk >> 3, c = chunk & 7;
        const int m = m0 + r;
        const int k = kb * kBK + c * 8;
        if (m < a.m && a.vec && k + 8 <= a.klog) {
            const float4* p = reinterpret_cast<const float4*>(a.x + static_cast<long long>(m) * a.xld + k);
            const float4 u = __ldg(p), w = __ldg(p + 1);
            v[i4 * 8 + 0] = u.x; v[i4 * 8 + 1] = u.y; v[i4 * 8 + 2] = u.z; v[i4 * 8 + 3] = u.w;
            v[i4 * 8 + 4] = w.x; v[i4 * 8 + 5] = w.y; v[i4 * 8 + 6] = w.z; v[i4 * 8 + 7] = w.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                v[i4 * 8 + i] =
                    (m < a.m && k + i < a.klog) ? __ldg(a.x + static_cast<long long>(m) * a.xld + k + i) : 0.0f;
        }
    }
}

__device__ __forceinline__ uint32_t chunk_offset_linear(int h, int i4, int t) {
    const int chunk = (4 * h + i4) * 128 + t;
    return sw128_offset(chunk >> 3, chunk & 7);
}

// Convolution: row r = output position m0 + r; packed k = tap * icp + ic.
// Thread t takes row t, chunks 4h .. 4h + 3 (32 channels of a tap): a
// warp's loads of one channel are 32 neighbouring positions.
__device__ __forceinline__ void load_conv(const GemmArgs& a, int m0, int kb, int h, int t, float (&v)[32]) {
    const ConvGeom& g = a.cg;
    const int m = m0 + t;
    const bool row_ok = m < a.m;
    const int ox = m % g.ow;
    const int oy = (m / g.ow) % g.oh;
    const int img = m / (g.ow * g.oh);
    const float* base = a.x + static_cast<long long>(img) * g.xnb[3];
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
        const int k = kb * kBK + (4 * h + i4) * 8;  // 8 channels of one tap (icp % 16 == 0)
        const int tap = k / g.icp;
        const int ic0 = k - tap * g.icp;
        const int ky = tap / g.kw, kx = tap - ky * g.kw;
        const int iy = oy * g.s1 + ky * g.d1 - g.p1;
        const int ix = ox * g.s0 + kx * g.d0 - g.p0;
        const bool in = row_ok && tap < g.kw * g.kh && iy >= 0 && iy < g.ih && ix >= 0 && ix < g.iw;
        const float* p = base + static_cast<long long>(iy) * g.xnb[1] + static_cast<long long>(ix) * g.xnb[0];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int ic = ic0 + i;
            v[i4 * 8 + i] = (in && ic < g.ic) ? __ldg(p + static_cast<long long>(ic) * g.xnb[2]) : 0.0f;
        }
    }
}

template <int MODE>
__device__ __forceinline__ void load_half(const GemmArgs& a, int m0, int kb, int h, int t, float (&v)[32]) {
    if (MODE == kModeLinear) load_linear(a, m0, kb, h, t, v);
    else load_conv(a, m0, kb, h, t, v);
}

// Splits and stores a half; returns true when a value was beyond FP16's range.
template <int MODE>
__device__ __forceinline__ bool store_half(const float (&v)[32], int h, int t, uint32_t a_hi, uint32_t a_lo) {
    bool over = false;
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = v[i4 * 8 + i];
        uint4 hi, lo;
        over |= split8(x, hi, lo);
        const uint32_t off = MODE == kModeLinear ? chunk_offset_linear(h, i4, t) : sw128_offset(t, 4 * h + i4);
        st_shared_v4(a_hi + off, hi);
        st_shared_v4(a_lo + off, lo);
    }
    return over;
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
__device__ __forceinline__ void store_conv(const GemmArgs& a, int m, int col0, const float (&v)[NV]) {
    if (m >= a.m) return;
    const ConvGeom& g = a.cg;
    const long long ox = m % g.ow;
    const long long oy = (m / g.ow) % g.oh;
    const long long img = m / (g.ow * g.oh);
    const long long base = ox * a.ynb[0] + oy * a.ynb[1] + img * a.ynb[3];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int col = col0 + j;
        if (col < a.n) {
            float* out = a.y + base + col * a.ynb[2];
            float val = v[j];
            if (a.chain.from_redirect) val = *out + val;
            *out = apply_chain(a.chain, val, ox, oy, col, img);
        }
    }
}

// ---------------------------------------------------------------- kernel

template <int MODE, int WMODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_split_kernel(const __grid_constant__ CUtensorMap wmap, const GemmArgs args) {
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
    const int m0 = blockIdx.x * kBM;
    const int n0 = blockIdx.y * BN;
    const int kblocks = args.kpad / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1 + 4);  // TMA arrive.expect_tx + the four converter warps
            mbar_init(&empty[s], 1);     // the MMA commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&hi_full[b], 1);
            mbar_init(&hi_empty[b], 8);  // the eight epilogue warps
        }
        mbar_init(lo_full, 1);
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
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
            int issued = 0;
            for (int kb = 0; kb < kblocks; ++kb) {
                const int s = kb % S::kStages;
                const uint32_t parity = ((kb / S::kStages) & 1) ^ 1;
                if (!mbar_wait(&empty[s], parity, abort, args.err)) break;
                mbar_arrive_expect_tx(&full[s], S::kBBytes * (S::kHasB1 ? 2 : 1));
                tma_load_2d(stage_b0(s), &wmap, &full[s], kb * kBK, n0);
                if (S::kHasB1) tma_load_2d(stage_b1(s), &wmap, &full[s], kb * kBK, args.b1_row + n0);
                ++issued;
            }
            if (*abort) {
                // Let the loads this thread started land before the CTA exits.
                for (int kb = (issued > S::kStages ? issued - S::kStages : 0); kb < issued; ++kb)
                    mbar_wait_quiet(&full[kb % S::kStages], (kb / S::kStages) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
            bool ok = true;
            for (int kb = 0; kb < kblocks && ok; ++kb) {
                const int s = kb % S::kStages;
                const int b = kb & 1;
                if (!mbar_wait(&full[s], (kb / S::kStages) & 1, abort, args.err)) { ok = false; break; }
                if (!mbar_wait(&hi_empty[b], ((kb >> 1) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t ahi = smem_u32(stage_a_hi(s)), alo = smem_u32(stage_a_lo(s));
                const uint32_t b0 = smem_u32(stage_b0(s)), b1 = smem_u32(stage_b1(s));
                const uint32_t d_hi = tmem + b * BN;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t fresh = kk > 0 ? 1u : 0u;
                    const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
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
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------ converters
        const int t = threadIdx.x - kConvWarp0 * 32;
        bool over = false;
        float v0[32], v1[32];
        if (kblocks > 0) {
            load_half<MODE>(args, m0, 0, 0, t, v0);
            load_half<MODE>(args, m0, 0, 1, t, v1);
        }
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % S::kStages;
            const uint32_t parity = ((kb / S::kStages) & 1) ^ 1;
            if (!mbar_wait(&empty[s], parity, abort, args.err)) break;
            const uint32_t ahi = smem_u32(stage_a_hi(s)), alo = smem_u32(stage_a_lo(s));
            const bool more = kb + 1 < kblocks;
            over |= store_half<MODE>(v0, 0, t, ahi, alo);
            if (more) load_half<MODE>(args, m0, kb + 1, 0, t, v0);
            over |= store_half<MODE>(v1, 1, t, ahi, alo);
            if (more) load_half<MODE>(args, m0, kb + 1, 1, t, v1);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
        if (over) atomicOr(args.err, kErrRange);
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
        for (int kb = 0; kb < kblocks; ++kb) {
            const int b = kb & 1;
            if (!mbar_wait(&hi_full[b], (kb >> 1) & 1, abort, args.err)) { ok = false; break; }
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
        if (ok && mbar_wait(lo_full, 0, abort, args.err)) {
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
            if (MODE == kModeLinear)
                store_linear<WMODE, NV>(args, smem, ew, q, lane, m0, col0, sum, gsum);
            else
                store_conv<NV>(args, m0 + q * 32 + lane, col0, sum);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, S::kTmemCols);
    }
}

}  // namespace sdb
