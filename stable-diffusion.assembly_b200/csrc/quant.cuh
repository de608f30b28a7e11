// The quantized linear layer (tuning bits = 2..8): the reference's integer
// products (quant.h, quant.cc) on the tensor cores.
//
// Inputs are unsigned bytes with a zero point, one scale and offset per row
// per group of k; weights signed, symmetric, one scale per output row per
// group (or per whole row).  A group's products are summed exactly in 32-bit
// integers by tcgen05.mma kind::i8 into tensor memory, and every group is
// folded into the FP32 result the way the reference's micro-kernel folds it
// (quant.cc:113-166):
//
//     t = fma(sa * sb, float(sum), t);  t = fma(-oa, ob, t)
//
// group after group in k order, from 0 (or the output's old value, for a
// residual written in place).  The FP32 arithmetic is the reference's,
// operation for operation, so the result is the reference's C++ form bit for
// bit.
//
// A CTA owns a tile of 128 rows by 128 product columns (128 packed weight
// rows: consecutive columns, or for the gated GELU 64 x columns and the
// matching 64 gate columns) and walks its tiles persistently.  Both operands
// are laid out in global memory tile by tile as shared memory wants them: a
// 64-byte stretch of k of 128 rows is one contiguous 8 KiB block, already in
// the 64-byte swizzle (quant_tile_offset), and a group's scales and offsets
// of 128 rows one 1 KiB block, so that every load is one bulk copy (tensor
// maps over 64-byte rows delivered about 9 bytes a clock to an SM here).
//
// All sixteen warps drain a group's sums while later groups' are being made
// in the others of four 128-column accumulators, and keep the tile's FP32
// running values in registers (32 a thread: a row, 32 columns, or 16 x and 16
// gate columns).  Lanes 0 have second roles between groups: the loads of a
// group a few groups ahead, each warp in turn, and -- the last warp to finish
// a group -- the MMAs of a later group into the accumulator it leaves.
// Sixteen warps, four an SM sub-partition, leave each thread 128 registers.
// The fold, not the tensor core, bounds the kernel: about 3.5 instructions an
// element a group (paired FP32 instructions, the integer-to-float conversion
// by the 1.5 * 2^23 trick) against an integer product issued in 1/4 of the
// time.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "gemm_wide.cuh"
#include "ptx.cuh"

namespace sdb {

constexpr int kQRows = 128;                              // tile rows
constexpr int kQCols = 128;                              // tile product columns
constexpr int kQStageK = 64;                             // bytes (= numbers) of k a stage holds
constexpr int kQStages = 6;
constexpr int kQRing = 10;                               // groups of scales in flight
constexpr int kQEpiWarps = 16;
constexpr int kQThreads = 32 * kQEpiWarps;
constexpr int kQABytes = kQRows * kQStageK;              // 8 KiB
constexpr int kQBBytes = kQCols * kQStageK;              // 8 KiB
constexpr int kQStageBytes = kQABytes + kQBBytes;
constexpr int kQScaleFloats = 2 * 128 + 2 * 128;         // A's (scales, offsets) x 128 rows, then B's
constexpr int kQBoxBytes = 32 * 64;                      // a 32-row x 16-column FP32 store box (two a warp)
constexpr int kQAcc = 4;                                 // accumulators of 128 columns in tensor memory
// mbarriers (stages, scale ring, accumulators, a drain for each warp), the
// fold counters, the TMEM slot and the abort flag.
constexpr int kQBarrierBytes = 8 * (2 * kQStages + 2 * kQRing + kQAcc + kQEpiWarps) + 4 * kQAcc + 8;
constexpr int kQSmemBytes =
    1024 + kQStages * kQStageBytes + kQRing * kQScaleFloats * 4 + 2 * kQEpiWarps * kQBoxBytes + kQBarrierBytes;
static_assert(kQSmemBytes <= 227 * 1024, "shared memory");

// The byte of row r (of 128), k-byte b (of 64) in a stage block: the 16-byte
// chunk b / 16 of row r at r * 64 + ((b / 16) ^ (r / 2) % 4) * 16 -- the
// layout a TMA load with CU_TENSOR_MAP_SWIZZLE_64B writes, which
// desc_kmajor_sw64 describes.
__host__ __device__ __forceinline__ int quant_tile_offset(int r, int b) {
    return r * 64 + ((((b >> 4) ^ (r >> 1)) & 3) << 4) + (b & 15);
}

struct QGemmArgs {
    const uint8_t* a;   // inputs: [tiles_m][nstages][8 KiB]
    const float* as;    // their scales: [tiles_m][groups][2][128]
    const uint8_t* w;   // weights: [tiles_n][nstages][8 KiB]
    const float* ws;    // their scales: [tiles_n][groups][2][128]
    int m;              // rows of the output
    int n;              // columns of the output (gated: of one half)
    int groups;         // groups of k
    int cpg;            // 32-byte chunks of k a group: group / 32
    int kchunks;        // groups * cpg
    int tiles_m, tiles_n, items;
    int batch_tiles;    // batched products (Winograd's xi, attention's heads): row tiles of one batch, whose
                        // weights are tiles_n tiles of their own; 0 for one product
    int batch_rep;      // batches sharing one set of weights (heads sharing keys); 1 otherwise
    int magic;          // the sums convert exactly by the 1.5 * 2^23 trick (|sum| < 2^22)
    int store;          // kStoreTma: whole 32 x 16 boxes through the output map; else direct
    float* y;
    long long ynb[4];   // output strides, elements
    long long rne1, rne2;
    Chain chain;
    unsigned* err;
};

// Instruction descriptor of kind::i8: A unsigned bytes, B signed bytes, S32
// accumulator, both K-major.
__host__ __device__ constexpr uint32_t idesc_u8s8_s32(int m, int n) {
    return (2u << 4)                                  // D format: S32
           | (0u << 7) | (1u << 10)                   // A: U8, B: S8
           | (static_cast<uint32_t>(n >> 3) << 17)
           | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ void unpack2(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}

__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// 32 lanes x 16 columns of 32-bit tensor memory, as raw bits.
__device__ __forceinline__ void tmem_ld16_bits(uint32_t addr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr)
        : "memory");
}

// A pair of 32-bit sums to floats, exactly: by the 1.5 * 2^23 trick for
// |sum| < 2^22 (the integer added to the bits of 1.5 * 2^23, which then
// subtracted), by conversion otherwise.
__device__ __forceinline__ uint64_t sums_to_floats(uint32_t a, uint32_t b, bool magic) {
    if (magic) {
        const uint64_t biased = pack2(__int_as_float(static_cast<int>(a) + 0x4B400000),
                                      __int_as_float(static_cast<int>(b) + 0x4B400000));
        return fadd2(biased, pack2(-12582912.0f, -12582912.0f));
    }
    return pack2(__int2float_rn(static_cast<int>(a)), __int2float_rn(static_cast<int>(b)));
}

// 16 columns of a group folded into the pairs t2[0..7]:
// t = fma(sa * sb, sum, t); t = fma(-oa, ob, t), each operation rounded to
// the nearest as the scalar ones are (a paired instruction rounds each half on
// its own); the columns' scales and offsets from shared memory.
__device__ __forceinline__ void qfold16(uint64_t* t2, const uint32_t* raw, uint64_t sa2, uint64_t noa2,
                                        const float* sb, const float* ob, bool magic) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(sb + j);
        const float4 o4 = *reinterpret_cast<const float4*>(ob + j);
        const uint64_t s01 = sums_to_floats(raw[j], raw[j + 1], magic);
        const uint64_t s23 = sums_to_floats(raw[j + 2], raw[j + 3], magic);
        uint64_t& t01 = t2[j / 2];
        uint64_t& t23 = t2[j / 2 + 1];
        t01 = ffma2(fmul2(sa2, pack2(b4.x, b4.y)), s01, t01);
        t23 = ffma2(fmul2(sa2, pack2(b4.z, b4.w)), s23, t23);
        t01 = ffma2(noa2, pack2(o4.x, o4.y), t01);
        t23 = ffma2(noa2, pack2(o4.z, o4.w), t23);
    }
}

// A warp's 32 rows x 16 columns out through the store map from one of its two
// boxes: the box's previous store (all but the latest bulk group) has read it.
__device__ __forceinline__ void store_box16_pair(const CUtensorMap* map, uint8_t* box, int lane, const float* v,
                                                 int x, int y) {
    if (lane == 0) bulk_wait_read_but_one();
    __syncwarp();
    stage_row16(box, lane, v);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, box, x, y);
        bulk_commit_group();
    }
}

template <bool GATED>
__global__ void __launch_bounds__(kQThreads, 1)
qgemm_kernel(const __grid_constant__ CUtensorMap ymap, const QGemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    // Offsets from the shared array itself (not through an integer), so that
    // the compiler keeps the scale reads as shared-memory loads it can schedule.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    float* scales = reinterpret_cast<float*>(smem + kQStages * kQStageBytes);
    uint8_t* staging = reinterpret_cast<uint8_t*>(scales + kQRing * kQScaleFloats);
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + 2 * kQEpiWarps * kQBoxBytes);
    uint64_t* empty = full + kQStages;
    uint64_t* sfull = empty + kQStages;
    uint64_t* sempty = sfull + kQRing;
    uint64_t* tfull = sempty + kQRing;
    uint64_t* drain = tfull + kQAcc;
    int* folds = reinterpret_cast<int*>(drain + kQEpiWarps);      // warps done, per accumulator
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(folds + kQAcc);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        // With groups of 32 a stage holds two groups, each of which releases it.
        for (int s = 0; s < kQStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], args.cpg == 1 ? 2 : 1);
        }
        for (int r = 0; r < kQRing; ++r) {
            mbar_init(&sfull[r], 1);
            mbar_init(&sempty[r], kQEpiWarps);
        }
        for (int b = 0; b < kQAcc; ++b) {
            mbar_init(&tfull[b], 1);
            folds[b] = 0;
        }
        for (int w = 0; w < kQEpiWarps; ++w) mbar_init(&drain[w], 1);
        *abort = 0;
        fence_barrier_init();
        if (args.store == kStoreTma) tma_prefetch_desc(&ymap);
    }
    if (warp == 0) tmem_alloc(tmem_slot, kQAcc * kQCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // The CTA's groups in order: item j = blockIdx.x + (seq / groups) * gridDim.x, group seq % groups.
    const int my_items = args.items > static_cast<int>(blockIdx.x)
                             ? (args.items - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                   static_cast<int>(gridDim.x)
                             : 0;
    const int total = my_items * args.groups;
    const int nstages = (args.kchunks + 1) / 2;   // stages an item takes
    // Groups loaded ahead: as many as the stages hold without reusing one that
    // a group not yet folded may still need (a warp folding group e has seen
    // the products of e complete).  A warp can be up to kQAcc - 1 groups ahead
    // of the slowest, so the scale ring holds ahead + kQAcc groups and its
    // slots are free when their loads are issued.
    const int ahead = max(1, min(kQRing - kQAcc, (2 * kQStages) / args.cpg));

    // ---- the loads of the CTA's group number g (lane 0 of some warp): its
    // scales into ring slot g % kQRing, and the stages its chunks begin.
    // Stages are numbered through the CTA's items, nstages an item; group gi
    // of an item needs its stages up to ((gi + 1) * cpg + 1) / 2.
    auto need = [&](int gi) { return gi < 0 ? 0 : ((gi + 1) * args.cpg + 1) / 2; };
    int produced[2] = {-1, -1};   // the last two groups this warp's lane 0 loaded
    auto produce = [&](int g) -> bool {
        if (g >= total) return true;
        produced[0] = produced[1];
        produced[1] = g;
        const int item = blockIdx.x + (g / args.groups) * gridDim.x, gi = g % args.groups;
        const int tm = item % args.tiles_m, tn = item / args.tiles_m;
        const int tw = args.batch_tiles ? tn + (tm / args.batch_tiles / args.batch_rep) * args.tiles_n : tn;
        const int slot = g % kQRing;
        if (!mbar_wait(&sempty[slot], ((g / kQRing) & 1) ^ 1, abort, args.err)) return false;
        float* sc = scales + slot * kQScaleFloats;
        mbar_arrive_expect_tx(&sfull[slot], kQScaleFloats * 4);
        bulk_load(sc, args.as + (static_cast<long long>(tm) * args.groups + gi) * 256, 1024, &sfull[slot]);
        bulk_load(sc + 256, args.ws + (static_cast<long long>(tw) * args.groups + gi) * 256, 1024, &sfull[slot]);
        const int base = (g / args.groups) * nstages;
        for (int ls = need(gi - 1); ls < need(gi); ++ls) {
            const int st_count = base + ls, s = st_count % kQStages;
            if (!mbar_wait(&empty[s], ((st_count / kQStages) & 1) ^ 1, abort, args.err)) return false;
            uint8_t* st = smem + s * kQStageBytes;
            mbar_arrive_expect_tx(&full[s], kQStageBytes);
            bulk_load(st, args.a + (static_cast<long long>(tm) * nstages + ls) * kQABytes, kQABytes, &full[s]);
            bulk_load(st + kQABytes, args.w + (static_cast<long long>(tw) * nstages + ls) * kQBBytes, kQBBytes,
                      &full[s]);
        }
        return true;
    };

    // ---- the products of the CTA's group number g into accumulator g % kQAcc,
    // by one lane: warp 1's for the first groups, then, for group g, the lane of
    // the last warp to finish folding group g - mma_ahead, which every other
    // warp has then left (the accumulator's previous use, when mma_ahead is
    // kQAcc; an older one otherwise).  Each issuing lane commits
    // the stages it read and the accumulator itself.
    constexpr uint32_t idesc = idesc_u8s8_s32(kQRows, kQCols);
    bool issued_any = false;
    auto issue = [&](int g) -> bool {
        if (g >= total) return true;
        issued_any = true;
        const int gi = g % args.groups, base = (g / args.groups) * nstages;
        const int buf = g % kQAcc;
        tc_fence_after();
        for (int i = 0; i < args.cpg; ++i) {
            const int c = gi * args.cpg + i;
            const int gs = base + (c >> 1), s = gs % kQStages;
            if ((c & 1) == 0 || i == 0) {
                if (!mbar_wait(&full[s], (gs / kQStages) & 1, abort, args.err)) return false;
                tc_fence_after();
            }
            const uint32_t a = smem_u32(smem + s * kQStageBytes) + (c & 1) * 32;
            mma_i8(tmem + buf * kQCols, desc_kmajor_sw64(a), desc_kmajor_sw64(a + kQABytes), idesc, i > 0 ? 1u : 0u);
            if (args.cpg == 1) {
                // Groups of 32 share a stage: each releases it once, and the
                // group alone in an item's last stage twice.
                mma_commit(&empty[s]);
                if ((c & 1) == 0 && c == args.kchunks - 1) mma_commit(&empty[s]);
            } else if ((c & 1) == 1 || c == args.kchunks - 1) {
                // A stage is released after its second chunk, or after its only
                // one (an item of an odd number of chunks: groups of 96 or 160).
                mma_commit(&empty[s]);
            }
        }
        mma_commit(&tfull[buf]);
        return true;
    };

    // Group g's loads are issued by warp g % kQEpiWarps: before its first
    // fold for g < ahead, after folding group g - ahead otherwise.
    bool ok = true;
    if (lane == 0)
        for (int g = warp; g < ahead && ok; g += kQEpiWarps) ok = produce(g);
    // The MMAs of a group are issued only once its loads have been: groups
    // [0, mma_ahead) by warp 1 here, group e + mma_ahead after the fold of e.
    const int mma_ahead = min(kQAcc, ahead);
    if (warp == 1 && lane == 0)
        for (int g = 0; g < mma_ahead && ok; ++g) ok = issue(g);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;

    // ---- every warp: the fold of each group, the tile's chain and stores
    const int q = warp & 3;                 // tensor-memory lane quarter
    const int part = warp >> 2;             // which quarter of the columns
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const bool magic = args.magic != 0;
    // Accumulator columns of t[0..15] and t[16..31]: 32 consecutive ones, or
    // (gated) 16 of the x half and the matching 16 of the gate half; the
    // scale of column c at sc[256 + c], its offset at sc[384 + c].
    const int c0 = GATED ? part * 16 : part * 32;
    const int c1 = GATED ? 64 + part * 16 : part * 32 + 16;
    const int s0 = 256 + c0;
    const int s1 = 256 + c1;
    // A group's accumulator and scales, waited for together: both tests in
    // one round trip (a completed barrier's test alone costs a few hundred
    // clocks), every lane observing both phases.
    auto warp_wait2 = [&](uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2) -> bool {
        const long long t0 = clock64();
        for (uint32_t it = 0;; ++it) {
            if (__all_sync(0xffffffffu, mbar_try_wait2(b1, p1, b2, p2) ? 1 : 0)) return true;
            if ((it & 255u) == 255u) {
                if (*abort) return false;
                if (clock64() - t0 > kWaitLimitCycles) {
                    if (lane == 0) {
                        *abort = 1;
                        if (args.err) atomicOr(args.err, kErrTimeout);
                    }
                    return false;
                }
            }
        }
    };
    int e = 0;   // groups folded
    for (int j = 0; j < my_items && ok; ++j) {
        const int item = blockIdx.x + j * gridDim.x;
        const int tm = item % args.tiles_m, tn = item / args.tiles_m;
        const long long m = static_cast<long long>(tm) * kQRows + row;
        const bool live = m < args.m;
        const long long mc = live ? m : args.m - 1;
        const long long i1 = mc % args.rne1, rest = mc / args.rne1;
        const long long i2 = rest % args.rne2, i3 = rest / args.rne2;
        float* yrow = args.y + i1 * args.ynb[1] + i2 * args.ynb[2] + i3 * args.ynb[3];
        // The output column of t[0]: plain, 32 consecutive columns; gated, 16 of them.
        const long long col = GATED ? static_cast<long long>(tn) * 64 + part * 16
                                    : static_cast<long long>(tn) * 128 + part * 32;
        uint64_t t2[16];
        uint8_t* box = staging + 2 * warp * kQBoxBytes;
        const int row0 = tm * kQRows + q * 32;
        if (!GATED && args.chain.from_redirect && args.store == kStoreTma) {
            // The sums start from the output's values, read coalesced a box at a
            // time (-0 + x is x for every x, zeros of either sign included).
#pragma unroll
            for (int c = 0; c < 32; c += 16) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = -0.0f;
                add_old_box16(args.y, args.n, row0, args.m, col + c, args.n, box + (c / 16) * kQBoxBytes, lane, o);
#pragma unroll
                for (int i = 0; i < 8; ++i) t2[c / 2 + i] = pack2(o[2 * i], o[2 * i + 1]);
            }
        } else if (!GATED && args.chain.from_redirect) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                t2[i] = pack2(yrow[min(col + 2 * i, args.n - 1LL) * args.ynb[0]],
                              yrow[min(col + 2 * i + 1, args.n - 1LL) * args.ynb[0]]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) t2[i] = 0ull;
        }
        for (int gi = 0; gi < args.groups; ++gi, ++e) {
            const int buf = e % kQAcc, slot = e % kQRing;
            if (!warp_wait2(&tfull[buf], (e / kQAcc) & 1, &sfull[slot], (e / kQRing) & 1)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t raw[32];
            const uint32_t base = lane_addr + buf * kQCols;
            tmem_ld16_bits(base + c0, *reinterpret_cast<uint32_t(*)[16]>(raw));
            tmem_ld16_bits(base + c1, *reinterpret_cast<uint32_t(*)[16]>(raw + 16));
            const float* sc = scales + slot * kQScaleFloats;
            const float sa = sc[row], oa = sc[128 + row];
            tmem_ld_wait();
            const uint64_t sa2 = pack2(sa, sa), noa2 = pack2(-oa, -oa);
            qfold16(t2, raw, sa2, noa2, sc + s0, sc + s0 + 128, magic);
            qfold16(t2 + 8, raw + 16, sa2, noa2, sc + s1, sc + s1 + 128, magic);
            tc_fence_before();
            __syncwarp();
            // The second roles: the loads of group e + ahead (this warp's turn);
            // then, the last warp to finish group e, the products of group
            // e + mma_ahead (into accumulator e % kQAcc when mma_ahead is kQAcc).
            bool lane_ok = true;
            if (lane == 0) {
                mbar_arrive(&sempty[slot]);
                if ((e + ahead) % kQEpiWarps == warp) lane_ok = produce(e + ahead);
                __threadfence_block();
                const int before = atomicAdd(&folds[buf], 1);
                if (before == kQEpiWarps * (e / kQAcc) + kQEpiWarps - 1) {
                    __threadfence_block();
                    lane_ok = issue(e + mma_ahead) && lane_ok;
                }
            }
            ok = __shfl_sync(0xffffffffu, lane_ok ? 1 : 0, 0) != 0;
            if (!ok) break;
        }
        if (!ok) break;
        float t[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) unpack2(t2[i], t[2 * i], t[2 * i + 1]);
        ChainRow cr;
        row_offsets(args.chain, cr, 0, i1, i2, i3);
        if (GATED) {
            apply_chain_cols<0, 16>(args.chain, cr, t, col, args.n - 1);
            apply_chain_cols<0, 16>(args.chain, cr, t + 16, args.n + col, 2LL * args.n - 1);
#pragma unroll
            for (int i = 0; i < 16; ++i) t[i] *= gelu(t[16 + i]);
            if (args.store == kStoreTma) {
                store_box16_pair(&ymap, box + (j & 1) * kQBoxBytes, lane, t, static_cast<int>(col), row0);
            } else if (live) {
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (col + i < args.n) yrow[(col + i) * args.ynb[0]] = t[i];
            }
        } else {
            apply_chain_cols<0, 32>(args.chain, cr, t, col, args.n - 1);
#pragma unroll
            for (int c = 0; c < 32; c += 16) {
                if (args.store == kStoreTma) {
                    store_box16_pair(&ymap, box + (c / 16) * kQBoxBytes, lane, t + c, static_cast<int>(col + c), row0);
                } else if (live) {
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        if (col + c + i < args.n) yrow[(col + c + i) * args.ynb[0]] = t[c + i];
                }
            }
        }
    }
    // Wind down.  On an abort the MMA lane waits for what it issued, the load
    // lane for the loads in flight.
    if (!ok && lane == 0 && issued_any) {
        mma_commit(&drain[warp]);
        mbar_wait_quiet(&drain[warp], 0, 100000000ull);
    }
    // Every load issued completes before the CTA leaves: on an abort each
    // loading lane waits (bounded) for the last loads it issued.
    if (!ok && lane == 0) {
        for (int i = 0; i < 2; ++i) {
            const int g = produced[i];
            if (g < 0) continue;
            mbar_wait_quiet(&sfull[g % kQRing], (g / kQRing) & 1, 100000000ull);
            const int gi = g % args.groups, base = (g / args.groups) * nstages;
            for (int ls = need(gi - 1); ls < need(gi); ++ls)
                mbar_wait_quiet(&full[(base + ls) % kQStages], ((base + ls) / kQStages) & 1, 100000000ull);
        }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kQAcc * kQCols);
    }
}

// Host side (quant.cu).
bool quantized_linear(int64_t rows);
int run_quantized_linear(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                         cudaStream_t st, bool gated);
bool quantized_conv();
int run_quantized_conv(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                       const sdb_chain* chain, cudaStream_t st);
bool quantized_winograd(const sdb_tensor* w, const sdb_tensor* dst, const int32_t params[6]);
bool quantized_attention(int64_t lk);
int run_quantized_attention(const sdb_tensor* q, const sdb_tensor* k, const sdb_tensor* v, const sdb_tensor* dst,
                            float scale, const sdb_chain* chain, cudaStream_t st);
int run_quantized_winograd(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const int32_t params[6],
                           const sdb_chain* chain, cudaStream_t st);

}  // namespace sdb
