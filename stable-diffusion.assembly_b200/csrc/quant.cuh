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
// A CTA owns a tile of 128 rows by 128 product columns (two boxes of 64
// packed weight rows: consecutive columns, or for the gated GELU 64 x columns
// and the matching 64 gate columns) and walks its tiles persistently.  Warp 0
// loads 64-byte stretches of k (SW64 boxes) and the groups' scales; warp 1
// issues the MMAs of each group into one of two 128-column accumulators;
// sixteen warps drain a group's sums while the next group's are being made,
// and keep the tile's FP32 running values in registers (32 a thread: a row,
// 32 columns, or 16 x and 16 gate columns).  The fold, not the tensor core,
// bounds the kernel: five FP32 operations an element a group against an
// integer product of 2 x 64 operations at twice the FP16 tensor rate.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/sdb.h"
#include "chain.cuh"
#include "ptx.cuh"

namespace sdb {

constexpr int kQRows = 128;                              // tile rows
constexpr int kQCols = 128;                              // tile product columns
constexpr int kQStageK = 64;                             // bytes (= numbers) of k a stage holds
constexpr int kQStages = 6;
constexpr int kQRing = 4;                                // groups of scales in flight
constexpr int kQEpiWarps = 16;
constexpr int kQThreads = 32 * (2 + kQEpiWarps);
constexpr int kQABytes = kQRows * kQStageK;              // 8 KiB
constexpr int kQBBytes = kQCols * kQStageK;              // 8 KiB
constexpr int kQStageBytes = kQABytes + kQBBytes;
constexpr int kQScaleFloats = 2 * 128 + 2 * 2 * 64;      // A's (scale, offset) x 128 rows, B's x 2 boxes of 64
constexpr int kQSmemBytes = 1024 + kQStages * kQStageBytes + kQRing * kQScaleFloats * 4 + 256;

struct QGemmArgs {
    int m;              // rows of the output
    int n;              // columns of the output (gated: of one half)
    int groups;         // groups of k
    int cpg;            // 32-byte chunks of k a group: group / 32
    int kchunks;        // groups * cpg
    int tiles_m, tiles_n, items;
    int b_second;       // gated: packed row of the first gate row
    int magic;          // the sums convert exactly by the 1.5 * 2^23 trick (|sum| < 2^22)
    float* y;
    long long ynb[4];   // output strides, elements
    long long rne1, rne2;
    Chain chain;
    unsigned* err;
};

// Shared-memory descriptor of a K-major operand tile in the 64-byte swizzle:
// rows of 64 bytes, 8-row atoms 512 bytes apart (what a TMA load with
// CU_TENSOR_MAP_SWIZZLE_64B writes); the tile base is 512-byte aligned and a
// step of 32 bytes of k moves the start address.
__device__ __forceinline__ uint64_t desc_kmajor_sw64(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(512 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(4) << 61;                      // swizzle: 64 B
    return d;
}

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

// Two columns of a row folded in: t = fma(sa * sb, sum, t); t = fma(-oa, ob, t),
// each operation rounded to the nearest as the scalar ones are (the paired
// instructions round each half on its own).
__device__ __forceinline__ void qfold2(float& t0, float& t1, float s0, float s1, uint64_t sa2, uint64_t noa2,
                                       float sb0, float sb1, float ob0, float ob1) {
    uint64_t t = pack2(t0, t1), sab;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(sab) : "l"(sa2), "l"(pack2(sb0, sb1)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(t) : "l"(sab), "l"(pack2(s0, s1)));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(t) : "l"(noa2), "l"(pack2(ob0, ob1)));
    unpack2(t, t0, t1);
}

// 32-bit sums to floats: exact in both forms for |sum| < 2^22.
__device__ __forceinline__ float sum_to_float(uint32_t bits, bool magic) {
    return magic ? __fsub_rn(__int_as_float(static_cast<int>(bits) + 0x4B400000), 12582912.0f)
                 : __int2float_rn(static_cast<int>(bits));
}

// 16 columns of a group folded into t[0..15]: the sums from tensor memory at
// `taddr`, the columns' scales and offsets from shared memory.
__device__ __forceinline__ void qfold16(float* t, uint32_t taddr, float sa, float oa, const float* sb,
                                        const float* ob, bool magic) {
    float raw[16];
    tmem_ld16(taddr, raw);
    tmem_ld_wait();
    const uint64_t sa2 = pack2(sa, sa), noa2 = pack2(-oa, -oa);
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(sb + j);
        const float4 o4 = *reinterpret_cast<const float4*>(ob + j);
        const float s0 = sum_to_float(__float_as_uint(raw[j]), magic);
        const float s1 = sum_to_float(__float_as_uint(raw[j + 1]), magic);
        const float s2 = sum_to_float(__float_as_uint(raw[j + 2]), magic);
        const float s3 = sum_to_float(__float_as_uint(raw[j + 3]), magic);
        qfold2(t[j], t[j + 1], s0, s1, sa2, noa2, b4.x, b4.y, o4.x, o4.y);
        qfold2(t[j + 2], t[j + 3], s2, s3, sa2, noa2, b4.z, b4.w, o4.z, o4.w);
    }
}

template <bool GATED>
__global__ void __launch_bounds__(kQThreads, 1)
qgemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap asmap,
             const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap wsmap,
             const QGemmArgs args) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* scales = reinterpret_cast<float*>(smem + kQStages * kQStageBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(scales + kQRing * kQScaleFloats);
    uint64_t* empty = full + kQStages;
    uint64_t* sfull = empty + kQStages;
    uint64_t* sempty = sfull + kQRing;
    uint64_t* tfull = sempty + kQRing;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kQStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < kQRing; ++r) {
            mbar_init(&sfull[r], 1);
            mbar_init(&sempty[r], kQEpiWarps);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kQEpiWarps);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&amap);
        tma_prefetch_desc(&asmap);
        tma_prefetch_desc(&wmap);
        tma_prefetch_desc(&wsmap);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * kQCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nstages = (args.kchunks + 1) / 2;   // stages an item takes

    auto rows_b = [&](int tn, int& r0, int& r1) {
        r0 = GATED ? tn * 64 : tn * 128;
        r1 = GATED ? args.b_second + tn * 64 : tn * 128 + 64;
    };

    bool ok = true;
    int st_count = 0, sc_count = 0;    // the producer's stages and scale groups issued
    if (warp == 0) {
        if (lane == 0) {
            for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
                const int tm = item % args.tiles_m, tn = item / args.tiles_m;
                int r0, r1;
                rows_b(tn, r0, r1);
                int next = 0;
                for (int gi = 0; gi < args.groups && ok; ++gi) {
                    const int slot = sc_count % kQRing;
                    if (!mbar_wait(&sempty[slot], ((sc_count / kQRing) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                    float* sc = scales + slot * kQScaleFloats;
                    mbar_arrive_expect_tx(&sfull[slot], kQScaleFloats * 4);
                    tma_load_2d(sc, &asmap, &sfull[slot], tm * kQRows, 2 * gi);
                    tma_load_2d(sc + 256, &wsmap, &sfull[slot], r0, 2 * gi);
                    tma_load_2d(sc + 384, &wsmap, &sfull[slot], r1, 2 * gi);
                    ++sc_count;
                    const int need = ((gi + 1) * args.cpg + 1) / 2;
                    for (; next < need; ++next) {
                        const int s = st_count % kQStages;
                        if (!mbar_wait(&empty[s], ((st_count / kQStages) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                        uint8_t* st = smem + s * kQStageBytes;
                        mbar_arrive_expect_tx(&full[s], kQStageBytes);
                        tma_load_2d(st, &amap, &full[s], next * kQStageK, tm * kQRows);
                        tma_load_2d(st + kQABytes, &wmap, &full[s], next * kQStageK, r0);
                        tma_load_2d(st + kQABytes + kQBBytes / 2, &wmap, &full[s], next * kQStageK, r1);
                        ++st_count;
                    }
                }
            }
            // On an abort, wait for the loads still in flight before leaving.
            if (!ok) {
                for (int i = (st_count > kQStages ? st_count - kQStages : 0); i < st_count; ++i)
                    mbar_wait_quiet(&full[i % kQStages], (i / kQStages) & 1, 100000000ull);
                for (int i = (sc_count > kQRing ? sc_count - kQRing : 0); i < sc_count; ++i)
                    mbar_wait_quiet(&sfull[i % kQRing], (i / kQRing) & 1, 100000000ull);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_u8s8_s32(kQRows, kQCols);
            int st_base = 0, gcount = 0;
            for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
                for (int gi = 0; gi < args.groups && ok; ++gi, ++gcount) {
                    const int buf = gcount & 1;
                    if (!mbar_wait(&tempty[buf], ((gcount >> 1) & 1) ^ 1, abort, args.err)) { ok = false; break; }
                    tc_fence_after();
                    for (int i = 0; i < args.cpg; ++i) {
                        const int c = gi * args.cpg + i;
                        const int gs = st_base + (c >> 1), s = gs % kQStages;
                        if ((c & 1) == 0) {
                            if (!mbar_wait(&full[s], (gs / kQStages) & 1, abort, args.err)) { ok = false; break; }
                            tc_fence_after();
                        }
                        const uint32_t a = smem_u32(smem + s * kQStageBytes) + (c & 1) * 32;
                        mma_i8(tmem + buf * kQCols, desc_kmajor_sw64(a), desc_kmajor_sw64(a + kQABytes), idesc,
                               i > 0 ? 1u : 0u);
                        if ((c & 1) == 1 || c == args.kchunks - 1) mma_commit(&empty[s]);
                    }
                    if (!ok) break;
                    mma_commit(&tfull[buf]);
                }
                st_base += nstages;
            }
            if (!ok) {
                mma_commit(drain);
                mbar_wait_quiet(drain, 0, 100000000ull);
            }
        }
    } else {
        // ---- the sixteen draining warps
        const int q = warp & 3;                 // tensor-memory lane quarter
        const int part = (warp - 2) >> 2;       // which quarter of the columns
        const int row = q * 32 + lane;
        const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const bool magic = args.magic != 0;
        // Accumulator columns of t[0..15] and t[16..31]: 32 consecutive ones,
        // or (gated) 16 of the x box and the matching 16 of the gate box; the
        // scales of column c at sc[256 + c / 64 * 128 + c % 64], offsets 64 on.
        const int c0 = GATED ? part * 16 : part * 32;
        const int c1 = GATED ? 64 + part * 16 : part * 32 + 16;
        const int s0 = 256 + (c0 >> 6) * 128 + (c0 & 63);
        const int s1 = 256 + (c1 >> 6) * 128 + (c1 & 63);
        int gcount = 0;
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, args.err) ? 1 : 0) != 0;
        };
        for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
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
            float t[32];
            if (!GATED && args.chain.from_redirect) {
#pragma unroll
                for (int j = 0; j < 32; ++j) t[j] = yrow[min(col + j, args.n - 1LL) * args.ynb[0]];
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) t[j] = 0.0f;
            }
            for (int gi = 0; gi < args.groups; ++gi, ++gcount) {
                const int buf = gcount & 1, slot = gcount % kQRing;
                if (!warp_wait(&tfull[buf], (gcount >> 1) & 1)) { ok = false; break; }
                if (!warp_wait(&sfull[slot], (gcount / kQRing) & 1)) { ok = false; break; }
                tc_fence_after();
                const float* sc = scales + slot * kQScaleFloats;
                const float sa = sc[row], oa = sc[128 + row];
                const uint32_t base = lane_addr + buf * kQCols;
                qfold16(t, base + c0, sa, oa, sc + s0, sc + s0 + 64, magic);
                qfold16(t + 16, base + c1, sa, oa, sc + s1, sc + s1 + 64, magic);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[buf]);
                    mbar_arrive(&sempty[slot]);
                }
            }
            if (!ok) break;
            // ---- the tile's chain and stores
            ChainRow cr;
            row_offsets(args.chain, cr, 0, i1, i2, i3);
            if (GATED) {
                apply_chain_cols<0, 16>(args.chain, cr, t, col, args.n - 1);
                apply_chain_cols<0, 16>(args.chain, cr, t + 16, args.n + col, 2LL * args.n - 1);
#pragma unroll
                for (int j = 0; j < 16; ++j) t[j] *= gelu(t[16 + j]);
                if (live) {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (col + j < args.n) yrow[(col + j) * args.ynb[0]] = t[j];
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; c += 16) {
                    apply_chain_cols<0, 16>(args.chain, cr, t + c, col + c, args.n - 1);
                    if (live) {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (col + c + j < args.n) yrow[(col + c + j) * args.ynb[0]] = t[c + j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * kQCols);
    }
}

// Host side (quant.cu).
bool quantized_linear(int64_t rows);
int run_quantized_linear(const sdb_tensor* w, const sdb_tensor* x, const sdb_tensor* dst, const sdb_chain* chain,
                         cudaStream_t st, bool gated);

}  // namespace sdb
