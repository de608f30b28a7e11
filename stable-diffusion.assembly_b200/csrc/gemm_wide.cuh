// The wide-tile tcgen05 GEMM: 128 rows x BN (up to 256) columns a tile, FP16
// weights, for the linear layers, the gated GEGLU product and the direct
// convolution.  The arithmetic: the activation split x = hi + lo 2^-11, each
// k-block's hi W + (lo W) 2^-11 in one tensor-memory accumulator (the lo
// products first, the first hi product scaling them as it adds), drained every
// k-block into FP32 registers with round-to-nearest.
//
// Why wide.  Each kind::f16 MMA reads its A and B tiles from shared memory, and
// TMA writes them there: at 128 x 128 a k-block moves ~112 KB through shared
// memory for 2 x 128 x 128 x 64 products, which the SM's 128 B/clk bound to
// ~900 cycles (measured: ~950), twice the tensor time.  At 128 x 256 the same
// products cost ~160 KB per 2 x 128 x 256 x 64, ~1250 cycles for twice the work.
//
// Tensor memory holds two such accumulators (columns 0 and 256), so the
// products of k-block kb + 1 run while the warps drain kb.  Sixteen warps (four
// per tensor-memory lane quarter, BN / 4 columns each) hold the running sums --
// 18 or more warps would cap a thread at 96 registers.  No warp is left over
// for the producers, so lane 0 of warp 0 also issues the TMA loads (after its
// drain) and lane 0 of warp 1 the MMAs (of the next k-block, before its drain:
// the issuing thread blocks while the tensor core takes them).
#pragma once

#include "gemm.cuh"

namespace sdb {

constexpr int kWideWarps = 16;
constexpr int kWideThreads = kWideWarps * 32;

template <int BN>
struct WideShape {
    static_assert(BN == 128 || BN == 192 || BN == 256, "tile width");
    static constexpr int kABytes = kBM * kBK * 2;             // one plane (hi or lo) of A
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = 2 * kABytes + kBBytes;
    static constexpr int kBoxBytes = 32 * 64;                 // a 32-row x 16-column FP32 store box
    static constexpr int kStagingBytes = kWideWarps * kBoxBytes;
    static constexpr int kBudget = 227 * 1024 - kStagingBytes - 1024 - 512;
    static constexpr int kStages = kBudget / kStageBytes >= 6 ? 6 : kBudget / kStageBytes;
    static constexpr int kLoCol = 256;                        // accumulators at [0, BN) and [256, 256 + BN)
    static constexpr int CPW = BN / 4;                        // accumulator columns a warp owns
    static constexpr int kSmemBytes = kStages * kStageBytes + kStagingBytes + 1024 + 512;
    static_assert(kStages >= 2, "too few stages");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// sum[j] += scale * tmem[addr + j] for j < N (N a multiple of 16), 32 columns
// at a time.
template <int N>
__device__ __forceinline__ void tmem_add(uint32_t addr, float* sum, float scale) {
#pragma unroll
    for (int c = 0; c < N; c += 32) {
        float a[16], b[16];
        tmem_ld16(addr + c, a);
        if (c + 16 < N) tmem_ld16(addr + c + 16, b);
        tmem_ld_wait();
        // Packed: two columns an instruction (fma(v, 1, s) is s + v exactly).
        if (scale == 1.0f) {
            add_packed<16>(sum + c, a);
            if (c + 16 < N) add_packed<16>(sum + c + 16, b);
        } else {
            fma_packed<16>(sum + c, a, scale);
            if (c + 16 < N) fma_packed<16>(sum + c + 16, b, scale);
        }
    }
}

// A 32-row x 16-column FP32 box for a TMA store in the 64-byte swizzle: row r's
// 16-byte chunk k at r * 64 + ((k ^ (r / 2) % 4) * 16) -- each eight lanes'
// vector stores cover the 32 banks once.
__device__ __forceinline__ void stage_row16(uint8_t* box, int lane, const float* v) {
    const uint32_t base = smem_u32(box) + lane * 64;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint4 q = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                   __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
        st_shared_v4(base + ((k ^ ((lane >> 1) & 3)) << 4), q);
    }
}

// One warp's 32 rows x 16 columns out through the store map (after the previous
// store from the box has read it).
__device__ __forceinline__ void store_box16(const CUtensorMap* map, uint8_t* box, int lane, const float* v, int x,
                                            int y) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    stage_row16(box, lane, v);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, box, x, y);
        bulk_commit_group();
    }
}

// v[0..15] += the existing output of this thread's row in the warp's 32 x 16
// box (rows row0.., columns col0.. of a row-major FP32 matrix, ld floats a
// row): the warp reads the box coalesced -- a float4 a lane, eight rows an
// instruction -- into the staging box in the store layout, then each thread
// takes its row.  Rows and columns past the valid ones read as 0.
__device__ __forceinline__ void add_old_box16(const float* y, long long ld, long long row0, long long rows,
                                              long long col0, long long cols, uint8_t* box, int lane, float* v) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    const uint32_t b = smem_u32(box);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = (lane >> 2) + 8 * i, c4 = lane & 3;
        float4 val = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (row0 + r < rows && col0 + 4 * c4 < cols)
            val = __ldg(reinterpret_cast<const float4*>(y + (row0 + r) * ld + col0 + 4 * c4));
        st_shared_v4(b + r * 64 + ((c4 ^ ((r >> 1) & 3)) << 4),
                     make_uint4(__float_as_uint(val.x), __float_as_uint(val.y), __float_as_uint(val.z),
                                __float_as_uint(val.w)));
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint4 o = ld_shared_v4(b + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4));
        v[4 * k] += __uint_as_float(o.x);
        v[4 * k + 1] += __uint_as_float(o.y);
        v[4 * k + 2] += __uint_as_float(o.z);
        v[4 * k + 3] += __uint_as_float(o.w);
    }
    __syncwarp();
}

// One output row of a linear-layer tile: where it goes and its chain operands.
struct LinearRow {
    bool live;         // inside the output
    ChainRow cr;
    float* yrow;
};

__device__ __forceinline__ LinearRow linear_row(const GemmArgs& args, int tm, int row) {
    LinearRow r;
    const long long m = static_cast<long long>(tm) * kBM + row;
    r.live = m < args.m;
    const long long mc = r.live ? m : args.m - 1;
    // The row's ggml coordinates: rows of a 2-D output are i1 itself (no division).
    long long i1 = mc, i2 = 0, i3 = 0;
    if (args.rne1 < args.m) {
        const long long rest = mc / args.rne1;
        i1 = mc - rest * args.rne1;
        i2 = rest % args.rne2;
        i3 = rest / args.rne2;
    }
    row_offsets(args.chain, r.cr, 0, i1, i2, i3);
    r.yrow = args.y + i1 * args.ynb[1] + i2 * args.ynb[2] + i3 * args.ynb[3];
    return r;
}

// Sixteen output columns cb .. cb + 15 of a warp's 32 rows (rows tm * 128 +
// q * 32 + lane) out of registers: the chain (bias, scale, residual, SiLU; a
// gated product x * GELU(gate) after both halves' chains, `gate` holding the
// gate half's sums) applied, stored by TMA (kStoreTma) or directly.
template <bool GATED>
__device__ __forceinline__ void store_linear_group(const GemmArgs& args, const CUtensorMap* ymap, const LinearRow& r,
                                                   float* v, float* gate, long long cb, int tm, int q, int lane,
                                                   uint8_t* box) {
    if (GATED) {
        apply_chain_cols<0, 16>(args.chain, r.cr, v, cb, args.n - 1);
        apply_chain_cols<0, 16>(args.chain, r.cr, gate, args.n + cb, 2LL * args.n - 1);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] *= gelu(gate[j]);
    } else {
        if (args.chain.from_redirect) {
            if (args.store == kStoreTma) {
                add_old_box16(args.y, args.n, static_cast<long long>(tm) * kBM + q * 32, args.m, cb, args.n, box, lane,
                              v);
            } else {
                float old[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) old[j] = r.yrow[min(cb + j, args.n - 1LL) * args.ynb[0]];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = old[j] + v[j];
            }
        }
        apply_chain_cols<0, 16>(args.chain, r.cr, v, cb, args.n - 1);
    }
    if (args.store == kStoreTma) {
        store_box16(ymap, box, lane, v, static_cast<int>(cb), tm * kBM + q * 32);
    } else if (r.live) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (cb + j < args.n) r.yrow[(cb + j) * args.ynb[0]] = v[j];
    }
}

// A finished linear-layer tile (or a split-K part of one) out of the sixteen
// draining warps' registers: warp (q, part) holds rows q * 32 + lane, columns
// colA .. colA + BN / 4 of the product (gated: BN / 8 of the x half, then the
// matching BN / 8 of the gate half).  Split-K parts go to the partial sums
// through `ymap` (the reduction applies the chain).
template <bool GATED, int BN>
__device__ __forceinline__ void store_linear_tile(const GemmArgs& args, const CUtensorMap* ymap, float* sum, int tm,
                                                  int tn, int split, int q, int lane, int colA, uint8_t* box) {
    constexpr int CPW = BN / 4;
    if (args.ksplit > 1) {
        const int prow = (split * args.tiles_m + tm) * kBM + q * 32;
#pragma unroll
        for (int c = 0; c < CPW; c += 16) store_box16(ymap, box, lane, sum + c, tn * BN + colA + c, prow);
        return;
    }
    const LinearRow r = linear_row(args, tm, q * 32 + lane);
    constexpr int NOUT = GATED ? CPW / 2 : CPW;     // output columns this warp writes
    const long long ocol0 = GATED ? static_cast<long long>(tn) * (BN / 2) + colA : static_cast<long long>(tn) * BN + colA;
#pragma unroll
    for (int c = 0; c < NOUT; c += 16)
        store_linear_group<GATED>(args, ymap, r, sum + c, GATED ? sum + CPW / 2 + c : nullptr, ocol0 + c, tm, q, lane,
                                  box);
}

template <int MODE, bool GATED, int BN>
__global__ void __launch_bounds__(kWideThreads, 1)
gemm_wide_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap,
                 const __grid_constant__ CUtensorMap ymap, const GemmArgs args) {
    using S = WideShape<BN>;
    constexpr int CPW = S::CPW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + S::kStages * S::kStageBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + S::kStagingBytes);
    uint64_t* empty = full + S::kStages;
    uint64_t* d_full = empty + S::kStages;   // [2] an accumulator's products completed
    uint64_t* d_empty = d_full + 2;          // [2] every warp drained it
    uint64_t* drain = d_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = warp & 3;           // tensor-memory lane quarter
    const int part = warp >> 2;       // which quarter of the tile's columns
    uint8_t* box = staging + warp * S::kBoxBytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&d_full[b], 1);
            mbar_init(&d_empty[b], kWideWarps);
        }
        mbar_init(drain, 1);
        *abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&amap);
        tma_prefetch_desc(&wmap);
        if (args.store == kStoreTma || args.ksplit > 1) tma_prefetch_desc(&ymap);
    }
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Items run column tile fastest, so that the CTAs working at one time on a row tile's column
    // tiles read its activations from DRAM once between them (the weights stay in L2).
    auto item_range = [&](int item, int& tm, int& tn, int& split, int& kb0, int& kb1) {
        tn = item % args.tiles_n;
        const int rest = item / args.tiles_n;
        tm = rest % args.tiles_m;
        split = rest / args.tiles_m;
        kb0 = split * args.per_split;
        kb1 = min(args.kblocks, kb0 + args.per_split);
    };
    // The global sequence of k-blocks this CTA consumes, item after item.
    int total_kb = 0;
    for (int item = blockIdx.x; item < args.items; item += gridDim.x) {
        int tm, tn, split, kb0, kb1;
        item_range(item, tm, tn, split, kb0, kb1);
        total_kb += kb1 - kb0;
    }

    // ---- producer (warp 0, lane 0): issues the loads of k-block number `it`.
    const ConvGeom& g = args.cg;
    const uint32_t tx_bytes = 2 * args.a_tx + S::kBBytes;
    int p_item = blockIdx.x, p_kb = 0, p_kb1 = 0, p_tm = 0, p_tn = 0;  // the producer's cursor
    int issued = 0;
    auto producer_next = [&]() -> bool {  // one more k-block's loads, if its stage is free
        if (issued >= total_kb) return true;
        while (p_kb >= p_kb1) {
            int split, kb0;
            item_range(p_item, p_tm, p_tn, split, kb0, p_kb1);
            p_kb = kb0;
            if (p_kb >= p_kb1) p_item += gridDim.x;
        }
        const int s = issued % S::kStages;
        if (!mbar_wait(&empty[s], ((issued / S::kStages) & 1) ^ 1, abort, args.err)) return false;
        mbar_arrive_expect_tx(&full[s], tx_bytes);
        uint8_t* st = smem + s * S::kStageBytes;
        const int kb = p_kb;
        if (MODE == kModeLinear) {
            tma_load_3d(st, &amap, &full[s], kb * kBK, p_tm * kBM, 0);
        } else {
            const int tx = p_tm % g.tw, ty = (p_tm / g.tw) % g.th, tz = p_tm / (g.tw * g.th);
            const int tap = kb / g.cblocks;
            const int cx0 = (kb - tap * g.cblocks) * kBK;
            const int ky = tap / g.kw, kx = tap - ky * g.kw;
            const int x = tx * g.owt * g.s0 - g.p0 + kx * g.d0, y = ty * g.oht * g.s1 - g.p1 + ky * g.d1;
            if (args.a_planes == 2) {
                tma_load_5d(st, &amap, &full[s], cx0, x, y, tz * g.nt, 0);
            } else {
                tma_load_5d(st, &amap, &full[s], cx0, x, y, tz * g.nt, 0);
                tma_load_5d(st + S::kABytes, &amap, &full[s], cx0, x, y, tz * g.nt, 1);
            }
        }
        if (GATED) {
            tma_load_2d(st + 2 * S::kABytes, &wmap, &full[s], kb * kBK, p_tn * (BN / 2));
            tma_load_2d(st + 2 * S::kABytes + S::kBBytes / 2, &wmap, &full[s], kb * kBK, args.b1_row + p_tn * (BN / 2));
        } else {
            tma_load_2d(st + 2 * S::kABytes, &wmap, &full[s], kb * kBK, p_tn * BN);
        }
        ++issued;
        if (++p_kb >= p_kb1) p_item += gridDim.x;
        return true;
    };

    // ---- MMA issuer (warp 1, lane 0): k-block number m_it of the CTA's sequence into
    // accumulator m_it % 2 (columns 0 and kLoCol): the lo products first into a fresh
    // accumulator, then the hi products, the first of them scaling the lo sum by 2^-11
    // (tcgen05.mma's scale of the input D), so that one accumulator holds the k-block's
    // hi W + (lo W) 2^-11.  The issuing thread blocks while the tensor core takes the
    // products, so it issues k-block kb + 1 before its warp drains kb: the products of
    // kb + 1 run while every warp drains kb.
    constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
    int m_it = 0;  // k-blocks issued
    auto issue_kblock = [&]() -> bool {
        const int s = m_it % S::kStages, b = m_it & 1;
        if (!mbar_wait(&full[s], (m_it / S::kStages) & 1, abort, args.err)) return false;
        if (!mbar_wait(&d_empty[b], ((static_cast<uint32_t>(m_it) >> 1) & 1u) ^ 1u, abort, args.err)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (b ? S::kLoCol : 0u);
        const uint32_t ahi = smem_u32(smem + s * S::kStageBytes), alo = ahi + S::kABytes;
        const uint32_t b0 = ahi + 2 * S::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16(d, desc_kmajor_sw128(alo + kk * 32), desc_kmajor_sw128(b0 + kk * 32), idesc, kk > 0 ? 1u : 0u);
        mma_f16_scale_lo(d, desc_kmajor_sw128(ahi), desc_kmajor_sw128(b0), idesc);
#pragma unroll
        for (int kk = 1; kk < kBK / 16; ++kk)
            mma_f16(d, desc_kmajor_sw128(ahi + kk * 32), desc_kmajor_sw128(b0 + kk * 32), idesc, 1u);
        mma_commit(&empty[s]);
        mma_commit(&d_full[b]);
        ++m_it;
        return true;
    };

    // Columns of the accumulator this warp owns: plain, [part * CPW, +CPW);
    // gated, CPW / 2 of the x half and the matching CPW / 2 of the gate half.
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int colA = GATED ? part * (CPW / 2) : part * CPW;
    const int colB = GATED ? BN / 2 + part * (CPW / 2) : 0;

    // Waits every lane of the warp makes together; the verdict is the warp's.
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, args.err) ? 1 : 0) != 0;
    };

    bool ok = true;
    if (warp == 0 && lane == 0)
        for (int i = 0; i < S::kStages && ok; ++i) ok = producer_next();
    if (warp == 1 && lane == 0 && total_kb > 0) ok = issue_kblock();
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    int e_it = 0;
    for (int item = blockIdx.x; item < args.items && ok; item += gridDim.x) {
        int tm, tn, split, kb0, kb1;
        item_range(item, tm, tn, split, kb0, kb1);
        float sum[CPW];
#pragma unroll
        for (int j = 0; j < CPW; ++j) sum[j] = 0.0f;
        for (int kb = kb0; kb < kb1 && ok; ++kb, ++e_it) {
            bool lane_ok = true;
            if (warp == 1 && lane == 0 && e_it + 1 < total_kb) lane_ok = issue_kblock();
            if (__shfl_sync(0xffffffffu, lane_ok ? 1 : 0, 0) == 0) { ok = false; break; }
            const int b = e_it & 1;
            if (!warp_wait(&d_full[b], (static_cast<uint32_t>(e_it) >> 1) & 1u)) { ok = false; break; }
            tc_fence_after();
            const uint32_t acc = lane_addr + (b ? S::kLoCol : 0u);
            if (GATED) {
                tmem_add<CPW / 2>(acc + colA, sum, 1.0f);
                tmem_add<CPW / 2>(acc + colB, sum + CPW / 2, 1.0f);
            } else {
                tmem_add<CPW>(acc + colA, sum, 1.0f);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[b]);
            // k-block e_it's products are done, so its stage is free: the next load never waits.
            if (warp == 0 && lane == 0) lane_ok = producer_next();
            if (__shfl_sync(0xffffffffu, lane_ok ? 1 : 0, 0) == 0) { ok = false; break; }
        }
        if (!ok) break;

        // ---- the tile's epilogue (the next item's products run meanwhile)
        const int row = q * 32 + lane;
        if (args.ksplit > 1 || MODE == kModeLinear) {
            store_linear_tile<GATED, BN>(args, &ymap, sum, tm, tn, split, q, lane, colA, box);
        } else {
            const ConvPos p = conv_pos(g, tm, row);
            const int ox = p.ok ? p.ox : 0, oy = p.ok ? p.oy : 0, img = p.ok ? p.img : 0;
            ChainRow cr;
            row_offsets(args.chain, cr, 2, ox, oy, img);
            float* ybase = args.y + ox * args.ynb[0] + static_cast<long long>(oy) * args.ynb[1] + img * args.ynb[3];
            const int ty = (tm / g.tw) % g.th, tz = tm / (g.tw * g.th);
            const int row0 = (tz * g.nt * g.oh + ty * g.oht) * g.ow;
#pragma unroll
            for (int c = 0; c < CPW; c += 16) {
                float* v = sum + c;
                const long long cb = static_cast<long long>(tn) * BN + colA + c;
                if (args.chain.from_redirect) {
                    if (args.store == kStoreTma) {
                        add_old_box16(args.y, args.n, row0 + q * 32, static_cast<long long>(g.n) * g.oh * g.ow, cb,
                                      args.n, box, lane, v);
                    } else {
                        float old[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) old[j] = ybase[min(cb + j, args.n - 1LL) * args.ynb[2]];
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = old[j] + v[j];
                    }
                }
                apply_chain_cols<2, 16>(args.chain, cr, v, cb, args.n - 1);
                if (args.store == kStoreTma) {
                    store_box16(&ymap, box, lane, v, static_cast<int>(cb), row0 + q * 32);
                } else if (p.ok) {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (cb + j < args.n) ybase[(cb + j) * args.ynb[2]] = v[j];
                }
            }
        }
    }
    // Wind down.  On an abort the MMA thread waits for what it issued.
    if (!ok && warp == 1 && lane == 0) {
        mma_commit(drain);
        mbar_wait_quiet(drain, 0, 100000000ull);
    }
    if (!ok && warp == 0 && lane == 0) {
        for (int i = (issued > S::kStages ? issued - S::kStages : 0); i < issued; ++i)
            mbar_wait_quiet(&full[i % S::kStages], (i / S::kStages) & 1, 100000000ull);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace sdb
