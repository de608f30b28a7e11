// Inline-PTX building blocks for sm_100a: mbarriers with bounded waits, TMA
// tile loads, tcgen05 tensor-memory allocation, MMA issue, commit and loads.
//
// Every wait in this library is bounded: a wait that has not completed after
// kWaitLimitNs nanoseconds of %globaltimer sets the kernel's abort flag and a
// bit in the device error word, and returns false; the kernel then winds down
// (waits, again bounded, for its own copies and MMAs in flight, frees tensor
// memory) and exits.  No kernel here traps or spins without a limit.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace sdb {

// Device error word bits (read back by sdb_device_status()).
enum : unsigned {
    kErrTimeout = 1u << 0,   // a bounded wait ran out
    kErrRange = 1u << 1,     // an activation was beyond the FP16 range of the split
    kErrBounds = 1u << 2,    // a checked index was out of bounds (SDB_CHECKS builds)
};

constexpr unsigned long long kWaitLimitNs = 2000ull * 1000ull * 1000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Both phases complete, tested in one round trip.
__device__ __forceinline__ bool mbar_try_wait2(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 q, [%3], %4;\n\t"
        "and.pred p, p, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(b1)), "r"(p1), "r"(smem_u32(b2)), "r"(p2)
        : "memory");
    return ok != 0;
}

// The same test, except that a thread whose phase is not complete yet is
// suspended (until the phase completes, or at the latest after about
// `hint_ns` nanoseconds) instead of returning at once: waiting warps then
// take no issue slots from the warps that work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `parity` to complete.  Returns false when the kernel
// is winding down: either another thread set *abort, or this wait ran past
// kWaitLimitCycles SM clocks (about 2 s at the B200's clocks), in which case
// it sets *abort and the timeout bit itself.  The SM-local clock64 keeps the
// check cheap; it is read only every 1024 tries.
constexpr long long kWaitLimitCycles = 4000ll * 1000ll * 1000ll;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 1023u) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                *abort = 1;
                if (err) atomicOr(err, kErrTimeout);
                return false;
            }
        }
    }
}

// mbar_wait for kernels where many warps wait while others work: the waiting
// thread is suspended between tests (at most ~20 us at a time, so that an
// abort is seen soon) instead of testing in a loop that takes issue slots
// from the working warps.  Waking takes longer than a test, so kernels whose
// waits are short and few keep mbar_wait.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendHintNs)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitLimitCycles) {
            *abort = 1;
            if (err) atomicOr(err, kErrTimeout);
            return false;
        }
    }
}

// A wait used while winding down: bounded, reports nothing.
__device__ __forceinline__ bool mbar_wait_quiet(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u && global_ns() - t0 > limit_ns) return false;
    }
}

// ---------------------------------------------------------------- fences

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

// A 2-D tile of the tensor map into shared memory, completing on `bar`.
// x is the innermost coordinate (in elements); callers keep x * element size
// a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y, int z,
                                            int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

// A contiguous run of `bytes` (a multiple of 16, both addresses 16-byte
// aligned) from global into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const void* desc, uint64_t* bar, int x, int y, int z,
                                            int w, int v) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
        "%7}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v)
        : "memory");
}

// A 2-D tile from shared memory to global memory through the tensor map
// (elements outside the tensor are not written).  The writing threads fence
// their shared-memory stores to the async proxy before one thread issues it.
__device__ __forceinline__ void tma_store_2d(const void* desc, const void* smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(desc)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until the shared-memory sources of this thread's bulk stores may be
// reused (.read) / until the stores are complete.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Until at most the most recent bulk group may still be reading shared memory.
__device__ __forceinline__ void bulk_wait_read_but_one() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// A contiguous run of shared memory to global memory (bytes and both
// addresses multiples of 16), in this thread's bulk group.
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
                 "r"(smem_u32(smem_src)), "r"(bytes)
                 : "memory");
}

// ---------------------------------------------------------------- tcgen05

// Allocates `ncols` columns of tensor memory (a power of two >= 32) for the
// CTA; the whole warp calls it; the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile in the 128-byte
// swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (the layout a TMA
// load with CU_TENSOR_MAP_SWIZZLE_128B writes).  The tile base is 1024-byte
// aligned; stepping K inside the 128-byte row moves the start address.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
    d |= static_cast<uint64_t>(1) << 16;                      // leading byte offset (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;              // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;                      // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;                      // swizzle: 128 B
    return d;
}

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

// Instruction descriptor of kind::f16 with FP16 A and B, FP32 accumulator,
// both operands K-major, an M x N tile.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
    return (1u << 4)                                  // D format: F32
           | (0u << 7) | (0u << 10)                   // A, B: F16
           | (0u << 15) | (0u << 16)                  // K-major A and B
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D = A B + D 2^-11: the product into an accumulator that holds the lo
// products of a split (each lo operand carries the split's 2^11), scaled to
// the hi product's units as the product is added (tcgen05.mma's scale of the
// input D, kind::f16).  So hi.hi + (hi.lo + lo.hi) 2^-11 lands in one
// accumulator: the lo products are issued first, then the first hi product
// with this scale, the rest plain.
__device__ __forceinline__ void mma_f16_scale_lo(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 1, 11;" ::"r"(tmem_d), "l"(adesc),
                 "l"(bdesc), "r"(idesc)
                 : "memory");
}

// The same two products with the A operand in tensor memory: `a_tmem` is the
// address of a 128-lane x 8-column block, lane m holding row m's 16 values of
// K as FP16 pairs (column c: k = 2c in the low half, 2c + 1 in the high).
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_f16_ta_scale_lo(uint32_t tmem_d, uint32_t a_tmem, uint64_t bdesc,
                                                    uint32_t idesc) {
    asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1, 11;" ::"r"(tmem_d), "r"(a_tmem),
                 "l"(bdesc), "r"(idesc)
                 : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued before has
// completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 columns of 32-bit tensor memory into 32 registers per thread:
// thread t of the warp gets lane (addr.lane + t), columns addr.col .. +31.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t addr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 / 8 columns of 32-bit words from registers into tensor memory.
__device__ __forceinline__ void tmem_st32_bits(uint32_t addr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st4_bits(uint32_t addr, const uint4& v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void tmem_st8_bits(uint32_t addr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// max(a, b, c) in one instruction.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float m;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
    return m;
}

// Two softmax weights (inside FP16's range) split as split_half does, as the
// FP16 pairs of two consecutive keys: hi = {fp16(p0), fp16(p1)} and
// lo = {fp16((p0 - hi0) 2^11), fp16((p1 - hi1) 2^11)}, the first key in the
// low half.  hi - p comes exact from the FP16 hi and the FP32 weight in one
// mixed-precision subtraction; the 2^11 (negated) in one packed multiply.
__device__ __forceinline__ void split_weights2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    float d0, d1;
    asm("{\n\t.reg .b16 h0, h1;\n\t"
        "cvt.rn.f16x2.f32 %0, %4, %3;\n\t"
        "mov.b32 {h0, h1}, %0;\n\t"
        "sub.f32.f16 %1, h0, %3;\n\t"
        "sub.f32.f16 %2, h1, %4;\n\t}"
        : "=r"(hi), "=f"(d0), "=f"(d1)
        : "f"(p0), "f"(p1));
    uint64_t d, s;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(d0), "f"(d1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(s) : "f"(-2048.0f));
    asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(d) : "l"(s));
    asm("{\n\t.reg .f32 a, b;\n\tmov.b64 {a, b}, %1;\n\tcvt.rn.f16x2.f32 %0, b, a;\n\t}" : "=r"(lo) : "l"(d));
}

// split8 in fewer instructions (split_weights2's packed form, the same pairs),
// with the range check left to the caller: `amax` takes the largest |x| (a
// value of 65520 or more rounds to an FP16 infinity).  NaNs pass the maximum
// unseen; they reach the output as NaNs.
__device__ __forceinline__ void split8_packed(const float (&x)[8], uint4& hi, uint4& lo, float& amax) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        split_weights2(x[2 * i], x[2 * i + 1], h[i], l[i]);
        amax = fmax3(amax, fabsf(x[2 * i]), fabsf(x[2 * i + 1]));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// sum[j] += v[j] for j < N (N even), two lanes of FP32 a packed add
// (add.rn.f32x2: each lane rounded to nearest as a scalar add would be).
template <int N>
__device__ __forceinline__ void add_packed(float* sum, const float* v) {
#pragma unroll
    for (int j = 0; j < N; j += 2) {
        uint64_t sp, vp;
        asm("mov.b64 %0, {%1, %2};" : "=l"(sp) : "f"(sum[j]), "f"(sum[j + 1]));
        asm("mov.b64 %0, {%1, %2};" : "=l"(vp) : "f"(v[j]), "f"(v[j + 1]));
        asm("add.rn.f32x2 %0, %0, %1;" : "+l"(sp) : "l"(vp));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(sum[j]), "=f"(sum[j + 1]) : "l"(sp));
    }
}

__device__ __forceinline__ void add16_packed(float* sum, const float (&v)[16]) { add_packed<16>(sum, v); }

// sum[j] = fma(v[j], scale, sum[j]) for j < N (N even), packed as add_packed.
template <int N>
__device__ __forceinline__ void fma_packed(float* sum, const float* v, float scale) {
    uint64_t sc;
    asm("mov.b64 %0, {%1, %1};" : "=l"(sc) : "f"(scale));
#pragma unroll
    for (int j = 0; j < N; j += 2) {
        uint64_t sp, vp;
        asm("mov.b64 %0, {%1, %2};" : "=l"(sp) : "f"(sum[j]), "f"(sum[j + 1]));
        asm("mov.b64 %0, {%1, %2};" : "=l"(vp) : "f"(v[j]), "f"(v[j + 1]));
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(sp) : "l"(vp), "l"(sc));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(sum[j]), "=f"(sum[j + 1]) : "l"(sp));
    }
}

// Descriptor of an operand tile in the no-swizzle canonical layout: 8 x 16-byte
// core matrices (128 contiguous bytes each); `lbo` bytes between core
// matrices adjacent along K, `sbo` bytes between those adjacent along M/N.
__device__ __forceinline__ uint64_t desc_noswizzle(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // version; layout type 0 = no swizzle
    return d;
}

// kind::f16 instruction descriptor with a chosen major-ness of B (0 K-major,
// 1 MN-major); A is K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32_bmajor(int m, int n, int b_mn_major) {
    return idesc_f16_f32(m, n) | (static_cast<uint32_t>(b_mn_major) << 16);
}

// ---------------------------------------------------------------- split

// x = hi + lo * 2^-11 with hi, lo in FP16: hi is x rounded to FP16, lo the
// remainder (exact in FP32) scaled by 2^11 so that it stays a normal FP16
// number down to |x| ~ 2^-14, then rounded.  |x - (hi + lo 2^-11)| is within
// 2^-22 |x| + 2^-36.  The product with an FP16 weight is then taken as two
// tensor-core products accumulated apart (the AMX-FP16 scheme of the
// reference, x86_64/amx_fp16.S:9-22, with the remainder kept normal).
constexpr float kLoScale = 2048.0f;
constexpr float kLoUnscale = 1.0f / 2048.0f;
constexpr float kHalfLimit = 65504.0f;

__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn((x - __half2float(hi)) * kLoScale);
}

// The FP32 value of the FP16 bits in the low half of `w`: the exponent and
// significand moved into FP32's fields and scaled by 2^112 (exact for normal
// and subnormal values alike) -- integer ops and one multiply, where a
// conversion instruction would take the slower conversion pipe.
__device__ __forceinline__ float half_bits_to_float(uint32_t w) {
    const uint32_t h = w & 0xffffu;
    const float mag = __uint_as_float((h & 0x7fffu) << 13) * 0x1p112f;
    return __uint_as_float(__float_as_uint(mag) | ((h & 0x8000u) << 16));
}

// Splits 8 floats into one 16-byte chunk of hi and one of lo (the same pair
// as split_half: hi = x rounded to FP16, lo = (x - hi) 2^11 rounded to FP16);
// returns true when any input is beyond the FP16 range.  Four packed
// conversions (two values each) for hi and four for lo.
// split8 for values known to be inside the FP16 range (softmax weights): no
// range check, and the hi part read back by the hardware's FP16 unpack.
__device__ __forceinline__ void split8_inrange(const float (&x)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn((x[2 * i] - hf.x) * kLoScale, (x[2 * i + 1] - hf.y) * kLoScale);
        h[i] = *reinterpret_cast<const uint32_t*>(&hh);
        l[i] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ bool split8(const float (&x)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
    bool over = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        h[i] = *reinterpret_cast<const uint32_t*>(&hh);
        const float r0 = (x[2 * i] - half_bits_to_float(h[i])) * kLoScale;
        const float r1 = (x[2 * i + 1] - half_bits_to_float(h[i] >> 16)) * kLoScale;
        const __half2 ll = __floats2half2_rn(r0, r1);
        l[i] = *reinterpret_cast<const uint32_t*>(&ll);
        over |= !(fabsf(x[2 * i]) <= kHalfLimit) | !(fabsf(x[2 * i + 1]) <= kHalfLimit);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
    return over;
}

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major 128B-swizzled
// tile whose rows are 128 bytes (64 FP16).
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

}  // namespace sdb
