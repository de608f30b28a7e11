// Split pre-pass kernels and the per-stream workspace (see split.cuh).
#include "split.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "chain.cuh"
#include "ptx.cuh"
#include "runtime.cuh"

namespace sdb {

namespace {

struct Space {
    void* ptr = nullptr;
    size_t bytes = 0;
};

std::mutex g_space_mutex;
std::map<std::pair<int, cudaStream_t>, Space> g_spaces;

// One thread per 8 consecutive values of a row: two float4 loads when the
// row is contiguous and aligned, one 16-byte store of hi and one of lo.
// I: the index type, 32-bit when every index fits (cheaper division).
// GN: the rows are an image's positions (channels along the row) read through
// a GroupNorm prologue (chain.cuh gn_in): the split of the normalised values.
template <typename I, bool GN = false>
__global__ void split_rows_kernel(const float* __restrict__ x, I ne0, I ne1, I ne2, I rows, long long xnb0,
                                  long long xnb1, long long xnb2, long long xnb3, I ld,
                                  uint16_t* __restrict__ out, unsigned* err, int vec, GnIn gn = GnIn{}) {
    const I chunks = ld / 8;
    const I total = rows * chunks;
    bool over = false;
    for (I idx = blockIdx.x * static_cast<I>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<I>(gridDim.x) * blockDim.x) {
        const I r = idx / chunks;
        const I c0 = (idx - r * chunks) * 8;
        const I i1 = r % ne1, i2 = (r / ne1) % ne2, i3 = r / (ne1 * ne2);
        const float* src = x + i1 * xnb1 + i2 * xnb2 + i3 * xnb3;
        float v[8];
        if (vec && c0 + 8 <= ne0) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(src + c0));
            const float4 b = __ldg(reinterpret_cast<const float4*>(src + c0 + 4));
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = c0 + i < ne0 ? __ldg(src + (c0 + i) * xnb0) : 0.0f;
        }
        if (GN) {
            const long long img = static_cast<long long>(r) / gn.positions;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (c0 + i < ne0) v[i] = gn_in(gn, v[i], gn_coef(gn, static_cast<int>(c0 + i), img));
        }
        uint4 hi, lo;
        over |= split8(v, hi, lo);
        *reinterpret_cast<uint4*>(out + static_cast<long long>(r) * ld + c0) = hi;
        *reinterpret_cast<uint4*>(out + (static_cast<long long>(rows) + r) * ld + c0) = lo;
    }
    if (over) atomicOr(err, kErrRange);
}

__global__ void split_rows_half_kernel(const __half* __restrict__ x, long long ne0, long long ne1, long long ne2,
                                       long long rows, long long xnb0, long long xnb1, long long xnb2, long long xnb3,
                                       long long ld, __half* __restrict__ out) {
    const long long total = rows * ld;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = idx / ld, c = idx - r * ld;
        const long long i1 = r % ne1, i2 = (r / ne1) % ne2, i3 = r / (ne1 * ne2);
        out[idx] = c < ne0 ? x[i1 * xnb1 + i2 * xnb2 + i3 * xnb3 + c * xnb0] : __float2half_rn(0.0f);
        out[rows * ld + idx] = __float2half_rn(0.0f);
    }
}

// One thread per 8 values of a row of a tile.
template <typename I>
__device__ __forceinline__ void split_tiles_body(const void* __restrict__ x, int half, I ne0, I ne1, I ne2, I heads,
                                                 long long xnb0, long long xnb1, long long xnb2, long long xnb3, I ld,
                                                 int tile, I ntiles, uint16_t* __restrict__ out, long long plane,
                                                 unsigned* err) {
    const I chunks = ld / 8;
    const I rows_pad = ntiles * tile;
    const I total = heads * rows_pad * chunks;
    bool over = false;
    for (I idx = blockIdx.x * static_cast<I>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<I>(gridDim.x) * blockDim.x) {
        // idx enumerates (head, row, chunk) with chunk fastest: neighbouring
        // threads read neighbouring 32-byte runs of a row.
        const I c = idx % chunks;
        const I row = (idx / chunks) % rows_pad;
        const I hh = idx / (chunks * rows_pad);
        const I i2 = hh % ne2, i3 = hh / ne2;
        float v[8];
        if (row < ne1) {
            const long long b = row * xnb1 + i2 * xnb2 + i3 * xnb3;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const I col = c * 8 + i;
                float val = 0.0f;
                if (col < ne0) {
                    const long long at = b + col * xnb0;
                    val = half ? __half2float(__ldg(reinterpret_cast<const __half*>(x) + at))
                               : __ldg(reinterpret_cast<const float*>(x) + at);
                }
                v[i] = val;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        uint4 hi, lo;
        over |= split8(v, hi, lo);
        const I t = row / tile, rr = row - t * tile;
        const long long at = ((static_cast<long long>(hh * ntiles + t) * chunks + c) * tile + rr) * 8;
        *reinterpret_cast<uint4*>(out + at) = hi;
        *reinterpret_cast<uint4*>(out + plane / 2 + at) = lo;
    }
    if (over) atomicOr(err, kErrRange);
}

template <typename I>
__global__ void split_tiles_kernel(const void* __restrict__ x, int half, I ne0, I ne1, I ne2, I heads,
                                   long long xnb0, long long xnb1, long long xnb2, long long xnb3, I ld, int tile,
                                   I ntiles, uint16_t* __restrict__ out, long long plane, unsigned* err) {
    split_tiles_body<I>(x, half, ne0, ne1, ne2, heads, xnb0, xnb1, xnb2, xnb3, ld, tile, ntiles, out, plane, err);
}

// Several split_tiles jobs in one launch: blockIdx.y picks the job.
template <typename I>
__global__ void split_tiles_many_kernel(const SplitTilesJobs jobs, unsigned* err) {
    const SplitTilesJob& j = jobs.job[blockIdx.y];
    split_tiles_body<I>(j.x, j.half, static_cast<I>(j.ne0), static_cast<I>(j.ne1), static_cast<I>(j.ne2),
                        static_cast<I>(j.heads), j.xnb[0], j.xnb[1], j.xnb[2], j.xnb[3], static_cast<I>(j.ld), j.tile,
                        static_cast<I>(j.ntiles), j.out, j.plane, err);
}

// Channels-last through shared memory: a block takes 64 channels x 32
// positions of one image row; reads run along W (coalesced), writes along C.
__global__ void split_nhwc_kernel(const float* __restrict__ x, long long W, long long H, long long C, long long N,
                                  long long xnb0, long long xnb1, long long xnb2, long long xnb3, long long cp,
                                  uint16_t* __restrict__ out, unsigned* err) {
    __shared__ float tile[64][33];
    const long long wblocks = (W + 31) / 32;
    const long long cblocks = (cp + 63) / 64;
    long long b = blockIdx.x;
    const long long wb = b % wblocks;
    b /= wblocks;
    const long long cb = b % cblocks;
    b /= cblocks;
    const long long y = b % H;
    const long long n = b / H;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    const long long w0 = wb * 32, c0 = cb * 64;
    for (int cc = ty; cc < 64; cc += 8) {
        const long long c = c0 + cc, w = w0 + tx;
        tile[cc][tx] = (c < C && w < W) ? __ldg(x + n * xnb3 + c * xnb2 + y * xnb1 + w * xnb0) : 0.0f;
    }
    __syncthreads();
    // 32 positions x 8 chunks of 8 channels: one chunk a thread.
    const int pos = threadIdx.x >> 3, chunk = threadIdx.x & 7;
    const long long w = w0 + pos, c = c0 + chunk * 8;
    bool over = false;
    if (w < W && c < cp) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = tile[chunk * 8 + i][pos];
        uint4 hi, lo;
        over = split8(v, hi, lo);
        const long long at = ((n * H + y) * W + w) * cp + c;
        const long long lo_at = (((N + n) * H + y) * W + w) * cp + c;
        *reinterpret_cast<uint4*>(out + at) = hi;
        *reinterpret_cast<uint4*>(out + lo_at) = lo;
    }
    if (over) atomicOr(err, kErrRange);
}

}  // namespace

int workspace(cudaStream_t stream, size_t bytes, void** out) {
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_space_mutex);
    Space& s = g_spaces[{dev, stream}];
    if (s.bytes < bytes) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        SDB_CUDA(cudaStreamIsCapturing(stream, &cap));
        if (cap != cudaStreamCaptureStatusNone)
            return fail(SDB_INVALID, "workspace must grow under stream capture: run the operation once before");
        if (s.ptr) {
            SDB_CUDA(cudaStreamSynchronize(stream));
            SDB_CUDA(cudaFree(s.ptr));
            s.ptr = nullptr;
            s.bytes = 0;
        }
        const size_t want = std::max(bytes, s.bytes + s.bytes / 2);
        SDB_CUDA(cudaMalloc(&s.ptr, want));
        s.bytes = want;
    }
    *out = s.ptr;
    return SDB_OK;
}

int split_rows(const float* x, const long long ne[4], const long long xnb[4], long long ld, uint16_t* out,
               unsigned* err, cudaStream_t stream, const GnIn* gn) {
    const long long rows = ne[1] * ne[2] * ne[3];
    const long long total = rows * (ld / 8);
    const int vec = xnb[0] == 1 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && xnb[1] % 4 == 0 &&
                    xnb[2] % 4 == 0 && xnb[3] % 4 == 0;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
    if (blocks == 0) return SDB_OK;
    const bool small = 2 * total * 8 < (1LL << 31);
    if (gn && gn->stats) {
        if (small)
            split_rows_kernel<unsigned, true><<<blocks, 256, 0, stream>>>(
                x, static_cast<unsigned>(ne[0]), static_cast<unsigned>(ne[1]), static_cast<unsigned>(ne[2]),
                static_cast<unsigned>(rows), xnb[0], xnb[1], xnb[2], xnb[3], static_cast<unsigned>(ld), out, err, vec,
                *gn);
        else
            split_rows_kernel<long long, true><<<blocks, 256, 0, stream>>>(x, ne[0], ne[1], ne[2], rows, xnb[0],
                                                                           xnb[1], xnb[2], xnb[3], ld, out, err, vec,
                                                                           *gn);
    } else if (small)
        split_rows_kernel<unsigned><<<blocks, 256, 0, stream>>>(
            x, static_cast<unsigned>(ne[0]), static_cast<unsigned>(ne[1]), static_cast<unsigned>(ne[2]),
            static_cast<unsigned>(rows), xnb[0], xnb[1], xnb[2], xnb[3], static_cast<unsigned>(ld), out, err, vec);
    else
        split_rows_kernel<long long><<<blocks, 256, 0, stream>>>(x, ne[0], ne[1], ne[2], rows, xnb[0], xnb[1],
                                                                 xnb[2], xnb[3], ld, out, err, vec);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int split_rows_half(const uint16_t* x, const long long ne[4], const long long xnb[4], long long ld, uint16_t* out,
                    cudaStream_t stream) {
    const long long rows = ne[1] * ne[2] * ne[3];
    const long long total = rows * ld;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
    if (blocks == 0) return SDB_OK;
    split_rows_half_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __half*>(x), ne[0], ne[1], ne[2], rows,
                                                       xnb[0], xnb[1], xnb[2], xnb[3], ld,
                                                       reinterpret_cast<__half*>(out));
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int split_tiles(const void* x, int half, const long long ne[4], const long long xnb[4], long long ld, int tile,
                uint16_t* out, unsigned* err, cudaStream_t stream) {
    const long long ntiles = (ne[1] + tile - 1) / tile;
    const long long heads = ne[2] * ne[3];
    const long long total = heads * ntiles * tile * (ld / 8);
    const long long plane = split_tiles_plane(ne, ld, tile);
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 32));
    if (blocks == 0) return SDB_OK;
    if (total * 8 < (1LL << 31))
        split_tiles_kernel<unsigned><<<blocks, 256, 0, stream>>>(
            x, half, static_cast<unsigned>(ne[0]), static_cast<unsigned>(ne[1]), static_cast<unsigned>(ne[2]),
            static_cast<unsigned>(heads), xnb[0], xnb[1], xnb[2], xnb[3], static_cast<unsigned>(ld), tile,
            static_cast<unsigned>(ntiles), out, plane, err);
    else
        split_tiles_kernel<long long><<<blocks, 256, 0, stream>>>(x, half, ne[0], ne[1], ne[2], heads, xnb[0], xnb[1],
                                                                  xnb[2], xnb[3], ld, tile, ntiles, out, plane, err);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int split_tiles_many(const SplitTilesJob* jobs, int count, unsigned* err, cudaStream_t stream) {
    if (count <= 0 || count > kSplitTilesJobs) return fail(SDB_INVALID, "split_tiles_many: 1..3 jobs");
    SplitTilesJobs all{};
    long long most = 0;
    for (int i = 0; i < count; ++i) {
        SplitTilesJob j = jobs[i];
        most = std::max(most, j.heads * j.ntiles * j.tile * (j.ld / 8));
        all.job[i] = j;
    }
    const int blocks = static_cast<int>(std::min<long long>((most + 255) / 256, 148LL * 32));
    if (blocks == 0) return SDB_OK;
    const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(count));
    if (most * 8 < (1LL << 31)) split_tiles_many_kernel<unsigned><<<grid, 256, 0, stream>>>(all, err);
    else split_tiles_many_kernel<long long><<<grid, 256, 0, stream>>>(all, err);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

SplitTilesJob split_tiles_job(const void* x, int half, const long long ne[4], const long long xnb[4], long long ld,
                              int tile, uint16_t* out) {
    SplitTilesJob j{};
    j.x = x;
    j.half = half;
    j.ne0 = ne[0];
    j.ne1 = ne[1];
    j.ne2 = ne[2];
    j.heads = ne[2] * ne[3];
    for (int d = 0; d < 4; ++d) j.xnb[d] = xnb[d];
    j.ld = ld;
    j.tile = tile;
    j.ntiles = (ne[1] + tile - 1) / tile;
    j.out = out;
    j.plane = split_tiles_plane(ne, ld, tile);
    return j;
}

int split_nhwc(const float* x, const long long ne[4], const long long xnb[4], long long cp, uint16_t* out,
               unsigned* err, cudaStream_t stream) {
    const long long W = ne[0], H = ne[1], C = ne[2], N = ne[3];
    const long long blocks = ((W + 31) / 32) * ((cp + 63) / 64) * H * N;
    if (blocks == 0) return SDB_OK;
    if (blocks > 0x7fffffffLL) return fail(SDB_NOT_SUPPORTED, "split_nhwc: too large");
    split_nhwc_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, W, H, C, N, xnb[0], xnb[1], xnb[2],
                                                                         xnb[3], cp, out, err);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

}  // namespace sdb
