// The split of FP32 activations into FP16 pairs, done once per operand, and
// the per-stream workspace it writes into.
//
// x = hi + lo 2^-11 (ptx.cuh split_half).  A product of the split pair with
// an FP16 weight is two tensor-core products; splitting each activation once,
// into a layout TMA can tile (rows of K for a linear layer, channels-last for
// a convolution, rows of head dims for attention), lets the product kernels
// be pure TMA + tcgen05 pipelines.  The pre-pass reads 4 bytes and writes 4
// bytes an element: it is bound by HBM bandwidth.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/sdb.h"

namespace sdb {

// Workspace memory of the current device for work on `stream`: at least
// `bytes`, 256-byte aligned, valid until the next call for the same stream.
// Grows by reallocation outside stream capture; under capture it must
// already be large enough (an SDB_INVALID status otherwise).
int workspace(cudaStream_t stream, size_t bytes, void** out);

// Rows: x viewed as [ne0 = row length, ne1, ne2, ne3] FP32 with element
// strides xnb, rows enumerated (i3, i2, i1) -> r = (i3 * ne2 + i2) * ne1 + i1.
// Writes hi rows [0, R) then lo rows [R, 2R) of `ld` FP16 each (ld >= ne0,
// a multiple of 8; columns past ne0 are zero).  R = ne1 * ne2 * ne3.
// With gn (stats not null), each row is an image's position, its values
// channels 0 .. ne0 - 1, read through the GroupNorm prologue (chain.cuh).
struct GnIn;
int split_rows(const float* x, const long long ne[4], const long long xnb[4], long long ld, uint16_t* out,
               unsigned* err, cudaStream_t stream, const GnIn* gn = nullptr);
// The rows of x through a LayerNorm (norm.cc:148-175) with its chain (gamma,
// beta) first, as sdb_norm computes them, then split the same way (norm.cu).
int layer_norm_split(const sdb_tensor* x, float eps, const sdb_chain* chain, long long ld, uint16_t* out,
                     unsigned* err, cudaStream_t stream);
struct LnIn {
    float eps;
    const sdb_chain* chain;
};
// The same for an FP16 source (hi = the value, lo = 0).
int split_rows_half(const uint16_t* x, const long long ne[4], const long long xnb[4], long long ld, uint16_t* out,
                    cudaStream_t stream);

// Tiles: x viewed as [ne0 = row length, ne1 = rows of a head, ne2, ne3]
// (FP32, or FP16 with `half`), the heads h = i3 * ne2 + i2 each cut into
// tiles of T rows (ceil(ne1 / T), rows past ne1 zero) and each tile stored
// as [chunk][row][8]: 8 consecutive values of a row, chunk = column / 8, for
// `ld` / 8 chunks (columns past ne0 zero).  This is the UMMA no-swizzle
// core-matrix layout, so a tile is one contiguous copy into shared memory.
// Writes the hi plane, then the lo plane right after it.
int split_tiles(const void* x, int half, const long long ne[4], const long long xnb[4], long long ld, int tile,
                uint16_t* out, unsigned* err, cudaStream_t stream);
// One split_tiles job, and up to three of them in one launch (attention's Q, K
// and V): the same output as three split_tiles calls.
struct SplitTilesJob {
    const void* x;
    int half;
    long long ne0, ne1, ne2, heads;
    long long xnb[4];
    long long ld;
    int tile;
    long long ntiles;
    uint16_t* out;
    long long plane;
};
constexpr int kSplitTilesJobs = 3;
struct SplitTilesJobs {
    SplitTilesJob job[kSplitTilesJobs];
};
SplitTilesJob split_tiles_job(const void* x, int half, const long long ne[4], const long long xnb[4], long long ld,
                              int tile, uint16_t* out);
int split_tiles_many(const SplitTilesJob* jobs, int count, unsigned* err, cudaStream_t stream);

// Bytes of one plane of split_tiles' output.
inline long long split_tiles_plane(const long long ne[4], long long ld, int tile) {
    return ne[2] * ne[3] * ((ne[1] + tile - 1) / tile) * tile * ld * 2;
}

// Channels-last: x [W, H, C, N] FP32 (element strides xnb) into
// [2N][H][W][cp] FP16: images [0, N) hi, [N, 2N) lo; channels past C zero.
int split_nhwc(const float* x, const long long ne[4], const long long xnb[4], long long cp, uint16_t* out,
               unsigned* err, cudaStream_t stream);

}  // namespace sdb
