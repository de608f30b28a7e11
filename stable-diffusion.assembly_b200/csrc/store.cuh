// The weight store: weights repacked once into the layout the GEMM reads,
// kept on the device and keyed by where they came from.  It stands in for the
// reference's store of packed panels (store.h:58-120, store.cc:202-266), with
// the same key (address, type, shape, strides, layout) and the same
// invalidation: sdb_forget() on any overlap with memory about to change.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>

#include "../../include/sdb.h"

namespace sdb {

enum class Layout : int {
    linear = 0,   // rows n of w [K, N]; k as is
    conv = 1,     // rows oc of w [KW, KH, IC, OC]; k = (ky * KW + kx) * icp + ic
    gated = 2,    // GEGLU: rows [0, half) x weights, [halfpad, halfpad + half) gate weights
    quantized = 3,        // linear, quantized (quant.cuh): int8 rows n, k padded to whole groups
    quantized_gated = 4,  // GEGLU, quantized: rows as `gated`
    winograd2 = 5,        // F(2x2, 3x3): U = G g G^T split, [plane][16 xi][ocp][kpad] (winograd.cuh)
    winograd4 = 6,        // F(4x4, 3x3): the same with 36 xi
    quantized_winograd2 = 7,  // F(2x2, 3x3) quantized: 16 xi of quantized rows oc (k = ic), as `quantized`
};

// What a quantized packing depends on (the reference's quantized_variant,
// mul_mat.cc:378-381): the group, the weights' greatest magnitude and whether
// each group has its own scale.
struct QuantSpec {
    int group = 64;
    int wmax = 127;
    bool weight_groups = true;
    int64_t variant() const {
        return static_cast<int64_t>(group) | static_cast<int64_t>(wmax) << 16 |
               static_cast<int64_t>(weight_groups ? 1 : 0) << 32;
    }
};

constexpr int kRowPad = 256;  // packed rows are padded to the widest GEMM tile

struct Packed {
    void* data = nullptr;     // FP16 [rows_total][kpad]
    size_t bytes = 0;
    int64_t rows_total = 0;
    int64_t kpad = 0;
    int64_t npad = 0;         // rows of one operand (hi) block
    int64_t b1_row = 0;       // row of the second operand (lo, or gate), 0 if none
    int icp = 0;              // conv: channels per tap
    bool split = false;       // FP32 weights: hi rows then lo rows
    CUtensorMap map64{};      // box {64, 64}
    CUtensorMap map80{};      // box {64, 80}
    CUtensorMap map96{};      // box {64, 96}
    CUtensorMap map160{};     // box {64, 160}
    CUtensorMap map128{};     // box {64, 128}
    CUtensorMap map192{};     // box {64, 192}
    CUtensorMap map256{};     // box {64, 256}
    CUtensorMap map128k32{};  // box {32, 128}, 64-byte swizzle (kWeightSplitK32)
    // Quantized layouts, in the quantized GEMM's tiles of 128 rows (quant.cuh):
    // data int8 [tiles][nstages][8 KiB], each block 64 bytes of k of the
    // tile's rows in the 64-byte swizzle; qscales FP32 [tiles][groups][2][128],
    // the rows' scales then their offsets (scale * sum of the group's
    // integers).  A tile's rows: 128 consecutive columns, or (gated) 64 x
    // columns then the matching 64 gate columns.
    void* qscales = nullptr;
    int group = 0, groups = 0, tiles = 0;
    cudaEvent_t ready = nullptr;
    bool done = false;        // the packing was seen complete
    bool owned_by_store = true;
    bool borrowed = false;    // data is the caller's memory (a transient packing): not freed here
    ~Packed();
};

// The packed form of w for `layout`, from the store or packed now on
// `stream`.  With the store off (tuning store=0) the result is packed anew
// and freed when the returned pointer is released (stream-ordered).
// Returns an sdb_status; *out is set on success.
int packed_weights(const sdb_tensor* w, Layout layout, int64_t n_logical, int64_t k_logical, int icp,
                   int64_t half, cudaStream_t stream, std::shared_ptr<Packed>* out);

// The quantized form of w (Layout::quantized, or quantized_gated with `half`),
// from the store or quantized now on `stream`, as the reference's
// quantize_weights_f16/_f32 quantize (quant.cc:204-244, 366-377).
int quantized_weights(const sdb_tensor* w, bool gated, int64_t n_logical, int64_t k_logical, int64_t half,
                      const QuantSpec& q, cudaStream_t stream, std::shared_ptr<Packed>* out);

// A linear layer's first operand packed as packed_weights(Layout::linear)
// packs it, into caller memory `dst` of at least transient_bytes(w, n, k)
// bytes, and not kept: for operands the graph itself writes between calls
// (the k and v of an attention computed as two products).  *out borrows dst.
size_t transient_bytes(const sdb_tensor* w, int64_t n_logical, int64_t k_logical);
int pack_transient(const sdb_tensor* w, int64_t n_logical, int64_t k_logical, void* dst, cudaStream_t stream,
                   Packed* out);

// The transformed kernels of a 3x3 convolution for Winograd's F(f x f, 3x3),
// f = 2 or 4 (winograd.cuh): from the store or transformed now on `stream`
// (the reference keeps them too, Layout::winograd, winograd.cc:2144-2160).
// Packed rows: xi * ocp + oc of the hi plane, then b1_row + the same of the
// lo plane; ocp = OC rounded up to 128, kpad = IC rounded up to 64.
// The arguments of the weight quantizer (store.cu quantize_weights_kernel):
// `batches` matrices of n logical rows each, packed tiles of 128 rows
// (rows / batches of them a batch, one after another); matrix bi at
// src + (bi / bdiv) * bnb_hi + (bi % bdiv) * bnb_lo.
struct QPackArgs {
    const uint8_t* src;
    int type;
    long long nb0, nb1;   // source strides in bytes (k, row)
    long long n;          // logical rows of a batch (gated: of one half)
    long long k;
    int gated;
    long long rows;       // packed rows in all: batches * tiles a batch * 128
    int group, groups, nstages, wmax, weight_groups;
    long long span;       // per-row scales (weight_groups 0): the numbers of k one scale covers, a multiple of group
    int batches, bdiv;
    long long bnb_hi, bnb_lo;
    int8_t* q;
    float* scales;
};
void launch_quantize_weights(const QPackArgs& a, cudaStream_t stream);

int quantized_winograd_weights(const sdb_tensor* w, const QuantSpec& q, int64_t span, cudaStream_t stream,
                               std::shared_ptr<Packed>* out);
int winograd_weights(const sdb_tensor* w, int f, cudaStream_t stream, std::shared_ptr<Packed>* out);

}  // namespace sdb
