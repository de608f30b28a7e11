// Host-side runtime shared by the entry points: per-thread error text, the
// per-device error word, tuning, launch accounting, CUDA-call checking.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>

#include "../../include/sdb.h"

namespace sdb {

// The knobs of sdb_set_tuning (the GPU analogue of the reference's Tuning,
// kernels.h:91-135).
struct Tuning {
    int64_t fuse = 1;            // match chains after operations (shim)
    int64_t fuse_residual = 1;   // and residual additions not in place
    int64_t winograd = 2;        // 0 direct, 1 F(2x2,3x3), 2 F(4x4,3x3) where it fits
    int64_t winograd_positions = 1024;  // the least outputs of an image Winograd is used for
    int64_t winograd4_positions = 256;  // with winograd = 2, the least outputs of an image for F(4x4)
    int64_t winograd_channels = 16;     // the least input channels Winograd is used for
    int64_t winograd_small_tiles = 256; // quantized: Winograd also for images of at most this many tiles in all
    int64_t winograd_kc = 256;          // quantized, per-row weight scales: the input channels a scale spans
    int64_t winograd_small_kc = 128;    //   and for images of few tiles
    int64_t store = 1;           // keep packed weights between calls
    int64_t todo = 1;            // ToDo K/V downsampling factor (1 = none)
    int64_t todo_tokens = 4096;  // least tokens of a grid downsampled
    int64_t bits = 0;            // 2..8: integer products, weights of that many bits (0: FP32)
    int64_t input_bits = 8;      // the inputs' bits, 2..8, unsigned with a zero point
    int64_t group = 64;          // numbers of k sharing a scale: 32, 64, 128 or 256
    int64_t weight_group = 1;    // the weights' scale per group: 1; per whole row: 0
    int64_t quantize = 7;        // with bits, what is quantized: 1 linear layers, 2 convolutions, 4 attention
    int64_t block_n = 0;         // GEMM tile width: 0 automatic; 128 or 256 (wide kernel), 128, 160 or 192 (fused kernel)
    int64_t attention_wg = 2;    // 2: Q and P in tensor memory, two query tiles a CTA, where it fits; 1: two-warpgroup; 0: the pair kernel
    int64_t gemm_fused = 1;      // linear layers: 1 the activations split inside the GEMM (FP32 rows by TMA) where it pays; 2 always; 0 the split pre-pass
};

Tuning& tuning();

void set_error(const std::string& what);
int fail(sdb_status status, const std::string& what);
int cuda_fail(cudaError_t e, const char* where);

// The device error word of the current device (allocated once per device).
unsigned* device_error_word();

void count_launch(uint64_t n = 1);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
// element_strides: TMA's traversal stride per dimension (nullptr: all 1).
CUresult encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, void* addr,
                           const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                           CUtensorMapSwizzle swizzle, const uint32_t* element_strides = nullptr);

int current_sm_count();

// The map of a row-major FP32 matrix (`cols` x `rows`, `ld` floats a row) for
// TMA stores of 32-row boxes of `box_cols` (32: 128-byte swizzle; 16: 64-byte).
bool store_map(CUtensorMap* map, void* base, long long cols, long long rows, long long ld, int box_cols);

#define SDB_CUDA(call)                                        \
    do {                                                      \
        cudaError_t e_ = (call);                              \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
    } while (0)

}  // namespace sdb
