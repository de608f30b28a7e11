// Element-wise math of the epilogues and the epilogue chain itself.
//
// exponential(), silu() and gelu() follow the reference's scalar_math.h:34-63:
// exp by Cody-Waite reduction x = n ln2 + r (n rounded by adding 1.5 * 2^23,
// ln2 in a high and a low part) and the degree-6 minimax polynomial of the
// Cephes library's expf for exp(r), 2^n built in the exponent field, the
// argument clamped to [-87.3, 88.73]; SiLU as x / (1 + exp(-x)); GELU by its
// tanh definition written as x / (1 + exp(-2y)), y = sqrt(2/pi)(x + 0.044715 x^3).
// The chain is the reference's Epilogue (fusion.h:51-91): up to six in-place
// additions / multiplications by a broadcast operand, or SiLU, applied in
// graph order to each output element, the element addressed by its four ggml
// coordinates (i0 fastest).
#pragma once

#include <cstdint>

#include "../../include/sdb.h"

namespace sdb {

__device__ __forceinline__ float exponential(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.73f);
    const float magic = 12582912.0f;  // 1.5 * 2^23
    const float z = fmaf(x, 1.44269504088896341f, magic);
    const float n = z - magic;
    float r = fmaf(n, -0.693359375f, x);
    r = fmaf(n, 2.12194440e-4f, r);
    float p = 1.9875691500e-4f;
    p = fmaf(p, r, 1.3981999507e-3f);
    p = fmaf(p, r, 8.3334519073e-3f);
    p = fmaf(p, r, 4.1665795894e-2f);
    p = fmaf(p, r, 1.6666665459e-1f);
    p = fmaf(p, r, 5.0000001201e-1f);
    p = fmaf(p * r, r, r) + 1.0f;
    const uint32_t e = static_cast<uint32_t>(__float_as_int(z) - 0x4b400000 + 127) << 23;
    return p * __uint_as_float(e);
}

__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, 1.0f + exponential(-x)); }

// The same SiLU as one out-of-line function: the tile epilogues unroll the
// chain over every column and every step, and SiLU inlined there (rare after
// a GEMM) would multiply their code past what the instruction cache holds.
static __device__ __noinline__ float silu_call(float x) { return silu(x); }

__device__ __forceinline__ float gelu(float x) {
    const float y = x * fmaf(0.044715f * x, x, 1.0f);
    return __fdiv_rn(x, 1.0f + exponential(-1.5957691216057308f * y));
}

// The chain as kernels take it (by value, in the launch parameters).
struct Chain {
    int count;
    int from_redirect;
    int kind[SDB_MAX_STEPS];
    const float* operand[SDB_MAX_STEPS];
    long long nb[SDB_MAX_STEPS][4];
};

__host__ inline Chain make_chain(const sdb_chain* c) {
    Chain k{};
    if (c == nullptr) return k;
    k.count = c->count;
    k.from_redirect = c->from_redirect;
    for (int s = 0; s < c->count && s < SDB_MAX_STEPS; ++s) {
        k.kind[s] = c->steps[s].kind;
        k.operand[s] = c->steps[s].operand;
        for (int d = 0; d < 4; ++d) k.nb[s][d] = c->steps[s].nb[d];
    }
    return k;
}

// Applies the chain to v, the output element at coordinates (i0, i1, i2, i3).
__device__ __forceinline__ float apply_chain(const Chain& c, float v, long long i0, long long i1, long long i2,
                                             long long i3) {
    for (int s = 0; s < c.count; ++s) {
        if (c.kind[s] == SDB_STEP_SILU) {
            v = silu(v);
            continue;
        }
        const long long at = i0 * c.nb[s][0] + i1 * c.nb[s][1] + i2 * c.nb[s][2] + i3 * c.nb[s][3];
        const float o = __ldg(c.operand[s] + at);
        v = c.kind[s] == SDB_STEP_ADD ? v + o : v * o;
    }
    return v;
}

// The chain for a tile epilogue: each thread owns one output row (an output
// position) and walks its columns, so the part of every operand's offset that
// depends on the row is computed once (row_offsets) and each element adds only
// column * stride (apply_chain_col).  col_dim names the ggml coordinate the
// columns run along (0 for a linear layer's features, 2 for a convolution's
// channels).  The step loop is unrolled so that the launch-parameter arrays
// are indexed statically.
struct ChainRow {
    long long off[SDB_MAX_STEPS];
};

__device__ __forceinline__ void row_offsets(const Chain& c, ChainRow& r, int col_dim, long long j0, long long j1,
                                            long long j2) {
    // j0..j2: the three row coordinates in ggml order without col_dim.
#pragma unroll
    for (int s = 0; s < SDB_MAX_STEPS; ++s) {
        if (col_dim == 0)
            r.off[s] = j0 * c.nb[s][1] + j1 * c.nb[s][2] + j2 * c.nb[s][3];
        else
            r.off[s] = j0 * c.nb[s][0] + j1 * c.nb[s][1] + j2 * c.nb[s][3];
    }
}

// The chain over NVAL consecutive columns col0.. of one row, in place: one
// step at a time over all the columns, so that a step's operand loads are
// issued together (columns past col_max read column col_max; their results
// are not stored).
template <int COL_DIM, int NVAL>
__device__ __forceinline__ void apply_chain_cols(const Chain& c, const ChainRow& r, float* v, long long col0,
                                                 long long col_max) {
#pragma unroll
    for (int s = 0; s < SDB_MAX_STEPS; ++s) {
        if (s >= c.count) break;
        if (c.kind[s] == SDB_STEP_SILU) {
#pragma unroll
            for (int j = 0; j < NVAL; ++j) v[j] = silu_call(v[j]);
        } else {
            const float* base = c.operand[s] + r.off[s];
            const long long stride = c.nb[s][COL_DIM];
            float o[NVAL];
#pragma unroll
            for (int j = 0; j < NVAL; ++j) o[j] = __ldg(base + min(col0 + j, col_max) * stride);
            if (c.kind[s] == SDB_STEP_ADD) {
#pragma unroll
                for (int j = 0; j < NVAL; ++j) v[j] += o[j];
            } else {
#pragma unroll
                for (int j = 0; j < NVAL; ++j) v[j] *= o[j];
            }
        }
    }
}

}  // namespace sdb

