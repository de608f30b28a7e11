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

// SiLU of the GroupNorm apply pass and its prologue form, x / (1 + e^-x) as the reference writes it (scalar_math.h:54-58), with
// e^-x by the same Cody-Waite reduction to |r| <= ln2 / 2 but 2^(r log2 e) from the hardware's
// ex2 (relative error about 2^-22) in place of the degree-6 polynomial, and the quotient by the
// hardware's reciprocal refined by one Newton step: within a few 2^-23 of the exact form, at a
// third of the instructions -- the pass is bound by issue, not by memory.
__device__ __forceinline__ float silu_apply(float x) {
    // Clamped at 87.3 on both sides (the reference's upper clamp is 88.73): 2^n stays finite, so
    // the Newton step never meets an infinity; past 87.3 the quotient is below FP32's normal range.
    const float t = fminf(fmaxf(-x, -87.3f), 87.3f);
    const float magic = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
    const float z = fmaf(t, 1.44269504088896341f, magic);
    const float n = z - magic;
    float r = fmaf(n, -0.693359375f, t);
    r = fmaf(n, 2.12194440e-4f, r);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(r * 1.44269504088896341f));
    e *= __uint_as_float(static_cast<uint32_t>(__float_as_int(z) - 0x4b400000 + 127) << 23);
    const float d = 1.0f + e;
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    y = fmaf(fmaf(-d, y, 1.0f), y, y);
    return x * y;
}


// GroupNorm read in place of its output (a prologue of the operation that
// consumes it: the Winograd input transform, the split of a convolution's or
// linear layer's activations): x' = (x - mean) * scale, then gamma and beta
// by one fmaf, then SiLU -- the apply pass's arithmetic (norm.cu,
// nhwc_gn_apply_kernel), so the fused operation sees the very numbers the
// GroupNorm node would have written.  stats [images][groups][2] (mean,
// 1 / sqrt(variance + eps)); stats null: no prologue.
struct GnIn {
    const float* stats;
    const float* gamma;   // [C], with beta, or both null
    const float* beta;
    int cpg;              // channels per group
    int groups;
    int silu;
    long long positions;  // rows (positions) of an image, for row-wise consumers
};

// The normalisation of one value whose channel's mean m, scale s, gamma ga and beta gb are known.
__device__ __forceinline__ float gn_apply(const GnIn& g, float x, float m, float s, float ga, float gb) {
    float v = (x - m) * s;
    if (g.gamma) v = fmaf(v, ga, gb);
    return g.silu ? silu_apply(v) : v;
}

// A channel's four numbers (consumers load them once for all the values of a channel they read).
struct GnCoef {
    float m, s, ga, gb;
};

__device__ __forceinline__ GnCoef gn_coef(const GnIn& g, int c, long long img) {
    const float* st = g.stats + (img * g.groups + c / g.cpg) * 2;
    GnCoef k{__ldg(st), __ldg(st + 1), 1.0f, 0.0f};
    if (g.gamma) {
        k.ga = __ldg(g.gamma + c);
        k.gb = __ldg(g.beta + c);
    }
    return k;
}

__device__ __forceinline__ float gn_in(const GnIn& g, float x, const GnCoef& k) {
    return gn_apply(g, x, k.m, k.s, k.ga, k.gb);
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
    // j0..j2: the three row coordinates in ggml order without col_dim; only the chain's steps.
#pragma unroll
    for (int s = 0; s < SDB_MAX_STEPS; ++s) {
        if (s >= c.count) break;
        if (col_dim == 0)
            r.off[s] = j0 * c.nb[s][1] + j1 * c.nb[s][2] + j2 * c.nb[s][3];
        else
            r.off[s] = j0 * c.nb[s][0] + j1 * c.nb[s][1] + j2 * c.nb[s][3];
    }
}

// The chain over NVAL consecutive columns col0.. of one row, in place: one
// step at a time over all the columns, so that a step's operand loads are
// issued together (columns past col_max read column col_max; their results
// are not stored).  An operand whose columns are consecutive floats (a bias,
// a residual row) is read a float4 at a time when the run is in range and
// aligned; else element by element.
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
            const float* run = base + col0 * stride;
            if (NVAL % 4 == 0 && stride == 1 && col0 + NVAL - 1 <= col_max &&
                (reinterpret_cast<uintptr_t>(run) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < NVAL; j += 4) {
                    const float4 f = __ldg(reinterpret_cast<const float4*>(run + j));
                    o[j] = f.x;
                    o[j + 1] = f.y;
                    o[j + 2] = f.z;
                    o[j + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < NVAL; ++j) o[j] = __ldg(base + min(col0 + j, col_max) * stride);
            }
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

