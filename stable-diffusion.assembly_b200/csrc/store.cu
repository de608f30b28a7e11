// The weight store and the packing kernel (see store.cuh).
#include "store.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "ptx.cuh"
#include "quant.cuh"
#include "runtime.cuh"
#include "winograd.cuh"

namespace sdb {

namespace {

struct PackArgs {
    const uint8_t* src;
    int type;             // SDB_TYPE_F16 / SDB_TYPE_F32
    long long nb[4];      // source strides in bytes
    int layout;
    long long n;          // logical rows (gated: 2 * half)
    long long k;          // logical K (linear) / IC (conv)
    int kw, kh, icp;
    long long half, halfpad;
    long long npad, kpad;
    long long rows;       // packed rows of one block (npad, or 2 * halfpad for gated)
    int split;
    __half* out;
    unsigned* err;
};

__global__ void pack_weights_kernel(const PackArgs p) {
    const long long total = p.rows * p.kpad;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = idx / p.kpad;
        const long long kp = idx - r * p.kpad;
        long long off = -1;
        if (p.layout == 0) {  // linear
            if (r < p.n && kp < p.k) off = kp * p.nb[0] + r * p.nb[1];
        } else if (p.layout == 1) {  // conv
            const long long tap = kp / p.icp, ic = kp - tap * p.icp;
            if (r < p.n && tap < static_cast<long long>(p.kw) * p.kh && ic < p.k) {
                const long long kx = tap % p.kw, ky = tap / p.kw;
                off = kx * p.nb[0] + ky * p.nb[1] + ic * p.nb[2] + r * p.nb[3];
            }
        } else {  // gated
            long long src_row = -1;
            if (r < p.half) src_row = r;
            else if (r >= p.halfpad && r - p.halfpad < p.half) src_row = p.half + (r - p.halfpad);
            if (src_row >= 0 && kp < p.k) off = kp * p.nb[0] + src_row * p.nb[1];
        }
        float w = 0.0f;
        if (off >= 0) {
            w = p.type == SDB_TYPE_F16 ? __half2float(*reinterpret_cast<const __half*>(p.src + off))
                                       : *reinterpret_cast<const float*>(p.src + off);
        }
        if (p.split) {
            __half hi, lo;
            split_half(w, hi, lo);
            if (!(fabsf(w) <= kHalfLimit)) atomicOr(p.err, kErrRange);
            p.out[idx] = hi;
            p.out[p.npad * p.kpad + idx] = lo;
        } else {
            p.out[idx] = __float2half_rn(w);  // exact for FP16 sources
        }
    }
}

// The reference's weight quantization (quant.cc:204-244): per packed row (an
// output feature), per group of `group` numbers of k (the last group's
// missing numbers zeros), m = max |w| over the group (or the whole row),
// s = m / wmax, inverse = s > 0 ? 1 / s : 0, q = clamp(rint(w * inverse),
// -wmax, wmax); the group's scale s and offset s * sum(q).  One warp a row;
// every operation rounds as the reference's scalar one does.  Written in the
// quantized GEMM's tiles (store.cuh, Packed).

template <int EPL>
__global__ void quantize_weights_kernel(const QPackArgs a) {
    const int lane = threadIdx.x & 31;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
    const long long per_batch = a.rows / a.batches;
    for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < a.rows;
         r += warps) {
        const long long tile = r >> 7;
        const int p = static_cast<int>(r & 127);
        const long long bi = r / per_batch, rr = r - bi * per_batch;
        long long src_row = -1;
        if (!a.gated) {
            if (rr < a.n) src_row = rr;
        } else {
            const long long c = (rr >> 7) * 64 + (p & 63);
            if (c < a.n) src_row = p < 64 ? c : a.n + c;
        }
        const uint8_t* row =
            src_row >= 0 ? a.src + (bi / a.bdiv) * a.bnb_hi + (bi % a.bdiv) * a.bnb_lo + src_row * a.nb1 : nullptr;
        auto load = [&](long long kk) -> float {
            if (row == nullptr || kk >= a.k) return 0.0f;
            const uint8_t* ptr = row + kk * a.nb0;
            return a.type == SDB_TYPE_F16 ? __half2float(*reinterpret_cast<const __half*>(ptr))
                                          : *reinterpret_cast<const float*>(ptr);
        };
        float row_max = 0.0f;
        for (int g = 0; g < a.groups; ++g) {
            if (!a.weight_groups && static_cast<long long>(g) * a.group % a.span == 0) {
                // The largest magnitude of the span of k this group begins.
                const long long k1 = min(a.k, static_cast<long long>(g) * a.group + a.span);
                row_max = 0.0f;
                for (long long kk = static_cast<long long>(g) * a.group + lane; kk < k1; kk += 32)
                    row_max = fmaxf(row_max, fabsf(load(kk)));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) row_max = fmaxf(row_max, __shfl_xor_sync(0xffffffffu, row_max, o));
            }
            float w[EPL];
            float m = row_max;
            const long long k0 = static_cast<long long>(g) * a.group + lane * EPL;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
                w[e] = load(k0 + e);
                if (a.weight_groups) m = fmaxf(m, fabsf(w[e]));
            }
            if (a.weight_groups) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            }
            const float s = __fdiv_rn(m, static_cast<float>(a.wmax));
            const float inverse = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
            int sum = 0;
            uint64_t bytes = 0;
#pragma unroll
            for (int e = 0; e < EPL; ++e) {
                const float v = fminf(fmaxf(rintf(__fmul_rn(w[e], inverse)), static_cast<float>(-a.wmax)),
                                      static_cast<float>(a.wmax));
                const int qi = static_cast<int>(v);
                sum += qi;
                bytes |= static_cast<uint64_t>(static_cast<uint8_t>(static_cast<int8_t>(qi))) << (8 * e);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (EPL == 1 || EPL == 2 || EPL == 4 || EPL == 8) {
                int8_t* dst =
                    a.q + (tile * a.nstages + (k0 >> 6)) * 8192 + quant_tile_offset(p, static_cast<int>(k0 & 63));
                if (EPL == 8) *reinterpret_cast<uint64_t*>(dst) = bytes;
                else if (EPL == 4) *reinterpret_cast<uint32_t*>(dst) = static_cast<uint32_t>(bytes);
                else if (EPL == 2) *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(bytes);
                else *reinterpret_cast<uint8_t*>(dst) = static_cast<uint8_t>(bytes);
            } else {
                // Runs of 3 or 5 bytes may cross a 16-byte chunk: byte by byte.
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    const long long kk = k0 + e;
                    a.q[(tile * a.nstages + (kk >> 6)) * 8192 + quant_tile_offset(p, static_cast<int>(kk & 63))] =
                        static_cast<int8_t>(static_cast<uint8_t>(bytes >> (8 * e)));
                }
            }
            if (lane == 0) {
                float* sc = a.scales + (tile * a.groups + g) * 256;
                sc[p] = s;
                sc[128 + p] = __fmul_rn(s, static_cast<float>(sum));
            }
        }
    }
}

struct Key {
    int dev;
    const void* data;
    int type;
    int64_t ne[4];
    int64_t nb[4];
    int layout;
    int icp;
    int64_t half;
    int64_t variant;
    bool operator<(const Key& o) const {
        return std::tie(dev, data, type, ne[0], ne[1], ne[2], ne[3], nb[0], nb[1], nb[2], nb[3], layout, icp, half,
                        variant) <
               std::tie(o.dev, o.data, o.type, o.ne[0], o.ne[1], o.ne[2], o.ne[3], o.nb[0], o.nb[1], o.nb[2],
                        o.nb[3], o.layout, o.icp, o.half, o.variant);
    }
};

std::mutex g_store_mutex;
std::map<Key, std::shared_ptr<Packed>> g_store;

// Bytes spanned by a tensor from its data pointer.
int64_t extent_bytes(const sdb_tensor* t) {
    int64_t last = 0;
    for (int d = 0; d < 4; ++d) last += (t->ne[d] - 1) * t->nb[d];
    return last + (t->type == SDB_TYPE_F16 ? 2 : 4);
}

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// The store's entry for `key`, if any (*found), made safe to read on `stream`.
int lookup(const Key& key, cudaStream_t stream, std::shared_ptr<Packed>* out, bool* found) {
    *found = false;
    const bool keep = tuning().store != 0;
    if (!keep) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        SDB_CUDA(cudaStreamIsCapturing(stream, &cap));
        if (cap != cudaStreamCaptureStatusNone) return fail(SDB_INVALID, "store=0 packs per call: not under capture");
        return SDB_OK;
    }
    std::lock_guard<std::mutex> lock(g_store_mutex);
    auto it = g_store.find(key);
    if (it == g_store.end()) return SDB_OK;
    // Wait for the packing only while it may still run.  Under stream
    // capture nothing may be queried: the packing must have finished
    // (been seen finished) before the capture began.
    Packed& pk = *it->second;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    SDB_CUDA(cudaStreamIsCapturing(stream, &cap));
    if (cap != cudaStreamCaptureStatusNone) {
        if (!pk.done) return fail(SDB_INVALID, "weights first used under stream capture: call once before");
    } else if (!pk.done) {
        // The packing's second use waits for it on the host, once: from then on the entry
        // is known complete, and a stream capture (which may not query events) may use it.
        SDB_CUDA(cudaEventSynchronize(pk.ready));
        pk.done = true;
    }
    *out = it->second;
    *found = true;
    return SDB_OK;
}

void remember(const Key& key, const std::shared_ptr<Packed>& p) {
    if (tuning().store == 0) return;
    std::lock_guard<std::mutex> lock(g_store_mutex);
    g_store[key] = p;
}

int make_maps(Packed& p) {
    const uint64_t dims[2] = {static_cast<uint64_t>(p.kpad), static_cast<uint64_t>(p.rows_total)};
    const uint64_t strides[1] = {static_cast<uint64_t>(p.kpad) * 2};
    for (int bn : {64, 80, 96, 128, 160, 192, 256}) {
        const uint32_t box[2] = {64, static_cast<uint32_t>(bn)};
        CUtensorMap* m = bn == 256 ? &p.map256 : bn == 192 ? &p.map192 : bn == 160 ? &p.map160
                       : bn == 128 ? &p.map128 : bn == 96 ? &p.map96 : bn == 80 ? &p.map80 : &p.map64;
        const CUresult r = encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.data, dims, strides, box,
                                             CU_TENSOR_MAP_SWIZZLE_128B);
        if (r != CUDA_SUCCESS) return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for packed weights");
    }
    const uint32_t box32[2] = {32, 128};
    if (encode_tensor_map(&p.map128k32, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.data, dims, strides, box32,
                          CU_TENSOR_MAP_SWIZZLE_64B) != CUDA_SUCCESS)
        return fail(SDB_CUDA_ERROR, "cuTensorMapEncodeTiled failed for packed weights");
    return SDB_OK;
}

}  // namespace

Packed::~Packed() {
    if (ready) cudaEventDestroy(ready);
    if (borrowed) return;
    if (data) cudaFree(data);
    if (qscales) cudaFree(qscales);
}

size_t transient_bytes(const sdb_tensor* w, int64_t n_logical, int64_t k_logical) {
    const int64_t rows = round_up(n_logical, kRowPad) * (w->type == SDB_TYPE_F32 ? 2 : 1);
    return static_cast<size_t>(rows * round_up(std::max<int64_t>(k_logical, 1), 64) * 2);
}

int pack_transient(const sdb_tensor* w, int64_t n_logical, int64_t k_logical, void* dst, cudaStream_t stream,
                   Packed* p) {
    const bool split = w->type == SDB_TYPE_F32;
    p->borrowed = true;
    p->data = dst;
    p->kpad = round_up(std::max<int64_t>(k_logical, 1), 64);
    p->split = split;
    p->npad = round_up(n_logical, kRowPad);
    p->rows_total = split ? 2 * p->npad : p->npad;
    p->b1_row = split ? p->npad : 0;
    p->bytes = static_cast<size_t>(p->rows_total * p->kpad * 2);
    if (int st = make_maps(*p); st != SDB_OK) return st;
    PackArgs a{};
    a.src = static_cast<const uint8_t*>(w->data);
    a.type = w->type;
    for (int d = 0; d < 4; ++d) a.nb[d] = w->nb[d];
    a.layout = static_cast<int>(Layout::linear);
    a.n = n_logical;
    a.k = k_logical;
    a.kw = a.kh = 1;
    a.icp = 1;
    a.npad = p->npad;
    a.kpad = p->kpad;
    a.rows = p->npad;
    a.split = split ? 1 : 0;
    a.out = static_cast<__half*>(dst);
    a.err = device_error_word();
    const long long total = a.rows * a.kpad;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    pack_weights_kernel<<<blocks, 256, 0, stream>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    return SDB_OK;
}

int packed_weights(const sdb_tensor* w, Layout layout, int64_t n_logical, int64_t k_logical, int icp, int64_t half,
                   cudaStream_t stream, std::shared_ptr<Packed>* out) {
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    const Key key{dev, w->data, w->type, {w->ne[0], w->ne[1], w->ne[2], w->ne[3]},
                  {w->nb[0], w->nb[1], w->nb[2], w->nb[3]}, static_cast<int>(layout), icp, half, 0};
    bool found = false;
    if (int s = lookup(key, stream, out, &found); s != SDB_OK || found) return s;
    auto p = std::make_shared<Packed>();
    const bool split = w->type == SDB_TYPE_F32;
    int64_t kdim;
    if (layout == Layout::conv) kdim = w->ne[0] * w->ne[1] * icp;
    else kdim = k_logical;
    p->kpad = round_up(std::max<int64_t>(kdim, 1), 64);
    p->icp = icp;
    p->split = split;
    if (layout == Layout::gated) {
        const int64_t halfpad = round_up(half, kRowPad);
        p->npad = 2 * halfpad;
        p->rows_total = 2 * halfpad;
        p->b1_row = halfpad;
    } else {
        p->npad = round_up(n_logical, kRowPad);
        p->rows_total = split ? 2 * p->npad : p->npad;
        p->b1_row = split ? p->npad : 0;
    }
    p->bytes = static_cast<size_t>(p->rows_total * p->kpad * 2);
    SDB_CUDA(cudaMalloc(&p->data, p->bytes));
    SDB_CUDA(cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming));
    if (int st = make_maps(*p); st != SDB_OK) return st;

    PackArgs a{};
    a.src = static_cast<const uint8_t*>(w->data);
    a.type = w->type;
    for (int d = 0; d < 4; ++d) a.nb[d] = w->nb[d];
    a.layout = static_cast<int>(layout);
    a.n = layout == Layout::gated ? 2 * half : n_logical;
    a.k = layout == Layout::conv ? w->ne[2] : k_logical;
    a.kw = static_cast<int>(w->ne[0]);
    a.kh = static_cast<int>(w->ne[1]);
    a.icp = icp > 0 ? icp : 1;
    a.half = half;
    a.halfpad = p->b1_row;
    a.npad = p->npad;
    a.kpad = p->kpad;
    a.rows = layout == Layout::gated ? p->rows_total : p->npad;
    a.split = split ? 1 : 0;
    a.out = static_cast<__half*>(p->data);
    a.err = device_error_word();
    const long long total = a.rows * a.kpad;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    pack_weights_kernel<<<blocks, 256, 0, stream>>>(a);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    SDB_CUDA(cudaEventRecord(p->ready, stream));
    remember(key, p);
    *out = p;
    return SDB_OK;
}

int quantized_weights(const sdb_tensor* w, bool gated, int64_t n_logical, int64_t k_logical, int64_t half,
                      const QuantSpec& q, cudaStream_t stream, std::shared_ptr<Packed>* out) {
    if (q.group % 32 != 0 || q.group < 32 || q.group > 256)
        return fail(SDB_NOT_SUPPORTED, "quantized products: group must be 32, 64, 128 or 256");
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    const Layout layout = gated ? Layout::quantized_gated : Layout::quantized;
    const Key key{dev, w->data, w->type, {w->ne[0], w->ne[1], w->ne[2], w->ne[3]},
                  {w->nb[0], w->nb[1], w->nb[2], w->nb[3]}, static_cast<int>(layout), 0, gated ? half : 0,
                  q.variant()};
    bool found = false;
    if (int s = lookup(key, stream, out, &found); s != SDB_OK || found) return s;

    auto p = std::make_shared<Packed>();
    p->group = q.group;
    p->groups = static_cast<int>((k_logical + q.group - 1) / q.group);
    p->kpad = static_cast<int64_t>(p->groups) * q.group;
    const int nstages = (p->groups * (q.group / 32) + 1) / 2;
    p->tiles = static_cast<int>(gated ? (half + 63) / 64 : (n_logical + 127) / 128);
    p->rows_total = static_cast<int64_t>(p->tiles) * 128;
    p->npad = p->rows_total;
    const size_t q_bytes = static_cast<size_t>(p->tiles) * nstages * 8192;
    const size_t s_bytes = static_cast<size_t>(p->tiles) * p->groups * 1024;
    p->bytes = q_bytes + s_bytes;
    SDB_CUDA(cudaMalloc(&p->data, q_bytes));
    SDB_CUDA(cudaMalloc(&p->qscales, s_bytes));
    // Bytes no group covers (the second half of an item's last stage with
    // groups of 32) are never read; zero them all the same.
    SDB_CUDA(cudaMemsetAsync(p->data, 0, q_bytes, stream));
    SDB_CUDA(cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming));
    QPackArgs a{};
    a.src = static_cast<const uint8_t*>(w->data);
    a.type = w->type;
    a.nb0 = w->nb[0];
    a.nb1 = w->nb[1];
    a.n = gated ? half : n_logical;
    a.k = k_logical;
    a.gated = gated ? 1 : 0;
    a.rows = p->rows_total;
    a.group = q.group;
    a.groups = p->groups;
    a.nstages = nstages;
    a.wmax = q.wmax;
    a.weight_groups = q.weight_groups ? 1 : 0;
    a.span = p->kpad;
    a.batches = 1;
    a.bdiv = 1;
    a.q = static_cast<int8_t*>(p->data);
    a.scales = static_cast<float*>(p->qscales);
    launch_quantize_weights(a, stream);
    SDB_CUDA(cudaGetLastError());
    SDB_CUDA(cudaEventRecord(p->ready, stream));
    remember(key, p);
    *out = p;
    return SDB_OK;
}

void launch_quantize_weights(const QPackArgs& a, cudaStream_t stream) {
    const int blocks = static_cast<int>(std::min<long long>((a.rows + 7) / 8, 148LL * 8));
    switch (a.group / 32) {
        case 1: quantize_weights_kernel<1><<<blocks, 256, 0, stream>>>(a); break;
        case 2: quantize_weights_kernel<2><<<blocks, 256, 0, stream>>>(a); break;
        case 3: quantize_weights_kernel<3><<<blocks, 256, 0, stream>>>(a); break;
        case 4: quantize_weights_kernel<4><<<blocks, 256, 0, stream>>>(a); break;
        case 5: quantize_weights_kernel<5><<<blocks, 256, 0, stream>>>(a); break;
        default: quantize_weights_kernel<8><<<blocks, 256, 0, stream>>>(a); break;
    }
    count_launch();
}

// F(2x2)'s transformed kernels quantized, xi by xi: U = G g G^T in FP32
// (winograd2_weights_f32_kernel, into a buffer freed after), then each xi's
// (oc, ic) matrix quantized like a linear layer's weights into tiles
// [xi][tiles][nstages][8 KiB] and scales [xi][tiles][groups][2][128]
// (winograd.cc:1907-1936).  span: with per-row scales, the input channels
// one scale covers (the reference's stretch of channels).
int quantized_winograd_weights(const sdb_tensor* w, const QuantSpec& q, int64_t span, cudaStream_t stream,
                               std::shared_ptr<Packed>* out) {
    if (q.group % 32 != 0 || q.group < 32 || q.group > 256)
        return fail(SDB_NOT_SUPPORTED, "quantized products: group must be 32, 64, 128 or 256");
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    const int64_t ic = w->ne[2], oc = w->ne[3];
    const Key key{dev, w->data, w->type, {w->ne[0], w->ne[1], w->ne[2], w->ne[3]},
                  {w->nb[0], w->nb[1], w->nb[2], w->nb[3]}, static_cast<int>(Layout::quantized_winograd2), 0,
                  q.weight_groups ? 0 : span, q.variant()};
    bool found = false;
    if (int s = lookup(key, stream, out, &found); s != SDB_OK || found) return s;

    constexpr int xi = 16;
    auto p = std::make_shared<Packed>();
    p->group = q.group;
    p->groups = static_cast<int>((ic + q.group - 1) / q.group);
    p->kpad = static_cast<int64_t>(p->groups) * q.group;
    const int nstages = (p->groups * (q.group / 32) + 1) / 2;
    p->tiles = static_cast<int>((oc + 127) / 128);
    p->rows_total = static_cast<int64_t>(p->tiles) * 128;
    p->npad = p->rows_total;
    const size_t q_xi = static_cast<size_t>(p->tiles) * nstages * 8192;
    const size_t s_xi = static_cast<size_t>(p->tiles) * p->groups * 1024;
    p->bytes = xi * (q_xi + s_xi);
    SDB_CUDA(cudaMalloc(&p->data, xi * q_xi));
    SDB_CUDA(cudaMalloc(&p->qscales, xi * s_xi));
    SDB_CUDA(cudaMemsetAsync(p->data, 0, xi * q_xi, stream));
    SDB_CUDA(cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming));
    float* u = nullptr;
    const size_t u_bytes = static_cast<size_t>(xi) * oc * ic * 4;
    SDB_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&u), u_bytes, stream));
    const long long total = ic * oc;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    winograd2_weights_f32_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(w->data), w->type, w->nb[0],
                                                             w->nb[1], w->nb[2], w->nb[3], static_cast<int>(ic),
                                                             static_cast<int>(oc), u);
    count_launch();
    SDB_CUDA(cudaGetLastError());
    QPackArgs a{};
    a.type = SDB_TYPE_F32;
    a.nb0 = 4;
    a.nb1 = 4 * ic;
    a.n = oc;
    a.k = ic;
    a.gated = 0;
    a.rows = p->rows_total;
    a.group = q.group;
    a.groups = p->groups;
    a.nstages = nstages;
    a.wmax = q.wmax;
    a.weight_groups = q.weight_groups ? 1 : 0;
    a.span = q.weight_groups ? p->kpad : span;
    // The sixteen xi as batches of the one launch: batch x reads U's plane x.
    a.src = reinterpret_cast<const uint8_t*>(u);
    a.batches = xi;
    a.bdiv = 1;
    a.bnb_hi = static_cast<long long>(oc) * ic * 4;
    a.rows = xi * p->rows_total;
    a.q = static_cast<int8_t*>(p->data);
    a.scales = static_cast<float*>(p->qscales);
    launch_quantize_weights(a, stream);
    SDB_CUDA(cudaGetLastError());
    SDB_CUDA(cudaFreeAsync(u, stream));
    SDB_CUDA(cudaEventRecord(p->ready, stream));
    remember(key, p);
    *out = p;
    return SDB_OK;
}

int winograd_weights(const sdb_tensor* w, int f, cudaStream_t stream, std::shared_ptr<Packed>* out) {
    if (f != 2 && f != 4) return fail(SDB_INVALID, "winograd: F(2x2) or F(4x4) only");
    int dev = 0;
    SDB_CUDA(cudaGetDevice(&dev));
    const Layout layout = f == 2 ? Layout::winograd2 : Layout::winograd4;
    const Key key{dev, w->data, w->type, {w->ne[0], w->ne[1], w->ne[2], w->ne[3]},
                  {w->nb[0], w->nb[1], w->nb[2], w->nb[3]}, static_cast<int>(layout), 0, 0, 0};
    bool found = false;
    if (int s = lookup(key, stream, out, &found); s != SDB_OK || found) return s;
    const int xi = f == 2 ? Wino<2>::kXi : Wino<4>::kXi;
    const int64_t ic = w->ne[2], oc = w->ne[3];
    auto p = std::make_shared<Packed>();
    p->kpad = round_up(ic, 64);
    const int64_t ocp = round_up(oc, 128);
    p->npad = xi * ocp;
    p->rows_total = 2 * p->npad;
    p->b1_row = p->npad;
    p->split = true;
    p->bytes = static_cast<size_t>(p->rows_total * p->kpad * 2);
    SDB_CUDA(cudaMalloc(&p->data, p->bytes));
    SDB_CUDA(cudaMemsetAsync(p->data, 0, p->bytes, stream));
    SDB_CUDA(cudaEventCreateWithFlags(&p->ready, cudaEventDisableTiming));
    if (int st = make_maps(*p); st != SDB_OK) return st;
    const long long total = ic * oc;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
    auto src = static_cast<const uint8_t*>(w->data);
    auto dst = static_cast<__half*>(p->data);
    if (f == 2)
        winograd_weights_kernel<2><<<blocks, 256, 0, stream>>>(src, w->type, w->nb[0], w->nb[1], w->nb[2], w->nb[3],
                                                               static_cast<int>(ic), static_cast<int>(oc), ocp,
                                                               p->kpad, dst, device_error_word());
    else
        winograd_weights_kernel<4><<<blocks, 256, 0, stream>>>(src, w->type, w->nb[0], w->nb[1], w->nb[2], w->nb[3],
                                                               static_cast<int>(ic), static_cast<int>(oc), ocp,
                                                               p->kpad, dst, device_error_word());
    count_launch();
    SDB_CUDA(cudaGetLastError());
    SDB_CUDA(cudaEventRecord(p->ready, stream));
    remember(key, p);
    *out = p;
    return SDB_OK;
}

}  // namespace sdb

extern "C" void sdb_forget(const void* begin, size_t size) {
    const auto b = reinterpret_cast<uintptr_t>(begin);
    const uintptr_t e = b + size;
    std::vector<std::shared_ptr<sdb::Packed>> dropped;
    {
        std::lock_guard<std::mutex> lock(sdb::g_store_mutex);
        for (auto it = sdb::g_store.begin(); it != sdb::g_store.end();) {
            const auto s = reinterpret_cast<uintptr_t>(it->first.data);
            sdb_tensor t{};
            t.type = it->first.type;
            for (int d = 0; d < 4; ++d) { t.ne[d] = it->first.ne[d]; t.nb[d] = it->first.nb[d]; }
            const uintptr_t se = s + static_cast<uintptr_t>(sdb::extent_bytes(&t));
            if (s < e && b < se) {
                dropped.push_back(it->second);
                it = sdb::g_store.erase(it);
            } else {
                ++it;
            }
        }
    }
    // Entries may still be read by kernels in flight: wait before freeing.
    if (!dropped.empty()) cudaDeviceSynchronize();
    dropped.clear();
}

extern "C" void sdb_store_stats(int64_t* entries, int64_t* bytes) {
    std::lock_guard<std::mutex> lock(sdb::g_store_mutex);
    int dev = 0;
    cudaGetDevice(&dev);
    int64_t n = 0, b = 0;
    for (const auto& kv : sdb::g_store) {
        if (kv.first.dev != dev) continue;
        ++n;
        b += static_cast<int64_t>(kv.second->bytes);
    }
    if (entries) *entries = n;
    if (bytes) *bytes = b;
}
