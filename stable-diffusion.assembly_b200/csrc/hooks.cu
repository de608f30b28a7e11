// The hook surface of sdasm.h over the sdb_* entry points: what ggml's patched
// CPU backend calls (the reference's sources/hooks.cc:29-196 and the chain
// matching of sources/fusion.cc:136-394), with the work done on a CUDA device.
//
// Per node, in the reference's order:
//   1. thread 0 forgets what was kept from the memory the node writes
//      (hooks.cc:107-111: every node offered, taken or not, may overwrite a
//      tensor whose packing is kept);
//   2. taken(): the operation and its operands, as the reference's
//      *_supported() test them, and as sdb_*_supported() can take them;
//   3. the chain after it (match_chain: in-place additions and multiplications
//      by broadcast operands, SiLU after a normalisation, a residual addition
//      not in place), or GEGLU's view/view/cont/gelu/mul after a linear layer;
//   4. thread 0 computes it on the device and waits; every thread returns the
//      same count of nodes, so that ggml's loop skips the fused ones.
//
// Memory.  ggml's buffers may be device or managed memory, which the kernels
// read in place, or host memory (the stock CPU backend).  A host tensor is
// staged per node through a device arena -- tensors whose bytes overlap share
// one staged region, so in-place chains and residual sums alias on the device
// as they do on the host -- and what the node writes is copied back.  Host
// weights (src[0] of MUL_MAT and CONV_2D) are mirrored on the device once and
// kept, with the packing the store makes of them, until sdasm_forget() names
// their memory: ggml calls it before it writes a buffer (patch 0004), and step
// 1 above covers what a graph's nodes write.
//
// Built into libsdb.so against include/ggml_mirror.h; inside ggml's CPU
// backend, against ggml's own headers (-DSDB_WITH_GGML).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cinttypes>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/sdasm.h"
#include "../../include/sdb.h"
#ifdef SDB_WITH_GGML
#include "ggml-cpu-impl.h"
#include "ggml.h"
#else
#include "../../include/ggml_mirror.h"
#endif
#include "runtime.cuh"

namespace sdb {
namespace hooks {
namespace {

enum class Op { none, conv2d, mul_mat, attention, group_norm, norm };

constexpr int kMaxSteps = SDB_MAX_STEPS;

// ---------------------------------------------------------------- tensors

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// The tensor holds elements of `type` of `size` bytes at element-aligned
// strides (memory.h holds<T>).
bool holds(const ggml_tensor* t, int type, size_t size) {
    if (t == nullptr || static_cast<int>(t->type) != type || !aligned(t->data, size)) return false;
    for (int k = 0; k < 4; ++k)
        if (t->nb[k] % size != 0) return false;
    return true;
}
bool holds_f32(const ggml_tensor* t) { return holds(t, GGML_TYPE_F32, 4); }
bool holds_f16(const ggml_tensor* t) { return holds(t, GGML_TYPE_F16, 2); }
bool holds_weights(const ggml_tensor* t) { return holds_f16(t) || holds_f32(t); }

bool overlaps(const void* a, size_t an, const void* b, size_t bn) {
    if (a == nullptr || b == nullptr || an == 0 || bn == 0) return false;
    const auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + bn && y < x + an;
}
bool tensors_overlap(const ggml_tensor* a, const ggml_tensor* b) {
    return overlaps(a->data, ggml_nbytes(a), b->data, ggml_nbytes(b));
}

// Same extents, strides, memory and type (fusion.cc:29-36).
bool same_layout(const ggml_tensor* a, const ggml_tensor* b) {
    for (int k = 0; k < 4; ++k)
        if (a->ne[k] != b->ne[k] || a->nb[k] != b->nb[k]) return false;
    return a->data == b->data && a->type == b->type;
}

float param_f32(const ggml_tensor* t, int i) {
    float f;
    std::memcpy(&f, &t->op_params[i], sizeof f);
    return f;
}

// The descriptor sdb.h takes, at `data` (a device address, or the tensor's
// own when only its shape is asked about).
sdb_tensor describe(const ggml_tensor* t, void* data) {
    sdb_tensor d{};
    d.type = static_cast<int32_t>(t->type);
    for (int k = 0; k < 4; ++k) {
        d.ne[k] = t->ne[k];
        d.nb[k] = static_cast<int64_t>(t->nb[k]);
    }
    // ggml may plan a graph before its tensors have memory: a stand-in address
    // of the alignment allocations have keeps the answer what it will be.
    d.data = data ? data : reinterpret_cast<void*>(uintptr_t{256});
    return d;
}
sdb_tensor describe(const ggml_tensor* t) { return describe(t, t->data); }

// ---------------------------------------------------------------- taken

Op taken(const ggml_tensor* node) {
    if (node == nullptr) return Op::none;
    const ggml_tensor* a = node->src[0];
    const ggml_tensor* b = node->src[1];
    switch (node->op) {
    case GGML_OP_CONV_2D: {
        // conv2d.cc:320-330 (winograd.cc:2107-2123 takes a subset of these).
        if (a == nullptr || b == nullptr) return Op::none;
        const int32_t* p = node->op_params;
        if (!(holds_weights(a) && ggml_is_contiguous(a) && holds_f32(b) && b->nb[0] == 4 && holds_f32(node) &&
              ggml_is_contiguous(node) && a->ne[2] == b->ne[2] && p[0] > 0 && p[1] > 0 && p[4] > 0 && p[5] > 0))
            return Op::none;
        const sdb_tensor w = describe(a), x = describe(b), y = describe(node);
        return sdb_conv2d_supported(&w, &x, &y, p) ? Op::conv2d : Op::none;
    }
    case GGML_OP_MUL_MAT: {
        // mul_mat.cc:181-194: one weight matrix, rows of x and of the result one
        // after another, and products big enough to pay for packing.
        if (a == nullptr || b == nullptr) return Op::none;
        if (!(holds_weights(a) && a->ne[2] == 1 && a->ne[3] == 1 && a->nb[0] == ggml_type_size(a->type) &&
              holds_f32(b) && ggml_is_contiguous(b) && holds_f32(node) && ggml_is_contiguous(node) &&
              a->extra == nullptr && b->ne[1] * b->ne[2] * b->ne[3] >= 16 && a->ne[0] >= 16))
            return Op::none;
        const sdb_tensor w = describe(a), x = describe(b), y = describe(node);
        return sdb_mul_mat_supported(&w, &x, &y) ? Op::mul_mat : Op::none;
    }
    case GGML_OP_FLASH_ATTN_EXT: {
        // attention.cc:828-845: no mask, no ALiBi, no soft cap.
        const ggml_tensor* v = node->src[2];
        if (a == nullptr || b == nullptr || v == nullptr || node->src[3] != nullptr || node->src[4] != nullptr)
            return Op::none;
        if (param_f32(node, 1) != 0.0f || param_f32(node, 2) != 0.0f) return Op::none;
        if (!(holds_f32(a) && holds_weights(b) && holds_weights(v) && a->nb[0] == 4 &&
              b->nb[0] == ggml_type_size(b->type) && v->nb[0] == ggml_type_size(v->type) && holds_f32(node) &&
              ggml_is_contiguous(node)))
            return Op::none;
        const sdb_tensor q = describe(a), k = describe(b), vv = describe(v), y = describe(node);
        return sdb_attention_supported(&q, &k, &vv, &y) ? Op::attention : Op::none;
    }
    case GGML_OP_GROUP_NORM:
        // norm.cc:94-98.
        return a != nullptr && holds_f32(a) && holds_f32(node) && ggml_is_contiguous(a) && ggml_is_contiguous(node) &&
                       ggml_are_same_shape(a, node) && node->op_params[0] > 0
                   ? Op::group_norm
                   : Op::none;
    case GGML_OP_NORM:
        // norm.cc:142-146.
        return a != nullptr && holds_f32(a) && holds_f32(node) && a->nb[0] == 4 && node->nb[0] == 4 &&
                       ggml_are_same_shape(a, node)
                   ? Op::norm
                   : Op::none;
    default:
        return Op::none;
    }
}

// ---------------------------------------------------------------- chains

struct Step {
    int kind = SDB_STEP_ADD;
    const ggml_tensor* operand = nullptr;
    int64_t nb[4] = {0, 0, 0, 0};  // elements; 0 along a broadcast dimension
};

// What a taken node computes with the nodes after it (fusion.h:61-91).
struct Chain {
    int count = 0;
    Step steps[kMaxSteps];
    int last_node = -1;
    const ggml_tensor* redirect = nullptr;  // the residual sum's tensor, written in place of the node's
    bool from_redirect = false;             // the sum begins from what redirect holds
    const ggml_tensor* gated_out = nullptr; // GEGLU: the gated GELU's output
    int gated_last = -1;
    bool empty() const { return count == 0 && !from_redirect; }
};

bool unary_is(const ggml_tensor* t, ggml_unary_op u) { return t->op == GGML_OP_UNARY && ggml_get_unary_op(t) == u; }

// Whether node `from` or any after it reads one of `tensors`, or a view of
// one (fusion.cc:314-327).
bool read_after(ggml_tensor* const* nodes, int n_nodes, int from, const std::vector<const ggml_tensor*>& tensors) {
    for (int i = from; i < n_nodes; ++i) {
        for (const ggml_tensor* s : nodes[i]->src)
            for (const ggml_tensor* t = s; t != nullptr; t = t->view_src)
                if (std::find(tensors.begin(), tensors.end(), t) != tensors.end()) return true;
    }
    return false;
}

// The chain after node `index` (fusion.cc:136-270).
Chain match_chain(ggml_tensor* const* nodes, int n_nodes, int index, bool silu, bool positions, bool redirect) {
    Chain e;
    const ggml_tensor* head = nodes[index];
    e.last_node = index;
    if (!holds_f32(head) || head->nb[0] != 4) return e;
    int j = index + 1;
    for (; j < n_nodes && e.count < kMaxSteps; ++j) {
        const ggml_tensor* node = nodes[j];
        if (ggml_op_is_empty(node->op)) continue;
        if ((node->flags & GGML_TENSOR_FLAG_COMPUTE) == 0 || !same_layout(node, head)) break;
        Step step;
        if (unary_is(node, GGML_UNARY_OP_SILU) && silu && node->src[0] != nullptr &&
            node->src[0]->data == head->data) {
            step.kind = SDB_STEP_SILU;
        } else if (node->op == GGML_OP_ADD || node->op == GGML_OP_MUL) {
            // In place through src[0]; the other operand broadcast to the output.
            const ggml_tensor* a = node->src[0];
            const ggml_tensor* b = node->src[1];
            if (a == nullptr || b == nullptr) break;
            if (a->data != head->data || !ggml_are_same_shape(a, head) || tensors_overlap(b, head) || !holds_f32(b) ||
                b->nb[0] != 4)
                break;
            bool fits = true;
            for (int k = 0; k < 4; ++k) {
                if (b->ne[k] != head->ne[k] && b->ne[k] != 1) fits = false;
                step.nb[k] = b->ne[k] == 1 ? 0 : static_cast<int64_t>(b->nb[k] / 4);
            }
            if (positions) {
                // An image's positions: one number for all of them, or rows as the output's.
                const bool broadcast = step.nb[0] == 0 && step.nb[1] == 0;
                const bool rows = step.nb[0] == 1 && step.nb[1] == head->ne[0];
                fits = fits && (broadcast || rows);
            }
            if (!fits) break;
            step.kind = node->op == GGML_OP_ADD ? SDB_STEP_ADD : SDB_STEP_MUL;
            step.operand = b;
        } else {
            break;
        }
        e.steps[e.count++] = step;
        e.last_node = j;
    }
    // A residual addition not in place, past any views (fusion.cc:200-269).
    for (; redirect && j < n_nodes && ggml_op_is_empty(nodes[j]->op); ++j) {
    }
    if (!redirect || j >= n_nodes || e.count >= kMaxSteps) return e;
    ggml_tensor* node = nodes[j];
    auto alike = [&](const ggml_tensor* t) {
        if (t == nullptr || !holds_f32(t)) return false;
        for (int k = 0; k < 4; ++k)
            if (t->ne[k] != head->ne[k] || t->nb[k] != head->nb[k]) return false;
        return true;
    };
    if (node->op != GGML_OP_ADD || (node->flags & GGML_TENSOR_FLAG_COMPUTE) == 0 || !alike(node) ||
        node->data == head->data)
        return e;
    const ggml_tensor* a = node->src[0];
    const ggml_tensor* b = node->src[1];
    const ggml_tensor* other = a != nullptr && a->data == head->data && alike(a)   ? b
                               : b != nullptr && b->data == head->data && alike(b) ? a
                                                                                   : nullptr;
    if (!alike(other) || tensors_overlap(other, head)) return e;
    // Nothing after reads the node's tensor or its chain's; none is an output.
    std::vector<const ggml_tensor*> unwritten;
    for (int i = index; i <= e.last_node; ++i) {
        const ggml_tensor* t = nodes[i];
        if (t->data != head->data) continue;
        if (t->flags & GGML_TENSOR_FLAG_OUTPUT) return e;
        unwritten.push_back(t);
    }
    if (read_after(nodes, n_nodes, j + 1, unwritten)) return e;
    if (other->data == node->data) {
        // The sum lands in the other operand's memory: begun from it, which only
        // additions before it may be reordered with.
        for (int s = 0; s < e.count; ++s)
            if (e.steps[s].kind != SDB_STEP_ADD) return e;
        e.from_redirect = true;
        e.last_node = j;
        e.redirect = node;
        return e;
    }
    Step step;
    step.kind = SDB_STEP_ADD;
    step.operand = other;
    for (int k = 0; k < 4; ++k) step.nb[k] = static_cast<int64_t>(other->nb[k] / 4);
    e.steps[e.count++] = step;
    e.last_node = j;
    e.redirect = node;
    return e;
}

// The redirect's memory is none of what the operation or its chain reads
// (fusion.cc:272-288).
bool redirect_apart(const ggml_tensor* node, const Chain& c) {
    if (c.redirect == nullptr) return true;
    for (const ggml_tensor* s : node->src)
        if (s != nullptr && s->data != nullptr && tensors_overlap(c.redirect, s)) return false;
    for (int i = 0; i < c.count; ++i)
        if (c.steps[i].operand != nullptr && tensors_overlap(c.redirect, c.steps[i].operand)) return false;
    return true;
}

// A view of `whole` that is its columns [begin, begin + width) (fusion.cc:331-343).
bool columns_of(const ggml_tensor* view, const ggml_tensor* whole, int64_t begin, int64_t width) {
    if (!holds_f32(view) || !holds_f32(whole) || view->ne[0] != width || view->nb[0] != 4 || begin > whole->ne[0] ||
        static_cast<const char*>(view->data) != static_cast<const char*>(whole->data) + begin * 4)
        return false;
    for (int k = 1; k < 4; ++k)
        if (view->ne[k] != whole->ne[k] || view->nb[k] != whole->nb[k]) return false;
    return true;
}

// GEGLU after a linear layer and its chain: view, view, cont of the gate, its
// GELU in place, x times that into a tensor of its own (fusion.cc:347-394).
void match_gated_gelu(ggml_tensor* const* nodes, int n_nodes, int index, Chain& c) {
    const int j = c.last_node + 1;
    if (j + 5 > n_nodes) return;
    const ggml_tensor* head = nodes[index];
    const ggml_tensor* v0 = nodes[j];
    const ggml_tensor* v1 = nodes[j + 1];
    const ggml_tensor* cont = nodes[j + 2];
    const ggml_tensor* gelu = nodes[j + 3];
    const ggml_tensor* mul = nodes[j + 4];
    if (head->type != GGML_TYPE_F32 || !ggml_is_contiguous(head) || head->ne[0] % 2 != 0 || v0->op != GGML_OP_VIEW ||
        v1->op != GGML_OP_VIEW || cont->op != GGML_OP_CONT || !unary_is(gelu, GGML_UNARY_OP_GELU) ||
        mul->op != GGML_OP_MUL)
        return;
    const ggml_tensor* gate = cont->src[0];
    const ggml_tensor* x = gate == v0 ? v1 : gate == v1 ? v0 : nullptr;
    const int64_t half = head->ne[0] / 2;
    if (x == nullptr || !columns_of(x, head, 0, half) || !columns_of(gate, head, half, half) ||
        gelu->src[0] != cont || gelu->data != cont->data || mul->src[0] != x || mul->src[1] != gelu ||
        mul->type != GGML_TYPE_F32 || !ggml_is_contiguous(mul) || !ggml_are_same_shape(mul, x))
        return;
    std::vector<const ggml_tensor*> unwritten;
    for (int i = index; i <= c.last_node; ++i) unwritten.push_back(nodes[i]);
    for (const ggml_tensor* t : {v0, v1, cont, gelu}) unwritten.push_back(t);
    for (const ggml_tensor* t : unwritten)
        if (t->flags & GGML_TENSOR_FLAG_OUTPUT) return;
    if (read_after(nodes, n_nodes, j + 5, unwritten)) return;
    c.gated_out = mul;
    c.gated_last = j + 4;
}

// The gated output's memory is none of what the product reads, and its
// layout is what sdb_mul_mat_gated writes (mul_mat.cc:1129-1150).
bool gated_supported(const ggml_tensor* node, const Chain& c) {
    const ggml_tensor* out = c.gated_out;
    const ggml_tensor* w = node->src[0];
    const ggml_tensor* x = node->src[1];
    const size_t on = ggml_nbytes(out);
    if (overlaps(out->data, on, w->data, ggml_nbytes(w)) || overlaps(out->data, on, x->data, ggml_nbytes(x)) ||
        overlaps(out->data, on, node->data, ggml_nbytes(node)))
        return false;
    for (int s = 0; s < c.count; ++s)
        if (c.steps[s].operand && overlaps(out->data, on, c.steps[s].operand->data, ggml_nbytes(c.steps[s].operand)))
            return false;
    if (!holds_f32(out) || out->nb[0] != 4 || out->ne[0] != node->ne[0] / 2) return false;
    const sdb_tensor dw = describe(w), dx = describe(x), dout = describe(out);
    return sdb_mul_mat_gated_supported(&dw, &dx, &dout) != 0;
}

// The chain of a taken node, as hooks.cc:123-152 matches it.
Chain chain_of(ggml_tensor* const* nodes, int n_nodes, int index, Op op) {
    Chain c;
    c.last_node = index;
    if (tuning().fuse == 0) return c;
    const ggml_tensor* node = nodes[index];
    const bool residual = tuning().fuse_residual != 0;
    switch (op) {
    case Op::conv2d:
    case Op::mul_mat: {
        const bool positions = op == Op::conv2d;
        c = match_chain(nodes, n_nodes, index, false, positions, residual);
        if (!redirect_apart(node, c)) c = match_chain(nodes, n_nodes, index, false, positions, false);
        if (op == Op::mul_mat && c.redirect == nullptr) {
            match_gated_gelu(nodes, n_nodes, index, c);
            if (c.gated_out != nullptr && !gated_supported(node, c)) {
                c.gated_out = nullptr;
                c.gated_last = -1;
            }
        }
        break;
    }
    case Op::group_norm:
    case Op::norm:
        c = match_chain(nodes, n_nodes, index, true, false, false);
        break;
    default:
        break;
    }
    return c;
}

int node_count(const Chain& c, int index) {
    if (c.gated_out != nullptr) return c.gated_last - index + 1;
    return c.empty() ? 1 : c.last_node - index + 1;
}

// ---------------------------------------------------------------- device memory

[[noreturn]] void die(const std::string& what) {
    std::fprintf(stderr, "sdasm (B200): %s\n", what.c_str());
    std::abort();
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(e));
}

int device_of_hooks() {
    static const int dev = [] {
        const char* s = std::getenv("SDASM_CUDA_DEVICE");
        return s ? std::atoi(s) : 0;
    }();
    return dev;
}

// Whether the kernels can read p in place (device or managed memory).
bool on_device(const void* p) {
    if (p == nullptr) return true;
    cudaPointerAttributes attr{};
    const cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

struct Mirror {
    size_t size = 0;
    uint8_t* base = nullptr;  // the allocation
    uint8_t* data = nullptr;  // the host bytes' copy, congruent with them modulo 256
};

struct DeviceState {
    cudaStream_t stream = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    std::map<uintptr_t, Mirror> mirrors;  // host weights' device copies, by host address
};

std::mutex g_mutex;  // one taken node at a time; guards the state below
std::unordered_map<int, DeviceState> g_devices;

DeviceState& device_state() {
    const int dev = device_of_hooks();
    check(cudaSetDevice(dev), "cudaSetDevice");
    DeviceState& d = g_devices[dev];
    if (d.stream == nullptr) check(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    return d;
}

// Drops host mirrors overlapping [begin, begin + size) and what the store
// packed from them.  Called with g_mutex held.
void drop_mirrors(const void* begin, size_t size) {
    for (auto& [dev, d] : g_devices) {
        for (auto it = d.mirrors.begin(); it != d.mirrors.end();) {
            if (overlaps(reinterpret_cast<const void*>(it->first), it->second.size, begin, size)) {
                check(cudaSetDevice(dev), "cudaSetDevice");
                sdb_forget(it->second.data, it->second.size);
                check(cudaFree(it->second.base), "cudaFree (weight mirror)");
                it = d.mirrors.erase(it);
            } else {
                ++it;
            }
        }
    }
}

uint8_t* weight_mirror(DeviceState& d, const ggml_tensor* t) {
    const auto host = reinterpret_cast<uintptr_t>(t->data);
    const size_t size = ggml_nbytes(t);
    auto it = d.mirrors.find(host);
    if (it != d.mirrors.end() && it->second.size == size) return it->second.data;
    drop_mirrors(t->data, size);
    Mirror m;
    m.size = size;
    check(cudaMalloc(&m.base, size + 256), "cudaMalloc (weight mirror)");
    m.data = m.base + (host & 255);
    check(cudaMemcpy(m.data, t->data, size, cudaMemcpyHostToDevice), "cudaMemcpy (weight mirror)");
    d.mirrors[host] = m;
    return m.data;
}

// The tensors of one node's computation and where the kernels find them.
class Staging {
public:
    explicit Staging(DeviceState& d) : d_(d) {}

    void weight(const ggml_tensor* t) { add(t, true, false); }
    void read(const ggml_tensor* t) { add(t, false, false); }
    void write(const ggml_tensor* t) { add(t, false, true); }

    // Copies the host tensors' bytes into the arena (overlapping ones as one
    // region), after which device() names each tensor's device address.
    void stage() {
        std::vector<Item*> host;
        for (Item& it : items_) {
            if (it.weight && !on_device(it.t->data)) {
                it.device = weight_mirror(d_, it.t);
            } else if (on_device(it.t->data)) {
                it.device = it.t->data;
            } else {
                host.push_back(&it);
            }
        }
        std::sort(host.begin(), host.end(), [](const Item* a, const Item* b) { return a->begin < b->begin; });
        for (Item* it : host) {
            if (regions_.empty() || it->begin >= regions_.back().end) regions_.push_back({it->begin, it->end, 0});
            else regions_.back().end = std::max(regions_.back().end, it->end);
        }
        size_t need = 0;
        for (Region& r : regions_) {
            need = (need + 255) / 256 * 256 + (r.begin & 255);
            r.offset = need;
            need += r.end - r.begin;
        }
        if (need > d_.arena_bytes) {
            if (d_.arena) {
                check(cudaStreamSynchronize(d_.stream), "cudaStreamSynchronize");
                check(cudaFree(d_.arena), "cudaFree (arena)");
            }
            d_.arena_bytes = std::max(need, d_.arena_bytes * 2);
            check(cudaMalloc(&d_.arena, d_.arena_bytes), "cudaMalloc (arena)");
        }
        for (const Region& r : regions_)
            check(cudaMemcpyAsync(d_.arena + r.offset, reinterpret_cast<const void*>(r.begin), r.end - r.begin,
                                  cudaMemcpyHostToDevice, d_.stream),
                  "cudaMemcpyAsync (staging)");
        for (Item* it : host) {
            const Region& r = region_of(it->begin);
            it->device = d_.arena + r.offset + (it->begin - r.begin);
        }
    }

    void* device(const ggml_tensor* t) const {
        for (const Item& it : items_)
            if (it.t == t) return it.device;
        return nullptr;
    }
    void* device_data(const void* host_ptr) const {
        for (const Item& it : items_)
            if (it.t->data == host_ptr) return it.device;
        return nullptr;
    }

    // Copies back what the node wrote to host memory, waits for the stream and
    // forgets whatever the store may have packed from the arena.
    void finish() {
        for (const Item& it : items_) {
            if (!it.write || on_device(it.t->data)) continue;
            check(cudaMemcpyAsync(it.t->data, it.device, it.end - it.begin, cudaMemcpyDeviceToHost, d_.stream),
                  "cudaMemcpyAsync (result)");
        }
        check(cudaStreamSynchronize(d_.stream), "cudaStreamSynchronize");
        if (!regions_.empty()) sdb_forget(d_.arena, d_.arena_bytes);
    }

private:
    struct Item {
        const ggml_tensor* t;
        uintptr_t begin, end;
        bool weight, write;
        void* device = nullptr;
    };
    struct Region {
        uintptr_t begin, end;
        size_t offset;
    };
    const Region& region_of(uintptr_t p) const {
        for (const Region& r : regions_)
            if (p >= r.begin && p < r.end) return r;
        die("staging: no region holds a tensor");
    }
    void add(const ggml_tensor* t, bool weight, bool write) {
        if (t == nullptr || t->data == nullptr) return;
        for (Item& it : items_)
            if (it.t == t) {
                it.write = it.write || write;
                return;
            }
        const auto b = reinterpret_cast<uintptr_t>(t->data);
        items_.push_back({t, b, b + ggml_nbytes(t), weight, write});
    }

    DeviceState& d_;
    std::vector<Item> items_;
    std::vector<Region> regions_;
};

// ---------------------------------------------------------------- computing

sdb_chain device_chain(const Chain& c, const Staging& s) {
    sdb_chain out{};
    out.count = c.count;
    for (int i = 0; i < c.count; ++i) {
        out.steps[i].kind = c.steps[i].kind;
        out.steps[i].operand = c.steps[i].operand ? static_cast<const float*>(s.device(c.steps[i].operand)) : nullptr;
        for (int k = 0; k < 4; ++k) out.steps[i].nb[k] = c.steps[i].nb[k];
    }
    out.redirect = c.redirect ? static_cast<float*>(s.device(c.redirect)) : nullptr;
    out.from_redirect = c.from_redirect ? 1 : 0;
    return out;
}

void compute(const ggml_tensor* node, Op op, const Chain& c) {
    std::lock_guard<std::mutex> guard(g_mutex);
    DeviceState& d = device_state();
    Staging s(d);
    const ggml_tensor* a = node->src[0];
    const ggml_tensor* b = node->src[1];
    switch (op) {
    case Op::conv2d:
    case Op::mul_mat:
        s.weight(a);
        s.read(b);
        break;
    case Op::attention:
        s.read(a);
        s.read(b);
        s.read(node->src[2]);
        break;
    case Op::group_norm:
    case Op::norm:
        s.read(a);
        break;
    case Op::none:
        return;
    }
    for (int i = 0; i < c.count; ++i) s.read(c.steps[i].operand);
    if (c.gated_out) s.write(c.gated_out);
    else if (c.redirect) s.write(c.redirect);
    else s.write(node);
    s.stage();

    const sdb_chain ch = device_chain(c, s);
    const sdb_chain* chp = c.empty() ? nullptr : &ch;
    const sdb_tensor y = describe(node, c.gated_out || c.redirect ? s.device(c.redirect ? c.redirect : c.gated_out)
                                                                  : s.device(node));
    int rc = SDB_OK;
    switch (op) {
    case Op::conv2d: {
        const sdb_tensor w = describe(a, s.device(a)), x = describe(b, s.device(b));
        rc = sdb_conv2d(&w, &x, &y, node->op_params, chp, d.stream);
        break;
    }
    case Op::mul_mat: {
        const sdb_tensor w = describe(a, s.device(a)), x = describe(b, s.device(b));
        if (c.gated_out) {
            const sdb_tensor out = describe(c.gated_out, s.device(c.gated_out));
            rc = sdb_mul_mat_gated(&w, &x, &out, chp, d.stream);
        } else {
            rc = sdb_mul_mat(&w, &x, &y, chp, d.stream);
        }
        break;
    }
    case Op::attention: {
        const ggml_tensor* v = node->src[2];
        const sdb_tensor q = describe(a, s.device(a)), k = describe(b, s.device(b)), vv = describe(v, s.device(v));
        rc = sdb_attention(&q, &k, &vv, &y, param_f32(node, 0), nullptr, d.stream);
        break;
    }
    case Op::group_norm: {
        const sdb_tensor x = describe(a, s.device(a));
        rc = sdb_group_norm(&x, &y, node->op_params[0], param_f32(node, 1), chp, d.stream);
        break;
    }
    case Op::norm: {
        const sdb_tensor x = describe(a, s.device(a));
        rc = sdb_norm(&x, &y, param_f32(node, 0), chp, d.stream);
        break;
    }
    case Op::none:
        break;
    }
    if (rc != SDB_OK) die(std::string("a taken node failed: ") + sdb_last_error());
    s.finish();
    const unsigned status = sdb_device_status(0);
    if (status != 0) die("the device error word is set: " + std::to_string(status));
}

void forget_written(const ggml_tensor* t) {
    if (t != nullptr && t->data != nullptr) sdasm_forget(t->data, ggml_nbytes(t));
}

// ---------------------------------------------------------------- profile

struct ProfileEntry {
    uint64_t count = 0, nanoseconds = 0, fused = 0;
};

struct Profile {
    std::mutex mutex;
    std::map<std::string, ProfileEntry> nodes;
    std::map<int, ProfileEntry> graphs;
};

Profile& profile() {
    static Profile* p = [] {
        auto* q = new Profile;
        std::atexit([] {
            Profile& pr = profile();
            const char* where = std::getenv("SDASM_PROFILE");
            FILE* f = stderr;
            if (where && std::strcmp(where, "1") != 0) f = std::fopen(where, "w");
            if (f == nullptr) f = stderr;
            std::lock_guard<std::mutex> guard(pr.mutex);
            std::fprintf(f, "sdasm profile (B200): graph nodes, runs, total ms\n");
            for (const auto& [n, e] : pr.graphs)
                std::fprintf(f, "graph %d nodes\t%" PRIu64 "\t%.3f\n", n, e.count, e.nanoseconds * 1e-6);
            std::fprintf(f, "node (op shape)\truns\tfused nodes\ttotal ms\n");
            for (const auto& [k, e] : pr.nodes)
                std::fprintf(f, "%s\t%" PRIu64 "\t%" PRIu64 "\t%.3f\n", k.c_str(), e.count, e.fused,
                             e.nanoseconds * 1e-6);
            if (f != stderr) std::fclose(f);
        });
        return q;
    }();
    return *p;
}

}  // namespace
}  // namespace hooks
}  // namespace sdb

using namespace sdb::hooks;

extern "C" {

bool sdasm_compute_forward(const ggml_compute_params* const params, const ggml_tensor* const node) {
    if (params == nullptr || params->use_ref || node == nullptr) return false;
    const Op op = taken(node);
    if (op == Op::none) return false;
    if (params->ith == 0) compute(node, op, Chain{});
    return true;
}

int sdasm_compute_nodes(const ggml_compute_params* const params, ggml_tensor* const* const nodes, int n_nodes,
                        int index) {
    if (params == nullptr || params->use_ref || nodes == nullptr || n_nodes <= 0 || index < 0 || index >= n_nodes)
        return 0;
    const ggml_tensor* node = nodes[index];
    // What the node writes was packed from nothing that is kept any more.
    if (params->ith == 0) forget_written(node);
    const Op op = taken(node);
    if (op == Op::none) return 0;
    const Chain c = chain_of(nodes, n_nodes, index, op);
    if (params->ith == 0) {
        forget_written(c.redirect);
        forget_written(c.gated_out);
        compute(node, op, c);
    }
    return node_count(c, index);
}

bool sdasm_work_size(const ggml_tensor* const node, int n_threads, size_t* const size) {
    (void)n_threads;
    if (taken(node) == Op::none) return false;
    // The kernels' workspace is device memory of their own.
    *size = 0;
    return true;
}

void sdasm_forget(const void* const begin, size_t size) {
    if (begin == nullptr || size == 0) return;
    {
        std::lock_guard<std::mutex> guard(g_mutex);
        drop_mirrors(begin, size);
    }
    sdb_forget(begin, size);
}

int sdasm_token_downsampling(int64_t width, int64_t height) { return sdb_token_downsampling(width, height); }

bool sdasm_profile_enabled(void) {
    static const bool on = [] {
        const char* s = std::getenv("SDASM_PROFILE");
        return s != nullptr && *s != '\0' && std::strcmp(s, "0") != 0;
    }();
    return on;
}

uint64_t sdasm_profile_now(void) {
    timespec ts{};
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return static_cast<uint64_t>(ts.tv_sec) * 1000000000ull + static_cast<uint64_t>(ts.tv_nsec);
}

void sdasm_profile_node(int n_nodes, const ggml_tensor* const node, int fused, uint64_t nanoseconds) {
    (void)n_nodes;
    if (!sdasm_profile_enabled() || node == nullptr) return;
    char key[160];
    std::snprintf(key, sizeof key, "op %d [%" PRId64 " %" PRId64 " %" PRId64 " %" PRId64 "]%s",
                  static_cast<int>(node->op), node->ne[0], node->ne[1], node->ne[2], node->ne[3],
                  taken(node) != Op::none ? " taken" : "");
    Profile& p = profile();
    std::lock_guard<std::mutex> guard(p.mutex);
    ProfileEntry& e = p.nodes[key];
    e.count += 1;
    e.fused += fused > 0 ? static_cast<uint64_t>(fused) : 0;
    e.nanoseconds += nanoseconds;
}

void sdasm_profile_graph(ggml_tensor* const* const nodes, int n_nodes, uint64_t nanoseconds) {
    (void)nodes;
    if (!sdasm_profile_enabled()) return;
    Profile& p = profile();
    std::lock_guard<std::mutex> guard(p.mutex);
    ProfileEntry& e = p.graphs[n_nodes];
    e.count += 1;
    e.nanoseconds += nanoseconds;
}

}  // extern "C"
