// Host runtime: errors, the device error word, tuning, tensor-map encoding.
#include "runtime.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

namespace sdb {

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::mutex g_word_mutex;
std::unordered_map<int, unsigned*> g_words;

bool parse_int(const char* s, const char* e, int64_t& out) {
    if (s == e) return false;
    bool neg = false;
    if (*s == '-') { neg = true; ++s; }
    if (s == e) return false;
    int64_t v = 0;
    for (; s != e; ++s) {
        if (*s < '0' || *s > '9') return false;
        v = v * 10 + (*s - '0');
    }
    out = neg ? -v : v;
    return true;
}

int64_t* knob(Tuning& t, const std::string& name) {
    if (name == "fuse") return &t.fuse;
    if (name == "fuse_residual") return &t.fuse_residual;
    if (name == "winograd") return &t.winograd;
    if (name == "winograd_positions") return &t.winograd_positions;
    if (name == "winograd4_positions") return &t.winograd4_positions;
    if (name == "winograd_channels") return &t.winograd_channels;
    if (name == "winograd_small_tiles") return &t.winograd_small_tiles;
    if (name == "winograd_kc") return &t.winograd_kc;
    if (name == "winograd_small_kc") return &t.winograd_small_kc;
    if (name == "store") return &t.store;
    if (name == "todo") return &t.todo;
    if (name == "todo_tokens") return &t.todo_tokens;
    if (name == "bits") return &t.bits;
    if (name == "group") return &t.group;
    if (name == "input_bits") return &t.input_bits;
    if (name == "weight_group") return &t.weight_group;
    if (name == "quantize") return &t.quantize;
    if (name == "block_n") return &t.block_n;
    if (name == "attention_wg") return &t.attention_wg;
    if (name == "gemm_fused") return &t.gemm_fused;
    return nullptr;
}

bool valid(const std::string& name, int64_t v) {
    if (name == "winograd") return v >= 0 && v <= 2;
    if (name == "bits") return v == 0 || (v >= 2 && v <= 8);
    if (name == "input_bits") return v >= 2 && v <= 8;
    if (name == "group") return v == 32 || v == 64 || v == 128 || v == 256;
    if (name == "weight_group") return v == 0 || v == 1;
    if (name == "quantize") return v >= 0 && v <= 7;
    if (name == "block_n") return v == 0 || v == 128 || v == 160 || v == 192 || v == 256;
    if (name == "todo") return v >= 1 && v <= 4;
    if (name == "attention_wg") return v >= 0 && v <= 2;
    if (name == "gemm_fused") return v >= 0 && v <= 2;
    return v >= 0;
}

Tuning initial_tuning() {
    Tuning t;
    if (const char* env = std::getenv("SDASM_TUNE")) {
        const char* p = env;
        while (*p) {
            const char* end = std::strchr(p, ',');
            if (!end) end = p + std::strlen(p);
            const char* eq = static_cast<const char*>(std::memchr(p, '=', static_cast<size_t>(end - p)));
            if (eq) {
                const std::string name(p, eq);
                int64_t v;
                int64_t* k = knob(t, name);
                if (k && parse_int(eq + 1, end, v) && valid(name, v)) *k = v;
            }
            p = *end ? end + 1 : end;
        }
    }
    return t;
}
}  // namespace

Tuning& tuning() {
    static Tuning t = initial_tuning();
    return t;
}

void set_error(const std::string& what) { g_last_error = what; }

int fail(sdb_status status, const std::string& what) {
    set_error(what);
    return status;
}

int cuda_fail(cudaError_t e, const char* where) {
    set_error(std::string(where) + ": " + cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? SDB_OUT_OF_MEMORY : SDB_CUDA_ERROR;
}

unsigned* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_word_mutex);
    auto it = g_words.find(dev);
    if (it != g_words.end()) return it->second;
    unsigned* w = nullptr;
    if (cudaMalloc(&w, sizeof(unsigned)) != cudaSuccess) return nullptr;
    if (cudaMemset(w, 0, sizeof(unsigned)) != cudaSuccess) return nullptr;
    g_words[dev] = w;
    return w;
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

CUresult encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, void* addr,
                           const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                           CUtensorMapSwizzle swizzle, const uint32_t* element_strides) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    if (!fn) return CUDA_ERROR_NOT_FOUND;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    for (uint32_t i = 0; element_strides && i < rank && i < 5; ++i) estr[i] = element_strides[i];
    return fn(map, type, rank, addr, reinterpret_cast<const cuuint64_t*>(dims),
              reinterpret_cast<const cuuint64_t*>(strides_bytes), reinterpret_cast<const cuuint32_t*>(box), estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int current_sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace sdb

extern "C" {

int sdb_set_tuning(const char* spec) {
    if (spec == nullptr) return sdb::fail(SDB_INVALID, "sdb_set_tuning: null spec");
    sdb::Tuning t = sdb::tuning();
    const char* p = spec;
    while (*p) {
        const char* end = std::strchr(p, ',');
        if (!end) end = p + std::strlen(p);
        const char* eq = static_cast<const char*>(std::memchr(p, '=', static_cast<size_t>(end - p)));
        if (!eq) return sdb::fail(SDB_INVALID, std::string("sdb_set_tuning: no '=' in '") + std::string(p, end) + "'");
        const std::string name(p, eq);
        int64_t v;
        int64_t* k = sdb::knob(t, name);
        if (!k) return sdb::fail(SDB_INVALID, "sdb_set_tuning: unknown name '" + name + "'");
        if (!sdb::parse_int(eq + 1, end, v) || !sdb::valid(name, v))
            return sdb::fail(SDB_INVALID, "sdb_set_tuning: bad value for '" + name + "'");
        *k = v;
        p = *end ? end + 1 : end;
    }
    sdb::tuning() = t;
    return SDB_OK;
}

int sdb_get_tuning(const char* name, int64_t* value) {
    if (name == nullptr || value == nullptr) return sdb::fail(SDB_INVALID, "sdb_get_tuning: null argument");
    int64_t* k = sdb::knob(sdb::tuning(), name);
    if (!k) return sdb::fail(SDB_INVALID, std::string("sdb_get_tuning: unknown name '") + name + "'");
    *value = *k;
    return SDB_OK;
}

unsigned sdb_device_status(int clear) {
    unsigned* w = sdb::device_error_word();
    if (!w) return ~0u;
    if (cudaDeviceSynchronize() != cudaSuccess) return ~0u;
    unsigned v = 0;
    if (cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return ~0u;
    if (clear && cudaMemset(w, 0, sizeof(unsigned)) != cudaSuccess) return ~0u;
    return v;
}

const char* sdb_last_error(void) { return sdb::g_last_error.c_str(); }

uint64_t sdb_launch_count(void) { return sdb::g_launches.load(); }

int sdb_token_downsampling(int64_t width, int64_t height) {
    const sdb::Tuning& t = sdb::tuning();
    if (t.todo < 2 || width <= 0 || height <= 0 || width * height < t.todo_tokens) return 1;
    return static_cast<int>(t.todo);
}

}  // extern "C"

namespace sdb {

bool store_map(CUtensorMap* map, void* base, long long cols, long long rows, long long ld, int box_cols) {
    const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 4};
    const uint32_t box[2] = {static_cast<uint32_t>(box_cols), 32};
    return encode_tensor_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                             box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B) == CUDA_SUCCESS;
}

}  // namespace sdb
