/*
 * ggml_mirror.h -- the parts of ggml's public types that the sdasm.h hook
 * layer reads, for building and testing that layer where ggml's own headers
 * are not present.
 *
 * The hook layer (stable-diffusion.assembly_b200/csrc/hooks.cu) is written
 * against ggml's field and function names.  Built inside ggml's CPU backend,
 * as the reference's hooks.cc is, it is compiled with -DSDB_WITH_GGML and
 * includes ggml.h and ggml-cpu-impl.h instead of this file, so the layout and
 * the numbering of ggml's enums are that build's own.  This mirror keeps:
 *   - struct ggml_tensor's fields in ggml's order (ggml.h: type, buffer,
 *     ne[4], nb[4], op, op_params[16], flags, src[10], view_src, view_offs,
 *     data, name[64], extra, padding[8]);
 *   - struct ggml_compute_params (ggml-cpu-impl.h: ith, nth, wsize, wdata,
 *     threadpool, use_ref);
 *   - ggml's type numbers for F32 and F16 (0 and 1) and its tensor flags;
 *   - the operations the hook layer tells apart, numbered here in an order of
 *     this file's own (SDB_GGML_OPS below; tests read the numbers from it);
 *   - the few helpers of ggml the layer calls (ggml_nbytes, ggml_is_contiguous,
 *     ggml_are_same_shape, ggml_op_is_empty, ggml_get_unary_op,
 *     ggml_type_size), with ggml's meaning, written here for the mirror.
 */
#ifndef SDB_GGML_MIRROR_H
#define SDB_GGML_MIRROR_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#define GGML_MAX_DIMS 4
#define GGML_MAX_OP_PARAMS 64
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1 };

/* The operations: X(name) in this file's order. */
#define SDB_GGML_OPS(X) \
    X(NONE) X(DUP) X(ADD) X(MUL) X(CONT) X(RESHAPE) X(VIEW) X(PERMUTE) X(TRANSPOSE) X(CPY) \
    X(MUL_MAT) X(CONV_2D) X(FLASH_ATTN_EXT) X(GROUP_NORM) X(NORM) X(UNARY) X(SCALE) X(SOFT_MAX)

enum ggml_op {
#define SDB_GGML_OP_ENUM(name) GGML_OP_##name,
    SDB_GGML_OPS(SDB_GGML_OP_ENUM)
#undef SDB_GGML_OP_ENUM
    GGML_OP_COUNT
};

enum ggml_unary_op { GGML_UNARY_OP_SILU = 0, GGML_UNARY_OP_GELU = 1 };

enum ggml_tensor_flag {
    GGML_TENSOR_FLAG_INPUT = 1,
    GGML_TENSOR_FLAG_OUTPUT = 2,
    GGML_TENSOR_FLAG_PARAM = 4,
    GGML_TENSOR_FLAG_LOSS = 8,
    GGML_TENSOR_FLAG_COMPUTE = 16
};

struct ggml_backend_buffer;
struct ggml_threadpool;

struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer *buffer;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    enum ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    struct ggml_tensor *src[GGML_MAX_SRC];
    struct ggml_tensor *view_src;
    size_t view_offs;
    void *data;
    char name[GGML_MAX_NAME];
    void *extra;
    char padding[8];
};

struct ggml_compute_params {
    int ith, nth;
    size_t wsize;
    void *wdata;
    struct ggml_threadpool *threadpool;
    bool use_ref;
};

static inline size_t ggml_type_size(enum ggml_type type) { return type == GGML_TYPE_F16 ? 2 : 4; }

/* Bytes from the first element to the end of the last (0 for an empty tensor). */
static inline size_t ggml_nbytes(const struct ggml_tensor *t) {
    size_t bytes = ggml_type_size(t->type);
    for (int k = 0; k < GGML_MAX_DIMS; ++k) {
        if (t->ne[k] <= 0) return 0;
        bytes += (size_t)(t->ne[k] - 1) * t->nb[k];
    }
    return bytes;
}

/* Elements one after another in memory: dimensions of extent 1 may have any stride. */
static inline bool ggml_is_contiguous(const struct ggml_tensor *t) {
    size_t expect = ggml_type_size(t->type);
    if (t->ne[0] != 1 && t->nb[0] != expect) return false;
    expect *= (size_t)t->ne[0];
    for (int k = 1; k < GGML_MAX_DIMS; ++k) {
        if (t->ne[k] == 1) continue;
        if (t->nb[k] != expect) return false;
        expect *= (size_t)t->ne[k];
    }
    return true;
}

static inline bool ggml_are_same_shape(const struct ggml_tensor *a, const struct ggml_tensor *b) {
    for (int k = 0; k < GGML_MAX_DIMS; ++k)
        if (a->ne[k] != b->ne[k]) return false;
    return true;
}

/* Operations that compute nothing: they only describe memory anew. */
static inline bool ggml_op_is_empty(enum ggml_op op) {
    return op == GGML_OP_NONE || op == GGML_OP_RESHAPE || op == GGML_OP_VIEW || op == GGML_OP_PERMUTE ||
           op == GGML_OP_TRANSPOSE;
}

static inline enum ggml_unary_op ggml_get_unary_op(const struct ggml_tensor *t) {
    return (enum ggml_unary_op)t->op_params[0];
}

#endif
