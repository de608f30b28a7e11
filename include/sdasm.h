/*
 * sdasm.h -- the hook surface that ggml's patched CPU backend calls, exported
 * by libsdb.so with the reference's signatures (sources/sdasm.h:38-78), so
 * that a ggml built with the reference's patches (patches/ggml/0001, 0003,
 * 0004) links against this library in place of the reference's and
 * stable-diffusion.cpp runs unchanged on top of it.
 *
 * The definitions (stable-diffusion.assembly_b200/csrc/hooks.cu) decide per
 * node whether it is taken, match the chain of element-wise nodes after it,
 * and hand it to the sdb_* entry points of sdb.h on a CUDA device.  ggml's
 * tensors may lie in device (or managed) memory, which the kernels read in
 * place, or in host memory, the stock CPU backend's buffers: those are staged
 * through device memory per node, and the weights among them are mirrored on
 * the device until sdasm_forget() names their memory.
 *
 * Threading, as the reference's: every thread of ggml's pool calls each hook
 * for every node and gets the same answer; thread params->ith == 0 does the
 * GPU work and waits for it before it returns (ggml's loop meets at a barrier
 * after every node).
 */
#ifndef SDB_SDASM_H
#define SDB_SDASM_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_compute_params;
struct ggml_tensor;

/* Computes <node> alone and returns true, or returns false when it is not taken
 * (ggml then computes it).  Replaces sdasm_compute_forward (sdasm.h:38,
 * hooks.cc:93-98). */
bool sdasm_compute_forward(const struct ggml_compute_params *const params, const struct ggml_tensor *const node);

/* Computes node <index> of the graph nodes[0 .. n_nodes - 1] with the chain of
 * nodes after it that change its output in place (bias, scale, SiLU, a residual
 * addition, the gated GELU of a GEGLU), and returns how many nodes that was; 0
 * when the node is not taken or the arguments name no node.  Replaces
 * sdasm_compute_nodes (sdasm.h:48-49, hooks.cc:100-164). */
int sdasm_compute_nodes(const struct ggml_compute_params *const params, struct ggml_tensor *const *const nodes,
                        int n_nodes, int index);

/* Sets *size to the bytes of ggml's work buffer a taken node needs (none: the
 * kernels keep their own device workspace) and returns true; false when the
 * node is not taken.  Replaces sdasm_work_size (sdasm.h:54, hooks.cc:174-196). */
bool sdasm_work_size(const struct ggml_tensor *const node, int n_threads, size_t *const size);

/* Drops what was kept from memory in [begin, begin + size): packed weights in
 * the device store, and device mirrors of host weights.  ggml calls it before
 * it writes a tensor's data or clears or frees a buffer (patch 0004).  Replaces
 * sdasm_forget (sdasm.h:59, store.cc:264-266). */
void sdasm_forget(const void *const begin, size_t size);

/* ToDo's K/V downsampling factor for an image's token grid of <width> by
 * <height>: 1 unless the tuning's todo asks for it and the grid has todo_tokens
 * tokens or more.  Replaces sdasm_token_downsampling (sdasm.h:67,
 * hooks.cc:166-172). */
int sdasm_token_downsampling(int64_t width, int64_t height);

/* The profile of the graphs, when SDASM_PROFILE is set in the environment:
 * ggml's patched loop (patch 0002) times each node and each graph with
 * sdasm_profile_now() and hands the nanoseconds over; the totals per operation
 * and shape are written to stderr (or to the file SDASM_PROFILE names, when it
 * is not "1") when the process exits.  Replace sdasm_profile_* (sdasm.h:75-78). */
bool sdasm_profile_enabled(void);
uint64_t sdasm_profile_now(void);
void sdasm_profile_node(int n_nodes, const struct ggml_tensor *const node, int fused, uint64_t nanoseconds);
void sdasm_profile_graph(struct ggml_tensor *const *const nodes, int n_nodes, uint64_t nanoseconds);

#ifdef __cplusplus
}
#endif

#endif
