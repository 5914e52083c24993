/*
 * lotus_graph.h - C ABI of the native PNNX graph runtime (one GPU per graph).
 *
 * Wraps lotus::Graph, the counterpart of the reference's lotus::Graph
 * (include/graph.hpp:15-43, source/graph.cpp): load a .pnnx.param/.pnnx.bin
 * pair for a fixed batch, take an NCHW fp32 input batch, run every layer,
 * expose the NCHW fp32 output.  All calls return 0 on success or a negative
 * LOTUS_ERR_* status with the text in lotus_last_error_string(), except
 * lotus_graph_create which returns NULL on failure.
 */
#ifndef LOTUS_GRAPH_H_
#define LOTUS_GRAPH_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#include "lotus_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lotus_graph lotus_graph;

#define LOTUS_GRAPH_NO_CUDA_GRAPH 1     /* flags: launch layers eagerly on every forward */
#define LOTUS_GRAPH_NO_RESIDUAL_FUSION 2 /* flags: keep pnnx.Expression add as its own kernel */
#define LOTUS_GRAPH_NO_S2D_STEM 4        /* flags: run a strided 3-channel stem conv directly */
#define LOTUS_GRAPH_NO_POOL_FUSION 8     /* flags: keep a max pool after a conv as its own kernel */
#define LOTUS_GRAPH_NO_CONCAT_FUSION 16  /* flags: copy torch.cat halves with a concat kernel */
#define LOTUS_GRAPH_NO_MEMORY_PLAN 32    /* flags: give every operand its own device buffer */

/* Graph(param, bin, batch) of the reference (source/graph.cpp:44-111) on
 * `device` (-1 = current). */
lotus_graph* lotus_graph_create(const char* param_path, const char* bin_path, int batch, int device, int flags);
void lotus_graph_destroy(lotus_graph* g);

/* Logical NCHW shapes of the input and output operands; *ndim <= 8. */
int lotus_graph_input_shape(const lotus_graph* g, int64_t* dims, int* ndim);
int lotus_graph_output_shape(const lotus_graph* g, int64_t* dims, int* ndim);
/* Device pointers of the fp32 input and output buffers (owned by the graph). */
float* lotus_graph_input_ptr(lotus_graph* g);
const float* lotus_graph_output_ptr(lotus_graph* g);
/* The graph's own stream. */
cudaStream_t lotus_graph_stream(const lotus_graph* g);

/* Asynchronous copies on `stream` (NULL = graph stream) from / to a host or
 * device buffer (unified addressing); `count` floats must equal the operand
 * size.  Host buffers should be pinned for the copy to be asynchronous. */
int lotus_graph_set_input(lotus_graph* g, const float* src, size_t count, cudaStream_t stream);
int lotus_graph_get_output(lotus_graph* g, float* dst, size_t count, cudaStream_t stream);

/* Enqueue one forward pass on `stream` (NULL = graph stream).  The first call
 * runs eagerly; later calls replay a captured CUDA graph unless the graph was
 * created with LOTUS_GRAPH_NO_CUDA_GRAPH. */
int lotus_graph_forward(lotus_graph* g, cudaStream_t stream);
/* Reference Graph::Forward(): forward on the graph stream and wait. */
int lotus_graph_forward_sync(lotus_graph* g);
/* Wait for all work queued on the graph stream.  Both waiting calls also read
 * (and clear) the device error word: if a kernel's bounded wait expired, its
 * output tiles were skipped, and the call returns LOTUS_ERR_CUDA naming the
 * code instead of reporting success.  Work queued with lotus_graph_forward
 * reports such an error at the next waiting call. */
int lotus_graph_synchronize(lotus_graph* g);

/* Pipelined inference from host memory (the serving path).  Enqueues, for one
 * batch: the copy of `host_in` (input-shape fp32 elements) to the device on a
 * host->device copy stream, the forward pass on the graph stream once that
 * copy has landed, and the copy of the output to `host_out` (output-shape
 * fp32 elements) on a device->host copy stream.  Two sets of device input and
 * output buffers alternate between consecutive submissions, so the input copy
 * of batch i+1 and the output copy of batch i overlap the forward of batch i.
 * Returns without waiting; both host buffers must stay valid (and should be
 * pinned, or the copies are not asynchronous) until lotus_graph_synchronize
 * returns.  The first call sets the pipeline up (allocates slot 1's buffers
 * and captures one CUDA graph per slot).  *slot (may be NULL) receives the
 * slot the batch used.  The reference has no counterpart: its
 * Graph::InitialiseInput / Forward / Output (source/graph.cpp:114-130) copy,
 * run and read back one batch at a time. */
int lotus_graph_submit(lotus_graph* g, const float* host_in, float* host_out, int* slot);
/* Copy streams of the pipelined path (which: 0 host->device, 1 device->host),
 * e.g. to bracket submissions with CUDA events. */
cudaStream_t lotus_graph_copy_stream(lotus_graph* g, int which);
/* Device output buffer of pipeline slot 0 or 1 (slot 0 is the graph's own
 * output buffer), valid on the graph stream after that slot's forward. */
float* lotus_graph_slot_output(lotus_graph* g, int slot);

/* Introspection for profiling and tests. */
int lotus_graph_layer_count(const lotus_graph* g);
const char* lotus_graph_layer_name(const lotus_graph* g, int i);
const char* lotus_graph_layer_type(const lotus_graph* g, int i);
double lotus_graph_layer_flops(const lotus_graph* g, int i);
double lotus_graph_layer_bytes(const lotus_graph* g, int i);
int lotus_graph_launches_per_forward(const lotus_graph* g);
/* Device bytes held by the graph's operands (activations, input and output;
 * weights and the split-K workspace not included).  With the memory plan,
 * operands whose lifetimes do not overlap share buffers. */
size_t lotus_graph_activation_bytes(const lotus_graph* g);
/* Device pointer, storage format (0 NCHW fp32, 1 NHWC fp16 with channel
 * stride roundup(C, 8)) and logical NCHW shape of a named operand; NULL if
 * the operand does not exist or was folded away. */
const void* lotus_graph_operand(const lotus_graph* g, const char* name, int* format, int64_t* dims, int* ndim);
/* Device pointer and size of layer i's prepacked weight (NULL if it has none). */
const void* lotus_graph_layer_weight(const lotus_graph* g, int i, size_t* bytes);
/* Mean device milliseconds per layer over `reps` eager runs into ms[layer_count]. */
int lotus_graph_profile_layers(lotus_graph* g, int reps, float* ms);

#ifdef __cplusplus
}
#endif

#endif /* LOTUS_GRAPH_H_ */
