/*
 * CUDA-target extensions of the SPINNV2 runtime API (B200, sm_100a).
 *
 * These entry points have no counterpart in the reference runtime: they expose
 * what a device backend adds (device selection, the stream kernels launch on,
 * device tensor pointers and layouts, asynchronous runs, conv math mode) and
 * the per-tensor read/write hooks the parity tests use to check single nodes.
 * The reference API in spkv2_runtime.h is unchanged by them.
 *
 * Activation layout: rank-4 activations live on the device channels-last
 * (NHWC) unless a layout-sensitive consumer or the graph boundary needs NCHW;
 * spkv2_cuda_tensor_layout reports the choice per tensor.  Host-visible data
 * (set_input, get_output, read/write_tensor) is always in the logical NCHW /
 * row-major order of the tensor record.
 */
#ifndef SPKV2_CUDA_H
#define SPKV2_CUDA_H

#include <stddef.h>
#include <stdint.h>
#include "spkv2_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Exported from libspkv2_runtime.so even when built with hidden visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* CUDA-target error codes (never returned by the reference runtime). */
#define SPKV2_ERR_CUDA          (-40) /* a CUDA runtime call failed */
#define SPKV2_ERR_DEVICE_ALLOC  (-41) /* device allocation failed */
#define SPKV2_ERR_NO_DEVICE     (-42) /* no usable sm_100 device */
#define SPKV2_ERR_UNSUPPORTED   (-43) /* node variant has no CUDA kernel */
#define SPKV2_ERR_LAUNCH        (-44) /* kernel launch failed */
#define SPKV2_ERR_NOT_PREPARED  (-45) /* call requires spkv2_prepare first */
#define SPKV2_ERR_PROTECTION    (-46) /* reserved; protection plans run (range guard, DMR) */
#define SPKV2_ERR_DEVICE_STATUS (-47) /* a kernel reported a bounded-wait timeout or a bad index */

/* fp32 Conv/Gemm math modes. */
#define SPKV2_CUDA_MATH_SPEC   0 /* follow each node's KernelSpec kind (default) */
#define SPKV2_CUDA_MATH_3XTF32 1 /* tcgen05 3xTF32 split: near-fp32 accuracy */
#define SPKV2_CUDA_MATH_TF32   2 /* tcgen05 plain TF32 */
#define SPKV2_CUDA_MATH_FP32   3 /* CUDA-core FFMA, exact fp32 products */

/* Physical layouts reported by spkv2_cuda_tensor_layout. */
#define SPKV2_CUDA_LAYOUT_ROWMAJOR 1 /* logical order (NCHW for rank 4) */
#define SPKV2_CUDA_LAYOUT_NHWC     2

/* Bind the context to a CUDA device.  Call between load and prepare; the
 * default is the calling thread's current device at prepare time. */
int spkv2_cuda_set_device(Spkv2Context *ctx, int device);
int spkv2_cuda_get_device(Spkv2Context *ctx, int *device);

/* Select the fp32 conv/gemm math mode (SPKV2_CUDA_MATH_*); before prepare. */
int spkv2_cuda_set_math_mode(Spkv2Context *ctx, int mode);

/* Enable (1, default) or disable (0) CUDA-graph replay of the node loop. */
int spkv2_cuda_set_graph_mode(Spkv2Context *ctx, int enabled);

/* The cudaStream_t every kernel of this context launches on. */
void *spkv2_cuda_stream(Spkv2Context *ctx);

/* Device address / physical layout of a tensor after prepare. */
void *spkv2_cuda_tensor_device_ptr(Spkv2Context *ctx, uint32_t tensor_id);
int spkv2_cuda_tensor_layout(Spkv2Context *ctx, uint32_t tensor_id);

/* Launch the whole graph without the final synchronisation (and without host
 * input/output staging).  Pair with spkv2_cuda_synchronize. */
int spkv2_cuda_run_async(Spkv2Context *ctx);
int spkv2_cuda_synchronize(Spkv2Context *ctx);

/* Run nodes [first, last) eagerly and synchronise (node-level tests). */
int spkv2_cuda_run_nodes(Spkv2Context *ctx, uint32_t first, uint32_t last);

/* Run every node once eagerly with a CUDA event after each, synchronise, and
 * write each node's device time in milliseconds to node_ms[node_index]
 * (count >= number of nodes). */
int spkv2_cuda_profile_nodes(Spkv2Context *ctx, float *node_ms, uint32_t count);

/* Copy a tensor between host memory (logical order) and its device storage. */
int spkv2_cuda_read_tensor(Spkv2Context *ctx, uint32_t tensor_id, void *host, size_t size);
int spkv2_cuda_write_tensor(Spkv2Context *ctx, uint32_t tensor_id, const void *host, size_t size);

/* Number of kernel launches one spkv2_run issues (after prepare). */
int spkv2_cuda_launches_per_run(Spkv2Context *ctx, uint32_t *count);

/* Name of the device kernel variant chosen for a node (after prepare). */
const char *spkv2_cuda_node_variant(Spkv2Context *ctx, uint32_t node_id);

/* Human-readable text for a runtime return code. */
const char *spkv2_cuda_status_string(int code);

/* Bounded-wait watchdog.  Every mbarrier / flag wait in the device kernels
 * gives up after about a second, records a role code in the context's device
 * status word and lets the kernel return; the next spkv2_run /
 * spkv2_cuda_synchronize then reports SPKV2_ERR_DEVICE_STATUS and the
 * context stays usable.  spkv2_cuda_last_device_code returns the code of the
 * last such timeout (1 A-operand producer, 2 TMA producer, 3 MMA issuer,
 * 4 epilogue, 5/6 operand or residual landing, 7 accumulator hand-off,
 * 9 watchdog probe).  Gather and GatherElements use the same word for an
 * index outside [-dim, dim) after wrapping: the element is written as 0,
 * nothing outside the input is read, and the code is 10.
 * spkv2_cuda_watchdog_probe (no reference counterpart) exercises that path on
 * purpose: one block waits on an mbarrier that nothing completes, with a
 * limit of wait_us microseconds (1 .. 2,000,000); it returns
 * SPKV2_ERR_DEVICE_STATUS with *code = 9.  Nothing faults or traps. */
int spkv2_cuda_watchdog_probe(Spkv2Context *ctx, uint32_t wait_us, int *code);
int spkv2_cuda_last_device_code(Spkv2Context *ctx);

/* FNV-1a 32 over `size` bytes: the SPK package checksum (the loader checks
 * it; the Python SPK writer calls it for large packages). */
uint32_t spkv2_fnv1a32(const void *data, size_t size);

/* Allocation-free GEMV: Y[M,N] = alpha * A[M,K] * B[K,N] + bias[N], all
 * row-major fp32 device pointers (bias: NULL, or a device pointer to at
 * least N floats; a host pointer or a shorter buffer is not detected and
 * faults asynchronously or reads the wrong memory), launched asynchronously on
 * `stream` (a cudaStream_t; NULL = legacy default stream).  This entry point
 * has no counterpart in the reference runtime.  It is for callers that must
 * not allocate device memory while they run - inside a CUDA stream capture,
 * in latency-bound loops where cudaMalloc would synchronise the device, or
 * in fixed-memory deployments (profiles with allow_runtime_malloc = false).
 * Its split-K scratch is a static 1 MiB device array that every GPU loading
 * this library holds until exit; the call itself allocates nothing.
 *   - M must be 1..8 and ksplit*M*N must fit 262144 floats (ksplit shrinks
 *     to fit, down to 1); otherwise it returns -14 (scratch overflow).
 *   - The first call on each device resolves the array's device address
 *     (cudaGetSymbolAddress) with that device current: make that first call
 *     before any stream capture begins.
 *   - All calls on a device share the one scratch array and every call fully
 *     rewrites the part it reads, so nothing needs clearing between calls;
 *     calls that overlap on the GPU (different streams, no ordering) race on
 *     it and must be serialised by the caller.
 * Returns 0, -1 for bad arguments, -14 for sizes beyond the scratch, or a
 * CUDA-target error code. */
int spkv2_cuda_gemv_noalloc(const float *A, const float *B, const float *bias, float *Y,
                            int M, int K, int N, float alpha, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* SPKV2_CUDA_H */
