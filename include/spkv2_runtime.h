/*
 * SPINNV2 runtime C API, implemented by the B200 CUDA target
 * (libspkv2_runtime.so built from spinnv2_b200/csrc).
 *
 * Every entry point keeps the name, signature, argument meaning and return
 * codes of the reference runtime's public API so that spkv2_run/spkv2_bench,
 * generated C and ctypes drivers link unchanged:
 *   reference runtime/include/spkv2_runtime.h:14-70
 *   (implementations: runtime/core/loader.c, runtime/core/executor.c,
 *    runtime/kernels/reference/kernels.c:18-59).
 *
 * CUDA-target semantics layered on top of the same contract:
 *   - spkv2_prepare* allocates ONE device activation arena and ONE device
 *     scratch arena sized from the SPK header and places every tensor at its
 *     memory-plan offset inside them.  A caller-supplied arena/scratch that is
 *     device memory is used as the arena itself; a host arena is only
 *     size-checked (it is the staging buffer of generated C).
 *   - bind_input/bind_output accept host pointers (staged: H2D at the start of
 *     spkv2_run, D2H at its end) or device pointers (used in place).
 *   - spkv2_run launches every node on the context's CUDA stream and
 *     synchronises before returning, so wall-clock timing stays meaningful.
 *   - Kernels registered with spkv2_register_kernel receive a context whose
 *     tensor data are DEVICE pointers; they launch on spkv2_cuda_stream(ctx).
 *   - There is no CPU fallback: a node with no CUDA kernel fails with -99.
 *
 * Return codes: 0 ok; the reference's negative codes keep their meaning
 * (-1 bad argument/allocation, -2 size/magic/version, -3 bounds, -4 missing
 * section or offset beyond arena, -5 checksum section missing or unbound
 * tensor at run, -6 checksum mismatch, -10 attribute bounds, -11 rank/axis,
 * -12 group, -13 missing scratch, -14 scratch overflow, -20..-26 fault and
 * protection, -99 no kernel).  CUDA-target codes are listed in spkv2_cuda.h.
 */
#ifndef SPKV2_RUNTIME_H
#define SPKV2_RUNTIME_H

#include <stddef.h>
#include <stdint.h>
#include "spkv2_format.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Exported from libspkv2_runtime.so even when built with hidden visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct Spkv2Context Spkv2Context;

/* Single-bit fault event (reference spkv2_runtime.h:14-22). */
typedef struct {
    uint32_t node_id;
    uint32_t tensor_id;
    uint64_t element_index;
    uint8_t bit_index;
    uint32_t invocation_index;
    uint64_t seed;
    int enabled;
} Spkv2FaultEvent;

typedef struct {
    uint64_t injected_faults;
    uint64_t detected_faults;
    uint64_t recovered_faults;
    uint64_t unrecovered_faults;
    uint64_t rerun_count;
} Spkv2ReliabilityStats;

typedef struct {
    uint32_t node_id;
    uint32_t tensor_id;
    float observed_min;
    float observed_max;
    uint64_t observations;
} Spkv2RangeObservation;

/* Kernel plug-in ABI (reference spkv2_runtime.h:40). */
typedef int (*Spkv2NodeKernelFn)(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch);

const char *spkv2_runtime_version(void);

/* reference runtime/core/loader.c:105-282 */
int spkv2_load_file(const char *path, Spkv2Context **out_ctx);
int spkv2_load_memory(const void *data, size_t size, Spkv2Context **out_ctx);
/* reference runtime/core/executor.c:189-247 */
int spkv2_prepare(Spkv2Context *ctx, void *arena, size_t arena_size);
int spkv2_prepare_with_scratch(
    Spkv2Context *ctx,
    void *arena,
    size_t arena_size,
    void *scratch,
    size_t scratch_size);
/* reference runtime/core/executor.c:249-333 */
int spkv2_set_input(Spkv2Context *ctx, int index, const void *data, size_t size);
int spkv2_bind_input(Spkv2Context *ctx, int index, void *data, size_t size);
int spkv2_bind_output(Spkv2Context *ctx, int index, void *data, size_t size);
int spkv2_get_output_size(Spkv2Context *ctx, int index, size_t *out_size);
int spkv2_get_output(Spkv2Context *ctx, int index, void *data, size_t size);
/* reference runtime/core/executor.c:500-536 */
int spkv2_run(Spkv2Context *ctx);
/* reference runtime/core/executor.c:335-398 */
int spkv2_set_fault_event(Spkv2Context *ctx, const Spkv2FaultEvent *event);
void spkv2_clear_fault_event(Spkv2Context *ctx);
int spkv2_get_reliability_stats(Spkv2Context *ctx, Spkv2ReliabilityStats *stats);
void spkv2_reset_reliability_stats(Spkv2Context *ctx);
int spkv2_get_range_observation(Spkv2Context *ctx, uint32_t node_id, Spkv2RangeObservation *observation);
void spkv2_reset_range_observations(Spkv2Context *ctx);
/* reference runtime/core/executor.c:107-183,539-541 */
void spkv2_profile_dump(void);
/* reference runtime/core/loader.c:284-305 */
void spkv2_free(Spkv2Context *ctx);

/* reference runtime/kernels/reference/kernels.c:18-30,57-59 */
int spkv2_register_kernel(uint16_t op_type, uint16_t backend, uint16_t kernel_kind,
                          Spkv2NodeKernelFn fn, int priority);
void spkv2_clear_user_kernels(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* SPKV2_RUNTIME_H */
