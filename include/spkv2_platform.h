/*
 * Platform layer of the B200 CUDA target.
 *
 * Host allocation and the CPU tuning knobs keep the reference's names and
 * signatures (reference runtime/include/spkv2_platform.h:10-61) so callers that
 * set them still link; on the CUDA target the GEMM tiling, thread-count,
 * parallel-threshold and core-affinity knobs are recorded and reported back
 * but do not steer any kernel (tiling is chosen per conv on the device).
 *
 * Added for the device: a replaceable device allocator.  Every device buffer
 * the runtime owns (arenas, uploaded weights, packed weight panels) goes
 * through spkv2_platform_device_malloc/free, so an embedding framework can
 * hand the runtime its own pool, and tests can simulate allocation failure.
 */
#ifndef SPKV2_PLATFORM_H
#define SPKV2_PLATFORM_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported from libspkv2_runtime.so even when built with hidden visibility. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

void *spkv2_platform_malloc(size_t size);
void *spkv2_platform_calloc(size_t count, size_t size);
void spkv2_platform_free(void *ptr);

void spkv2_set_num_threads(int n);
int  spkv2_get_num_threads(void);

void spkv2_set_gemm_tiling(int kc, int nc);
int  spkv2_get_gemm_kc(void);
int  spkv2_get_gemm_nc(void);
void spkv2_auto_tune_gemm(int l1_bytes, int l2_bytes);

void spkv2_set_parallel_cost_threshold(int threshold_ns);
int  spkv2_get_parallel_cost_threshold(void);
int  spkv2_should_parallelize(int count, int cost_per_unit_ns);

#define SPKV2_CORES_ALL    0
#define SPKV2_CORES_BIG    1
#define SPKV2_CORES_LITTLE 2

typedef struct {
    int num_big;
    int num_little;
    int big_core_ids[16];
    int little_core_ids[16];
    int detected;
} Spkv2CoreTopology;

void spkv2_detect_topology(void);
const Spkv2CoreTopology *spkv2_get_topology(void);
void spkv2_set_affinity(int core_type);

/* ---- device memory (CUDA target) ---- */

/* Allocate / free device memory on the CURRENT CUDA device.  Returns NULL on
 * failure.  Default implementation: cudaMalloc / cudaFree. */
void *spkv2_platform_device_malloc(size_t size);
void spkv2_platform_device_free(void *ptr);

typedef void *(*Spkv2DeviceMallocFn)(size_t size, void *user);
typedef void (*Spkv2DeviceFreeFn)(void *ptr, void *user);

/* Replace the device allocator for all contexts prepared afterwards.  Passing
 * NULL for both restores cudaMalloc/cudaFree.  Returns -1 if exactly one of
 * the two functions is NULL. */
int spkv2_platform_set_device_allocator(Spkv2DeviceMallocFn alloc_fn,
                                        Spkv2DeviceFreeFn free_fn,
                                        void *user);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* SPKV2_PLATFORM_H */
