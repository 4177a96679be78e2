// Platform layer of the CUDA target.
//
// Host allocation and the CPU tuning knobs keep the reference signatures
// (runtime/platform/platform.c:29-71,254-256); the knobs are stored and read
// back but steer nothing on the device.  Device allocation goes through a
// replaceable allocator (default cudaMalloc/cudaFree).
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include "context.h"
#include "spkv2_platform.h"

namespace {

int g_threads = 0;
int g_gemm_kc = 256;
int g_gemm_nc = 256;
int g_parallel_threshold = 50000;
Spkv2CoreTopology g_topology{};
Spkv2DeviceMallocFn g_dev_alloc = nullptr;
Spkv2DeviceFreeFn g_dev_free = nullptr;
void *g_dev_user = nullptr;

int env_int(const char *name, int fallback) {
  const char *v = getenv(name);
  return (v && *v) ? atoi(v) : fallback;
}

struct EnvInit {
  EnvInit() {
    g_threads = env_int("SPKV2_NUM_THREADS", 0);
    g_gemm_kc = env_int("SPKV2_GEMM_KC", 256);
    g_gemm_nc = env_int("SPKV2_GEMM_NC", 256);
    g_parallel_threshold = env_int("SPKV2_PARALLEL_THRESHOLD", 50000);
  }
} g_env_init;

}  // namespace

namespace spkv2 {

void *device_alloc(size_t bytes) { return spkv2_platform_device_malloc(bytes); }
void device_free(void *ptr) {
  if (ptr) spkv2_platform_device_free(ptr);
}

}  // namespace spkv2

extern "C" {

void *spkv2_platform_malloc(size_t size) { return malloc(size); }
void *spkv2_platform_calloc(size_t count, size_t size) { return calloc(count, size); }
void spkv2_platform_free(void *ptr) { free(ptr); }

void spkv2_set_num_threads(int n) { g_threads = n < 0 ? 0 : n; }
int spkv2_get_num_threads(void) { return g_threads; }

void spkv2_set_gemm_tiling(int kc, int nc) {
  if (kc > 0) g_gemm_kc = kc;
  if (nc > 0) g_gemm_nc = nc;
}
int spkv2_get_gemm_kc(void) { return g_gemm_kc; }
int spkv2_get_gemm_nc(void) { return g_gemm_nc; }
void spkv2_auto_tune_gemm(int l1_bytes, int l2_bytes) {
  (void)l1_bytes;
  (void)l2_bytes;
}

void spkv2_set_parallel_cost_threshold(int threshold_ns) { g_parallel_threshold = threshold_ns; }
int spkv2_get_parallel_cost_threshold(void) { return g_parallel_threshold; }
int spkv2_should_parallelize(int count, int cost_per_unit_ns) {
  return (long long)count * cost_per_unit_ns > g_parallel_threshold ? 1 : 0;
}

void spkv2_detect_topology(void) { g_topology.detected = 1; }
const Spkv2CoreTopology *spkv2_get_topology(void) { return &g_topology; }
void spkv2_set_affinity(int core_type) { (void)core_type; }

void *spkv2_platform_device_malloc(size_t size) {
  if (g_dev_alloc) return g_dev_alloc(size, g_dev_user);
  void *p = nullptr;
  if (cudaMalloc(&p, size) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

void spkv2_platform_device_free(void *ptr) {
  if (!ptr) return;
  if (g_dev_free) {
    g_dev_free(ptr, g_dev_user);
    return;
  }
  cudaFree(ptr);
}

int spkv2_platform_set_device_allocator(Spkv2DeviceMallocFn alloc_fn, Spkv2DeviceFreeFn free_fn, void *user) {
  if ((alloc_fn == nullptr) != (free_fn == nullptr)) return -1;
  g_dev_alloc = alloc_fn;
  g_dev_free = free_fn;
  g_dev_user = user;
  return 0;
}

}  // extern "C"
