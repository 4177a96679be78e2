// Built-in CUDA kernels of the B200 target: prepare/run entry points that the
// registry (runtime/registry.cpp) binds to SPK op codes.  Every run function
// has the plug-in ABI  int fn(Spkv2Context*, const Spkv2NodeRecord*, void*)
// and launches asynchronously on the context's stream; prepare functions
// build the per-node plan (packed weights, tile choice) once at prepare time.
#pragma once

#include <cuda_runtime.h>

#include "../runtime/context.h"

namespace spkv2 {

typedef int (*PrepareFn)(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec);

#define SPKV2_DECLARE_OP(name)                                                                  \
  int name##_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec); \
  int name##_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch);

SPKV2_DECLARE_OP(conv)
SPKV2_DECLARE_OP(gemm)
SPKV2_DECLARE_OP(eltwise)
SPKV2_DECLARE_OP(copy)
SPKV2_DECLARE_OP(pool)
SPKV2_DECLARE_OP(resize)
SPKV2_DECLARE_OP(concat)
SPKV2_DECLARE_OP(split)
SPKV2_DECLARE_OP(transpose)
SPKV2_DECLARE_OP(tile)
SPKV2_DECLARE_OP(gather_elements)
SPKV2_DECLARE_OP(slice)
SPKV2_DECLARE_OP(gather)
SPKV2_DECLARE_OP(reduce)
SPKV2_DECLARE_OP(softmax)
SPKV2_DECLARE_OP(topk)

#undef SPKV2_DECLARE_OP

// Watchdog self-test: a block whose bounded mbarrier wait never completes
// gives up after `wait_us` and records code 9 in *d_status (watchdog.cu).
int watchdog_probe(int *d_status, uint32_t wait_us, cudaStream_t stream);

// XOR `mask` into one 32-bit word on the device (fault-event injection).
int launch_bit_flip(uint32_t *word, uint32_t mask, cudaStream_t stream);

// Protection-plan checks (protect.cu); both synchronise the stream.
struct GuardRange {
  uint64_t out_of_range = 0;  // elements non-finite or outside [lo, hi]
  bool any = false;           // some element is not NaN (min / max valid)
  bool first_nan = false;     // element 0 is NaN
  float min = 0.0f, max = 0.0f;
};
int guard_range_scan(const float *x, uint64_t n, float lo, float hi, uint32_t *d_out, GuardRange *res,
                     cudaStream_t stream);
int guard_bytes_differ(const void *a, const void *b, uint64_t bytes, uint32_t *d_out, bool *differ,
                       cudaStream_t stream);

// Copy a tensor between host memory in logical order and its device storage
// in the tensor's physical layout; synchronises the stream.
int copy_tensor_to_host(const TensorState &t, void *host, cudaStream_t stream);
int copy_tensor_from_host(const TensorState &t, const void *host, cudaStream_t stream);

}  // namespace spkv2
