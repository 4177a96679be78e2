// Internal state of one SPK model bound to one B200.
//
// Mirrors the role of the reference runtime's Spkv2Context
// (runtime/core/context.h:15-59): the mapped package tables, per-tensor
// state, arena/scratch, a per-node cache for prepared kernels and the
// reliability bookkeeping.  The CUDA target adds the device, the stream, the
// device copies of arena/scratch/weights, the physical layout of each tensor
// and the captured CUDA graph.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "spkv2_cuda.h"
#include "spkv2_format.h"
#include "spkv2_runtime.h"

namespace spkv2 {

enum Layout : uint8_t { kRowMajor = SPKV2_CUDA_LAYOUT_ROWMAJOR, kNHWC = SPKV2_CUDA_LAYOUT_NHWC };

struct TensorState {
  const Spkv2TensorRecord *record = nullptr;
  uint8_t *data = nullptr;        // device address of the tensor's storage
  Layout layout = kRowMajor;      // physical layout of `data`
  uint8_t *default_data = nullptr;  // storage assigned at prepare
  uint8_t *owned_storage = nullptr; // private device buffer of an EXTERNAL tensor
  void *host_binding = nullptr;     // host pointer staged in/out around a run
  bool external_device = false;     // bound to caller device memory
  bool bound = false;               // EXTERNAL tensor has been bound/set
};

// Per-node prepared kernel state lives in ctx->node_cache[node_id]; every
// built-in kernel keeps a NodePlan there.  `variant` names the device kernel.
struct NodePlan {
  virtual ~NodePlan() {}
  std::string variant;
  int launches = 1;  // kernel launches per execution of the node
};

}  // namespace spkv2

struct Spkv2Context {
  // ---- package (reference context.h:15-37) ----
  uint8_t *owned_model = nullptr;
  size_t owned_model_size = 0;
  const uint8_t *model_data = nullptr;
  size_t model_size = 0;
  Spkv2Header header{};
  const Spkv2SectionEntry *sections = nullptr;
  const Spkv2TensorRecord *tensor_records = nullptr;
  const Spkv2NodeRecord *node_records = nullptr;
  const Spkv2MemoryPlanRecord *memory_plan_records = nullptr;
  size_t memory_plan_count = 0;
  const Spkv2KernelSpecRecord *kernel_spec_records = nullptr;
  size_t kernel_spec_count = 0;
  const Spkv2ProtectionRecord *protection_records = nullptr;
  size_t protection_count = 0;
  const uint8_t *attrs = nullptr;
  size_t attrs_size = 0;
  const uint8_t *weights = nullptr;  // host copy inside the package
  size_t weights_size = 0;
  const Spkv2QuantParamRecord *quant_param_records = nullptr;
  size_t quant_param_count = 0;
  const uint8_t *quant_data = nullptr;
  size_t quant_data_size = 0;
  std::vector<uint32_t> output_ids;

  // ---- tensors ----
  std::vector<spkv2::TensorState> tensors;

  // ---- device ----
  int device = -1;  // -1: current device at prepare
  bool prepared = false;
  cudaStream_t stream = nullptr;
  uint8_t *d_arena = nullptr;
  bool owns_arena = false;
  size_t arena_size = 0;
  uint8_t *d_scratch = nullptr;
  bool owns_scratch = false;
  size_t scratch_size = 0;
  uint8_t *d_weights = nullptr;
  int math_mode = SPKV2_CUDA_MATH_SPEC;
  int graph_mode = 1;
  int *d_status = nullptr;  // device-side status word written by bounded waits
  // Stream-K workspace shared by the tcgen05 convs (grown at prepare; they
  // run in stream order) and the arrival counters of each plan that uses it.
  float *d_sk_ws = nullptr;
  size_t sk_ws_bytes = 0;
  std::vector<std::pair<void *, size_t>> sk_counters;
  int last_device_code = 0; // code of the last bounded wait that gave up

  // ---- per-node cache (reference context.h:46-48) ----
  std::vector<void *> node_cache;
  std::vector<void (*)(void *)> node_cache_dtors;

  // ---- graph replay ----
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  bool graph_dirty = true;   // bindings changed since the last capture
  bool validated = false;    // an eager run succeeded since graph_dirty was set
  uint64_t run_count = 0;

  // ---- reliability (reference context.h:55-58) ----
  Spkv2FaultEvent fault_event{};
  Spkv2ReliabilityStats reliability_stats{};
  std::vector<Spkv2RangeObservation> range_observations;
  std::vector<uint32_t> node_invocation_counts;
  // Protection plan: record index per node (-1: none; the first record
  // naming the node, as the reference's linear lookup), whether any record
  // is active (runs then go node by node, eagerly), and a small device
  // buffer for the range-scan / compare results.
  std::vector<int32_t> protection_of_node;
  bool protected_run = false;
  uint32_t *d_guard = nullptr;
};

namespace spkv2 {

// ---- shared helpers (runtime/*.cpp) ----
int execute_node(Spkv2Context *ctx, const Spkv2NodeRecord *node);
int prepare_node(Spkv2Context *ctx, const Spkv2NodeRecord *node);
int get_attr(const Spkv2Context *ctx, const Spkv2NodeRecord *node, Spkv2AttrRecord *attr);
const Spkv2KernelSpecRecord *spec_for_node(const Spkv2Context *ctx, const Spkv2NodeRecord *node);
const Spkv2QuantParamRecord *find_quant_param(const Spkv2Context *ctx, uint32_t tensor_id);
const float *quant_scales(const Spkv2Context *ctx, const Spkv2QuantParamRecord *qp);
int assign_layouts(Spkv2Context *ctx);
int cuda_status(cudaError_t err);
size_t elem_count(const Spkv2TensorRecord *r);
size_t dtype_size(uint16_t dtype);
void *device_alloc(size_t bytes);
void device_free(void *ptr);

template <class T>
T *node_plan(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  if (node->id >= ctx->node_cache.size()) return nullptr;
  return static_cast<T *>(static_cast<NodePlan *>(ctx->node_cache[node->id]));
}

void set_node_plan(Spkv2Context *ctx, const Spkv2NodeRecord *node, NodePlan *plan);

}  // namespace spkv2
