// Prepare / bind / run for the CUDA target.
//
// Contract kept from the reference executor (runtime/core/executor.c):
//   prepare_with_scratch  :193-247  arena (-2 if too small), scratch (-2),
//                                   weight bounds (-3), arena bounds (-4)
//   set/bind input/output :249-333  size must equal the record (-2), index
//                                   past the last input/output (-3)
//   run                   :500-536  unbound tensor (-5), nodes in order
//   fault events          :335-398  single-bit flip after the node's n-th run
//   profiler              :96-183   SPKV2_PROFILE=1, same dump format
// Device specifics: one device arena + one device scratch placed from the
// memory plan, weights uploaded once, host-bound IO staged around each run,
// node loop captured into a CUDA graph from the second run on.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <vector>

#include "../kernels/kernels.h"
#include "context.h"
#include "spkv2_platform.h"

using namespace spkv2;

namespace {

// ---------------- profiler (process-global like the reference) -------------
constexpr int kProfOps = 64;
constexpr int kProfNodes = 4096;
int g_prof_enabled = -1;
double g_prof_op_ms[kProfOps];
int g_prof_op_count[kProfOps];
double g_prof_node_ms[kProfNodes];
int g_prof_node_count[kProfNodes];
int g_prof_runs = 0;
const Spkv2Context *g_prof_ctx = nullptr;

void prof_init() {
  if (g_prof_enabled >= 0) return;
  const char *v = getenv("SPKV2_PROFILE");
  g_prof_enabled = (v && v[0] && v[0] != '0') ? 1 : 0;
  memset(g_prof_op_ms, 0, sizeof(g_prof_op_ms));
  memset(g_prof_op_count, 0, sizeof(g_prof_op_count));
  memset(g_prof_node_ms, 0, sizeof(g_prof_node_ms));
  memset(g_prof_node_count, 0, sizeof(g_prof_node_count));
  g_prof_runs = 0;
}

const char *op_label(uint16_t op) {
  switch (op) {
    case SPKV2_OP_ADD: return "Add";
    case SPKV2_OP_CONV: return "Conv";
    case SPKV2_OP_MUL: return "Mul";
    case SPKV2_OP_SUB: return "Sub";
    case SPKV2_OP_DIV: return "Div";
    case SPKV2_OP_RELU: return "Relu";
    case SPKV2_OP_SIGMOID: return "Sigmoid";
    case SPKV2_OP_GEMM: return "Gemm";
    case SPKV2_OP_MATMUL: return "MatMul";
    case SPKV2_OP_CONCAT: return "Concat";
    case SPKV2_OP_SPLIT: return "Split";
    case SPKV2_OP_RESHAPE: return "Reshape";
    case SPKV2_OP_RESIZE: return "Resize";
    case SPKV2_OP_TRANSPOSE: return "Transpose";
    case SPKV2_OP_MAXPOOL: return "MaxPool";
    case SPKV2_OP_SOFTMAX: return "Softmax";
    case SPKV2_OP_TOPK: return "TopK";
    case SPKV2_OP_FLATTEN: return "Flatten";
    case SPKV2_OP_UNSQUEEZE: return "Unsqueeze";
    case SPKV2_OP_TILE: return "Tile";
    case SPKV2_OP_GATHERELEMENTS: return "GatherElements";
    case SPKV2_OP_REDUCEMAX: return "ReduceMax";
    case SPKV2_OP_REDUCEMEAN: return "ReduceMean";
    case SPKV2_OP_CAST: return "Cast";
    case SPKV2_OP_MOD: return "Mod";
    case SPKV2_OP_SLICE: return "Slice";
    case SPKV2_OP_GATHER: return "Gather";
    default: return "Unknown";
  }
}

void prof_dump_impl(const Spkv2Context *ctx) {
  fprintf(stderr, "\n[SPKV2_PROFILE] per-op totals over %d runs:\n", g_prof_runs);
  fprintf(stderr, "  %-20s %8s %12s %12s\n", "op", "count", "total_ms", "avg_ms");
  std::vector<int> ops;
  for (int i = 0; i < kProfOps; ++i)
    if (g_prof_op_count[i] > 0) ops.push_back(i);
  std::stable_sort(ops.begin(), ops.end(), [](int a, int b) { return g_prof_op_ms[a] > g_prof_op_ms[b]; });
  double total = 0;
  for (int op : ops) total += g_prof_op_ms[op];
  const int runs = g_prof_runs > 0 ? g_prof_runs : 1;
  for (int op : ops) {
    fprintf(stderr, "  %-20s %8d %12.3f %12.4f (%5.1f%%)\n", op_label(uint16_t(op)), g_prof_op_count[op] / runs,
            g_prof_op_ms[op], g_prof_op_ms[op] / std::max(1, g_prof_op_count[op]),
            total > 0 ? 100.0 * g_prof_op_ms[op] / total : 0.0);
  }
  fprintf(stderr, "  %-20s %8s %12.3f\n", "TOTAL", "", total);
  if (!ctx) return;
  fprintf(stderr, "\n[SPKV2_PROFILE] conv nodes over %d runs:\n", g_prof_runs);
  fprintf(stderr, "  %-5s %-18s %8s %10s %22s %12s %10s\n", "node", "algo", "count", "avg_ms",
          "N,C,H,W->OC,k,s,p,g", "total_ms", "scratch");
  for (uint32_t i = 0; i < ctx->header.num_nodes && i < uint32_t(kProfNodes); ++i) {
    const Spkv2NodeRecord *nd = &ctx->node_records[i];
    if (nd->op_type != SPKV2_OP_CONV || g_prof_node_count[i] == 0 || nd->input_count < 2) continue;
    const Spkv2TensorRecord *x = ctx->tensors[nd->inputs[0]].record;
    const Spkv2TensorRecord *w = ctx->tensors[nd->inputs[1]].record;
    Spkv2AttrRecord a;
    if (x->rank != 4 || w->rank != 4 || get_attr(ctx, nd, &a) != 0) continue;
    char shape[128];
    snprintf(shape, sizeof(shape), "%u,%u,%u,%u->%u,%ux%u,%dx%d,%d/%d/%d/%d,%d", x->shape[0], x->shape[1],
             x->shape[2], x->shape[3], w->shape[0], w->shape[2], w->shape[3], a.strides[0], a.strides[1],
             a.pads[0], a.pads[1], a.pads[2], a.pads[3], a.group);
    const char *variant = spkv2_cuda_node_variant(const_cast<Spkv2Context *>(ctx), nd->id);
    fprintf(stderr, "  %-5u %-18s %8d %10.4f %22s %12.3f %10u\n", nd->id, variant ? variant : "?",
            g_prof_node_count[i] / runs, g_prof_node_ms[i] / std::max(1, g_prof_node_count[i]), shape,
            g_prof_node_ms[i], nd->scratch_bytes);
  }
  fprintf(stderr, "\nnode_id,op_type,avg_ms,total_ms,count\n");
  for (uint32_t i = 0; i < ctx->header.num_nodes && i < uint32_t(kProfNodes); ++i) {
    if (g_prof_node_count[i] == 0) continue;
    const Spkv2NodeRecord *nd = &ctx->node_records[i];
    fprintf(stderr, "%u,%s,%.9f,%.9f,%d\n", nd->id, op_label(nd->op_type),
            g_prof_node_ms[i] / double(g_prof_node_count[i]), g_prof_node_ms[i], g_prof_node_count[i] / runs);
  }
  fprintf(stderr, "\n");
}

// ---------------- device helpers ----------------

bool is_device_pointer(const void *p, int device) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error of an unregistered host pointer
    return false;
  }
  return (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) && attr.device == device;
}

void release_device_state(Spkv2Context *ctx) {
  if (ctx->device >= 0) cudaSetDevice(ctx->device);
  if (ctx->graph_exec) cudaGraphExecDestroy(ctx->graph_exec);
  if (ctx->graph) cudaGraphDestroy(ctx->graph);
  ctx->graph_exec = nullptr;
  ctx->graph = nullptr;
  ctx->sk_counters.clear();  // owned by the plans released below
  for (size_t i = 0; i < ctx->node_cache.size(); ++i) {
    if (!ctx->node_cache[i]) continue;
    if (ctx->node_cache_dtors[i])
      ctx->node_cache_dtors[i](ctx->node_cache[i]);
    else
      delete static_cast<NodePlan *>(ctx->node_cache[i]);
    ctx->node_cache[i] = nullptr;
    ctx->node_cache_dtors[i] = nullptr;
  }
  for (auto &t : ctx->tensors) {
    if (t.owned_storage) device_free(t.owned_storage);
    t.owned_storage = nullptr;
  }
  if (ctx->owns_arena) device_free(ctx->d_arena);
  if (ctx->owns_scratch) device_free(ctx->d_scratch);
  device_free(ctx->d_weights);
  device_free(ctx->d_status);
  device_free(ctx->d_guard);
  ctx->d_guard = nullptr;
  device_free(ctx->d_sk_ws);
  ctx->d_sk_ws = nullptr;
  ctx->sk_ws_bytes = 0;
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  ctx->d_arena = ctx->d_scratch = ctx->d_weights = nullptr;
  ctx->d_status = nullptr;
  ctx->owns_arena = ctx->owns_scratch = false;
  ctx->stream = nullptr;
  ctx->prepared = false;
}

int input_tensor_id(const Spkv2Context *ctx, int index, uint32_t *id) {
  int seen = 0;
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    if (ctx->tensor_records[i].role != SPKV2_ROLE_INPUT) continue;
    if (seen++ == index) {
      *id = i;
      return 0;
    }
  }
  return -3;
}

int output_tensor_id(const Spkv2Context *ctx, int index, uint32_t *id) {
  if (!ctx->output_ids.empty() && size_t(index) < ctx->output_ids.size()) {
    uint32_t t = ctx->output_ids[size_t(index)];
    if (t >= ctx->header.num_tensors || ctx->tensor_records[t].role != SPKV2_ROLE_OUTPUT) return -3;
    *id = t;
    return 0;
  }
  int seen = 0;
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    if (ctx->tensor_records[i].role != SPKV2_ROLE_OUTPUT) continue;
    if (seen++ == index) {
      *id = i;
      return 0;
    }
  }
  return -3;
}

// Binds `data` as the storage of tensor `id`: a device pointer on the
// context's device replaces the device storage; anything else is a host
// staging buffer copied around each run.
int bind_tensor(Spkv2Context *ctx, uint32_t id, void *data) {
  TensorState &t = ctx->tensors[id];
  if (ctx->prepared && is_device_pointer(data, ctx->device)) {
    if (t.layout != kRowMajor) return SPKV2_ERR_UNSUPPORTED;
    t.data = static_cast<uint8_t *>(data);
    t.host_binding = nullptr;
    t.external_device = true;
    ctx->graph_dirty = true;
    ctx->validated = false;
  } else {
    if (t.external_device) {
      t.data = t.default_data;
      t.external_device = false;
      ctx->graph_dirty = true;
      ctx->validated = false;
    }
    t.host_binding = data;
  }
  t.bound = true;
  return 0;
}

int stage_inputs(Spkv2Context *ctx) {
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    TensorState &t = ctx->tensors[i];
    if (t.record->role != SPKV2_ROLE_INPUT || !t.host_binding) continue;
    int rc = cuda_status(cudaMemcpyAsync(t.data, t.host_binding, size_t(t.record->size_bytes),
                                         cudaMemcpyHostToDevice, ctx->stream));
    if (rc) return rc;
  }
  return 0;
}

int stage_outputs(Spkv2Context *ctx) {
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    TensorState &t = ctx->tensors[i];
    if (t.record->role != SPKV2_ROLE_OUTPUT || !t.host_binding) continue;
    int rc = cuda_status(cudaMemcpyAsync(t.host_binding, t.data, size_t(t.record->size_bytes),
                                         cudaMemcpyDeviceToHost, ctx->stream));
    if (rc) return rc;
  }
  return 0;
}

// Physical element offset of logical (row-major) element `e` of tensor t.
uint64_t physical_index(const TensorState &t, uint64_t e) {
  if (t.layout != kNHWC) return e;
  const uint32_t *s = t.record->shape;
  uint64_t C = s[1], H = s[2], W = s[3];
  uint64_t w = e % W, h = (e / W) % H, c = (e / (W * H)) % C, n = e / (W * H * C);
  return ((n * H + h) * W + w) * C + c;
}

// Flip one bit of an fp32 output element after the node's n-th invocation
// (reference executor.c:377-398); the flip runs as a device kernel.
int maybe_inject_fault(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  Spkv2FaultEvent &ev = ctx->fault_event;
  if (!ev.enabled || node->id != ev.node_id) return 0;
  if (node->id >= ctx->node_invocation_counts.size()) return -20;
  if (++ctx->node_invocation_counts[node->id] != ev.invocation_index) return 0;
  if (ev.tensor_id >= ctx->header.num_tensors) return -21;
  const Spkv2TensorRecord *rec = &ctx->tensor_records[ev.tensor_id];
  bool is_output = false;
  for (uint16_t i = 0; i < node->output_count; ++i) is_output |= node->outputs[i] == ev.tensor_id;
  if (!is_output || rec->dtype != SPKV2_DTYPE_FP32) return -22;
  if (ev.element_index >= rec->size_bytes / 4) return -23;
  const TensorState &t = ctx->tensors[ev.tensor_id];
  uint32_t *word = reinterpret_cast<uint32_t *>(t.data) + physical_index(t, ev.element_index);
  int rc = launch_bit_flip(word, 1u << ev.bit_index, ctx->stream);
  if (rc) return rc;
  ctx->reliability_stats.injected_faults++;
  return 0;
}

int execute_once(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  int rc = execute_node(ctx, node);
  return rc ? rc : maybe_inject_fault(ctx, node);
}

// Range scan of the protected output; records the observation when asked
// (reference record_output_range, first execution only) and returns in
// *ok whether every element is finite and inside [lower, upper] (reference
// output_in_range).
int check_range(Spkv2Context *ctx, const Spkv2ProtectionRecord &r, bool record, bool *ok) {
  const TensorState &t = ctx->tensors[r.tensor_id];
  const uint64_t n = t.record->size_bytes / sizeof(float);
  GuardRange g;
  int rc = guard_range_scan(reinterpret_cast<const float *>(t.data), n, r.lower_bound, r.upper_bound, ctx->d_guard,
                            &g, ctx->stream);
  if (rc) return rc;
  if (record && n > 0 && r.node_id < ctx->range_observations.size()) {
    // Reference semantics: min = max = element 0, then `<` / `>` updates;
    // a NaN element 0 stays NaN, later NaNs never win a comparison.
    const float mn = g.first_nan ? NAN : g.min, mx = g.first_nan ? NAN : g.max;
    Spkv2RangeObservation &o = ctx->range_observations[r.node_id];
    o.node_id = r.node_id;
    o.tensor_id = r.tensor_id;
    if (o.observations == 0) {
      o.observed_min = mn;
      o.observed_max = mx;
    } else {
      if (mn < o.observed_min) o.observed_min = mn;
      if (mx > o.observed_max) o.observed_max = mx;
    }
    o.observations++;
  }
  *ok = g.out_of_range == 0;
  return 0;
}

int device_copy(void *dst, const void *src, size_t bytes, cudaStream_t s) {
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
}

// One node under its protection record (reference core/executor.c:445-498):
// range_guard_rerun runs once, scans, and reruns once when the output is
// out of range; dmr_compare_rerun runs twice into two scratch copies and,
// when they differ, a third run votes.  Statistics as the reference.  Each
// check synchronises the stream, so protected runs go node by node.
int execute_protected(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  const int32_t idx = node->id < ctx->protection_of_node.size() ? ctx->protection_of_node[node->id] : -1;
  if (idx < 0 || ctx->protection_records[idx].mode == SPKV2_PROTECT_NONE) return execute_once(ctx, node);
  const Spkv2ProtectionRecord &r = ctx->protection_records[idx];
  if (r.tensor_id >= ctx->header.num_tensors || node->output_count != 1 || node->outputs[0] != r.tensor_id)
    return -24;
  Spkv2ReliabilityStats &st = ctx->reliability_stats;
  if (r.mode == SPKV2_PROTECT_RANGE_GUARD_RERUN) {
    int rc = execute_once(ctx, node);
    bool ok = false;
    if (rc == 0) rc = check_range(ctx, r, true, &ok);
    if (rc != 0 || ok) return rc;
    st.detected_faults++;
    st.rerun_count++;
    if ((rc = execute_once(ctx, node))) return rc;
    if ((rc = check_range(ctx, r, false, &ok))) return rc;
    if (ok)
      st.recovered_faults++;
    else
      st.unrecovered_faults++;
    return 0;
  }
  if (r.mode == SPKV2_PROTECT_DMR_COMPARE_RERUN) {
    TensorState &t = ctx->tensors[r.tensor_id];
    const size_t bytes = size_t(t.record->size_bytes);
    if (!ctx->d_scratch || r.scratch_offset > ctx->scratch_size || bytes * 2u > ctx->scratch_size - r.scratch_offset)
      return -25;
    uint8_t *first = ctx->d_scratch + r.scratch_offset;
    uint8_t *second = first + bytes;
    int rc = execute_once(ctx, node);
    if (rc == 0) rc = device_copy(first, t.data, bytes, ctx->stream);
    if (rc == 0) rc = execute_once(ctx, node);
    if (rc == 0) rc = device_copy(second, t.data, bytes, ctx->stream);
    bool differ = false;
    if (rc == 0) rc = guard_bytes_differ(first, second, bytes, ctx->d_guard, &differ, ctx->stream);
    if (rc != 0 || !differ) return rc;
    st.detected_faults++;
    st.rerun_count++;
    if ((rc = execute_once(ctx, node))) return rc;
    if ((rc = guard_bytes_differ(first, t.data, bytes, ctx->d_guard, &differ, ctx->stream))) return rc;
    if (!differ) {
      st.recovered_faults++;  // the output already holds the agreeing bytes
      return 0;
    }
    if ((rc = guard_bytes_differ(second, t.data, bytes, ctx->d_guard, &differ, ctx->stream))) return rc;
    if (!differ)
      st.recovered_faults++;
    else
      st.unrecovered_faults++;
    return 0;
  }
  return -26;
}

int run_nodes_eager(Spkv2Context *ctx, uint32_t first, uint32_t last, bool profile) {
  std::vector<cudaEvent_t> ev;
  if (profile) {
    ev.resize(size_t(last - first) + 1);
    for (auto &e : ev) cudaEventCreate(&e);
    cudaEventRecord(ev[0], ctx->stream);
  }
  int rc = 0;
  for (uint32_t i = first; i < last && rc == 0; ++i) {
    const Spkv2NodeRecord *node = &ctx->node_records[i];
    rc = ctx->protected_run ? execute_protected(ctx, node) : execute_once(ctx, node);
    if (rc == 0) rc = cuda_status(cudaGetLastError());
    if (profile) cudaEventRecord(ev[i - first + 1], ctx->stream);
  }
  if (profile) {
    cudaStreamSynchronize(ctx->stream);
    if (rc == 0) {
      for (uint32_t i = first; i < last; ++i) {
        float ms = 0;
        cudaEventElapsedTime(&ms, ev[i - first], ev[i - first + 1]);
        const Spkv2NodeRecord *nd = &ctx->node_records[i];
        if (nd->op_type < kProfOps) {
          g_prof_op_ms[nd->op_type] += ms;
          g_prof_op_count[nd->op_type]++;
        }
        if (nd->id < uint32_t(kProfNodes)) {
          g_prof_node_ms[nd->id] += ms;
          g_prof_node_count[nd->id]++;
        }
      }
      g_prof_runs++;
    }
    for (auto &e : ev) cudaEventDestroy(e);
  }
  return rc;
}

int launch_graph(Spkv2Context *ctx) {
  if (ctx->graph_dirty || !ctx->graph_exec) {
    if (ctx->graph_exec) cudaGraphExecDestroy(ctx->graph_exec);
    if (ctx->graph) cudaGraphDestroy(ctx->graph);
    ctx->graph_exec = nullptr;
    ctx->graph = nullptr;
    int rc = cuda_status(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    if (rc) return rc;
    int krc = 0;
    for (uint32_t i = 0; i < ctx->header.num_nodes && krc == 0; ++i)
      krc = execute_node(ctx, &ctx->node_records[i]);
    cudaGraph_t g = nullptr;
    cudaError_t end = cudaStreamEndCapture(ctx->stream, &g);
    if (krc) {
      if (g) cudaGraphDestroy(g);
      return krc;
    }
    if ((rc = cuda_status(end))) return rc;
    ctx->graph = g;
    if ((rc = cuda_status(cudaGraphInstantiate(&ctx->graph_exec, g, 0)))) return rc;
    ctx->graph_dirty = false;
  }
  return cuda_status(cudaGraphLaunch(ctx->graph_exec, ctx->stream));
}

// Launches all nodes on the stream.  With graph mode on, the first run after
// a (re)binding runs eagerly; the next one captures the node loop into a CUDA
// graph that later runs replay.
int launch_all(Spkv2Context *ctx) {
  prof_init();
  g_prof_ctx = ctx;
  std::fill(ctx->node_invocation_counts.begin(), ctx->node_invocation_counts.end(), 0u);
  if (g_prof_enabled || ctx->fault_event.enabled || ctx->protected_run || !ctx->graph_mode)
    return run_nodes_eager(ctx, 0, ctx->header.num_nodes, g_prof_enabled > 0);
  if (ctx->graph_dirty && !ctx->validated) {
    int rc = run_nodes_eager(ctx, 0, ctx->header.num_nodes, false);
    if (rc == 0) ctx->validated = true;
    return rc;
  }
  return launch_graph(ctx);
}

// Reads (and clears) the status word that kernels with bounded waits set on
// timeout; call after the stream has been synchronised.
int take_device_status(Spkv2Context *ctx) {
  int st = 0;
  if (!ctx->d_status) return 0;
  if (cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return SPKV2_ERR_CUDA;
  if (st != 0) {
    ctx->last_device_code = st;
    cudaMemset(ctx->d_status, 0, sizeof(int));
    // A launch that gave up mid-way may leave stream-K arrival counts behind.
    for (const auto &c : ctx->sk_counters) cudaMemset(c.first, 0, c.second);
    return SPKV2_ERR_DEVICE_STATUS;
  }
  return 0;
}

int check_runnable(Spkv2Context *ctx) {
  if (!ctx) return -1;
  if (!ctx->prepared) return -5;
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    const TensorState &t = ctx->tensors[i];
    if (t.record->role == SPKV2_ROLE_WEIGHT) continue;
    if (t.record->memory_class == SPKV2_MEMORY_EXTERNAL && !t.bound) return -5;
    if (!t.data && t.record->size_bytes > 0) return -5;
  }
  return 0;
}

}  // namespace

namespace spkv2 {

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return 0;
  if (err == cudaErrorMemoryAllocation) return SPKV2_ERR_DEVICE_ALLOC;
  if (err == cudaErrorLaunchFailure || err == cudaErrorInvalidConfiguration) return SPKV2_ERR_LAUNCH;
  return SPKV2_ERR_CUDA;
}

size_t dtype_size(uint16_t dtype) {
  switch (dtype) {
    case SPKV2_DTYPE_INT8: return 1;
    case SPKV2_DTYPE_FP16: return 2;
    default: return 4;
  }
}

size_t elem_count(const Spkv2TensorRecord *r) {
  size_t n = 1;
  for (uint16_t i = 0; i < r->rank; ++i) n *= r->shape[i];
  return n;
}

void set_node_plan(Spkv2Context *ctx, const Spkv2NodeRecord *node, NodePlan *plan) {
  if (node->id >= ctx->node_cache.size()) {
    delete plan;
    return;
  }
  if (ctx->node_cache[node->id]) delete static_cast<NodePlan *>(ctx->node_cache[node->id]);
  ctx->node_cache[node->id] = static_cast<void *>(plan);
  ctx->node_cache_dtors[node->id] = nullptr;
}

}  // namespace spkv2

extern "C" {

int spkv2_prepare(Spkv2Context *ctx, void *arena, size_t arena_size) {
  return spkv2_prepare_with_scratch(ctx, arena, arena_size, nullptr, 0);
}

int spkv2_prepare_with_scratch(Spkv2Context *ctx, void *arena, size_t arena_size, void *scratch,
                               size_t scratch_size) {
  if (!ctx) return -1;
  const uint64_t need_arena = ctx->header.activation_arena_bytes;
  const uint64_t need_scratch = ctx->header.scratch_arena_bytes;
  if (arena && arena_size < need_arena) return -2;
  if (need_scratch > 0 && scratch && scratch_size < need_scratch) return -2;
  if (ctx->prepared) release_device_state(ctx);

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return SPKV2_ERR_NO_DEVICE;
  }
  if (ctx->device < 0 && cudaGetDevice(&ctx->device) != cudaSuccess) return SPKV2_ERR_NO_DEVICE;
  if (ctx->device >= ndev) return SPKV2_ERR_NO_DEVICE;
  int rc = cuda_status(cudaSetDevice(ctx->device));
  if (rc) return rc;
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, ctx->device);
  if (major != 10) return SPKV2_ERR_NO_DEVICE;  // kernels are built for sm_100a only
  ctx->protection_of_node.assign(ctx->header.num_nodes, -1);
  ctx->protected_run = false;
  for (size_t i = 0; i < ctx->protection_count; ++i) {
    const Spkv2ProtectionRecord &r = ctx->protection_records[i];
    if (r.node_id < ctx->header.num_nodes && ctx->protection_of_node[r.node_id] < 0)
      ctx->protection_of_node[r.node_id] = int32_t(i);
    ctx->protected_run |= r.mode != SPKV2_PROTECT_NONE;
  }

  if ((rc = cuda_status(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking)))) return rc;

  // Activation arena: a device arena from the caller is used as is; a host
  // arena (generated C's static buffer) only passes the size check.
  if (arena && is_device_pointer(arena, ctx->device)) {
    ctx->d_arena = static_cast<uint8_t *>(arena);
    ctx->arena_size = arena_size;
  } else {
    ctx->arena_size = size_t(need_arena);
    ctx->d_arena = static_cast<uint8_t *>(device_alloc(std::max<size_t>(ctx->arena_size, 256)));
    ctx->owns_arena = true;
    if (!ctx->d_arena) {
      release_device_state(ctx);
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    cudaMemsetAsync(ctx->d_arena, 0, ctx->arena_size, ctx->stream);
  }
  if (need_scratch > 0) {
    if (scratch && is_device_pointer(scratch, ctx->device)) {
      ctx->d_scratch = static_cast<uint8_t *>(scratch);
      ctx->scratch_size = scratch_size;
    } else {
      ctx->scratch_size = size_t(need_scratch);
      ctx->d_scratch = static_cast<uint8_t *>(device_alloc(ctx->scratch_size));
      ctx->owns_scratch = true;
      if (!ctx->d_scratch) {
        release_device_state(ctx);
        return SPKV2_ERR_DEVICE_ALLOC;
      }
      cudaMemsetAsync(ctx->d_scratch, 0, ctx->scratch_size, ctx->stream);
    }
  }
  // Weights: one upload of the weight section.
  if (ctx->weights_size > 0) {
    ctx->d_weights = static_cast<uint8_t *>(device_alloc(ctx->weights_size));
    if (!ctx->d_weights) {
      release_device_state(ctx);
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    if ((rc = cuda_status(cudaMemcpy(ctx->d_weights, ctx->weights, ctx->weights_size, cudaMemcpyHostToDevice)))) {
      release_device_state(ctx);
      return rc;
    }
  }
  ctx->d_status = static_cast<int *>(device_alloc(sizeof(int) * 4));
  if (!ctx->d_status) {
    release_device_state(ctx);
    return SPKV2_ERR_DEVICE_ALLOC;
  }
  cudaMemsetAsync(ctx->d_status, 0, sizeof(int) * 4, ctx->stream);
  if (ctx->protected_run) {
    ctx->d_guard = static_cast<uint32_t *>(device_alloc(sizeof(uint32_t) * 8));
    if (!ctx->d_guard) {
      release_device_state(ctx);
      return SPKV2_ERR_DEVICE_ALLOC;
    }
  }

  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) {
    TensorState &t = ctx->tensors[i];
    const Spkv2TensorRecord *r = t.record;
    t.host_binding = nullptr;
    t.external_device = false;
    t.bound = false;
    if (r->role == SPKV2_ROLE_WEIGHT) {
      if (r->data_offset > ctx->weights_size || r->size_bytes > ctx->weights_size - r->data_offset) {
        release_device_state(ctx);
        return -3;
      }
      t.data = ctx->d_weights + r->data_offset;
    } else if (r->memory_class == SPKV2_MEMORY_EXTERNAL) {
      // Caller-bound tensor: private device storage backs host bindings.
      t.owned_storage = static_cast<uint8_t *>(device_alloc(std::max<size_t>(size_t(r->size_bytes), 16)));
      if (!t.owned_storage) {
        release_device_state(ctx);
        return SPKV2_ERR_DEVICE_ALLOC;
      }
      t.data = t.owned_storage;
    } else {
      if (r->data_offset + r->size_bytes > need_arena) {
        release_device_state(ctx);
        return -4;
      }
      t.data = ctx->d_arena + r->data_offset;
    }
    t.default_data = t.data;
  }
  if ((rc = assign_layouts(ctx))) {
    release_device_state(ctx);
    return rc;
  }
  for (uint32_t i = 0; i < ctx->header.num_nodes; ++i) {
    if ((rc = prepare_node(ctx, &ctx->node_records[i]))) {
      release_device_state(ctx);
      return rc;
    }
  }
  if ((rc = cuda_status(cudaStreamSynchronize(ctx->stream)))) {
    release_device_state(ctx);
    return rc;
  }
  ctx->prepared = true;
  ctx->graph_dirty = true;
  ctx->validated = false;
  ctx->run_count = 0;
  return 0;
}

int spkv2_set_input(Spkv2Context *ctx, int index, const void *data, size_t size) {
  if (!ctx || !data || index < 0) return -1;
  uint32_t id;
  int rc = input_tensor_id(ctx, index, &id);
  if (rc) return rc;
  TensorState &t = ctx->tensors[id];
  if (size != t.record->size_bytes) return -2;
  if (t.host_binding) {
    memcpy(t.host_binding, data, size);
    return 0;
  }
  if (!ctx->prepared || !t.data) return -5;
  cudaSetDevice(ctx->device);
  rc = cuda_status(cudaMemcpyAsync(t.data, data, size, cudaMemcpyHostToDevice, ctx->stream));
  if (rc) return rc;
  if (t.record->memory_class == SPKV2_MEMORY_EXTERNAL) t.bound = true;
  return cuda_status(cudaStreamSynchronize(ctx->stream));
}

int spkv2_bind_input(Spkv2Context *ctx, int index, void *data, size_t size) {
  if (!ctx || !data || index < 0) return -1;
  uint32_t id;
  int rc = input_tensor_id(ctx, index, &id);
  if (rc) return rc;
  if (size != ctx->tensor_records[id].size_bytes) return -2;
  return bind_tensor(ctx, id, data);
}

int spkv2_bind_output(Spkv2Context *ctx, int index, void *data, size_t size) {
  if (!ctx || !data || index < 0) return -1;
  uint32_t id;
  int rc = output_tensor_id(ctx, index, &id);
  if (rc) return rc;
  if (size != ctx->tensor_records[id].size_bytes) return -2;
  return bind_tensor(ctx, id, data);
}

int spkv2_get_output_size(Spkv2Context *ctx, int index, size_t *out_size) {
  if (!ctx || !out_size || index < 0) return -1;
  uint32_t id;
  int rc = output_tensor_id(ctx, index, &id);
  if (rc) return rc;
  *out_size = size_t(ctx->tensor_records[id].size_bytes);
  return 0;
}

int spkv2_get_output(Spkv2Context *ctx, int index, void *data, size_t size) {
  if (!ctx || !data || index < 0) return -1;
  uint32_t id;
  int rc = output_tensor_id(ctx, index, &id);
  if (rc) return rc;
  TensorState &t = ctx->tensors[id];
  if (size != t.record->size_bytes) return -2;
  if (t.host_binding) {
    if (t.host_binding != data) memcpy(data, t.host_binding, size);
    return 0;
  }
  if (!ctx->prepared || !t.data) return -5;
  cudaSetDevice(ctx->device);
  rc = cuda_status(cudaMemcpyAsync(data, t.data, size, cudaMemcpyDeviceToHost, ctx->stream));
  if (rc) return rc;
  return cuda_status(cudaStreamSynchronize(ctx->stream));
}

int spkv2_run(Spkv2Context *ctx) {
  int rc = check_runnable(ctx);
  if (rc) return rc;
  cudaSetDevice(ctx->device);
  if ((rc = stage_inputs(ctx))) return rc;
  if ((rc = launch_all(ctx))) {
    cudaStreamSynchronize(ctx->stream);
    return rc;
  }
  if ((rc = stage_outputs(ctx))) return rc;
  if ((rc = cuda_status(cudaStreamSynchronize(ctx->stream)))) return rc;
  if ((rc = take_device_status(ctx))) return rc;
  ctx->run_count++;
  return 0;
}

int spkv2_set_fault_event(Spkv2Context *ctx, const Spkv2FaultEvent *event) {
  if (!ctx || !event || event->bit_index >= 32u) return -1;
  if (event->node_id >= ctx->header.num_nodes || event->tensor_id >= ctx->header.num_tensors) return -2;
  ctx->fault_event = *event;
  return 0;
}

void spkv2_clear_fault_event(Spkv2Context *ctx) {
  if (ctx) memset(&ctx->fault_event, 0, sizeof(ctx->fault_event));
}

int spkv2_get_reliability_stats(Spkv2Context *ctx, Spkv2ReliabilityStats *stats) {
  if (!ctx || !stats) return -1;
  *stats = ctx->reliability_stats;
  return 0;
}

void spkv2_reset_reliability_stats(Spkv2Context *ctx) {
  if (ctx) memset(&ctx->reliability_stats, 0, sizeof(ctx->reliability_stats));
}

int spkv2_get_range_observation(Spkv2Context *ctx, uint32_t node_id, Spkv2RangeObservation *observation) {
  if (!ctx || !observation || node_id >= ctx->range_observations.size()) return -1;
  *observation = ctx->range_observations[node_id];
  return 0;
}

void spkv2_reset_range_observations(Spkv2Context *ctx) {
  if (!ctx) return;
  std::fill(ctx->range_observations.begin(), ctx->range_observations.end(), Spkv2RangeObservation{});
}

void spkv2_profile_dump(void) {
  if (g_prof_enabled > 0 && g_prof_runs > 0) prof_dump_impl(g_prof_ctx);
}

void spkv2_free(Spkv2Context *ctx) {
  if (!ctx) return;
  release_device_state(ctx);
  if (g_prof_ctx == ctx) g_prof_ctx = nullptr;
  if (ctx->owned_model) spkv2_platform_free(ctx->owned_model);
  delete ctx;
}

// ---------------- CUDA-target extensions ----------------

int spkv2_cuda_set_device(Spkv2Context *ctx, int device) {
  if (!ctx || device < 0) return -1;
  if (ctx->prepared) return -1;
  ctx->device = device;
  return 0;
}

int spkv2_cuda_get_device(Spkv2Context *ctx, int *device) {
  if (!ctx || !device) return -1;
  *device = ctx->device;
  return 0;
}

int spkv2_cuda_set_math_mode(Spkv2Context *ctx, int mode) {
  if (!ctx || mode < SPKV2_CUDA_MATH_SPEC || mode > SPKV2_CUDA_MATH_FP32) return -1;
  if (ctx->prepared) return -1;
  ctx->math_mode = mode;
  return 0;
}

int spkv2_cuda_set_graph_mode(Spkv2Context *ctx, int enabled) {
  if (!ctx) return -1;
  ctx->graph_mode = enabled ? 1 : 0;
  ctx->graph_dirty = true;
  ctx->validated = false;
  return 0;
}

void *spkv2_cuda_stream(Spkv2Context *ctx) { return ctx ? static_cast<void *>(ctx->stream) : nullptr; }

void *spkv2_cuda_tensor_device_ptr(Spkv2Context *ctx, uint32_t tensor_id) {
  if (!ctx || !ctx->prepared || tensor_id >= ctx->header.num_tensors) return nullptr;
  return ctx->tensors[tensor_id].data;
}

int spkv2_cuda_tensor_layout(Spkv2Context *ctx, uint32_t tensor_id) {
  if (!ctx || !ctx->prepared || tensor_id >= ctx->header.num_tensors) return -1;
  return int(ctx->tensors[tensor_id].layout);
}

int spkv2_cuda_run_async(Spkv2Context *ctx) {
  int rc = check_runnable(ctx);
  if (rc) return rc;
  cudaSetDevice(ctx->device);
  rc = launch_all(ctx);
  if (rc == 0) ctx->run_count++;
  return rc;
}

int spkv2_cuda_synchronize(Spkv2Context *ctx) {
  if (!ctx || !ctx->prepared) return SPKV2_ERR_NOT_PREPARED;
  cudaSetDevice(ctx->device);
  int rc = cuda_status(cudaStreamSynchronize(ctx->stream));
  return rc ? rc : take_device_status(ctx);
}

int spkv2_cuda_run_nodes(Spkv2Context *ctx, uint32_t first, uint32_t last) {
  int rc = check_runnable(ctx);
  if (rc) return rc;
  if (first > last || last > ctx->header.num_nodes) return -3;
  cudaSetDevice(ctx->device);
  rc = run_nodes_eager(ctx, first, last, false);
  int src = cuda_status(cudaStreamSynchronize(ctx->stream));
  if (rc == 0 && src == 0) src = take_device_status(ctx);
  return rc ? rc : src;
}

int spkv2_cuda_profile_nodes(Spkv2Context *ctx, float *node_ms, uint32_t count) {
  int rc = check_runnable(ctx);
  if (rc) return rc;
  if (!node_ms || count < ctx->header.num_nodes) return -1;
  cudaSetDevice(ctx->device);
  const uint32_t n = ctx->header.num_nodes;
  std::vector<cudaEvent_t> ev(size_t(n) + 1);
  for (auto &e : ev) cudaEventCreate(&e);
  cudaEventRecord(ev[0], ctx->stream);
  for (uint32_t i = 0; i < n && rc == 0; ++i) {
    rc = execute_node(ctx, &ctx->node_records[i]);
    cudaEventRecord(ev[i + 1], ctx->stream);
  }
  int src = cuda_status(cudaStreamSynchronize(ctx->stream));
  if (rc == 0 && src == 0)
    for (uint32_t i = 0; i < n; ++i) cudaEventElapsedTime(&node_ms[i], ev[i], ev[i + 1]);
  for (auto &e : ev) cudaEventDestroy(e);
  return rc ? rc : src;
}

int spkv2_cuda_read_tensor(Spkv2Context *ctx, uint32_t tensor_id, void *host, size_t size) {
  if (!ctx || !host) return -1;
  if (!ctx->prepared) return SPKV2_ERR_NOT_PREPARED;
  if (tensor_id >= ctx->header.num_tensors) return -3;
  const TensorState &t = ctx->tensors[tensor_id];
  if (size != t.record->size_bytes) return -2;
  cudaSetDevice(ctx->device);
  return copy_tensor_to_host(t, host, ctx->stream);
}

int spkv2_cuda_write_tensor(Spkv2Context *ctx, uint32_t tensor_id, const void *host, size_t size) {
  if (!ctx || !host) return -1;
  if (!ctx->prepared) return SPKV2_ERR_NOT_PREPARED;
  if (tensor_id >= ctx->header.num_tensors) return -3;
  const TensorState &t = ctx->tensors[tensor_id];
  if (size != t.record->size_bytes) return -2;
  cudaSetDevice(ctx->device);
  return copy_tensor_from_host(t, host, ctx->stream);
}

int spkv2_cuda_watchdog_probe(Spkv2Context *ctx, uint32_t wait_us, int *code) {
  if (!ctx || wait_us == 0 || wait_us > 2000000u) return -1;
  if (!ctx->prepared || !ctx->d_status) return SPKV2_ERR_NOT_PREPARED;
  cudaSetDevice(ctx->device);
  int rc = watchdog_probe(ctx->d_status, wait_us, ctx->stream);
  if (rc) return rc;
  if ((rc = cuda_status(cudaStreamSynchronize(ctx->stream)))) return rc;
  rc = take_device_status(ctx);
  if (code) *code = rc ? ctx->last_device_code : 0;
  return rc;
}

int spkv2_cuda_last_device_code(Spkv2Context *ctx) { return ctx ? ctx->last_device_code : 0; }

int spkv2_cuda_launches_per_run(Spkv2Context *ctx, uint32_t *count) {
  if (!ctx || !count) return -1;
  if (!ctx->prepared) return SPKV2_ERR_NOT_PREPARED;
  uint32_t n = 0;
  for (uint32_t i = 0; i < ctx->header.num_nodes; ++i) {
    NodePlan *p = static_cast<NodePlan *>(ctx->node_cache[i]);
    n += p ? uint32_t(p->launches) : 1u;
  }
  *count = n;
  return 0;
}

const char *spkv2_cuda_node_variant(Spkv2Context *ctx, uint32_t node_id) {
  if (!ctx || node_id >= ctx->node_cache.size() || !ctx->node_cache[node_id]) return nullptr;
  return static_cast<NodePlan *>(ctx->node_cache[node_id])->variant.c_str();
}

const char *spkv2_cuda_status_string(int code) {
  switch (code) {
    case 0: return "ok";
    case -1: return "bad argument or host allocation failure";
    case -2: return "size, magic or version mismatch";
    case -3: return "index or bounds error";
    case -4: return "missing section or offset beyond arena";
    case -5: return "checksum section missing, or tensor unbound at run";
    case -6: return "checksum mismatch";
    case -10: return "attribute record out of bounds";
    case -11: return "bad rank or axis";
    case -12: return "bad group";
    case -13: return "missing scratch";
    case -14: return "scratch overflow";
    case -99: return "no kernel for node";
    case SPKV2_ERR_CUDA: return "CUDA runtime error";
    case SPKV2_ERR_DEVICE_ALLOC: return "device allocation failed";
    case SPKV2_ERR_NO_DEVICE: return "no usable sm_100 device";
    case SPKV2_ERR_UNSUPPORTED: return "node variant unsupported on the CUDA target";
    case SPKV2_ERR_LAUNCH: return "kernel launch failed";
    case SPKV2_ERR_NOT_PREPARED: return "context not prepared";
    case SPKV2_ERR_PROTECTION: return "protection plan error";
    case SPKV2_ERR_DEVICE_STATUS: return "device kernel reported a timeout or an out-of-range index";
    default: return (code <= -20 && code >= -26) ? "fault or protection error" : "unknown";
  }
}

}  // extern "C"
