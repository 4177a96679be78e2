// Kernel registry and node dispatch for the CUDA target.
//
// Keeps the reference registry's contract (runtime/kernels/reference/
// kernels.c:5-30,144-245): 64 user slots; spkv2_register_kernel returns -1
// for a NULL function and -2 when the slots are full; user entries are
// scanned first and a built-in replaces the current best only with a strictly
// higher priority (built-ins have priority 0); a kernel returning -99 moves
// dispatch to the spec's fallback_kernel_spec_id.
//
// Difference by design: every built-in is a CUDA kernel, and a built-in
// serves its op whatever (backend, kind) the KernelSpec names, so SPKs
// compiled for the CPU profiles also run on the device.  There is no CPU
// kernel anywhere on this path; an op without a CUDA kernel returns -99.
#include <string.h>

#include "../kernels/kernels.h"
#include "context.h"

using namespace spkv2;

namespace {

constexpr int kUserSlots = 64;

struct UserEntry {
  uint16_t op, backend, kind;
  int priority;
  Spkv2NodeKernelFn fn;
};

UserEntry g_user[kUserSlots];
int g_user_count = 0;

struct Builtin {
  uint16_t op;
  Spkv2NodeKernelFn run;
  PrepareFn prepare;
};

const Builtin kBuiltins[] = {
    {SPKV2_OP_CONV, conv_run, conv_prepare},
    {SPKV2_OP_GEMM, gemm_run, gemm_prepare},
    {SPKV2_OP_MATMUL, gemm_run, gemm_prepare},
    {SPKV2_OP_ADD, eltwise_run, eltwise_prepare},
    {SPKV2_OP_SUB, eltwise_run, eltwise_prepare},
    {SPKV2_OP_MUL, eltwise_run, eltwise_prepare},
    {SPKV2_OP_DIV, eltwise_run, eltwise_prepare},
    {SPKV2_OP_MOD, eltwise_run, eltwise_prepare},
    {SPKV2_OP_RELU, eltwise_run, eltwise_prepare},
    {SPKV2_OP_SIGMOID, eltwise_run, eltwise_prepare},
    {SPKV2_OP_CLIP, eltwise_run, eltwise_prepare},
    {SPKV2_OP_LEAKYRELU, eltwise_run, eltwise_prepare},
    {SPKV2_OP_CAST, copy_run, copy_prepare},
    {SPKV2_OP_FLATTEN, copy_run, copy_prepare},
    {SPKV2_OP_RESHAPE, copy_run, copy_prepare},
    {SPKV2_OP_UNSQUEEZE, copy_run, copy_prepare},
    {SPKV2_OP_MAXPOOL, pool_run, pool_prepare},
    {SPKV2_OP_AVERAGEPOOL, pool_run, pool_prepare},
    {SPKV2_OP_GLOBALAVGPOOL, pool_run, pool_prepare},
    {SPKV2_OP_RESIZE, resize_run, resize_prepare},
    {SPKV2_OP_CONCAT, concat_run, concat_prepare},
    {SPKV2_OP_SPLIT, split_run, split_prepare},
    {SPKV2_OP_TRANSPOSE, transpose_run, transpose_prepare},
    {SPKV2_OP_TILE, tile_run, tile_prepare},
    {SPKV2_OP_GATHERELEMENTS, gather_elements_run, gather_elements_prepare},
    {SPKV2_OP_SLICE, slice_run, slice_prepare},
    {SPKV2_OP_GATHER, gather_run, gather_prepare},
    {SPKV2_OP_REDUCEMEAN, reduce_run, reduce_prepare},
    {SPKV2_OP_REDUCEMAX, reduce_run, reduce_prepare},
    {SPKV2_OP_SOFTMAX, softmax_run, softmax_prepare},
    {SPKV2_OP_TOPK, topk_run, topk_prepare},
};

const Builtin *builtin_for(uint16_t op) {
  for (const Builtin &b : kBuiltins)
    if (b.op == op) return &b;
  return nullptr;
}

// The (backend REF, kind REFERENCE) spec used when a node has no valid spec
// (reference kernels.c:169-190).
Spkv2KernelSpecRecord ref_spec_for(uint32_t node_id) {
  Spkv2KernelSpecRecord s;
  memset(&s, 0, sizeof(s));
  s.id = 0xFFFFFFFFu;
  s.node_id = node_id;
  s.kernel_kind = SPKV2_KERNEL_REFERENCE;
  s.backend = SPKV2_BACKEND_REF;
  s.dtype = SPKV2_DTYPE_FP32;
  s.layout = SPKV2_LAYOUT_NCHW;
  s.weight_layout = 1;
  s.fallback_kernel_spec_id = 0xFFFFFFFFu;
  s.required_feature_mask = 1;
  return s;
}

const Spkv2KernelSpecRecord *spec_by_id(const Spkv2Context *ctx, uint32_t id) {
  if (id == 0xFFFFFFFFu || id >= ctx->kernel_spec_count) return nullptr;
  return &ctx->kernel_spec_records[id];
}

Spkv2NodeKernelFn find_kernel(uint16_t op, const Spkv2KernelSpecRecord *spec) {
  Spkv2NodeKernelFn best = nullptr;
  int best_priority = -1;
  for (int i = 0; i < g_user_count; ++i) {
    const UserEntry &e = g_user[i];
    if (e.op == op && e.backend == spec->backend && e.kind == spec->kernel_kind && e.priority > best_priority) {
      best = e.fn;
      best_priority = e.priority;
    }
  }
  const Builtin *b = builtin_for(op);
  if (b && 0 > best_priority) best = b->run;
  return best;
}

int run_with_spec(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  Spkv2NodeKernelFn fn = find_kernel(node->op_type, spec);
  if (!fn) return -99;
  if (spec->scratch_bytes > ctx->scratch_size) return -14;
  if (spec->scratch_bytes > 0 && spec->scratch_offset > ctx->scratch_size - spec->scratch_bytes) return -14;
  void *scratch = spec->scratch_bytes > 0 ? ctx->d_scratch + spec->scratch_offset : nullptr;
  return fn(ctx, node, scratch);
}

}  // namespace

namespace spkv2 {

const Spkv2KernelSpecRecord *spec_for_node(const Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  const Spkv2KernelSpecRecord *s = spec_by_id(ctx, node->kernel_spec_id);
  return (s && s->node_id == node->id) ? s : nullptr;
}

int execute_node(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  Spkv2KernelSpecRecord ref = ref_spec_for(node->id);
  const Spkv2KernelSpecRecord *spec = spec_for_node(ctx, node);
  if (!spec) spec = &ref;
  int rc = run_with_spec(ctx, node, spec);
  if (rc != -99) return rc;
  const Spkv2KernelSpecRecord *fb = spec_by_id(ctx, spec->fallback_kernel_spec_id);
  if (fb) return run_with_spec(ctx, node, fb);
  // No CPU reference kernel exists on this target: the built-in CUDA kernel
  // of the op is the last resort, and -99 if the op has none.
  const Builtin *b = builtin_for(node->op_type);
  return b ? b->run(ctx, node, nullptr) : -99;
}

int prepare_node(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  Spkv2KernelSpecRecord ref = ref_spec_for(node->id);
  const Spkv2KernelSpecRecord *spec = spec_for_node(ctx, node);
  if (!spec) spec = &ref;
  const Builtin *b = builtin_for(node->op_type);
  Spkv2NodeKernelFn fn = find_kernel(node->op_type, spec);
  if (b && fn == b->run) return b->prepare(ctx, node, spec);
  if (!fn && !b) return -99;
  return 0;  // user kernel: prepares itself
}

int get_attr(const Spkv2Context *ctx, const Spkv2NodeRecord *node, Spkv2AttrRecord *attr) {
  if (node->attr_offset > ctx->attrs_size || node->attr_size > ctx->attrs_size - node->attr_offset ||
      node->attr_size < sizeof(Spkv2AttrRecord))
    return -10;
  memcpy(attr, ctx->attrs + node->attr_offset, sizeof(Spkv2AttrRecord));
  return 0;
}

const Spkv2QuantParamRecord *find_quant_param(const Spkv2Context *ctx, uint32_t tensor_id) {
  for (size_t i = 0; i < ctx->quant_param_count; ++i)
    if (ctx->quant_param_records[i].tensor_id == tensor_id) return &ctx->quant_param_records[i];
  return nullptr;
}

const float *quant_scales(const Spkv2Context *ctx, const Spkv2QuantParamRecord *qp) {
  if (!qp || !ctx->quant_data) return nullptr;
  if (qp->data_offset + uint64_t(qp->num_channels) * 4 > ctx->quant_data_size) return nullptr;
  return reinterpret_cast<const float *>(ctx->quant_data + qp->data_offset);
}

}  // namespace spkv2

extern "C" {

int spkv2_register_kernel(uint16_t op_type, uint16_t backend, uint16_t kernel_kind, Spkv2NodeKernelFn fn,
                          int priority) {
  if (!fn) return -1;
  if (g_user_count >= kUserSlots) return -2;
  g_user[g_user_count++] = UserEntry{op_type, backend, kernel_kind, priority, fn};
  return 0;
}

void spkv2_clear_user_kernels(void) { g_user_count = 0; }

}  // extern "C"
