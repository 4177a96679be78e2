// Physical layout of every tensor on the device.
//
// The SPK records every activation in logical NCHW / row-major order and the
// memory plan fixes only byte offsets and sizes.  Channels-last (NHWC) has the
// same byte size, so the plan stays valid when a rank-4 activation is stored
// NHWC, which is what the implicit-GEMM convs want (K contiguous per pixel).
//
// Rules:
//   1. Non-rank-4 tensors, weights, graph inputs/outputs and caller-bound
//      (EXTERNAL) tensors stay row-major: the host sees logical order.
//   2. A rank-4 tensor with C == 1 or H*W == 1 is the same bytes either way and
//      is recorded as row-major.
//   3. Tensors that share arena bytes while both are live (the planner's
//      in-place Relu/Flatten/Reshape aliases and Concat sub-region aliases,
//      compiler/planner/memory_plan.py:275-379) form an alias group.  A group
//      is NHWC only if every member is an NHWC candidate with the same shape
//      at the same offset; otherwise every member is row-major.
#include <algorithm>
#include <numeric>
#include <vector>

#include "context.h"

namespace spkv2 {

namespace {

struct DisjointSet {
  std::vector<int> parent;
  explicit DisjointSet(size_t n) : parent(n) { std::iota(parent.begin(), parent.end(), 0); }
  int find(int x) {
    while (parent[x] != x) x = parent[x] = parent[parent[x]];
    return x;
  }
  void unite(int a, int b) { parent[find(a)] = find(b); }
};

bool nhwc_candidate(const Spkv2TensorRecord *r) {
  if (r->role != SPKV2_ROLE_ACTIVATION) return false;
  if (r->memory_class != SPKV2_MEMORY_ACTIVATION_ARENA) return false;
  if (r->rank != 4) return false;
  if (r->dtype != SPKV2_DTYPE_FP32 && r->dtype != SPKV2_DTYPE_INT8) return false;
  return r->shape[1] > 1 && uint64_t(r->shape[2]) * r->shape[3] > 1;
}

}  // namespace

int assign_layouts(Spkv2Context *ctx) {
  const uint32_t nt = ctx->header.num_tensors;
  const uint32_t nn = ctx->header.num_nodes;
  std::vector<int64_t> first(nt, -1), last(nt, -1);
  for (uint32_t i = 0; i < nt; ++i) {
    const Spkv2TensorRecord *r = ctx->tensors[i].record;
    if (r->role == SPKV2_ROLE_INPUT) first[i] = 0;
    if (r->role == SPKV2_ROLE_OUTPUT) last[i] = int64_t(nn) + 1;
  }
  for (uint32_t n = 0; n < nn; ++n) {
    const Spkv2NodeRecord *node = &ctx->node_records[n];
    for (uint16_t k = 0; k < node->output_count && k < 4; ++k) {
      uint32_t t = node->outputs[k];
      if (t >= nt) return -3;
      if (first[t] < 0) first[t] = n;
      last[t] = std::max<int64_t>(last[t], n);
    }
    for (uint16_t k = 0; k < node->input_count && k < 8; ++k) {
      uint32_t t = node->inputs[k];
      if (t >= nt) return -3;
      if (first[t] < 0) first[t] = n;
      last[t] = std::max<int64_t>(last[t], n);
    }
  }
  // Arena tensors ordered by offset; union those that overlap in bytes and
  // in lifetime.
  std::vector<uint32_t> arena;
  for (uint32_t i = 0; i < nt; ++i) {
    const Spkv2TensorRecord *r = ctx->tensors[i].record;
    if (r->role == SPKV2_ROLE_WEIGHT || r->memory_class == SPKV2_MEMORY_EXTERNAL || r->size_bytes == 0) continue;
    if (first[i] < 0) continue;  // never touched by a node
    arena.push_back(i);
  }
  std::sort(arena.begin(), arena.end(), [&](uint32_t a, uint32_t b) {
    return ctx->tensors[a].record->data_offset < ctx->tensors[b].record->data_offset;
  });
  DisjointSet groups(nt);
  for (size_t a = 0; a < arena.size(); ++a) {
    const Spkv2TensorRecord *ra = ctx->tensors[arena[a]].record;
    const uint64_t end_a = ra->data_offset + ra->size_bytes;
    for (size_t b = a + 1; b < arena.size(); ++b) {
      const Spkv2TensorRecord *rb = ctx->tensors[arena[b]].record;
      if (rb->data_offset >= end_a) break;
      if (first[arena[a]] <= last[arena[b]] && first[arena[b]] <= last[arena[a]])
        groups.unite(int(arena[a]), int(arena[b]));
    }
  }
  // A group is NHWC only if all of its members agree.
  std::vector<int> group_ok(nt, 1);
  std::vector<const Spkv2TensorRecord *> group_rep(nt, nullptr);
  for (uint32_t i = 0; i < nt; ++i) {
    const Spkv2TensorRecord *r = ctx->tensors[i].record;
    int g = groups.find(int(i));
    if (!nhwc_candidate(r)) {
      group_ok[g] = 0;
      continue;
    }
    const Spkv2TensorRecord *rep = group_rep[g];
    if (!rep) {
      group_rep[g] = r;
    } else if (rep->data_offset != r->data_offset || rep->dtype != r->dtype ||
               memcmp(rep->shape, r->shape, sizeof(uint32_t) * 4) != 0) {
      group_ok[g] = 0;
    }
  }
  for (uint32_t i = 0; i < nt; ++i) {
    int g = groups.find(int(i));
    ctx->tensors[i].layout = (nhwc_candidate(ctx->tensors[i].record) && group_ok[g]) ? kNHWC : kRowMajor;
  }
  return 0;
}

}  // namespace spkv2
