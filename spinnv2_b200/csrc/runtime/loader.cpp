// SPK package loading for the CUDA target.
//
// Validation order and return codes follow the reference loader
// (runtime/core/loader.c:105-282): magic/version -> -2, directory or section
// out of bounds -> -3, missing tensor/node/attribute/weight section or short
// tables -> -4, checksum section missing -> -5, FNV-1a mismatch -> -6.  The
// metadata "outputs" list fixes the output order (loader.c:46-103).
#include <ctype.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <new>

#include "context.h"
#include "spkv2_platform.h"

namespace {

const Spkv2SectionEntry *section_of(const Spkv2Context *ctx, uint32_t kind) {
  for (uint32_t i = 0; i < ctx->header.section_count; ++i)
    if (ctx->sections[i].kind == kind) return &ctx->sections[i];
  return nullptr;
}

uint32_t fnv1a(const uint8_t *p, size_t n) {
  uint32_t h = 0x811C9DC5u;  // FNV-1a 32-bit offset basis
  for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 0x01000193u;
  return h;
}

// Reads the integer list that follows the key "outputs" in the metadata JSON.
// A malformed or short list leaves the default (tensor-table order) in place.
void read_output_order(Spkv2Context *ctx, const Spkv2SectionEntry *meta) {
  if (!meta || meta->size == 0 || ctx->header.num_outputs == 0) return;
  const char *s = reinterpret_cast<const char *>(ctx->model_data + meta->offset);
  const char *end = s + meta->size;
  static const char kKey[] = "\"outputs\"";
  const size_t klen = sizeof(kKey) - 1;
  for (const char *p = s; p + klen <= end; ++p) {
    if (memcmp(p, kKey, klen) != 0) continue;
    const char *q = p + klen;
    while (q < end && isspace((unsigned char)*q)) ++q;
    if (q >= end || *q != ':') continue;
    ++q;
    while (q < end && isspace((unsigned char)*q)) ++q;
    if (q >= end || *q != '[') continue;
    ++q;
    std::vector<uint32_t> ids;
    for (;;) {
      while (q < end && isspace((unsigned char)*q)) ++q;
      if (q >= end) return;
      if (*q == ']') break;
      char buf[32];
      size_t n = 0;
      while (q < end && n + 1 < sizeof(buf) && isdigit((unsigned char)*q)) buf[n++] = *q++;
      if (n == 0) return;
      buf[n] = 0;
      unsigned long v = strtoul(buf, nullptr, 10);
      if (v >= ctx->header.num_tensors || ids.size() >= ctx->header.num_outputs) return;
      ids.push_back(static_cast<uint32_t>(v));
      while (q < end && isspace((unsigned char)*q)) ++q;
      if (q < end && *q == ',') { ++q; continue; }
      if (q < end && *q == ']') break;
      return;
    }
    if (ids.size() == ctx->header.num_outputs) ctx->output_ids = ids;
    return;
  }
}

}  // namespace

extern "C" {

const char *spkv2_runtime_version(void) { return "0.0.0-m0+cuda_b200"; }

uint32_t spkv2_fnv1a32(const void *data, size_t size) {
  return data ? fnv1a(static_cast<const uint8_t *>(data), size) : 0u;
}

int spkv2_load_memory(const void *data, size_t size, Spkv2Context **out_ctx) {
  if (!data || !out_ctx || size < sizeof(Spkv2Header)) return -1;
  Spkv2Context *ctx = new (std::nothrow) Spkv2Context();
  if (!ctx) return -1;
  memcpy(&ctx->header, data, sizeof(Spkv2Header));
  if (ctx->header.magic != SPKV2_MAGIC || ctx->header.version_major != SPKV2_VERSION_MAJOR) {
    delete ctx;
    return -2;
  }
  const uint64_t dir_off = ctx->header.header_size;
  const uint64_t dir_len = uint64_t(ctx->header.section_count) * sizeof(Spkv2SectionEntry);
  if (dir_off > size || dir_len > size - dir_off) {
    delete ctx;
    return -3;
  }
  ctx->model_data = static_cast<const uint8_t *>(data);
  ctx->model_size = size;
  ctx->sections = reinterpret_cast<const Spkv2SectionEntry *>(ctx->model_data + dir_off);
  for (uint32_t i = 0; i < ctx->header.section_count; ++i) {
    const Spkv2SectionEntry &s = ctx->sections[i];
    if (s.offset > size || s.size > size - s.offset) {
      delete ctx;
      return -3;
    }
  }
  const Spkv2SectionEntry *tensor_sec = section_of(ctx, SPKV2_SECTION_TENSOR_TABLE);
  const Spkv2SectionEntry *node_sec = section_of(ctx, SPKV2_SECTION_NODE_TABLE);
  const Spkv2SectionEntry *attr_sec = section_of(ctx, SPKV2_SECTION_ATTRIBUTES);
  const Spkv2SectionEntry *weight_sec = section_of(ctx, SPKV2_SECTION_WEIGHTS);
  const Spkv2SectionEntry *plan_sec = section_of(ctx, SPKV2_SECTION_MEMORY_PLAN);
  const Spkv2SectionEntry *spec_sec = section_of(ctx, SPKV2_SECTION_KERNEL_SPEC);
  const Spkv2SectionEntry *quant_sec = section_of(ctx, SPKV2_SECTION_QUANTIZATION);
  const Spkv2SectionEntry *prot_sec = section_of(ctx, SPKV2_SECTION_PROTECTION_PLAN);
  const Spkv2SectionEntry *sum_sec = section_of(ctx, SPKV2_SECTION_CHECKSUM);
  const Spkv2SectionEntry *meta_sec = section_of(ctx, SPKV2_SECTION_METADATA);
  if (!tensor_sec || !node_sec || !attr_sec || !weight_sec ||
      tensor_sec->size < uint64_t(ctx->header.num_tensors) * sizeof(Spkv2TensorRecord) ||
      node_sec->size < uint64_t(ctx->header.num_nodes) * sizeof(Spkv2NodeRecord)) {
    delete ctx;
    return -4;
  }
  if (ctx->header.checksum_type == 1) {
    if (!sum_sec || sum_sec->size < 4) {
      delete ctx;
      return -5;
    }
    uint32_t stored;
    memcpy(&stored, ctx->model_data + sum_sec->offset, 4);
    if (stored != fnv1a(ctx->model_data, size_t(sum_sec->offset))) {
      delete ctx;
      return -6;
    }
  }
  ctx->tensor_records = reinterpret_cast<const Spkv2TensorRecord *>(ctx->model_data + tensor_sec->offset);
  ctx->node_records = reinterpret_cast<const Spkv2NodeRecord *>(ctx->model_data + node_sec->offset);
  if (plan_sec && plan_sec->size >= uint64_t(ctx->header.num_tensors) * sizeof(Spkv2MemoryPlanRecord)) {
    ctx->memory_plan_records = reinterpret_cast<const Spkv2MemoryPlanRecord *>(ctx->model_data + plan_sec->offset);
    ctx->memory_plan_count = size_t(plan_sec->size / sizeof(Spkv2MemoryPlanRecord));
  }
  if (spec_sec && spec_sec->size >= uint64_t(ctx->header.num_nodes) * sizeof(Spkv2KernelSpecRecord)) {
    ctx->kernel_spec_records = reinterpret_cast<const Spkv2KernelSpecRecord *>(ctx->model_data + spec_sec->offset);
    ctx->kernel_spec_count = size_t(spec_sec->size / sizeof(Spkv2KernelSpecRecord));
  }
  // Quantisation section: the records come first; the first record's
  // data_offset marks where the record array ends.
  if (quant_sec && quant_sec->size >= sizeof(Spkv2QuantParamRecord)) {
    const uint8_t *base = ctx->model_data + quant_sec->offset;
    Spkv2QuantParamRecord first;
    memcpy(&first, base, sizeof(first));
    size_t n = size_t(first.data_offset / sizeof(Spkv2QuantParamRecord));
    if (first.data_offset > 0 && n > 0 && n * sizeof(Spkv2QuantParamRecord) <= quant_sec->size) {
      ctx->quant_param_records = reinterpret_cast<const Spkv2QuantParamRecord *>(base);
      ctx->quant_param_count = n;
      ctx->quant_data = base;
      ctx->quant_data_size = size_t(quant_sec->size);
    }
  }
  if (prot_sec && prot_sec->size >= sizeof(Spkv2ProtectionRecord)) {
    ctx->protection_records = reinterpret_cast<const Spkv2ProtectionRecord *>(ctx->model_data + prot_sec->offset);
    ctx->protection_count = size_t(prot_sec->size / sizeof(Spkv2ProtectionRecord));
  }
  ctx->attrs = ctx->model_data + attr_sec->offset;
  ctx->attrs_size = size_t(attr_sec->size);
  ctx->weights = ctx->model_data + weight_sec->offset;
  ctx->weights_size = size_t(weight_sec->size);

  ctx->tensors.resize(ctx->header.num_tensors);
  for (uint32_t i = 0; i < ctx->header.num_tensors; ++i) ctx->tensors[i].record = &ctx->tensor_records[i];
  read_output_order(ctx, meta_sec);
  ctx->node_cache.assign(ctx->header.num_nodes, nullptr);
  ctx->node_cache_dtors.assign(ctx->header.num_nodes, nullptr);
  ctx->node_invocation_counts.assign(ctx->header.num_nodes, 0);
  ctx->range_observations.assign(ctx->header.num_nodes, Spkv2RangeObservation{});
  *out_ctx = ctx;
  return 0;
}

int spkv2_load_file(const char *path, Spkv2Context **out_ctx) {
  if (!path || !out_ctx) return -1;
  FILE *fp = fopen(path, "rb");
  if (!fp) return -1;
  if (fseek(fp, 0, SEEK_END) != 0) {
    fclose(fp);
    return -1;
  }
  long n = ftell(fp);
  if (n <= 0) {
    fclose(fp);
    return -1;
  }
  rewind(fp);
  uint8_t *buf = static_cast<uint8_t *>(spkv2_platform_malloc(size_t(n)));
  if (!buf) {
    fclose(fp);
    return -1;
  }
  size_t got = fread(buf, 1, size_t(n), fp);
  fclose(fp);
  if (got != size_t(n)) {
    spkv2_platform_free(buf);
    return -1;
  }
  int rc = spkv2_load_memory(buf, size_t(n), out_ctx);
  if (rc != 0) {
    spkv2_platform_free(buf);
    return rc;
  }
  (*out_ctx)->owned_model = buf;
  (*out_ctx)->owned_model_size = size_t(n);
  return 0;
}

}  // extern "C"
