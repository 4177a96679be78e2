// Concat, Split, Transpose, Tile and GatherElements.
//
// Semantics (reference):
//   Concat  reference/tensor/concat.c:5-30   inputs stacked along `axis`
//   Split   reference/tensor/split.c:5-30    output sizes from the output
//           records along `axis`
//   Transpose reference/shape/transpose.c:3  y[coords] = x[coords permuted by
//           attr.extra]; with no perm attribute the mapping is the identity
//   Tile    reference/shape/tile.c            x coord = y coord mod x dim
//   GatherElements reference/tensor/gather_elements.c:3-25  fp32 indices,
//           negative indices wrap by the axis size
//   Slice   reference/tensor/slice.c:4-56   one axis: starts[0], ends[0],
//           axes[0] (default 0), steps[0] (default 1) read from constant
//           inputs; negative start/end wrap by the axis size, end clamps to
//           it, start clamps at 0; out extent (end - start + step - 1) / step
//   Gather  reference/tensor/gather.c:4-44  y = data[..., idx[j], ...] along
//           `axis`, output shape data[:axis] + idx.shape + data[axis+1:],
//           fp32 indices, negative indices wrap by the axis size
// An index that is still out of range after wrapping (the reference reads
// outside the tensor) writes 0 and records device code 10 in the context's
// status word, so the run returns SPKV2_ERR_DEVICE_STATUS instead of
// touching memory outside the input.
// Device design: every kernel walks one tensor in physical order and reaches
// the others through per-dim strides, so NHWC and NCHW operands mix freely;
// Concat/Split move four elements per thread when the innermost physical dim
// allows it.  Concat inputs that the memory plan placed inside the output
// (sub-region aliases) are copied onto themselves, which is a no-op.
#include <string.h>

#include <type_traits>

#include "common.cuh"

namespace spkv2 {

namespace {

constexpr int kMaxParts = 8;

struct PartDesc {
  int rank;                      // iteration rank (physical order of the big tensor)
  int64_t dim[kMaxRank];         // big tensor dims in iteration order
  int64_t big_stride[kMaxRank];  // big tensor strides in iteration order
  int axis_pos;                  // position of the axis in iteration order
  int parts;
  int64_t begin[kMaxParts + 1];  // axis offset of each part
  int64_t part_stride[kMaxParts][kMaxRank];
  void *ptr[kMaxParts];
};

struct PartPlan : NodePlan {
  PartDesc d;
  int vec = 1;
  int esize = 4;
  int64_t total = 0;
  // Dense fast path: big and every part contiguous in the big tensor's
  // physical order, so each of `rows` outer rows of the big tensor is the
  // parts' rows side by side: part k owns elements [seg[k], seg[k+1]) of a
  // big row of seg[parts] elements (all in 16-byte vectors).
  bool rows_path = false;
  uint32_t rows = 0;
  uint32_t seg[kMaxParts + 1] = {};
};

// Dense row copy of 16-byte vectors, part-major: blockIdx.y selects part k
// (uniform per block, so its row width, offset and pointer are read once),
// and the part is walked in its own contiguous order.  Vector v of part k
// is at row v / w_k, column v % w_k of its rows of w_k vectors; in the big
// tensor it sits at row * W + off_k + column.  One division per vector and
// no search over the parts; each block moves kRowsPerBlock vectors of one
// part, four 16-byte loads in flight per thread (blocks past a smaller
// part's end exit at once).  32-bit indices: the plan checks the sizes.
struct PartRows {
  uint32_t W;                   // big row width, vectors
  uint32_t off[kMaxParts];      // part k's column offset in a big row
  uint32_t n[kMaxParts];        // vectors of part k
  FastDiv w[kMaxParts];         // part k's row width
  void *ptr[kMaxParts];
};

constexpr int kRowsThreads = 256, kRowsUnroll = 4, kRowsIters = 4;
constexpr uint32_t kRowsPerBlock = kRowsThreads * kRowsUnroll * kRowsIters;

template <bool GATHER>
__global__ void __launch_bounds__(kRowsThreads) rows_kernel(uint4 *__restrict__ big, PartRows r) {
  const int k = blockIdx.y;
  const uint32_t n = r.n[k];
  const uint32_t base = blockIdx.x * kRowsPerBlock;
  if (base >= n) return;
  const FastDiv w = r.w[k];
  const uint32_t off = r.off[k], W = r.W;
  uint4 *part = static_cast<uint4 *>(r.ptr[k]);
#pragma unroll 1
  for (int it = 0; it < kRowsIters; ++it) {
    const uint32_t v0 = base + uint32_t(it * kRowsUnroll * kRowsThreads) + threadIdx.x;
    uint4 val[kRowsUnroll];
    uint4 *dst[kRowsUnroll];
#pragma unroll
    for (int u = 0; u < kRowsUnroll; ++u) {
      const uint32_t v = v0 + uint32_t(u * kRowsThreads);
      dst[u] = nullptr;
      if (v < n) {
        const uint32_t row = w.div(v);
        uint4 *b = big + (size_t(row) * W + off + (v - row * w.d));
        val[u] = GATHER ? __ldg(part + v) : __ldg(b);
        dst[u] = GATHER ? b : part + v;
      }
    }
#pragma unroll
    for (int u = 0; u < kRowsUnroll; ++u)
      if (dst[u]) *dst[u] = val[u];
  }
}

// GATHER (Concat): big = output, parts = inputs.  Split: big = input,
// parts = outputs.
template <typename T, int V, bool GATHER>
__global__ void part_kernel(T *big, PartDesc d, int64_t total) {
  typedef typename std::conditional<sizeof(T) == 4, float4, char4>::type VT;
  const int64_t inner = d.dim[d.rank - 1] / V;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i;
    int64_t coord[kMaxRank];
    coord[d.rank - 1] = (rem % inner) * V;
    rem /= inner;
    for (int k = d.rank - 2; k >= 0; --k) {
      coord[k] = rem % d.dim[k];
      rem /= d.dim[k];
    }
    const int64_t a = coord[d.axis_pos];
    int p = 0;
    while (p + 1 < d.parts && a >= d.begin[p + 1]) ++p;
    int64_t ob = 0, op = 0;
    for (int k = 0; k < d.rank; ++k) {
      ob += coord[k] * d.big_stride[k];
      op += (k == d.axis_pos ? a - d.begin[p] : coord[k]) * d.part_stride[p][k];
    }
    T *part = static_cast<T *>(d.ptr[p]);
    if (V == 4) {
      if (GATHER)
        *reinterpret_cast<VT *>(big + ob) = *reinterpret_cast<const VT *>(part + op);
      else
        *reinterpret_cast<VT *>(part + op) = *reinterpret_cast<const VT *>(big + ob);
    } else {
      if (GATHER)
        big[ob] = part[op];
      else
        part[op] = big[ob];
    }
  }
}

int prepare_parts(Spkv2Context *ctx, const Spkv2NodeRecord *node, bool concat) {
  Spkv2AttrRecord attr;
  int rc = get_attr(ctx, node, &attr);
  if (rc) return rc;
  const uint16_t nparts = concat ? node->input_count : node->output_count;
  if (nparts < 1 || nparts > kMaxParts) return SPKV2_ERR_UNSUPPORTED;
  const TensorState &big = ctx->tensors[concat ? node->outputs[0] : node->inputs[0]];
  const int rank = big.record->rank;
  const int axis = attr.axis < 0 ? attr.axis + rank : attr.axis;
  if (axis < 0 || axis >= rank) return -11;
  const View vb = make_view(big);
  int order[kMaxRank];
  for (int i = 0; i < rank; ++i) order[i] = i;
  std::stable_sort(order, order + rank, [&](int a, int b) { return vb.stride[a] > vb.stride[b]; });
  PartPlan *p = new PartPlan();
  PartDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  d.rank = rank;
  d.parts = nparts;
  for (int j = 0; j < rank; ++j) {
    d.dim[j] = vb.dim[order[j]];
    d.big_stride[j] = vb.stride[order[j]];
    if (order[j] == axis) d.axis_pos = j;
  }
  const size_t esize = dtype_size(big.record->dtype);
  // Four elements per thread need: big innermost stride 1 and extent % 4,
  // every other stride of every tensor % 4, parts contiguous innermost,
  // part extents along an innermost axis % 4, 4-element-aligned pointers.
  bool vec = d.big_stride[rank - 1] == 1 && d.dim[rank - 1] % 4 == 0 &&
             reinterpret_cast<uintptr_t>(big.data) % (4 * esize) == 0;
  for (int j = 0; j + 1 < rank; ++j) vec = vec && d.big_stride[j] % 4 == 0;
  int64_t off = 0;
  for (int k = 0; k < nparts; ++k) {
    const TensorState &t = ctx->tensors[concat ? node->inputs[k] : node->outputs[k]];
    if (t.record->rank != rank || t.record->dtype != big.record->dtype) {
      delete p;
      return SPKV2_ERR_UNSUPPORTED;
    }
    const View vp = make_view(t);
    for (int j = 0; j < rank; ++j)
      if (j != axis && vp.dim[j] != vb.dim[j]) {
        delete p;
        return -3;
      }
    d.begin[k] = off;
    off += vp.dim[axis];
    for (int j = 0; j < rank; ++j) d.part_stride[k][j] = vp.stride[order[j]];
    vec = vec && d.part_stride[k][rank - 1] == 1 && reinterpret_cast<uintptr_t>(t.data) % (4 * esize) == 0;
    for (int j = 0; j + 1 < rank; ++j) vec = vec && d.part_stride[k][j] % 4 == 0;
    if (d.axis_pos == rank - 1) vec = vec && vp.dim[axis] % 4 == 0;
  }
  d.begin[nparts] = off;
  if (off != vb.dim[axis]) {
    delete p;
    return -3;
  }
  p->vec = vec ? 4 : 1;
  p->esize = int(esize);
  p->total = vb.count() / p->vec;
  // Dense fast path (see PartPlan): every tensor contiguous in the big
  // tensor's physical order, 16-byte rows segments, 32-bit vector indices.
  {
    bool dense = vb.count() * int64_t(esize) / 16 < (int64_t(1) << 31) &&
                 reinterpret_cast<uintptr_t>(big.data) % 16 == 0;
    int64_t expect = 1;
    for (int j = rank - 1; j >= 0; --j) {
      dense = dense && d.big_stride[j] == expect;
      expect *= d.dim[j];
    }
    int64_t inner = 1, outer = 1;
    for (int j = d.axis_pos + 1; j < rank; ++j) inner *= d.dim[j];
    for (int j = 0; j < d.axis_pos; ++j) outer *= d.dim[j];
    for (int k = 0; k < nparts && dense; ++k) {
      const int64_t ext = d.begin[k + 1] - d.begin[k];
      int64_t pe = 1;
      for (int j = rank - 1; j >= 0; --j) {
        dense = dense && d.part_stride[k][j] == pe;
        pe *= j == d.axis_pos ? ext : d.dim[j];
      }
      dense = dense && (ext * inner * int64_t(esize)) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(ctx->tensors[concat ? node->inputs[k] : node->outputs[k]].data) % 16 == 0;
    }
    if (dense && outer > 0) {
      p->rows_path = true;
      p->rows = uint32_t(outer);
      for (int k = 0; k <= nparts; ++k) p->seg[k] = uint32_t(d.begin[k] * inner * int64_t(esize) / 16);
      p->variant = concat ? "concat_rows16" : "split_rows16";
      set_node_plan(ctx, node, p);
      return 0;
    }
  }
  p->variant = vec ? (concat ? "concat_vec4" : "split_vec4") : (concat ? "concat" : "split");
  set_node_plan(ctx, node, p);
  return 0;
}

template <bool GATHER>
int run_parts(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  PartPlan *p = node_plan<PartPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->total == 0) return 0;
  PartDesc d = p->d;
  for (int k = 0; k < d.parts; ++k) d.ptr[k] = ctx->tensors[GATHER ? node->inputs[k] : node->outputs[k]].data;
  void *big = ctx->tensors[GATHER ? node->outputs[0] : node->inputs[0]].data;
  if (p->rows_path) {
    PartRows r;
    memset(&r, 0, sizeof(r));
    r.W = p->seg[d.parts];
    uint32_t most = 0;
    for (int k = 0; k < d.parts; ++k) {
      const uint32_t wk = p->seg[k + 1] - p->seg[k];
      r.off[k] = p->seg[k];
      r.w[k] = FastDiv(wk);
      r.n[k] = p->rows * wk;
      r.ptr[k] = d.ptr[k];
      most = std::max(most, r.n[k]);
    }
    if (most == 0) return 0;
    const dim3 grid(unsigned((most + kRowsPerBlock - 1) / kRowsPerBlock), unsigned(d.parts));
    rows_kernel<GATHER><<<grid, kRowsThreads, 0, ctx->stream>>>(static_cast<uint4 *>(big), r);
    return cuda_status(cudaGetLastError());
  }
  const int g = grid_for(p->total, 256);
  if (p->esize == 1) {
    if (p->vec == 4)
      part_kernel<int8_t, 4, GATHER><<<g, 256, 0, ctx->stream>>>(static_cast<int8_t *>(big), d, p->total);
    else
      part_kernel<int8_t, 1, GATHER><<<g, 256, 0, ctx->stream>>>(static_cast<int8_t *>(big), d, p->total);
  } else {
    if (p->vec == 4)
      part_kernel<float, 4, GATHER><<<g, 256, 0, ctx->stream>>>(static_cast<float *>(big), d, p->total);
    else
      part_kernel<float, 1, GATHER><<<g, 256, 0, ctx->stream>>>(static_cast<float *>(big), d, p->total);
  }
  return cuda_status(cudaGetLastError());
}

// ---------------- strided gather copy (Transpose, Tile) ----------------

struct GatherDesc {
  int rank;
  int64_t dim[kMaxRank];      // output dims in output physical order
  int64_t ostride[kMaxRank];  // output strides
  int64_t istride[kMaxRank];  // input stride per output dim
  int64_t imod[kMaxRank];     // input coordinate = output coordinate mod imod
};

struct GatherPlan : NodePlan {
  GatherDesc d;
  int esize = 4;
  int64_t total = 0;
  int64_t x_offset = 0;  // elements: Slice's start along its axis
};

template <typename T>
__global__ void gather_copy_kernel(T *__restrict__ y, const T *__restrict__ x, GatherDesc d, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, oy = 0, ox = 0;
    for (int k = d.rank - 1; k >= 0; --k) {
      const int64_t c = rem % d.dim[k];
      rem /= d.dim[k];
      oy += c * d.ostride[k];
      ox += (c % d.imod[k]) * d.istride[k];
    }
    y[oy] = x[ox];
  }
}

// perm[d] = input dim feeding output dim d; tile=true uses the modulus.
// Slice: output coordinate c of dim `step_dim` reads input coordinate
// start + c * step (step >= 1).
int prepare_gather(Spkv2Context *ctx, const Spkv2NodeRecord *node, const int *perm, bool tile, const char *name,
                   int step_dim = -1, int64_t start = 0, int64_t step = 1) {
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.record->dtype != ty.record->dtype || tx.record->rank != ty.record->rank) return SPKV2_ERR_UNSUPPORTED;
  const View vx = make_view(tx), vy = make_view(ty);
  const int rank = vy.rank;
  int order[kMaxRank];
  for (int i = 0; i < rank; ++i) order[i] = i;
  std::stable_sort(order, order + rank, [&](int a, int b) { return vy.stride[a] > vy.stride[b]; });
  GatherPlan *p = new GatherPlan();
  GatherDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  d.rank = rank;
  for (int j = 0; j < rank; ++j) {
    const int od = order[j];
    const int id = perm[od];
    if (id < 0 || id >= rank) {
      delete p;
      return -11;
    }
    d.dim[j] = vy.dim[od];
    d.ostride[j] = vy.stride[od];
    d.istride[j] = vx.stride[id] * (od == step_dim ? step : 1);
    d.imod[j] = tile ? std::max<int64_t>(vx.dim[id], 1) : std::max<int64_t>(vy.dim[od], 1);
  }
  if (step_dim >= 0) p->x_offset = start * vx.stride[perm[step_dim]];
  p->esize = int(dtype_size(ty.record->dtype));
  p->total = vy.count();
  p->variant = name;
  set_node_plan(ctx, node, p);
  return 0;
}

int run_gather(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  GatherPlan *p = node_plan<GatherPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->total == 0) return 0;
  void *y = ctx->tensors[node->outputs[0]].data;
  const uint8_t *x = ctx->tensors[node->inputs[0]].data + p->x_offset * p->esize;
  const int g = grid_for(p->total, 256);
  if (p->esize == 1)
    gather_copy_kernel<uint8_t><<<g, 256, 0, ctx->stream>>>(static_cast<uint8_t *>(y), x, p->d, p->total);
  else
    gather_copy_kernel<uint32_t><<<g, 256, 0, ctx->stream>>>(static_cast<uint32_t *>(y),
                                                             reinterpret_cast<const uint32_t *>(x), p->d, p->total);
  return cuda_status(cudaGetLastError());
}

// ---------------- GatherElements ----------------

struct GEDesc {
  int rank;
  int axis;
  int64_t dim[kMaxRank];      // output (= index) dims, logical order
  int64_t ystride[kMaxRank];
  int64_t istride[kMaxRank];
  int64_t dstride[kMaxRank];
  int64_t axis_dim;
};

struct GEPlan : NodePlan {
  GEDesc d;
  int64_t total = 0;
};

constexpr int kIndexRangeCode = 10;  // device status code: an index outside [-dim, dim)

__global__ void gather_elements_kernel(float *__restrict__ y, const float *__restrict__ data,
                                       const float *__restrict__ idx, GEDesc d, int64_t total, int *status) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, oy = 0, oi = 0, od = 0;
    int64_t coord[kMaxRank];
    for (int k = d.rank - 1; k >= 0; --k) {
      coord[k] = rem % d.dim[k];
      rem /= d.dim[k];
      oy += coord[k] * d.ystride[k];
      oi += coord[k] * d.istride[k];
    }
    int64_t g = int64_t(idx[oi]);
    if (g < 0) g += d.axis_dim;
    if (g < 0 || g >= d.axis_dim) {
      y[oy] = 0.0f;
      atomicCAS(status, 0, kIndexRangeCode);
      continue;
    }
    coord[d.axis] = g;
    for (int k = 0; k < d.rank; ++k) od += coord[k] * d.dstride[k];
    y[oy] = data[od];
  }
}

// ---------------- Gather (one index tensor along one axis) ----------------

struct GatherIdxDesc {
  int rank;                   // output rank (data rank - 1 + index rank)
  int64_t dim[kMaxRank];      // output dims in output physical order
  int64_t ystride[kMaxRank];  // output strides
  int64_t dstride[kMaxRank];  // data strides of the data dims (0 on index dims)
  int64_t istride[kMaxRank];  // index-tensor strides of the index dims (0 elsewhere)
  int64_t axis_stride;        // data stride along the gather axis
  int64_t axis_dim;
};

struct GatherIdxPlan : NodePlan {
  GatherIdxDesc d;
  int esize = 4;
  int64_t total = 0;
};

template <typename T>
__global__ void gather_index_kernel(T *__restrict__ y, const T *__restrict__ data, const float *__restrict__ idx,
                                    GatherIdxDesc d, int64_t total, int *status) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, oy = 0, od = 0, oi = 0;
    for (int k = d.rank - 1; k >= 0; --k) {
      const int64_t c = rem % d.dim[k];
      rem /= d.dim[k];
      oy += c * d.ystride[k];
      od += c * d.dstride[k];
      oi += c * d.istride[k];
    }
    int64_t g = int64_t(idx[oi]);
    if (g < 0) g += d.axis_dim;
    if (g < 0 || g >= d.axis_dim) {
      y[oy] = T(0);
      atomicCAS(status, 0, kIndexRangeCode);
      continue;
    }
    y[oy] = data[od + g * d.axis_stride];
  }
}

}  // namespace

int concat_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->output_count < 1) return -3;
  return prepare_parts(ctx, node, true);
}
int concat_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) { return run_parts<true>(ctx, node); }

int split_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 1) return -3;
  return prepare_parts(ctx, node, false);
}
int split_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) { return run_parts<false>(ctx, node); }

int transpose_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 1 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  int perm[kMaxRank];
  const int rank = ctx->tensors[node->outputs[0]].record->rank;
  for (int i = 0; i < rank; ++i) perm[i] = a.extra_count > 0 ? a.extra[i] : i;
  return prepare_gather(ctx, node, perm, false, "transpose");
}
int transpose_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) { return run_gather(ctx, node); }

int tile_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 1 || node->output_count < 1) return -3;
  int perm[kMaxRank];
  for (int i = 0; i < kMaxRank; ++i) perm[i] = i;
  return prepare_gather(ctx, node, perm, true, "tile");
}
int tile_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) { return run_gather(ctx, node); }

int gather_elements_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 2 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &td = ctx->tensors[node->inputs[0]];
  const TensorState &ti = ctx->tensors[node->inputs[1]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (td.record->dtype != SPKV2_DTYPE_FP32 || ti.record->dtype != SPKV2_DTYPE_FP32 ||
      ty.record->dtype != SPKV2_DTYPE_FP32)
    return SPKV2_ERR_UNSUPPORTED;
  const int rank = td.record->rank;
  const int axis = a.axis < 0 ? a.axis + rank : a.axis;
  if (axis < 0 || axis >= rank || ti.record->rank != rank || ty.record->rank != rank) return -11;
  const View vd = make_view(td), vi = make_view(ti), vy = make_view(ty);
  GEPlan *p = new GEPlan();
  GEDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  d.rank = rank;
  d.axis = axis;
  d.axis_dim = vd.dim[axis];
  for (int k = 0; k < rank; ++k) {
    d.dim[k] = vi.dim[k];
    d.ystride[k] = vy.stride[k];
    d.istride[k] = vi.stride[k];
    d.dstride[k] = vd.stride[k];
  }
  p->total = vi.count();
  p->variant = "gather_elements";
  set_node_plan(ctx, node, p);
  return 0;
}

int gather_elements_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  GEPlan *p = node_plan<GEPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->total == 0) return 0;
  gather_elements_kernel<<<grid_for(p->total, 256), 256, 0, ctx->stream>>>(
      reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data),
      reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data),
      reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data), p->d, p->total, ctx->d_status);
  return cuda_status(cudaGetLastError());
}

namespace {

// Optional input k of a node is present when the node lists it and the slot
// is not the 0xFFFF "absent" marker (reference tensor/slice.c:20-30).
bool has_input(const Spkv2NodeRecord *node, int k) { return node->input_count > k && node->inputs[k] != 0xFFFF; }

// First value of a constant fp32 input, if it is one.
bool first_const(const Spkv2Context *ctx, uint32_t tid, float *v) {
  size_t n = 0;
  const float *p = host_weight_f32(ctx, tid, &n);
  if (!p || n < 1) return false;
  *v = p[0];
  return true;
}

}  // namespace

int slice_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 3 || node->output_count < 1) return -3;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  const int rank = tx.record->rank;
  if (ty.record->rank != rank || rank < 1 || rank > kMaxRank) return -11;
  float fs = 0, fe = 0, fa = 0, fst = 1;
  // starts / ends / axes / steps must be package constants: the kernel's
  // geometry is fixed at prepare.
  if (!first_const(ctx, node->inputs[1], &fs) || !first_const(ctx, node->inputs[2], &fe)) return SPKV2_ERR_UNSUPPORTED;
  if (has_input(node, 3) && !first_const(ctx, node->inputs[3], &fa)) return SPKV2_ERR_UNSUPPORTED;
  if (has_input(node, 4) && !first_const(ctx, node->inputs[4], &fst)) return SPKV2_ERR_UNSUPPORTED;
  int64_t start = int64_t(fs), end = int64_t(fe), step = int64_t(int(fst));
  int axis = int(fa);
  if (axis < 0) axis += rank;
  if (axis < 0 || axis >= rank) return -11;
  if (step < 1) return SPKV2_ERR_UNSUPPORTED;  // the reference's extent formula assumes a positive step
  const int64_t dim = tx.record->shape[axis];
  if (start < 0) start += dim;
  if (end < 0) end += dim;
  if (end > dim) end = dim;
  if (start < 0) start = 0;
  const int64_t out = std::max<int64_t>(0, (end - start + step - 1) / step);
  for (int k = 0; k < rank; ++k)
    if (int64_t(ty.record->shape[k]) != (k == axis ? out : int64_t(tx.record->shape[k]))) return -3;
  if (out > 0 && start + (out - 1) * step >= dim) return -3;
  if (tx.record->dtype != ty.record->dtype) return SPKV2_ERR_UNSUPPORTED;
  int perm[kMaxRank];
  for (int i = 0; i < rank; ++i) perm[i] = i;
  return prepare_gather(ctx, node, perm, false, "slice", axis, start, step);
}
int slice_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) { return run_gather(ctx, node); }

int gather_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 2 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &td = ctx->tensors[node->inputs[0]];
  const TensorState &ti = ctx->tensors[node->inputs[1]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (ti.record->dtype != SPKV2_DTYPE_FP32 || td.record->dtype != ty.record->dtype) return SPKV2_ERR_UNSUPPORTED;
  const size_t esize = dtype_size(td.record->dtype);
  if (esize != 1 && esize != 4) return SPKV2_ERR_UNSUPPORTED;
  const int dr = td.record->rank, ir = ti.record->rank, yr = ty.record->rank;
  const int axis = a.axis < 0 ? a.axis + dr : a.axis;
  if (axis < 0 || axis >= dr || yr != dr - 1 + ir || yr > kMaxRank || yr < 1) return -11;
  const View vd = make_view(td), vi = make_view(ti), vy = make_view(ty);
  // Logical output dim k: data dim k (k < axis), index dim k - axis, or data
  // dim k - ir + 1.
  int64_t dstr[kMaxRank] = {}, istr[kMaxRank] = {};
  for (int k = 0; k < yr; ++k) {
    int64_t want;
    if (k < axis) {
      want = vd.dim[k];
      dstr[k] = vd.stride[k];
    } else if (k < axis + ir) {
      want = vi.dim[k - axis];
      istr[k] = vi.stride[k - axis];
    } else {
      want = vd.dim[k - ir + 1];
      dstr[k] = vd.stride[k - ir + 1];
    }
    if (vy.dim[k] != want) return -3;
  }
  // Constant indices are checked here, once; activations on the device.
  size_t n = 0;
  if (const float *iv = host_weight_f32(ctx, node->inputs[1], &n)) {
    for (size_t j = 0; j < n; ++j) {
      int64_t g = int64_t(iv[j]);
      if (g < 0) g += vd.dim[axis];
      if (g < 0 || g >= vd.dim[axis]) return -3;
    }
  }
  int order[kMaxRank];
  for (int i = 0; i < yr; ++i) order[i] = i;
  std::stable_sort(order, order + yr, [&](int x, int y) { return vy.stride[x] > vy.stride[y]; });
  GatherIdxPlan *p = new GatherIdxPlan();
  GatherIdxDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  d.rank = yr;
  for (int j = 0; j < yr; ++j) {
    d.dim[j] = vy.dim[order[j]];
    d.ystride[j] = vy.stride[order[j]];
    d.dstride[j] = dstr[order[j]];
    d.istride[j] = istr[order[j]];
  }
  d.axis_stride = vd.stride[axis];
  d.axis_dim = vd.dim[axis];
  p->esize = int(esize);
  p->total = vy.count();
  p->variant = "gather_index";
  set_node_plan(ctx, node, p);
  return 0;
}

int gather_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  GatherIdxPlan *p = node_plan<GatherIdxPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->total == 0) return 0;
  void *y = ctx->tensors[node->outputs[0]].data;
  const void *x = ctx->tensors[node->inputs[0]].data;
  const float *idx = reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data);
  const int g = grid_for(p->total, 256);
  if (p->esize == 1)
    gather_index_kernel<uint8_t><<<g, 256, 0, ctx->stream>>>(static_cast<uint8_t *>(y), static_cast<const uint8_t *>(x),
                                                             idx, p->d, p->total, ctx->d_status);
  else
    gather_index_kernel<uint32_t><<<g, 256, 0, ctx->stream>>>(
        static_cast<uint32_t *>(y), static_cast<const uint32_t *>(x), idx, p->d, p->total, ctx->d_status);
  return cuda_status(cudaGetLastError());
}

}  // namespace spkv2
