// Elementwise ops (Add/Sub/Mul/Div/Mod with broadcast, Relu, Sigmoid, Clip,
// LeakyRelu), shape-only copies (Flatten/Reshape/Unsqueeze/Cast), the
// fault-injection bit flip and host<->device tensor transfer.
//
// Semantics follow the reference kernels:
//   Add  reference/math/add.c:3-20        y = act(a + b), numpy broadcast
//   Sub/Mul/Div/Mod reference/math/binary.c:3-33 (Mod on truncated ints)
//   Relu reference/activation/relu.c      y = x > 0 ? x : 0
//   Sigmoid reference/activation/sigmoid.c y = 1 / (1 + expf(-x))
//   Clip/LeakyRelu reference/activation/clip_leakyrelu.c
//   Flatten/Reshape/Cast/Unsqueeze reference/shape/{flatten,copy,unsqueeze}.c:
//     the output is the input's elements in logical row-major order.
// Device design: memory-bound, so one pass over the output in its physical
// order with 128-bit accesses on the contiguous fast path, a grid-stride loop
// sized to the SM count, and strided gathers for broadcast or mixed layouts.
#include <string.h>

#include "common.cuh"

namespace spkv2 {

namespace {

enum EltOp : int { kAdd, kSub, kMul, kDiv, kMod, kRelu, kSigmoid, kClip, kLeakyRelu };

struct EltPlan : NodePlan {
  int op = kAdd;
  int act = 0;
  float alpha = 0.01f;
  bool fast = false;  // all operands contiguous with identical views
  IterSpace<3> it;
  int64_t count = 0;
};

__device__ __forceinline__ float elt_apply(int op, float a, float b, int act, float alpha, float lo, float hi) {
  switch (op) {
    case kAdd: return apply_act(a + b, act);
    case kSub: return a - b;
    case kMul: return a * b;
    case kDiv: return a / b;
    case kMod: return float(int(a) % int(b));
    case kRelu: return a > 0.0f ? a : 0.0f;
    case kSigmoid: return 1.0f / (1.0f + expf(-a));
    case kClip: {
      float v = a;
      if (v < lo) v = lo;
      if (v > hi) v = hi;
      return v;
    }
    case kLeakyRelu: return a >= 0.0f ? a : a * alpha;
  }
  return a;
}

__global__ void elt_fast_kernel(float *__restrict__ y, const float *__restrict__ a, const float *__restrict__ b,
                                int64_t n, int op, int act, float alpha, const float *lo_p, const float *hi_p) {
  const float lo = lo_p ? *lo_p : -INFINITY;
  const float hi = hi_p ? *hi_p : INFINITY;
  const int64_t n4 = n / 4;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(a) |
                     (b ? reinterpret_cast<uintptr_t>(b) : 0)) & 15) == 0;
  int64_t start = 0;
  if (vec) {
    // Four float4s per thread per pass, all loads issued before any math:
    // a unary op (one input stream) otherwise keeps only one 16-byte load
    // in flight per thread, too few to cover HBM latency.
    constexpr int U = 4;
    const float4 *a4 = reinterpret_cast<const float4 *>(a);
    const float4 *b4 = reinterpret_cast<const float4 *>(b);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    for (int64_t i0 = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i0 < n4; i0 += U * stride) {
      float4 va[U], vb[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * stride;
        va[u] = i < n4 ? __ldg(a4 + i) : make_float4(0, 0, 0, 0);
        vb[u] = b && i < n4 ? __ldg(b4 + i) : make_float4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < n4) {
          float4 r;
          r.x = elt_apply(op, va[u].x, vb[u].x, act, alpha, lo, hi);
          r.y = elt_apply(op, va[u].y, vb[u].y, act, alpha, lo, hi);
          r.z = elt_apply(op, va[u].z, vb[u].z, act, alpha, lo, hi);
          r.w = elt_apply(op, va[u].w, vb[u].w, act, alpha, lo, hi);
          y4[i] = r;
        }
      }
    }
    start = n4 * 4;
  }
  for (int64_t i = start + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += stride)
    y[i] = elt_apply(op, a[i], b ? b[i] : 0.0f, act, alpha, lo, hi);
}

__global__ void elt_strided_kernel(float *__restrict__ y, const float *__restrict__ a, const float *__restrict__ b,
                                   IterSpace<3> it, int64_t n, int op, int act, float alpha, const float *lo_p,
                                   const float *hi_p) {
  const float lo = lo_p ? *lo_p : -INFINITY;
  const float hi = hi_p ? *hi_p : INFINITY;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, oy = 0, oa = 0, ob = 0;
    for (int d = it.rank - 1; d >= 0; --d) {
      const int64_t c = rem % it.dim[d];
      rem /= it.dim[d];
      oy += c * it.stride[0][d];
      oa += c * it.stride[1][d];
      ob += c * it.stride[2][d];
    }
    y[oy] = elt_apply(op, a[oa], b ? b[ob] : 0.0f, act, alpha, lo, hi);
  }
}

bool same_view(const View &x, const View &y) {
  if (x.rank != y.rank) return false;
  for (int i = 0; i < x.rank; ++i)
    if (x.dim[i] != y.dim[i] || (x.dim[i] != 1 && x.stride[i] != y.stride[i])) return false;
  return true;
}

// ---------------- logical-order copy between layouts ----------------

// Physical element offset of logical row-major element `e` in a rank-4
// tensor [N,C,H,W] stored NHWC.
__device__ __forceinline__ int64_t nhwc_offset(int64_t e, int64_t C, int64_t H, int64_t W) {
  const int64_t w = e % W;
  int64_t r = e / W;
  const int64_t h = r % H;
  r /= H;
  const int64_t c = r % C;
  const int64_t n = r / C;
  return ((n * H + h) * W + w) * C + c;
}

// dst[phys_out(e)] = src[phys_in(e)] for every logical element e; each side
// is row-major or NHWC with its own [C,H,W].
template <typename T>
__global__ void relayout_kernel(T *__restrict__ dst, const T *__restrict__ src, int64_t n, int in_nhwc,
                                int64_t iC, int64_t iH, int64_t iW, int out_nhwc, int64_t oC, int64_t oH,
                                int64_t oW) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t si = in_nhwc ? nhwc_offset(e, iC, iH, iW) : e;
    const int64_t di = out_nhwc ? nhwc_offset(e, oC, oH, oW) : e;
    dst[di] = src[si];
  }
}

// NHWC -> NCHW (and back) through a shared-memory tile of kTransP positions x
// 32 channels, so both the reads and the writes are coalesced; used for host
// transfers and for copies between an NHWC and a row-major view.  A block is
// 32 x 8 threads; each thread moves kTransP / 8 elements, all its global loads
// issued before its first shared-memory store (the loops are unrolled), so a
// block keeps 8 KB of loads in flight.  Row stride 33 keeps both the row and
// the column accesses of the tile free of bank conflicts.
constexpr int kTransP = 64;

template <typename T>
__global__ void __launch_bounds__(256) transpose_hw_c_kernel(T *__restrict__ dst, const T *__restrict__ src, int64_t N,
                                                             int64_t P, int64_t C, int to_nchw) {
  __shared__ T tile[kTransP][33];  // [position][channel]
  constexpr int kRows = kTransP / 8;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t n = blockIdx.z;
  const int64_t p0 = int64_t(blockIdx.x) * kTransP, c0 = int64_t(blockIdx.y) * 32;
  if (to_nchw) {  // src [N,P,C] -> dst [N,C,P]
    const int64_t c = c0 + tx;
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = ty + 8 * i;  // tile position
      if (p0 + r < P && c < C) tile[r][tx] = src[(n * P + p0 + r) * C + c];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int j = ty + 8 * i, cl = j % 32, pl = (j / 32) * 32 + tx;
      if (p0 + pl < P && c0 + cl < C) dst[(n * C + c0 + cl) * P + p0 + pl] = tile[pl][cl];
    }
  } else {  // src [N,C,P] -> dst [N,P,C]
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int j = ty + 8 * i, cl = j % 32, pl = (j / 32) * 32 + tx;
      if (p0 + pl < P && c0 + cl < C) tile[pl][cl] = src[(n * C + c0 + cl) * P + p0 + pl];
    }
    __syncthreads();
    const int64_t c = c0 + tx;
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = ty + 8 * i;
      if (p0 + r < P && c < C) dst[(n * P + p0 + r) * C + c] = tile[r][tx];
    }
  }
}

// 4-byte elements with C % 4 == 0, P % 4 == 0 and 16-byte aligned tensors:
// 16-byte accesses on both sides.  A block moves a tile of 32 channels x 128
// positions (16 KB) through shared memory held channel-major, tile[c][p];
// the NHWC side moves 4 channels of one position per float4 (a warp covers
// 4 positions x 32 channels, four 128-byte rows), the [N, C, P] side 4
// positions of one channel per float4 (a warp covers one 512-byte channel
// run).  The position quads of channel row c are stored XOR-swizzled by
// (c / 4) % 8, so the scalar side's 32 lanes (8 channel quads x 4
// positions) hit 32 distinct banks and the float4 side still reads or
// writes whole 16-byte groups.  Four float4s per thread, loads first.
constexpr int kTrP4 = 128;

__device__ __forceinline__ int tr_col(int c, int p) { return ((((p >> 2) ^ ((c >> 2) & 7))) << 2) | (p & 3); }

__global__ void __launch_bounds__(256) transpose_hw_c_vec_kernel(float *__restrict__ dst, const float *__restrict__ src,
                                                                 int64_t P, int64_t C, int to_nchw) {
  __shared__ __align__(16) float tile[32][kTrP4];
  const int t = threadIdx.x;
  const int64_t n = blockIdx.z;
  const int64_t p0 = int64_t(blockIdx.x) * kTrP4, c0 = int64_t(blockIdx.y) * 32;
  float4 v[4];
  if (to_nchw) {  // src [N,P,C] -> dst [N,C,P]
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, pl = f >> 3, cq = f & 7;
      const bool in = p0 + pl < P && c0 + 4 * cq < C;
      v[i] = in ? __ldg(reinterpret_cast<const float4 *>(src + (n * P + p0 + pl) * C + c0 + 4 * cq))
                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, pl = f >> 3, c = 4 * (f & 7);
      tile[c][tr_col(c, pl)] = v[i].x;
      tile[c + 1][tr_col(c + 1, pl)] = v[i].y;
      tile[c + 2][tr_col(c + 2, pl)] = v[i].z;
      tile[c + 3][tr_col(c + 3, pl)] = v[i].w;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, c = f >> 5, q = f & 31;
      if (c0 + c < C && p0 + 4 * q < P)
        *reinterpret_cast<float4 *>(dst + (n * C + c0 + c) * P + p0 + 4 * q) =
            *reinterpret_cast<const float4 *>(&tile[c][tr_col(c, 4 * q)]);
    }
  } else {  // src [N,C,P] -> dst [N,P,C]
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, c = f >> 5, q = f & 31;
      const bool in = c0 + c < C && p0 + 4 * q < P;
      v[i] = in ? __ldg(reinterpret_cast<const float4 *>(src + (n * C + c0 + c) * P + p0 + 4 * q))
                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, c = f >> 5, q = f & 31;
      *reinterpret_cast<float4 *>(&tile[c][tr_col(c, 4 * q)]) = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = t + 256 * i, pl = f >> 3, c = 4 * (f & 7);
      if (p0 + pl < P && c0 + c < C)
        *reinterpret_cast<float4 *>(dst + (n * P + p0 + pl) * C + c0 + c) =
            make_float4(tile[c][tr_col(c, pl)], tile[c + 1][tr_col(c + 1, pl)], tile[c + 2][tr_col(c + 2, pl)],
                        tile[c + 3][tr_col(c + 3, pl)]);
    }
  }
}

template <typename T>
int launch_transpose_hw_c(T *dst, const T *src, const Spkv2TensorRecord *r, int to_nchw, cudaStream_t s) {
  const int64_t N = r->shape[0], C = r->shape[1], P = int64_t(r->shape[2]) * r->shape[3];
  if (N > 65535 || ceil_div(C, 32) > 65535) return SPKV2_ERR_UNSUPPORTED;
  if (sizeof(T) == 4 && C % 4 == 0 && P % 4 == 0 &&
      ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
    dim3 grid(unsigned(ceil_div(P, kTrP4)), unsigned(ceil_div(C, 32)), unsigned(N));
    transpose_hw_c_vec_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<float *>(dst), reinterpret_cast<const float *>(src),
                                                   P, C, to_nchw);
    return cuda_status(cudaGetLastError());
  }
  dim3 grid(unsigned(ceil_div(P, kTransP)), unsigned(ceil_div(C, 32)), unsigned(N));
  transpose_hw_c_kernel<T><<<grid, dim3(32, 8), 0, s>>>(dst, src, N, P, C, to_nchw);
  return cuda_status(cudaGetLastError());
}

struct CopyPlan : NodePlan {
  bool same_storage = false;
};

__global__ void bit_flip_kernel(uint32_t *word, uint32_t mask) { *word ^= mask; }

}  // namespace

// ---------------- Elementwise ----------------

int eltwise_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  (void)spec;
  EltPlan *p = new EltPlan();
  switch (node->op_type) {
    case SPKV2_OP_ADD: p->op = kAdd; break;
    case SPKV2_OP_SUB: p->op = kSub; break;
    case SPKV2_OP_MUL: p->op = kMul; break;
    case SPKV2_OP_DIV: p->op = kDiv; break;
    case SPKV2_OP_MOD: p->op = kMod; break;
    case SPKV2_OP_RELU: p->op = kRelu; break;
    case SPKV2_OP_SIGMOID: p->op = kSigmoid; break;
    case SPKV2_OP_CLIP: p->op = kClip; break;
    case SPKV2_OP_LEAKYRELU: p->op = kLeakyRelu; break;
    default: delete p; return -99;
  }
  const bool binary = p->op <= kMod;
  if (node->output_count < 1 || node->input_count < (binary ? 2 : 1)) {
    delete p;
    return -3;
  }
  Spkv2AttrRecord attr;
  memset(&attr, 0, sizeof(attr));
  attr.alpha = 0.01f;
  if (p->op == kAdd || p->op == kLeakyRelu) {
    int rc = get_attr(ctx, node, &attr);
    if (rc) {
      delete p;
      return rc;
    }
  }
  p->act = p->op == kAdd ? attr.fused_activation : 0;
  p->alpha = attr.alpha;
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  for (uint16_t i = 0; i < (binary ? 2 : 1); ++i)
    if (ctx->tensors[node->inputs[i]].record->dtype != SPKV2_DTYPE_FP32) {
      delete p;
      return SPKV2_ERR_UNSUPPORTED;
    }
  if (ty.record->dtype != SPKV2_DTYPE_FP32) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }
  View vy = make_view(ty);
  View vin[2];
  vin[0] = make_view(ctx->tensors[node->inputs[0]]);
  if (binary) vin[1] = make_view(ctx->tensors[node->inputs[1]]);
  p->count = vy.count();
  p->fast = same_view(vy, vin[0]) && (!binary || same_view(vy, vin[1])) && is_rowmajor(vy) == is_rowmajor(vin[0]);
  if (p->fast) {
    // identical views: physical order is shared, so a flat pass is exact
  }
  p->it = make_iter<3>(vy, vin, binary ? 2 : 1);
  p->variant = p->fast ? "eltwise_vec4" : "eltwise_strided";
  set_node_plan(ctx, node, p);
  return 0;
}

int eltwise_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch) {
  (void)scratch;
  EltPlan *p = node_plan<EltPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->count == 0) return 0;
  float *y = reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data);
  const float *a = reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data);
  const float *b = p->op <= kMod ? reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data) : nullptr;
  const float *lo = nullptr, *hi = nullptr;
  if (p->op == kClip) {
    if (node->input_count >= 2) lo = reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data);
    if (node->input_count >= 3) hi = reinterpret_cast<const float *>(ctx->tensors[node->inputs[2]].data);
  }
  const int threads = 256;
  if (p->fast) {
    elt_fast_kernel<<<grid_for(ceil_div(p->count, 16), threads), threads, 0, ctx->stream>>>(y, a, b, p->count, p->op,
                                                                                              p->act, p->alpha, lo, hi);
  } else {
    elt_strided_kernel<<<grid_for(p->count, threads), threads, 0, ctx->stream>>>(y, a, b, p->it, p->count, p->op,
                                                                                  p->act, p->alpha, lo, hi);
  }
  return cuda_status(cudaGetLastError());
}

// ---------------- Flatten / Reshape / Unsqueeze / Cast ----------------

int copy_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  (void)spec;
  if (node->input_count < 1 || node->output_count < 1) return -3;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.record->dtype != ty.record->dtype || tx.record->size_bytes != ty.record->size_bytes)
    return SPKV2_ERR_UNSUPPORTED;
  CopyPlan *p = new CopyPlan();
  p->same_storage = tx.data == ty.data;
  if (p->same_storage && tx.layout != ty.layout) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;  // the layout pass keeps aliased views row-major
  }
  p->launches = p->same_storage ? 0 : 1;
  p->variant = p->same_storage ? "alias" : (tx.layout == ty.layout ? "memcpy" : "relayout");
  set_node_plan(ctx, node, p);
  return 0;
}

int copy_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch) {
  (void)scratch;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.data == ty.data) return 0;
  const size_t bytes = size_t(ty.record->size_bytes);
  if (tx.layout == ty.layout) return cuda_status(cudaMemcpyAsync(ty.data, tx.data, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  const int64_t n = int64_t(elem_count(ty.record));
  const uint32_t *is = tx.record->shape, *os = ty.record->shape;
  const int in_nhwc = tx.layout == kNHWC, out_nhwc = ty.layout == kNHWC;
  // One side NHWC, the other row-major: the logical (row-major) element
  // order is shared, so the copy is a [N, H*W, C] <-> [N, C, H*W] transpose of
  // the NHWC side's dims through shared-memory tiles (both sides coalesced).
  if (in_nhwc != out_nhwc) {
    const Spkv2TensorRecord *r = in_nhwc ? tx.record : ty.record;
    if (r->rank == 4) {
      const int rc = dtype_size(ty.record->dtype) == 1
                         ? launch_transpose_hw_c(reinterpret_cast<uint8_t *>(ty.data),
                                                 reinterpret_cast<const uint8_t *>(tx.data), r, in_nhwc, ctx->stream)
                         : launch_transpose_hw_c(reinterpret_cast<uint32_t *>(ty.data),
                                                 reinterpret_cast<const uint32_t *>(tx.data), r, in_nhwc, ctx->stream);
      if (rc != SPKV2_ERR_UNSUPPORTED) return rc;
    }
  }
  if (dtype_size(ty.record->dtype) == 1) {
    relayout_kernel<uint8_t><<<grid_for(n, 256), 256, 0, ctx->stream>>>(ty.data, tx.data, n, in_nhwc, is[1], is[2],
                                                                        is[3], out_nhwc, os[1], os[2], os[3]);
  } else {
    relayout_kernel<uint32_t><<<grid_for(n, 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<uint32_t *>(ty.data), reinterpret_cast<const uint32_t *>(tx.data), n, in_nhwc, is[1], is[2],
        is[3], out_nhwc, os[1], os[2], os[3]);
  }
  return cuda_status(cudaGetLastError());
}

// ---------------- utilities ----------------

int launch_bit_flip(uint32_t *word, uint32_t mask, cudaStream_t stream) {
  bit_flip_kernel<<<1, 1, 0, stream>>>(word, mask);
  return cuda_status(cudaGetLastError());
}

int copy_tensor_to_host(const TensorState &t, void *host, cudaStream_t stream) {
  const size_t bytes = size_t(t.record->size_bytes);
  if (t.layout != kNHWC) {
    int rc = cuda_status(cudaMemcpyAsync(host, t.data, bytes, cudaMemcpyDeviceToHost, stream));
    return rc ? rc : cuda_status(cudaStreamSynchronize(stream));
  }
  void *tmp = device_alloc(bytes);
  if (!tmp) return SPKV2_ERR_DEVICE_ALLOC;
  int rc = dtype_size(t.record->dtype) == 1
               ? launch_transpose_hw_c<uint8_t>(static_cast<uint8_t *>(tmp), t.data, t.record, 1, stream)
               : launch_transpose_hw_c<uint32_t>(static_cast<uint32_t *>(tmp),
                                                 reinterpret_cast<const uint32_t *>(t.data), t.record, 1, stream);
  if (!rc) rc = cuda_status(cudaMemcpyAsync(host, tmp, bytes, cudaMemcpyDeviceToHost, stream));
  if (!rc) rc = cuda_status(cudaStreamSynchronize(stream));
  device_free(tmp);
  return rc;
}

int copy_tensor_from_host(const TensorState &t, const void *host, cudaStream_t stream) {
  const size_t bytes = size_t(t.record->size_bytes);
  if (t.layout != kNHWC) {
    int rc = cuda_status(cudaMemcpyAsync(t.data, host, bytes, cudaMemcpyHostToDevice, stream));
    return rc ? rc : cuda_status(cudaStreamSynchronize(stream));
  }
  void *tmp = device_alloc(bytes);
  if (!tmp) return SPKV2_ERR_DEVICE_ALLOC;
  int rc = cuda_status(cudaMemcpyAsync(tmp, host, bytes, cudaMemcpyHostToDevice, stream));
  if (!rc)
    rc = dtype_size(t.record->dtype) == 1
             ? launch_transpose_hw_c<uint8_t>(t.data, static_cast<const uint8_t *>(tmp), t.record, 0, stream)
             : launch_transpose_hw_c<uint32_t>(reinterpret_cast<uint32_t *>(t.data),
                                               static_cast<const uint32_t *>(tmp), t.record, 0, stream);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(stream));
  device_free(tmp);
  return rc;
}

}  // namespace spkv2
