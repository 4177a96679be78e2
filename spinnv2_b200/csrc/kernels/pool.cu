// MaxPool / AveragePool / GlobalAveragePool and nearest Resize.
//
// Semantics (reference):
//   MaxPool  reference/pool/maxpool.c:5-43   window max, padding skipped,
//            -inf when the window holds no input element
//   AveragePool reference/pool/avgpool.c     sum / (number of in-range taps)
//   GlobalAveragePool reference/pool/avgpool.c  sum * (1 / (H*W))
//   Resize   reference/shape/resize.c:5-31   nearest, asymmetric:
//            ih = min(floor(oh / (OH / H)), H - 1) in fp32
// INT8 MaxPool (quantised models) keeps the input's scale and returns the
// largest int8 code, -128 for an empty window.
// Device design: one thread per output element (four channels per thread
// when both tensors are NHWC with C % 4 == 0), iterating the output in its
// physical order so stores coalesce; NHWC reads are coalesced along C.
#include <string.h>

#include "common.cuh"

namespace spkv2 {

namespace {

struct Geo {
  int N, C, H, W, OH, OW;
  int kh, kw, sh, sw, ph, pw;
  // element strides (n, c, h, w) of input and output
  int64_t xs[4], ys[4];
};

enum PoolKind : int { kMax, kAvg, kGlobalAvg };

struct PoolPlan : NodePlan {
  Geo g;
  int kind = kMax;
  int vec = 1;
  int band = 0;  // > 0: stride-1 fp32 max pool, output rows per thread
  bool out_nhwc = false;
  bool is_int8 = false;
};

template <typename T>
struct PoolTraits;
template <>
struct PoolTraits<float> {
  __device__ static float lowest() { return -INFINITY; }
};
template <>
struct PoolTraits<int8_t> {
  __device__ static int8_t lowest() { return -128; }
};

// Output coordinate of linear index i in the output's physical order.
__device__ __forceinline__ void out_coords(int64_t i, const Geo &g, bool nhwc, int C, int &n, int &c, int &oh,
                                           int &ow) {
  if (nhwc) {
    c = int(i % C);
    i /= C;
    ow = int(i % g.OW);
    i /= g.OW;
    oh = int(i % g.OH);
    n = int(i / g.OH);
  } else {
    ow = int(i % g.OW);
    i /= g.OW;
    oh = int(i % g.OH);
    i /= g.OH;
    c = int(i % C);
    n = int(i / C);
  }
}

template <typename T>
__global__ void pool_kernel(T *__restrict__ y, const T *__restrict__ x, Geo g, int kind, bool out_nhwc,
                            int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int n, c, oh, ow;
    out_coords(i, g, out_nhwc, g.C, n, c, oh, ow);
    const T *xb = x + n * g.xs[0] + c * g.xs[1];
    float acc = 0.0f;
    T best = PoolTraits<T>::lowest();
    int count = 0;
    for (int r = 0; r < g.kh; ++r) {
      const int ih = oh * g.sh + r - g.ph;
      if (ih < 0 || ih >= g.H) continue;
      for (int s = 0; s < g.kw; ++s) {
        const int iw = ow * g.sw + s - g.pw;
        if (iw < 0 || iw >= g.W) continue;
        const T v = xb[ih * g.xs[2] + iw * g.xs[3]];
        if (kind == kMax) {
          if (v > best) best = v;
        } else {
          acc += float(v);
          ++count;
        }
      }
    }
    T out;
    if (kind == kMax)
      out = best;
    else if (kind == kAvg)
      out = T(count > 0 ? acc / float(count) : 0.0f);
    else
      out = T(acc * (1.0f / float(g.H * g.W)));
    y[n * g.ys[0] + c * g.ys[1] + oh * g.ys[2] + ow * g.ys[3]] = out;
  }
}

// Both tensors NHWC, C % 4 == 0, fp32 max pooling: one float4 of channels
// per thread.
__global__ void maxpool_nhwc4_kernel(float *__restrict__ y, const float *__restrict__ x, Geo g, int64_t total4) {
  const int C4 = g.C / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total4; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c4 = int(r % C4);
    r /= C4;
    const int ow = int(r % g.OW);
    r /= g.OW;
    const int oh = int(r % g.OH);
    const int n = int(r / g.OH);
    float4 best = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    const float *xb = x + int64_t(n) * g.H * g.W * g.C + c4 * 4;
    for (int rr = 0; rr < g.kh; ++rr) {
      const int ih = oh * g.sh + rr - g.ph;
      if (ih < 0 || ih >= g.H) continue;
      for (int s = 0; s < g.kw; ++s) {
        const int iw = ow * g.sw + s - g.pw;
        if (iw < 0 || iw >= g.W) continue;
        const float4 v = *reinterpret_cast<const float4 *>(xb + (int64_t(ih) * g.W + iw) * g.C);
        best.x = v.x > best.x ? v.x : best.x;
        best.y = v.y > best.y ? v.y : best.y;
        best.z = v.z > best.z ? v.z : best.z;
        best.w = v.w > best.w ? v.w : best.w;
      }
    }
    reinterpret_cast<float4 *>(y)[i] = best;
  }
}

// Stride-1 max pool with a square KH x KH window (the SPPF 5x5 windows), NHWC
// fp32, C % 4 == 0: thread (n, band, ow, c4) walks its output column down a
// band of `band` output rows keeping the maxima of the last KH input rows
// (each over the KH window columns) in registers, so an output costs one new
// row's KH loads instead of KH x KH.  The host picks the band height so that
// the threads fill the resident slots of the GPU about once (a whole-height
// walk is a chain of dependent rows; very short bands re-read more rows).
// Offsets within an image are 32-bit (the plan checks H*W*C < 2^31).  Max is
// order-independent, so results equal the direct window scan; rows and
// columns outside the image are skipped as there.
template <int KH>
__global__ void __launch_bounds__(128) maxpool_nhwc4_s1_kernel(float *__restrict__ y, const float *__restrict__ x,
                                                                Geo g, int band, int64_t columns) {
  const int C4 = g.C / 4;
  const int bands = (g.OH + band - 1) / band;
  const int row_elems = g.W * g.C;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < columns; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c4 = int(r % C4);
    r /= C4;
    const int ow = int(r % g.OW);
    r /= g.OW;
    const int b = int(r % bands);
    const int n = int(r / bands);
    const float *xb = x + int64_t(n) * g.H * row_elems + c4 * 4;
    float4 *yb = reinterpret_cast<float4 *>(y + int64_t(n) * g.OH * g.OW * g.C + ow * g.C + c4 * 4);
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    auto row_max = [&](int ih) {
      float4 best = ninf;
      if (ih < 0 || ih >= g.H) return best;
      const float *xr = xb + ih * row_elems;
#pragma unroll
      for (int s = 0; s < KH; ++s) {
        const int iw = ow + s - g.pw;
        if (iw < 0 || iw >= g.W) continue;
        const float4 v = *reinterpret_cast<const float4 *>(xr + iw * g.C);
        best.x = v.x > best.x ? v.x : best.x;
        best.y = v.y > best.y ? v.y : best.y;
        best.z = v.z > best.z ? v.z : best.z;
        best.w = v.w > best.w ? v.w : best.w;
      }
      return best;
    };
    const int oh0 = b * band, oh1 = min(g.OH, oh0 + band);
    float4 rm[KH];  // rm[j]: max of input row oh - ph + j
#pragma unroll
    for (int j = 0; j + 1 < KH; ++j) rm[j + 1] = row_max(oh0 + j - g.ph);
    for (int oh = oh0; oh < oh1; ++oh) {
#pragma unroll
      for (int j = 0; j + 1 < KH; ++j) rm[j] = rm[j + 1];
      rm[KH - 1] = row_max(oh - g.ph + KH - 1);
      float4 best = rm[0];
#pragma unroll
      for (int j = 1; j < KH; ++j) {
        best.x = rm[j].x > best.x ? rm[j].x : best.x;
        best.y = rm[j].y > best.y ? rm[j].y : best.y;
        best.z = rm[j].z > best.z ? rm[j].z : best.z;
        best.w = rm[j].w > best.w ? rm[j].w : best.w;
      }
      yb[int64_t(oh) * g.OW * C4] = best;
    }
  }
}

// Band height for the stride-1 kernel: as many bands per output column as
// fill the GPU's resident 128-thread blocks once, at least one row each.
template <int KH>
int s1_band(const Geo &g) {
  int dev = 0, sms = 148, per_sm = 8;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, maxpool_nhwc4_s1_kernel<KH>, 128, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 8;
  const int64_t resident = int64_t(sms) * per_sm * 128;
  const int64_t cols = int64_t(g.N) * g.OW * (g.C / 4);
  const int64_t bands = std::max<int64_t>(1, std::min<int64_t>(g.OH, resident / std::max<int64_t>(cols, 1)));
  return int((g.OH + bands - 1) / bands);
}

// Both tensors NHWC int8, C % 16 == 0: 16 channels (one 16-byte load) per
// thread, per-byte signed max on 32-bit words; an empty window gives -128.
__global__ void maxpool_nhwc16_i8_kernel(int8_t *__restrict__ y, const int8_t *__restrict__ x, Geo g,
                                         int64_t total16) {
  const int C16 = g.C / 16;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total16; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c16 = int(r % C16);
    r /= C16;
    const int ow = int(r % g.OW);
    r /= g.OW;
    const int oh = int(r % g.OH);
    const int n = int(r / g.OH);
    uint4 best = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
    const int8_t *xb = x + int64_t(n) * g.H * g.W * g.C + c16 * 16;
    for (int rr = 0; rr < g.kh; ++rr) {
      const int ih = oh * g.sh + rr - g.ph;
      if (ih < 0 || ih >= g.H) continue;
      for (int s = 0; s < g.kw; ++s) {
        const int iw = ow * g.sw + s - g.pw;
        if (iw < 0 || iw >= g.W) continue;
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(xb + (int64_t(ih) * g.W + iw) * g.C));
        best.x = __vmaxs4(best.x, v.x);
        best.y = __vmaxs4(best.y, v.y);
        best.z = __vmaxs4(best.z, v.z);
        best.w = __vmaxs4(best.w, v.w);
      }
    }
    reinterpret_cast<uint4 *>(y)[i] = best;
  }
}

void strides_of(const TensorState &t, int64_t s[4]) {
  View v = make_view(t);
  for (int i = 0; i < 4; ++i) s[i] = v.stride[i];
}

struct ResizeGeo {
  int N, C, H, W, OH, OW;
  int64_t xs[4], ys[4];
  bool out_nhwc;
};

struct ResizePlan : NodePlan {
  ResizeGeo g;
  bool vec4 = false;
  bool int_factor = false;  // OH % H == 0 and OW % W == 0
  int esize = 4;
};

template <typename T>
__global__ void resize_nearest_kernel(T *__restrict__ y, const T *__restrict__ x, ResizeGeo g, int64_t total) {
  const float scale_h = float(g.OH) / float(g.H);
  const float scale_w = float(g.OW) / float(g.W);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    int n, c, oh, ow;
    if (g.out_nhwc) {
      c = int(r % g.C);
      r /= g.C;
      ow = int(r % g.OW);
      r /= g.OW;
      oh = int(r % g.OH);
      n = int(r / g.OH);
    } else {
      ow = int(r % g.OW);
      r /= g.OW;
      oh = int(r % g.OH);
      r /= g.OH;
      c = int(r % g.C);
      n = int(r / g.C);
    }
    int ih = int(floorf(float(oh) / scale_h));
    if (ih >= g.H) ih = g.H - 1;
    int iw = int(floorf(float(ow) / scale_w));
    if (iw >= g.W) iw = g.W - 1;
    y[n * g.ys[0] + c * g.ys[1] + oh * g.ys[2] + ow * g.ys[3]] =
        x[n * g.xs[0] + c * g.xs[1] + ih * g.xs[2] + iw * g.xs[3]];
  }
}

__global__ void resize_nearest_nhwc4_kernel(float4 *__restrict__ y, const float4 *__restrict__ x, ResizeGeo g,
                                            int64_t total4) {
  const float scale_h = float(g.OH) / float(g.H);
  const float scale_w = float(g.OW) / float(g.W);
  const int C4 = g.C / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total4; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c4 = int(r % C4);
    r /= C4;
    const int ow = int(r % g.OW);
    r /= g.OW;
    const int oh = int(r % g.OH);
    const int n = int(r / g.OH);
    int ih = int(floorf(float(oh) / scale_h));
    if (ih >= g.H) ih = g.H - 1;
    int iw = int(floorf(float(ow) / scale_w));
    if (iw >= g.W) iw = g.W - 1;
    y[i] = x[((int64_t(n) * g.H + ih) * g.W + iw) * C4 + c4];
  }
}

// Integer scale factors (OH = fh * H, OW = fw * W), NHWC fp32, C % 4 == 0:
// thread (n, ih, iw, c4) reads its input float4 once and writes the fh x fw
// outputs it feeds.  For these factors floor(oh / (OH / H)) in fp32 equals
// oh / fh, so the outputs are those of the per-output index formula.
__global__ void resize_nearest_int_nhwc4_kernel(float4 *__restrict__ y, const float4 *__restrict__ x, ResizeGeo g,
                                                int fh, int fw, int64_t in4) {
  const int C4 = g.C / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < in4; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int c4 = int(r % C4);
    r /= C4;
    const int iw = int(r % g.W);
    r /= g.W;
    const int ih = int(r % g.H);
    const int n = int(r / g.H);
    const float4 v = x[i];
    float4 *yb = y + ((int64_t(n) * g.OH + int64_t(ih) * fh) * g.OW + int64_t(iw) * fw) * C4 + c4;
    for (int a = 0; a < fh; ++a)
      for (int b = 0; b < fw; ++b) yb[(int64_t(a) * g.OW + b) * C4] = v;
  }
}

}  // namespace

int pool_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  (void)spec;
  if (node->input_count < 1 || node->output_count < 1) return -3;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.record->rank != 4 || ty.record->rank != 4) return -11;
  if (tx.record->dtype != ty.record->dtype) return SPKV2_ERR_UNSUPPORTED;
  const bool is_int8 = tx.record->dtype == SPKV2_DTYPE_INT8;
  if (!is_int8 && tx.record->dtype != SPKV2_DTYPE_FP32) return SPKV2_ERR_UNSUPPORTED;
  PoolPlan *p = new PoolPlan();
  p->kind = node->op_type == SPKV2_OP_MAXPOOL ? kMax : node->op_type == SPKV2_OP_AVERAGEPOOL ? kAvg : kGlobalAvg;
  if (is_int8 && p->kind != kMax) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }
  Geo &g = p->g;
  memset(&g, 0, sizeof(g));
  g.N = int(tx.record->shape[0]);
  g.C = int(tx.record->shape[1]);
  g.H = int(tx.record->shape[2]);
  g.W = int(tx.record->shape[3]);
  g.OH = int(ty.record->shape[2]);
  g.OW = int(ty.record->shape[3]);
  if (p->kind == kGlobalAvg) {
    g.kh = g.H;
    g.kw = g.W;
    g.sh = g.sw = 1;
  } else {
    Spkv2AttrRecord a;
    int rc = get_attr(ctx, node, &a);
    if (rc) {
      delete p;
      return rc;
    }
    g.kh = a.kernel_shape[0];
    g.kw = a.kernel_shape[1];
    g.sh = a.strides[0];
    g.sw = a.strides[1];
    g.ph = a.pads[0];
    g.pw = a.pads[1];
  }
  strides_of(tx, g.xs);
  strides_of(ty, g.ys);
  p->out_nhwc = ty.layout == kNHWC;
  p->is_int8 = is_int8;
  p->vec = (!is_int8 && p->kind == kMax && tx.layout == kNHWC && ty.layout == kNHWC && g.C % 4 == 0) ? 4 : 1;
  if (is_int8 && p->kind == kMax && tx.layout == kNHWC && ty.layout == kNHWC && g.C % 16 == 0 &&
      reinterpret_cast<uintptr_t>(tx.data) % 16 == 0 && reinterpret_cast<uintptr_t>(ty.data) % 16 == 0)
    p->vec = 16;
  const bool s1 = g.sh == 1 && g.sw == 1 && g.kh == g.kw && (g.kh == 3 || g.kh == 5 || g.kh == 7) &&
                  int64_t(g.H) * g.W * g.C < (int64_t(1) << 31);
  if (p->vec == 4 && s1) p->band = g.kh == 3 ? s1_band<3>(g) : g.kh == 5 ? s1_band<5>(g) : s1_band<7>(g);
  p->variant = p->vec == 4    ? (s1 ? "maxpool_nhwc_vec4_s1rows" : "maxpool_nhwc_vec4")
               : p->vec == 16 ? "maxpool_nhwc_i8_vec16"
                              : "pool_generic";
  set_node_plan(ctx, node, p);
  return 0;
}

int pool_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch) {
  (void)scratch;
  PoolPlan *p = node_plan<PoolPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  const Geo &g = p->g;
  const int64_t total = int64_t(g.N) * g.C * g.OH * g.OW;
  if (total == 0) return 0;
  void *y = ctx->tensors[node->outputs[0]].data;
  const void *x = ctx->tensors[node->inputs[0]].data;
  // Vector paths need 16-byte aligned tensors (a rebinding may move them).
  const bool aligned = (reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 16 == 0;
  if (p->vec == 4 && aligned && p->band > 0) {
    const int64_t columns = int64_t(g.N) * ((g.OH + p->band - 1) / p->band) * g.OW * (g.C / 4);
    const int grid = grid_for(columns, 128);
    if (g.kh == 3)
      maxpool_nhwc4_s1_kernel<3><<<grid, 128, 0, ctx->stream>>>(static_cast<float *>(y),
                                                                   static_cast<const float *>(x), g, p->band, columns);
    else if (g.kh == 5)
      maxpool_nhwc4_s1_kernel<5><<<grid, 128, 0, ctx->stream>>>(static_cast<float *>(y),
                                                                   static_cast<const float *>(x), g, p->band, columns);
    else
      maxpool_nhwc4_s1_kernel<7><<<grid, 128, 0, ctx->stream>>>(static_cast<float *>(y),
                                                                   static_cast<const float *>(x), g, p->band, columns);
  } else if (p->vec == 4 && aligned) {
    maxpool_nhwc4_kernel<<<grid_for(total / 4, 256), 256, 0, ctx->stream>>>(
        static_cast<float *>(y), static_cast<const float *>(x), g, total / 4);
  } else if (p->vec == 16 && aligned) {
    maxpool_nhwc16_i8_kernel<<<grid_for(total / 16, 256), 256, 0, ctx->stream>>>(
        static_cast<int8_t *>(y), static_cast<const int8_t *>(x), g, total / 16);
  } else if (p->is_int8) {
    pool_kernel<int8_t><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
        static_cast<int8_t *>(y), static_cast<const int8_t *>(x), g, p->kind, p->out_nhwc, total);
  } else {
    pool_kernel<float><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
        static_cast<float *>(y), static_cast<const float *>(x), g, p->kind, p->out_nhwc, total);
  }
  return cuda_status(cudaGetLastError());
}

int resize_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  (void)spec;
  if (node->input_count < 1 || node->output_count < 1) return -3;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.record->rank != 4 || ty.record->rank != 4) return -11;
  if (tx.record->dtype != ty.record->dtype) return SPKV2_ERR_UNSUPPORTED;
  ResizePlan *p = new ResizePlan();
  ResizeGeo &g = p->g;
  g.N = int(ty.record->shape[0]);
  g.C = int(ty.record->shape[1]);
  g.OH = int(ty.record->shape[2]);
  g.OW = int(ty.record->shape[3]);
  g.H = int(tx.record->shape[2]);
  g.W = int(tx.record->shape[3]);
  strides_of(tx, g.xs);
  strides_of(ty, g.ys);
  g.out_nhwc = ty.layout == kNHWC;
  p->esize = int(dtype_size(ty.record->dtype));
  p->vec4 = p->esize == 4 && tx.layout == kNHWC && ty.layout == kNHWC && g.C % 4 == 0;
  // Integer factors below 2^8 keep fp32's floor(oh / f) equal to oh / f.
  p->int_factor = g.H > 0 && g.W > 0 && g.OH % g.H == 0 && g.OW % g.W == 0 && g.OH / g.H <= 256 && g.OW / g.W <= 256;
  p->variant = p->vec4 ? (p->int_factor ? "resize_nearest_nhwc_vec4_int" : "resize_nearest_nhwc_vec4")
                       : "resize_nearest_generic";
  set_node_plan(ctx, node, p);
  return 0;
}

int resize_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *scratch) {
  (void)scratch;
  ResizePlan *p = node_plan<ResizePlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  const ResizeGeo &g = p->g;
  const int64_t total = int64_t(g.N) * g.C * g.OH * g.OW;
  if (total == 0) return 0;
  void *y = ctx->tensors[node->outputs[0]].data;
  const void *x = ctx->tensors[node->inputs[0]].data;
  if (p->vec4 && p->int_factor) {
    const int64_t in4 = int64_t(g.N) * g.H * g.W * (g.C / 4);
    resize_nearest_int_nhwc4_kernel<<<grid_for(in4, 256), 256, 0, ctx->stream>>>(
        static_cast<float4 *>(y), static_cast<const float4 *>(x), g, g.OH / g.H, g.OW / g.W, in4);
  } else if (p->vec4) {
    resize_nearest_nhwc4_kernel<<<grid_for(total / 4, 256), 256, 0, ctx->stream>>>(
        static_cast<float4 *>(y), static_cast<const float4 *>(x), g, total / 4);
  } else if (p->esize == 1) {
    resize_nearest_kernel<uint8_t><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
        static_cast<uint8_t *>(y), static_cast<const uint8_t *>(x), g, total);
  } else {
    resize_nearest_kernel<uint32_t><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
        static_cast<uint32_t *>(y), static_cast<const uint32_t *>(x), g, total);
  }
  return cuda_status(cudaGetLastError());
}

}  // namespace spkv2
