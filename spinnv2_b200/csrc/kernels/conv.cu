// Conv: prepare (numeric mode, quantisation constants, packed weights,
// kernel choice) and the CUDA-core implicit-GEMM kernels.
//
// Semantics (reference/conv/conv.c:3-62, optimized/conv/conv.c:926-1196):
//   y = act(conv(x, W) + b [+ residual])   residual = inputs[3], added before
//   the activation; act 1 = Relu, 2 = SiLU x / (1 + expf(-x)); groups,
//   strides, pads, dilations as in the attribute record.
// INT8 (this target's requantisation contract for int8 networks; no
// reference counterpart on x86 - the reference INT8 conv is
// ARM-dotprod-only, conv_int8.c:13):
//   acc  = sum over k of int32(w_q) * int32(x_q)              (exact int32)
//   acc' = acc + b_q[c]                                        (int32 bias)
//   v    = fp32(acc') * M[c],  M[c] = fp32(s_x * s_w[c]) / s_y (host, fp32)
//   v    = v + fp32(r_q) * R,  R = s_r / s_y                  (residual)
//   y_q  = clamp(round_half_even(v), relu ? 0 : -128, 127)
//   Every fp32 step is one IEEE-rounded operation (no FMA contraction) so the
//   CPU oracle reproduces it bit for bit.
// fp32 conv with an int8 output (the quantised model's first conv):
//   y_q = clamp(round_half_even(act(conv + b) * (1 / s_y)), -128, 127).
//
// GEMM view: rows = output pixels (n, oh, ow), columns = output channels,
// K = (r, s, c) with c fastest so an NHWC pixel's channels are contiguous.
#include <string.h>

#include "conv.h"

namespace spkv2 {

namespace {

// ---- weight packing: OIHW -> [groups][K][Mg], k = (r*KW + s)*Cg + c ----
template <typename T>
__global__ void pack_simt_kernel(T *__restrict__ dst, const T *__restrict__ w, ConvGeo g) {
  const int64_t total = int64_t(g.M) * g.K;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / g.K);
    const int k = int(i % g.K);
    const int c = k % g.Cg, rs = k / g.Cg, s = rs % g.KW, r = rs / g.KW;
    const int grp = m / g.Mg, ml = m % g.Mg;
    dst[(int64_t(grp) * g.K + k) * g.Mg + ml] = w[((int64_t(m) * g.Cg + c) * g.KH + r) * g.KW + s];
  }
}

constexpr int kBM = 64, kBN = 64, kBK = 16;

// A-operand element (pixel p, reduction index k) of the implicit GEMM.
template <typename T>
__device__ __forceinline__ T load_a(const T *__restrict__ x, const ConvGeo &g, int grp, int64_t p, int k) {
  if (p >= g.P || k >= g.K) return T(0);
  const int ow = int(p % g.OW);
  const int64_t t = p / g.OW;
  const int oh = int(t % g.OH);
  const int n = int(t / g.OH);
  const int c = k % g.Cg, rs = k / g.Cg, s = rs % g.KW, r = rs / g.KW;
  const int ih = oh * g.sh - g.ph + r * g.dh;
  const int iw = ow * g.sw - g.pw + s * g.dw;
  if (ih < 0 || ih >= g.H || iw < 0 || iw >= g.W) return T(0);
  return x[n * g.xs[0] + int64_t(grp * g.Cg + c) * g.xs[1] + ih * g.xs[2] + iw * g.xs[3]];
}

// fp32 implicit GEMM on CUDA cores: 64 pixels x 64 channels per block,
// 4x4 outputs per thread; grid (pixel tiles, channel tiles, groups).
template <int MODE>
__global__ void __launch_bounds__(256) conv_simt_f32_kernel(const float *__restrict__ x, const float *__restrict__ wp,
                                                            const float *__restrict__ bias,
                                                            const float *__restrict__ res, void *__restrict__ y,
                                                            ConvGeo g) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int grp = blockIdx.z;
  const int64_t p0 = int64_t(blockIdx.x) * kBM;
  const int n0 = blockIdx.y * kBN;
  const float *wg = wp + int64_t(grp) * g.K * g.Mg;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += kBK) {
    for (int e = tid; e < kBM * kBK; e += 256) {
      const int kk = e % kBK, mm = e / kBK;
      As[kk][mm] = load_a<float>(x, g, grp, p0 + mm, k0 + kk);
      const int kb = e / kBN, nn = e % kBN;
      Bs[kb][nn] = (k0 + kb < g.K && n0 + nn < g.Mg) ? wg[int64_t(k0 + kb) * g.Mg + n0 + nn] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t p = p0 + ty * 4 + i;
    if (p >= g.P) continue;
    const int ow = int(p % g.OW);
    const int64_t t = p / g.OW;
    const int oh = int(t % g.OH);
    const int n = int(t / g.OH);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ml = n0 + tx * 4 + j;
      if (ml >= g.Mg) continue;
      const int m = grp * g.Mg + ml;
      float v = acc[i][j];
      if (g.has_bias) v += bias[m];
      if (g.has_res) v += res[n * g.rs[0] + m * g.rs[1] + oh * g.rs[2] + ow * g.rs[3]];
      v = apply_act(v, g.act);
      const int64_t yo = n * g.ys[0] + m * g.ys[1] + oh * g.ys[2] + ow * g.ys[3];
      if (MODE == kConvF32)
        static_cast<float *>(y)[yo] = v;
      else
        static_cast<int8_t *>(y)[yo] = sat_rne_i8(__fmul_rn(v, g.out_scale_inv), -128);
    }
  }
}

// INT8 implicit GEMM on CUDA cores (exact int32 accumulation) with the
// requantising epilogue.
// OUT32: int32 output acc + b_q (no requantisation).
template <bool OUT32>
__global__ void __launch_bounds__(256) conv_simt_i8_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ wp,
                                                           const int32_t *__restrict__ bias_q,
                                                           const float *__restrict__ scale_m,
                                                           const int8_t *__restrict__ res, void *__restrict__ yv,
                                                           ConvGeo g) {
  __shared__ int32_t As[kBK][kBM + 4];
  __shared__ int32_t Bs[kBK][kBN + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int grp = blockIdx.z;
  const int64_t p0 = int64_t(blockIdx.x) * kBM;
  const int n0 = blockIdx.y * kBN;
  const int8_t *wg = wp + int64_t(grp) * g.K * g.Mg;
  int32_t acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += kBK) {
    for (int e = tid; e < kBM * kBK; e += 256) {
      const int kk = e % kBK, mm = e / kBK;
      As[kk][mm] = load_a<int8_t>(x, g, grp, p0 + mm, k0 + kk);
      const int kb = e / kBN, nn = e % kBN;
      Bs[kb][nn] = (k0 + kb < g.K && n0 + nn < g.Mg) ? wg[int64_t(k0 + kb) * g.Mg + n0 + nn] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += As[kk][ty * 4 + i] * Bs[kk][tx * 4 + j];
    }
    __syncthreads();
  }
  const int lo = g.act == 1 ? 0 : -128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t p = p0 + ty * 4 + i;
    if (p >= g.P) continue;
    const int ow = int(p % g.OW);
    const int64_t t = p / g.OW;
    const int oh = int(t % g.OH);
    const int n = int(t / g.OH);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ml = n0 + tx * 4 + j;
      if (ml >= g.Mg) continue;
      const int m = grp * g.Mg + ml;
      const int32_t a = acc[i][j] + (g.has_bias ? bias_q[m] : 0);
      const int64_t yo = n * g.ys[0] + m * g.ys[1] + oh * g.ys[2] + ow * g.ys[3];
      if (OUT32) {
        static_cast<int32_t *>(yv)[yo] = a;
        continue;
      }
      float v = __fmul_rn(float(a), scale_m[m]);
      if (g.has_res)
        v = __fadd_rn(v, __fmul_rn(float(res[n * g.rs[0] + m * g.rs[1] + oh * g.rs[2] + ow * g.rs[3]]), g.res_scale));
      static_cast<int8_t *>(yv)[yo] = sat_rne_i8(v, lo);
    }
  }
}

void strides4(const TensorState &t, int64_t s[4]) {
  View v = make_view(t);
  for (int i = 0; i < 4; ++i) s[i] = v.stride[i];
}

float per_tensor_scale(const Spkv2Context *ctx, uint32_t tid, bool *ok) {
  const float *s = quant_scales(ctx, find_quant_param(ctx, tid));
  if (!s) {
    *ok = false;
    return 1.0f;
  }
  return s[0];
}

}  // namespace

int conv_simt_launch(const ConvPlan &p, const void *x, void *y, const void *res, cudaStream_t s) {
  const ConvGeo &g = p.g;
  dim3 grid(unsigned(ceil_div(g.P, kBM)), unsigned(ceil_div(g.Mg, kBN)), unsigned(g.groups));
  if (grid.y > 65535 || grid.z > 65535) return SPKV2_ERR_UNSUPPORTED;
  switch (p.mode) {
    case kConvF32:
      conv_simt_f32_kernel<kConvF32><<<grid, 256, 0, s>>>(static_cast<const float *>(x),
                                                          static_cast<const float *>(p.w_simt), p.bias_f,
                                                          static_cast<const float *>(res), y, g);
      break;
    case kConvF32ToI8:
      conv_simt_f32_kernel<kConvF32ToI8><<<grid, 256, 0, s>>>(static_cast<const float *>(x),
                                                              static_cast<const float *>(p.w_simt), p.bias_f,
                                                              static_cast<const float *>(res), y, g);
      break;
    case kConvI8:
      conv_simt_i8_kernel<false><<<grid, 256, 0, s>>>(static_cast<const int8_t *>(x),
                                                      static_cast<const int8_t *>(p.w_simt), p.bias_q, p.scale_m,
                                                      static_cast<const int8_t *>(res), y, g);
      break;
    case kConvI8ToI32:
      conv_simt_i8_kernel<true><<<grid, 256, 0, s>>>(static_cast<const int8_t *>(x),
                                                     static_cast<const int8_t *>(p.w_simt), p.bias_q, nullptr,
                                                     nullptr, y, g);
      break;
    default: return SPKV2_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaGetLastError());
}

// ---------------- weights-only INT8 (the reference compiler's format) ----------------
//
// Reference runtime/kernels/optimized/conv/conv_int8.c:22-56,86-119: the
// fp32 input is quantised per tensor, q = sat8(rne(x * fp32(1 / s_x))) (its
// vector lanes; the scalar tail rounds half away from zero and is only
// reached when an image's C*H*W is not a multiple of 16), the int8 conv
// accumulates in int32, and y = act(fma(acc, s_w[c] * s_x, b[c]) + res).

namespace {

// x (any layout, strides g.xs) -> dense NHWC int8.
__global__ void quantize_w8_kernel(int8_t *__restrict__ xq, const float *__restrict__ x, ConvGeo g, float inv,
                                   int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % g.C);
    const int64_t pix = i / g.C;
    const int w = int(pix % g.W), h = int((pix / g.W) % g.H), n = int(pix / (int64_t(g.W) * g.H));
    const float v = __fmul_rn(x[n * g.xs[0] + c * g.xs[1] + h * g.xs[2] + w * g.xs[3]], inv);
    int q = __float2int_rn(v);
    q = q < -128 ? -128 : q > 127 ? 127 : q;
    xq[i] = int8_t(q);
  }
}

// Dense NHWC int32 accumulators -> y (strides g.ys), fused dequantisation.
__global__ void dequant_w8_kernel(float *__restrict__ y, const int32_t *__restrict__ acc, const float *__restrict__ cs,
                                  const float *__restrict__ bias, const float *__restrict__ res, ConvGeo g,
                                  int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i % g.M);
    const int64_t pix = i / g.M;
    const int ow = int(pix % g.OW), oh = int((pix / g.OW) % g.OH), n = int(pix / (int64_t(g.OW) * g.OH));
    float v = fmaf(float(acc[i]), cs[m], bias ? bias[m] : 0.0f);
    if (res) v = __fadd_rn(v, res[n * g.rs[0] + m * g.rs[1] + oh * g.rs[2] + ow * g.rs[3]]);
    v = apply_act(v, g.act);
    y[n * g.ys[0] + m * g.ys[1] + oh * g.ys[2] + ow * g.ys[3]] = v;
  }
}

}  // namespace

int prepare_w8(Spkv2Context *ctx, const Spkv2NodeRecord *node, ConvPlan &p, const void *w_dev) {
  const ConvGeo &g = p.g;
  if (g.groups != 1) return SPKV2_ERR_UNSUPPORTED;
  bool ok = true;
  const float sx = per_tensor_scale(ctx, node->inputs[0], &ok);
  const Spkv2QuantParamRecord *wq = find_quant_param(ctx, node->inputs[1]);
  const float *sw = quant_scales(ctx, wq);
  if (!ok || !sw || wq->num_channels != uint32_t(g.M)) return SPKV2_ERR_UNSUPPORTED;
  p.w8_inv_sx = 1.0f / sx;
  std::vector<float> cs(size_t(ceil_div(g.M, 32) * 32), 0.0f);
  for (int c = 0; c < g.M; ++c) cs[size_t(c)] = sw[c] * sx;
  p.w8_cs = static_cast<float *>(device_alloc(sizeof(float) * cs.size()));
  p.w8_xq = static_cast<int8_t *>(device_alloc(size_t(g.N) * g.C * g.H * g.W + 16));
  p.w8_acc = static_cast<int32_t *>(device_alloc(sizeof(int32_t) * size_t(g.P) * g.M + 16));
  if (!p.w8_cs || !p.w8_xq || !p.w8_acc) return SPKV2_ERR_DEVICE_ALLOC;
  int rc = cuda_status(cudaMemcpyAsync(p.w8_cs, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice,
                                       ctx->stream));
  if (rc == 0) rc = cuda_status(cudaStreamSynchronize(ctx->stream));  // the host vector must outlive the copy
  if (rc) return rc;
  // The int8 conv: dense NHWC int8 in, dense NHWC int32 out, no bias,
  // residual or activation (those are applied by the dequantisation).
  ConvPlan *q = new ConvPlan();
  p.w8_inner = q;
  q->mode = kConvI8ToI32;
  q->g = g;
  ConvGeo &gi = q->g;
  gi.xs[0] = int64_t(g.H) * g.W * g.C, gi.xs[1] = 1, gi.xs[2] = int64_t(g.W) * g.C, gi.xs[3] = g.C;
  gi.ys[0] = int64_t(g.OH) * g.OW * g.M, gi.ys[1] = 1, gi.ys[2] = int64_t(g.OW) * g.M, gi.ys[3] = g.M;
  gi.has_bias = 0;
  gi.has_res = 0;
  gi.act = 0;
  rc = SPKV2_ERR_UNSUPPORTED;
  if (ctx->math_mode != SPKV2_CUDA_MATH_FP32) rc = conv_tc_i8_prepare(*q, w_dev, p.w8_xq, p.w8_acc, nullptr, ctx->stream);
  if (rc != 0 && rc != SPKV2_ERR_UNSUPPORTED) return rc;
  if (!q->w_tc) {
    q->w_simt = device_alloc(size_t(g.M) * g.K);
    if (!q->w_simt) return SPKV2_ERR_DEVICE_ALLOC;
    pack_simt_kernel<int8_t><<<grid_for(int64_t(g.M) * g.K, 256), 256, 0, ctx->stream>>>(
        static_cast<int8_t *>(q->w_simt), static_cast<const int8_t *>(w_dev), g);
    if ((rc = cuda_status(cudaGetLastError()))) return rc;
    q->variant = "simt_int8_i32out";
  }
  p.launches = 2 + q->launches;
  p.variant = "w8_" + q->variant;
  return 0;
}

int run_w8(Spkv2Context *ctx, const ConvPlan &p, const float *x, float *y, const float *res) {
  const ConvGeo &g = p.g;
  const int64_t nx = int64_t(g.N) * g.C * g.H * g.W, ny = g.P * g.M;
  quantize_w8_kernel<<<grid_for(nx, 256), 256, 0, ctx->stream>>>(p.w8_xq, x, g, p.w8_inv_sx, nx);
  int rc = cuda_status(cudaGetLastError());
  if (rc) return rc;
  const ConvPlan &q = *p.w8_inner;
  rc = q.w_tc ? conv_tc_i8_launch(q, p.w8_xq, p.w8_acc, nullptr, ctx->d_status, ctx->stream)
              : conv_simt_launch(q, p.w8_xq, p.w8_acc, nullptr, ctx->stream);
  if (rc) return rc;
  dequant_w8_kernel<<<grid_for(ny, 256), 256, 0, ctx->stream>>>(y, p.w8_acc, p.w8_cs, p.bias_f, res, g, ny);
  return cuda_status(cudaGetLastError());
}

int conv_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *spec) {
  if (node->input_count < 2 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &tw = ctx->tensors[node->inputs[1]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  const Spkv2TensorRecord *xr = tx.record, *wr = tw.record, *yr = ty.record;
  if (xr->rank != 4 || wr->rank != 4 || yr->rank != 4) return -11;
  if (wr->role != SPKV2_ROLE_WEIGHT) return SPKV2_ERR_UNSUPPORTED;
  const int group = a.group > 0 ? a.group : 1;
  if (xr->shape[1] % group != 0 || wr->shape[0] % group != 0) return -12;
  if (wr->shape[1] != xr->shape[1] / group) return -12;

  ConvPlan *p = new ConvPlan();
  ConvGeo &g = p->g;
  g.N = int(xr->shape[0]);
  g.C = int(xr->shape[1]);
  g.H = int(xr->shape[2]);
  g.W = int(xr->shape[3]);
  g.M = int(wr->shape[0]);
  g.KH = int(wr->shape[2]);
  g.KW = int(wr->shape[3]);
  g.OH = int(yr->shape[2]);
  g.OW = int(yr->shape[3]);
  g.sh = a.strides[0];
  g.sw = a.strides[1];
  g.ph = a.pads[0];
  g.pw = a.pads[1];
  g.dh = a.dilations[0] > 0 ? a.dilations[0] : 1;
  g.dw = a.dilations[1] > 0 ? a.dilations[1] : 1;
  g.groups = group;
  g.Cg = g.C / group;
  g.Mg = g.M / group;
  g.K = g.KH * g.KW * g.Cg;
  g.P = int64_t(g.N) * g.OH * g.OW;
  g.act = a.fused_activation;
  g.has_bias = node->input_count > 2;
  g.has_res = node->input_count > 3;
  strides4(tx, g.xs);
  strides4(ty, g.ys);
  if (g.has_res) strides4(ctx->tensors[node->inputs[3]], g.rs);

  // Numeric mode from the tensor dtypes.
  const uint16_t dx = xr->dtype, dw = wr->dtype, dy = yr->dtype;
  if (dx == SPKV2_DTYPE_FP32 && dw == SPKV2_DTYPE_FP32 && dy == SPKV2_DTYPE_FP32)
    p->mode = kConvF32;
  else if (dx == SPKV2_DTYPE_FP32 && dw == SPKV2_DTYPE_FP32 && dy == SPKV2_DTYPE_INT8)
    p->mode = kConvF32ToI8;
  else if (dx == SPKV2_DTYPE_INT8 && dw == SPKV2_DTYPE_INT8 && dy == SPKV2_DTYPE_INT8)
    p->mode = kConvI8;
  else if (dx == SPKV2_DTYPE_INT8 && dw == SPKV2_DTYPE_INT8 && dy == SPKV2_DTYPE_INT32)
    p->mode = kConvI8ToI32;
  else if (dx == SPKV2_DTYPE_FP32 && dw == SPKV2_DTYPE_INT8 && dy == SPKV2_DTYPE_FP32)
    p->mode = kConvW8;
  else {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }
  const bool int_acc = p->mode == kConvI8 || p->mode == kConvI8ToI32;
  bool ok = true;
  if (g.has_bias) {
    const TensorState &tb = ctx->tensors[node->inputs[2]];
    const uint16_t want = int_acc ? SPKV2_DTYPE_INT32 : SPKV2_DTYPE_FP32;
    if (tb.record->dtype != want || elem_count(tb.record) != size_t(g.M)) ok = false;
    if (!int_acc) p->bias_f = reinterpret_cast<const float *>(tb.data);
  }
  if (g.has_res) {
    const uint16_t want = p->mode == kConvI8 ? SPKV2_DTYPE_INT8 : SPKV2_DTYPE_FP32;
    if (ctx->tensors[node->inputs[3]].record->dtype != want || p->mode == kConvI8ToI32) ok = false;
  }
  if (p->mode == kConvF32ToI8) {
    const float sy = per_tensor_scale(ctx, node->outputs[0], &ok);
    g.out_scale_inv = 1.0f / sy;
  }
  if (int_acc && g.act == 2) ok = false;  // SiLU has no int8 requant form
  if (p->mode == kConvI8ToI32 && g.act != 0) ok = false;
  // Per-channel int32 bias and requant multipliers, padded to a multiple of
  // 32 channels (zeros) so the epilogue may read whole 16-byte vectors.
  const size_t mpad = size_t(ceil_div(g.M, 32) * 32);
  if (ok && int_acc && g.has_bias) {
    p->bias_q = static_cast<int32_t *>(device_alloc(sizeof(int32_t) * mpad));
    if (!p->bias_q) {
      delete p;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    cudaMemsetAsync(p->bias_q, 0, sizeof(int32_t) * mpad, ctx->stream);
    cudaMemcpyAsync(p->bias_q, ctx->tensors[node->inputs[2]].data, sizeof(int32_t) * size_t(g.M),
                    cudaMemcpyDeviceToDevice, ctx->stream);
  }
  if (ok && p->mode == kConvI8) {
    const float sx = per_tensor_scale(ctx, node->inputs[0], &ok);
    const float sy = per_tensor_scale(ctx, node->outputs[0], &ok);
    const Spkv2QuantParamRecord *wq = find_quant_param(ctx, node->inputs[1]);
    const float *sw = quant_scales(ctx, wq);
    if (!sw || wq->num_channels != uint32_t(g.M)) ok = false;
    if (ok) {
      std::vector<float> m(mpad, 0.0f);
      for (int c = 0; c < g.M; ++c) {
        const float t = sx * sw[c];
        m[size_t(c)] = t / sy;
      }
      p->scale_m = static_cast<float *>(device_alloc(sizeof(float) * mpad));
      if (!p->scale_m) {
        delete p;
        return SPKV2_ERR_DEVICE_ALLOC;
      }
      cudaMemcpyAsync(p->scale_m, m.data(), sizeof(float) * mpad, cudaMemcpyHostToDevice, ctx->stream);
      // The host vector must outlive the copy.
      if ((rc = cuda_status(cudaStreamSynchronize(ctx->stream)))) {
        delete p;
        return rc;
      }
      if (g.has_res) {
        const float sr = per_tensor_scale(ctx, node->inputs[3], &ok);
        g.res_scale = sr / sy;
      }
    }
  }
  if (!ok) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }

  if (p->mode == kConvW8) {
    if ((rc = prepare_w8(ctx, node, *p, tw.data))) {
      delete p;
      return rc;
    }
    set_node_plan(ctx, node, p);
    return 0;
  }

  // Math mode: the context override, else the KernelSpec kind.
  int math = ctx->math_mode;
  if (math == SPKV2_CUDA_MATH_SPEC) {
    const uint16_t kind = spec ? spec->kernel_kind : uint16_t(SPKV2_KERNEL_REFERENCE);
    math = kind == SPKV2_KERNEL_TC_TF32 ? SPKV2_CUDA_MATH_TF32
           : kind == SPKV2_KERNEL_SIMT_FP32 ? SPKV2_CUDA_MATH_FP32
                                             : SPKV2_CUDA_MATH_3XTF32;
  }
  p->math = math;

  // Weights the compiler stored pre-packed (weight_layout TC_PANEL_F32X2):
  // the tensor-core path reads them in place; the CUDA-core path unpacks
  // them to OIHW first.
  const bool prepacked = spec && spec->weight_layout == SPKV2_WEIGHT_LAYOUT_TC_PANEL_F32X2;
  const int panel_npad = int(ceil_div(g.M, 256) * 256), panel_kpad = int(ceil_div(g.K, 32) * 32);
  if (prepacked && (dw != SPKV2_DTYPE_FP32 || g.groups != 1 ||
                    uint64_t(wr->size_bytes) != uint64_t(2) * panel_npad * panel_kpad * sizeof(float))) {
    delete p;
    return -2;  // the record's size does not match the panel of its shape
  }
  const void *w_oihw = tw.data;  // OIHW weights for the packers below
  float *w_unpacked = nullptr;

  // Tensor-core path first; the CUDA-core kernel takes every shape it
  // declines (and every conv in FP32 math mode).
  if (math != SPKV2_CUDA_MATH_FP32) {
    const void *r_dev = g.has_res ? ctx->tensors[node->inputs[3]].data : nullptr;
    rc = int_acc ? conv_tc_i8_prepare(*p, tw.data, tx.data, ty.data, r_dev, ctx->stream)
         : prepacked ? conv_tc_prepare_ex(*p, nullptr, tx.data, ty.data, false, ctx->stream, r_dev,
                                          reinterpret_cast<const float *>(tw.data), panel_npad)
                     : conv_tc_prepare(*p, tw.data, tx.data, ty.data, r_dev, ctx->stream);
    if (rc == 0 && !int_acc) rc = conv_tc_attach(ctx, *p);
    if (rc != 0 && rc != SPKV2_ERR_UNSUPPORTED) {
      delete p;
      return rc;
    }
  }
  if (!p->w_tc && prepacked) {
    w_unpacked = static_cast<float *>(device_alloc(size_t(g.M) * g.K * sizeof(float)));
    if (!w_unpacked || (rc = conv_unpack_panel(w_unpacked, reinterpret_cast<const float *>(tw.data), g, panel_npad,
                                               panel_kpad, ctx->stream))) {
      device_free(w_unpacked);
      delete p;
      return w_unpacked ? rc : SPKV2_ERR_DEVICE_ALLOC;
    }
    w_oihw = w_unpacked;
  }
  if (!p->w_tc) {
    const size_t esz = int_acc ? 1 : 4;
    p->w_simt = device_alloc(size_t(g.M) * g.K * esz);
    if (!p->w_simt) {
      device_free(w_unpacked);
      delete p;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    const int64_t total = int64_t(g.M) * g.K;
    if (esz == 1)
      pack_simt_kernel<int8_t><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
          static_cast<int8_t *>(p->w_simt), reinterpret_cast<const int8_t *>(w_oihw), g);
    else
      pack_simt_kernel<float><<<grid_for(total, 256), 256, 0, ctx->stream>>>(
          static_cast<float *>(p->w_simt), reinterpret_cast<const float *>(w_oihw), g);
    rc = cuda_status(cudaGetLastError());
    if (w_unpacked) {  // the pack above reads it: free it once that finished
      const int src = cuda_status(cudaStreamSynchronize(ctx->stream));
      device_free(w_unpacked);
      rc = rc ? rc : src;
    }
    if (rc) {
      delete p;
      return rc;
    }
    p->variant = int_acc ? (p->mode == kConvI8ToI32 ? "simt_int8_i32out" : "simt_int8") : "simt_fp32";
  }
  set_node_plan(ctx, node, p);
  return 0;
}

int conv_tc_attach(Spkv2Context *ctx, const ConvPlan &p) {
  const size_t need = conv_tc_sk_workspace_bytes(p);
  if (need > ctx->sk_ws_bytes) {
    // Nothing in flight may still use the old buffer; a captured graph
    // holding its address is re-captured.
    int rc = cuda_status(cudaStreamSynchronize(ctx->stream));
    if (rc) return rc;
    device_free(ctx->d_sk_ws);
    ctx->d_sk_ws = static_cast<float *>(device_alloc(need));
    ctx->sk_ws_bytes = ctx->d_sk_ws ? need : 0;
    ctx->graph_dirty = true;
    if (!ctx->d_sk_ws) return SPKV2_ERR_DEVICE_ALLOC;
  }
  size_t bytes = 0;
  if (void *cnt = conv_tc_sk_counters(p, &bytes)) ctx->sk_counters.emplace_back(cnt, bytes);
  return 0;
}

int conv_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  ConvPlan *p = node_plan<ConvPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->g.P == 0 || p->g.M == 0) return 0;
  const void *x = ctx->tensors[node->inputs[0]].data;
  void *y = ctx->tensors[node->outputs[0]].data;
  const void *res = p->g.has_res ? ctx->tensors[node->inputs[3]].data : nullptr;
  if (p->mode == kConvW8) return run_w8(ctx, *p, static_cast<const float *>(x), static_cast<float *>(y),
                                        static_cast<const float *>(res));
  if (p->w_tc)
    return p->tc_i8 ? conv_tc_i8_launch(*p, x, y, res, ctx->d_status, ctx->stream)
                    : conv_tc_launch(*p, x, y, res, ctx->d_status, ctx->stream, ctx->d_sk_ws);
  return conv_simt_launch(*p, x, y, res, ctx->stream);
}

}  // namespace spkv2
