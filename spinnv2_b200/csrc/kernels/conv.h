// Conv node plan shared by the CUDA-core (SIMT) and tcgen05 conv kernels.
#pragma once

#include "common.cuh"

namespace spkv2 {

// Numeric mode of a conv node, from the dtypes of x / w / y.
enum ConvMode : int {
  kConvF32 = 0,     // fp32 x, fp32 w -> fp32 y
  kConvF32ToI8 = 1, // fp32 x, fp32 w -> int8 y   (quantising epilogue)
  kConvI8 = 2,      // int8 x, int8 w -> int8 y   (int32 acc, requantised)
  kConvI8ToI32 = 3, // int8 x, int8 w -> int32 y  (acc + int32 bias, no requantisation)
  kConvW8 = 4,      // fp32 x, int8 w -> fp32 y   (weights-only int8: x quantised per tensor on
                    //  the fly, int8 conv to int32, y = act(fma(acc, s_w[c] s_x, b) + res))
};

// Geometry and epilogue parameters, passed by value to the kernels.
struct ConvGeo {
  int N, C, H, W;       // input
  int M, OH, OW;        // output channels and spatial size
  int KH, KW, sh, sw, ph, pw, dh, dw;
  int groups, Cg, Mg;   // per-group input / output channels
  int K;                // KH * KW * Cg, ordered (r, s, c) with c fastest
  int64_t P;            // N * OH * OW output pixels
  int64_t xs[4], ys[4], rs[4];  // element strides (n, c, h, w) of x, y, residual
  int act;              // 0 none, 1 Relu, 2 SiLU
  int has_bias, has_res;
  float out_scale_inv;  // 1 / s_y            (kConvF32ToI8)
  float res_scale;      // s_r / s_y          (kConvI8 with residual)
};

// Tile width (output channels per tile) for the tcgen05 kernels: the one
// with the shortest estimated run, waves x K steps x cycles per K step.
// One wave = one tile per SM; a K step is four M=128 MMAs whose issue cost,
// measured on B200 for TF32 (K=8) and INT8 (K=32), is max(48, N/2) cycles
// each (narrow tiles are bound by shared-memory operand reads).  Ties go to
// the wider tile.
inline int pick_block_n(int64_t P, int M, int64_t K_steps, int sms, int min_bn, int max_bn) {
  const int64_t m_tiles = (P + 127) / 128;
  int best = max_bn;
  int64_t best_cost = -1;
  for (int bn = max_bn; bn >= min_bn; bn /= 2) {
    if (bn > 32 && (bn / 2) >= M) continue;  // a narrower tile already covers Cout
    const int64_t tiles = m_tiles * ((M + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = waves * K_steps * 4 * (bn / 2 > 48 ? bn / 2 : 48);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

void conv_tc_release(void *state);
void conv_tc_i8_release(void *state);

struct ConvPlan : NodePlan {
  ConvGeo g{};
  int mode = kConvF32;
  int math = 0;            // SPKV2_CUDA_MATH_* actually used
  void *w_simt = nullptr;  // [groups][K][Mg] packed weights (fp32 or int8)
  void *w_tc = nullptr;    // tcgen05 operand panels (see conv_tc.cu)
  bool w_tc_borrowed = false;  // w_tc points into the device weight section (pre-packed SPK panel)
  int32_t *bias_q = nullptr;  // int32 requantisation bias (kConvI8)
  float *scale_m = nullptr;   // per-channel requant multiplier M[c] (kConvI8)
  const float *bias_f = nullptr;  // fp32 bias (device weights)
  int tc_block_n = 0;      // tcgen05 tile width in output channels
  int tc_kpad = 0;         // padded K of the tcgen05 panels
  void *tc_state = nullptr;  // tensor maps + launch configuration (conv_tc.cu / conv_tc_i8.cu)
  bool tc_i8 = false;        // tc_state belongs to the kind::i8 kernel
  // kConvW8: the int8 conv over the quantised input, its buffers and the
  // per-channel dequantisation scale s_w[c] * s_x.
  ConvPlan *w8_inner = nullptr;
  int8_t *w8_xq = nullptr;
  int32_t *w8_acc = nullptr;
  float *w8_cs = nullptr;
  float w8_inv_sx = 1.0f;
  ~ConvPlan() override {
    delete w8_inner;
    device_free(w8_xq);
    device_free(w8_acc);
    device_free(w8_cs);
    if (tc_state) tc_i8 ? conv_tc_i8_release(tc_state) : conv_tc_release(tc_state);
    device_free(w_simt);
    if (!w_tc_borrowed) device_free(w_tc);
    device_free(bias_q);
    device_free(scale_m);
  }
};

int conv_simt_launch(const ConvPlan &p, const void *x, void *y, const void *res, cudaStream_t s);

// tcgen05 path (conv_tc.cu): returns 0 when the node is eligible and its
// operand panels were built; SPKV2_ERR_UNSUPPORTED when the shape is not.
int conv_tc_prepare(ConvPlan &p, const void *w_raw_dev, const void *x_dev, const void *y_dev, const void *r_dev,
                    cudaStream_t s);
// w_kn: the weights are a [K][Cout] matrix (Gemm B, transB = 0), not OIHW.
// panel / panel_npad: the weights already stored as the tcgen05 panel
// (SPK weight_layout TC_PANEL_F32X2, Npad rows per part); used in place when
// the conv keeps its channel count as the GEMM K order's (no row packing,
// no channel padding), else SPKV2_ERR_UNSUPPORTED.
int conv_tc_prepare_ex(ConvPlan &p, const void *w_raw_dev, const void *x_dev, const void *y_dev, bool w_kn,
                       cudaStream_t s, const void *r_dev = nullptr, const float *panel = nullptr,
                       int panel_npad = 0);
// TC_PANEL_F32X2 panel -> OIHW fp32 (w = part0 + part1, exact), on `s`.
int conv_unpack_panel(float *oihw, const float *panel, const ConvGeo &g, int npad, int kpad, cudaStream_t s);
// sk_ws: the context's stream-K workspace (conv_tc_attach sized it); may be
// null for plans that do not use stream-K.
int conv_tc_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s,
                   float *sk_ws);
// Stream-K needs of a prepared tcgen05 plan: workspace bytes for partial
// tiles (one buffer per context, shared by all convs since they run in
// stream order) and the plan's arrival counters (zero between launches).
size_t conv_tc_sk_workspace_bytes(const ConvPlan &p);
void *conv_tc_sk_counters(const ConvPlan &p, size_t *bytes);
// Grows the context's stream-K workspace to what plan p needs and registers
// its counters (re-zeroed after a device-side abort).  Called at prepare.
int conv_tc_attach(Spkv2Context *ctx, const ConvPlan &p);

// tcgen05 kind::i8 path (conv_tc_i8.cu) for kConvI8 / kConvI8ToI32.
int conv_tc_i8_prepare(ConvPlan &p, const void *w_dev, const void *x_dev, const void *y_dev, const void *r_dev,
                       cudaStream_t s);
int conv_tc_i8_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s);

}  // namespace spkv2
