// Gemm: Y[M,N] = alpha * op(A)[M,K] * op(B)[K,N] + C[n].
//
// Semantics (reference/mm/gemm.c:3-33, reference/mm/gemm_cpu_direct.c:3-37,
// optimized/mm/gemm.c:9-85): beta is ignored, C is read as a per-column bias
// c[n], transA/transB are honoured.
// Device design (fp32 CUDA-core, exact fp32 products):
//   M <= 8, no transposes  - weight-streaming GEMV: a warp reads 32 adjacent
//     columns of B per k (coalesced), K is split over warps and blocks, and a
//     second kernel sums the partial results in a fixed order (deterministic).
//   otherwise, no transposes - 64x64x16 shared-memory tiles, 4x4 per thread.
//   with transposes        - one thread per output, strided loads.
// MatMul (reference/mm/matmul.c:3-50): Y[..., M, N] = A[..., M, K] *
// B[..., K, N] with numpy-style broadcasting of the leading (batch) dims
// (a size-1 or missing dim repeats); no bias, no alpha.  Device design: the
// 64x64x16 tiled kernel over element strides (any operand may be an NHWC
// rank-4 activation), one grid z-slice per batch matrix.
#include <atomic>
#include <string.h>

#include "conv.h"

namespace spkv2 {

namespace {

constexpr int kGemvMaxM = 8;
constexpr int kGemvWarps = 8;
constexpr int kTcMinRows = 16;  // from this many rows a Gemm runs as a tcgen05 1x1 conv

struct GemmPlan : NodePlan {
  int M = 0, K = 0, N = 0;
  int trans_a = 0, trans_b = 0;
  float alpha = 1.0f;
  int ksplit = 1;
  float *partials = nullptr;  // [ksplit][M][N] for the GEMV path
  ConvPlan *tc = nullptr;     // Y = A * B + bias as a 1x1 conv over [M,1,1,K]
  ~GemmPlan() override {
    device_free(partials);
    delete tc;
  }
};

// grid (ceil(N/32), ksplit); block 32 x kGemvWarps.  Each block reduces its
// warps in shared memory and writes one partial per (split, m, n).
__global__ void gemv_partial_kernel(float *__restrict__ part, const float *__restrict__ A, const float *__restrict__ B,
                                    int M, int K, int N, int k_per_block) {
  __shared__ float red[kGemvWarps][kGemvMaxM][32];
  const int lane = threadIdx.x, warp = threadIdx.y;
  const int n = blockIdx.x * 32 + lane;
  const int k0 = blockIdx.y * k_per_block;
  const int k1 = min(K, k0 + k_per_block);
  float acc[kGemvMaxM];
#pragma unroll
  for (int m = 0; m < kGemvMaxM; ++m) acc[m] = 0.0f;
  if (n < N) {
    for (int k = k0 + warp; k < k1; k += kGemvWarps) {
      const float b = B[int64_t(k) * N + n];
#pragma unroll
      for (int m = 0; m < kGemvMaxM; ++m)
        if (m < M) acc[m] = fmaf(A[int64_t(m) * K + k], b, acc[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < kGemvMaxM; ++m) red[warp][m][lane] = acc[m];
  __syncthreads();
  if (warp == 0 && n < N) {
    for (int m = 0; m < M; ++m) {
      float s = 0.0f;
      for (int w = 0; w < kGemvWarps; ++w) s += red[w][m][lane];
      part[(int64_t(blockIdx.y) * M + m) * N + n] = s;
    }
  }
}

__global__ void gemv_finish_kernel(float *__restrict__ Y, const float *__restrict__ part, const float *__restrict__ bias,
                                   int M, int N, int ksplit, float alpha) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int k = 0; k < ksplit; ++k) s += part[int64_t(k) * total + i];
    Y[i] = alpha * s + (bias ? bias[i % N] : 0.0f);
  }
}

// 64x64 output tile, K step 16, 256 threads each owning a 4x4 sub-tile.
__global__ void __launch_bounds__(256) sgemm_tile_kernel(float *__restrict__ Y, const float *__restrict__ A,
                                                         const float *__restrict__ B, const float *__restrict__ bias,
                                                         int M, int K, int N, float alpha) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = tid; e < 64 * 16; e += 256) {
      const int mm = e / 16, kk = e % 16;
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? A[int64_t(m) * K + k] : 0.0f;
      const int kb = e / 64, nn = e % 64;
      const int kg = k0 + kb, n = n0 + nn;
      Bs[kb][nn] = (kg < K && n < N) ? B[int64_t(kg) * N + n] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
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
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) Y[int64_t(m) * N + n] = alpha * acc[i][j] + (bias ? bias[n] : 0.0f);
    }
  }
}

// Batched strided matmul.  Batch index b (blockIdx.z + k * gridDim.z)
// decomposes over the output's leading dims; each operand's stride per
// leading dim is 0 where it broadcasts.
struct MatmulDesc {
  int M, K, N;
  int nb;                 // leading (batch) dims of the output
  int64_t bdim[kMaxRank];
  int64_t as[kMaxRank], bs[kMaxRank], ys[kMaxRank];  // per-batch-dim strides
  int64_t a_m, a_k, b_k, b_n, y_m, y_n;              // matrix strides
  int64_t batches;
};

struct MatmulPlan : NodePlan {
  MatmulDesc d;
};

__global__ void __launch_bounds__(256) matmul_tile_kernel(float *__restrict__ Y, const float *__restrict__ A,
                                                          const float *__restrict__ B, MatmulDesc d) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  for (int64_t bi = blockIdx.z; bi < d.batches; bi += gridDim.z) {
    int64_t rem = bi, oa = 0, ob = 0, oy = 0;
    for (int k = d.nb - 1; k >= 0; --k) {
      const int64_t c = rem % d.bdim[k];
      rem /= d.bdim[k];
      oa += c * d.as[k];
      ob += c * d.bs[k];
      oy += c * d.ys[k];
    }
    const float *a = A + oa;
    const float *b = B + ob;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < d.K; k0 += 16) {
      for (int e = tid; e < 64 * 16; e += 256) {
        const int mm = e / 16, kk = e % 16;
        const int m = m0 + mm, k = k0 + kk;
        As[kk][mm] = (m < d.M && k < d.K) ? a[m * d.a_m + k * d.a_k] : 0.0f;
        const int kb = e / 64, nn = e % 64;
        const int kg = k0 + kb, n = n0 + nn;
        Bs[kb][nn] = (kg < d.K && n < d.N) ? b[kg * d.b_k + n * d.b_n] : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty * 4 + i;
      if (m >= d.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n < d.N) Y[oy + m * d.y_m + n * d.y_n] = acc[i][j];
      }
    }
  }
}

int matmul_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  const TensorState &ta = ctx->tensors[node->inputs[0]];
  const TensorState &tb = ctx->tensors[node->inputs[1]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (ta.record->dtype != SPKV2_DTYPE_FP32 || tb.record->dtype != SPKV2_DTYPE_FP32 ||
      ty.record->dtype != SPKV2_DTYPE_FP32)
    return SPKV2_ERR_UNSUPPORTED;
  const View va = make_view(ta), vb = make_view(tb), vy = make_view(ty);
  if (va.rank < 2 || vb.rank < 2 || vy.rank < 2) return -11;
  const int ar = va.rank, br = vb.rank, yr = vy.rank;
  MatmulPlan *p = new MatmulPlan();
  MatmulDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  d.M = int(vy.dim[yr - 2]);
  d.N = int(vy.dim[yr - 1]);
  d.K = int(va.dim[ar - 1]);
  bool ok = va.dim[ar - 2] == d.M && vb.dim[br - 2] == d.K && vb.dim[br - 1] == d.N && yr - 2 <= kMaxRank;
  d.nb = yr - 2;
  d.batches = 1;
  for (int k = 0; k < d.nb && ok; ++k) {
    d.bdim[k] = vy.dim[k];
    d.ys[k] = vy.stride[k];
    d.batches *= vy.dim[k];
    // Right-aligned operand dims; a size-1 or missing dim broadcasts.
    const int ad = k - (yr - ar), bd = k - (yr - br);
    d.as[k] = (ad < 0 || va.dim[ad] == 1) ? 0 : va.stride[ad];
    d.bs[k] = (bd < 0 || vb.dim[bd] == 1) ? 0 : vb.stride[bd];
    if (ad >= 0 && va.dim[ad] != 1 && va.dim[ad] != vy.dim[k]) ok = false;
    if (bd >= 0 && vb.dim[bd] != 1 && vb.dim[bd] != vy.dim[k]) ok = false;
  }
  if (!ok) {
    delete p;
    return -11;
  }
  d.a_m = va.stride[ar - 2];
  d.a_k = va.stride[ar - 1];
  d.b_k = vb.stride[br - 2];
  d.b_n = vb.stride[br - 1];
  d.y_m = vy.stride[yr - 2];
  d.y_n = vy.stride[yr - 1];
  p->variant = "matmul_tile64_fp32";
  set_node_plan(ctx, node, p);
  return 0;
}

int matmul_run(Spkv2Context *ctx, const Spkv2NodeRecord *node) {
  MatmulPlan *p = node_plan<MatmulPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  const MatmulDesc &d = p->d;
  if (d.M == 0 || d.N == 0 || d.batches == 0) return 0;
  dim3 grid(unsigned(ceil_div(d.N, 64)), unsigned(ceil_div(d.M, 64)), unsigned(std::min<int64_t>(d.batches, 65535)));
  matmul_tile_kernel<<<grid, 256, 0, ctx->stream>>>(reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data),
                                                    reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data),
                                                    reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data),
                                                    d);
  return cuda_status(cudaGetLastError());
}

__global__ void gemm_naive_kernel(float *__restrict__ Y, const float *__restrict__ A, const float *__restrict__ B,
                                  const float *__restrict__ bias, int M, int K, int N, int ta, int tb, float alpha) {
  const int64_t total = int64_t(M) * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / N), n = int(i % N);
    float s = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float av = ta ? A[int64_t(k) * M + m] : A[int64_t(m) * K + k];
      const float bv = tb ? B[int64_t(n) * K + k] : B[int64_t(k) * N + n];
      s = fmaf(av, bv, s);
    }
    Y[i] = alpha * s + (bias ? bias[n] : 0.0f);
  }
}

}  // namespace

// ---------------- allocation-free GEMV entry point ----------------
//
// Some callers cannot allocate device memory at call time: code that runs
// inside a CUDA stream capture (allocation is not a capturable operation),
// real-time loops where cudaMalloc's implicit device synchronisation would
// break the latency budget, and deployments built from the fixed-memory
// target profiles (allow_runtime_malloc = false) whose memory is budgeted
// ahead of time.  spkv2_cuda_gemv_noalloc serves them: the split-K partial
// sums live in the file-scope array below, sized once at load time, and the
// call itself allocates nothing.

namespace {

// 1 MiB of split-K partials: ksplit * M * N must not exceed this many floats.
constexpr size_t kNoAllocPartials = 262144;
__device__ __align__(256) float g_noalloc_partials[kNoAllocPartials];

constexpr int kMaxDevices = 64;
// Per-device cache of the array's device address.  Atomic slots: host
// threads making their first call on one device at the same time each
// resolve the address (the same value) and store it without a data race.
std::atomic<float *> g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_partials on the current device.  In host code
// the array's name is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress, once per device, with that device current.
int noalloc_scratch(float **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SPKV2_ERR_NO_DEVICE;
  float *cached = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!cached) {
    void *p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (err != cudaSuccess || !p) return cuda_status(err == cudaSuccess ? cudaErrorInvalidSymbol : err);
    cached = static_cast<float *>(p);
    g_noalloc_ptr[dev].store(cached, std::memory_order_release);
  }
  *out = cached;
  return 0;
}

}  // namespace

int gemm_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 2 || node->output_count < 1) return -3;
  if (node->op_type == SPKV2_OP_MATMUL) return matmul_prepare(ctx, node);
  if (node->op_type != SPKV2_OP_GEMM) return SPKV2_ERR_UNSUPPORTED;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &ta = ctx->tensors[node->inputs[0]];
  const TensorState &tb = ctx->tensors[node->inputs[1]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (ta.record->rank != 2 || tb.record->rank != 2 || ty.record->rank != 2) return -11;
  if (ta.record->dtype != SPKV2_DTYPE_FP32 || tb.record->dtype != SPKV2_DTYPE_FP32 ||
      ty.record->dtype != SPKV2_DTYPE_FP32)
    return SPKV2_ERR_UNSUPPORTED;
  GemmPlan *p = new GemmPlan();
  p->trans_a = a.trans_a;
  p->trans_b = a.trans_b;
  p->alpha = a.alpha;
  p->M = int(a.trans_a ? ta.record->shape[1] : ta.record->shape[0]);
  p->K = int(a.trans_a ? ta.record->shape[0] : ta.record->shape[1]);
  p->N = int(a.trans_b ? tb.record->shape[0] : tb.record->shape[1]);
  // The reference adds c[n] to column n whatever C's shape (a [M, N] C
  // contributes its first row); a C with fewer than N elements would be read
  // past its end there, and is rejected here.
  if (node->input_count > 2 && elem_count(ctx->tensors[node->inputs[2]].record) < size_t(p->N)) {
    delete p;
    return -11;
  }
  if (!p->trans_a && !p->trans_b && p->M <= kGemvMaxM) {
    p->ksplit = std::max(1, std::min(16, p->K / 128));
    p->partials = static_cast<float *>(device_alloc(size_t(p->ksplit) * p->M * p->N * sizeof(float) + 16));
    if (!p->partials) {
      delete p;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    p->launches = 2;
    p->variant = "gemv_splitk_fp32";
  } else if (!p->trans_a && !p->trans_b) {
    p->variant = "sgemm_tile64_fp32";
    const int math = ctx->math_mode == SPKV2_CUDA_MATH_SPEC ? SPKV2_CUDA_MATH_3XTF32 : ctx->math_mode;
    if (p->M >= kTcMinRows && p->alpha == 1.0f && math != SPKV2_CUDA_MATH_FP32) {
      // A [M,K] row-major is an NHWC [M,1,1,K] activation; Y [M,N] likewise.
      ConvPlan *c = new ConvPlan();
      ConvGeo &g = c->g;
      g.N = p->M, g.C = p->K, g.H = g.W = 1, g.M = p->N, g.OH = g.OW = 1;
      g.KH = g.KW = 1, g.sh = g.sw = 1, g.ph = g.pw = 0, g.dh = g.dw = 1;
      g.groups = 1, g.Cg = p->K, g.Mg = p->N, g.K = p->K, g.P = p->M;
      g.xs[0] = p->K, g.xs[1] = 1, g.xs[2] = p->K, g.xs[3] = p->K;
      g.ys[0] = p->N, g.ys[1] = 1, g.ys[2] = p->N, g.ys[3] = p->N;
      g.act = 0;
      g.has_bias = node->input_count > 2 ? 1 : 0;
      g.has_res = 0;
      c->mode = kConvF32;
      c->math = math;
      c->bias_f = g.has_bias ? reinterpret_cast<const float *>(ctx->tensors[node->inputs[2]].data) : nullptr;
      int trc = conv_tc_prepare_ex(*c, tb.data, ta.data, ty.data, true, ctx->stream);
      if (trc == 0) trc = conv_tc_attach(ctx, *c);
      if (trc == 0) {
        p->tc = c;
        p->launches = c->launches;
        p->variant = "gemm_as_" + c->variant;
      } else {
        delete c;
        if (trc != SPKV2_ERR_UNSUPPORTED) {
          delete p;
          return trc;
        }
      }
    }
  } else {
    p->variant = "gemm_naive_fp32";
  }
  set_node_plan(ctx, node, p);
  return 0;
}

int gemm_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  if (node->op_type == SPKV2_OP_MATMUL) return matmul_run(ctx, node);
  GemmPlan *p = node_plan<GemmPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->M == 0 || p->N == 0) return 0;
  float *Y = reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data);
  const float *A = reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data);
  const float *B = reinterpret_cast<const float *>(ctx->tensors[node->inputs[1]].data);
  const float *bias = node->input_count > 2 ? reinterpret_cast<const float *>(ctx->tensors[node->inputs[2]].data) : nullptr;
  if (p->tc) return conv_tc_launch(*p->tc, A, Y, nullptr, ctx->d_status, ctx->stream, ctx->d_sk_ws);
  if (p->partials) {
    const int kpb = int(ceil_div(p->K, p->ksplit));
    dim3 grid(unsigned(ceil_div(p->N, 32)), unsigned(p->ksplit));
    gemv_partial_kernel<<<grid, dim3(32, kGemvWarps), 0, ctx->stream>>>(p->partials, A, B, p->M, p->K, p->N, kpb);
    gemv_finish_kernel<<<grid_for(int64_t(p->M) * p->N, 256), 256, 0, ctx->stream>>>(Y, p->partials, bias, p->M, p->N,
                                                                                      p->ksplit, p->alpha);
  } else if (!p->trans_a && !p->trans_b) {
    dim3 grid(unsigned(ceil_div(p->N, 64)), unsigned(ceil_div(p->M, 64)));
    sgemm_tile_kernel<<<grid, 256, 0, ctx->stream>>>(Y, A, B, bias, p->M, p->K, p->N, p->alpha);
  } else {
    gemm_naive_kernel<<<grid_for(int64_t(p->M) * p->N, 256), 256, 0, ctx->stream>>>(Y, A, B, bias, p->M, p->K, p->N,
                                                                                     p->trans_a, p->trans_b, p->alpha);
  }
  return cuda_status(cudaGetLastError());
}

}  // namespace spkv2

extern "C" int spkv2_cuda_gemv_noalloc(const float *A, const float *B, const float *bias, float *Y, int M, int K,
                                       int N, float alpha, void *stream) {
  using namespace spkv2;
  if (!A || !B || !Y || M < 1 || K < 1 || N < 1) return -1;
  if (M > kGemvMaxM) return -14;  // rows beyond the GEMV kernel's register tile
  int ksplit = std::max(1, std::min(16, K / 128));
  while (ksplit > 1 && size_t(ksplit) * M * N > kNoAllocPartials) --ksplit;
  if (size_t(ksplit) * M * N > kNoAllocPartials) return -14;  // partials exceed the static scratch
  float *part = nullptr;
  int rc = noalloc_scratch(&part);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int kpb = int(ceil_div(K, ksplit));
  dim3 grid(unsigned(ceil_div(N, 32)), unsigned(ksplit));
  gemv_partial_kernel<<<grid, dim3(32, kGemvWarps), 0, s>>>(part, A, B, M, K, N, kpb);
  gemv_finish_kernel<<<grid_for(int64_t(M) * N, 256), 256, 0, s>>>(Y, part, bias, M, N, ksplit, alpha);
  return cuda_status(cudaGetLastError());
}
