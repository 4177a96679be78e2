// ReduceMean / ReduceMax, Softmax and TopK.
//
// Semantics (reference):
//   Reduce  reference/reduce/reduce.c:5-45   axes from input[1] (fp32 data),
//           else attr.extra, else all dims; keepdims; ReduceMax starts at -inf;
//           ReduceMean adds x/denom element by element in row-major order
//           (denom = fp32 product of the reduced dims).  INT8 ReduceMean (the
//           quantised models' global pool) sums the codes exactly in int32 and
//           returns (float)sum * (s_x / denom) with the factor formed in fp32.
//   Softmax reference/activation/softmax.c:5-41   max-shifted expf, divide by
//           the sum
//   TopK    reference/tensor/topk.c:5-124   k from input[1]; values and fp32
//           indices sorted (descending if largest), ties to the smaller index,
//           equal values at the k-th place keep the earlier indices
// Device design: reductions run one thread per output element looping over
// the reduced index space in the reference's order (bit-exact with it;
// adjacent reduced axes forming one strided run are walked as one); the
// threads of a warp take adjacent outputs, so NHWC global pooling reads
// coalesce along C.  Softmax uses a warp per row when the axis is innermost in
// row-major tensors (a block per row for a few rows of 512 or more), else one
// thread per row over any layouts.
// TopK (one block per row) radix-selects the k smallest (value, index) keys
// and sorts those (k <= 2048; rows of any length, keys in shared memory up
// to 16384 elements, recomputed from global memory beyond), else
// bitonic-sorts the whole row in shared memory (up to 16384 elements).
#include <string.h>

#include "common.cuh"

namespace spkv2 {

namespace {

struct ReduceDesc {
  int keep_rank;
  int64_t keep_dim[kMaxRank];
  int64_t keep_xstride[kMaxRank];
  int64_t keep_ystride[kMaxRank];
  int red_rank;
  int64_t red_dim[kMaxRank];
  int64_t red_xstride[kMaxRank];
  float denom;
  int o32;                       // output count < 2^31: coordinates by 32-bit multiply-shift divisions
  FastDiv keep_div[kMaxRank];    // keep_dim[k]
};

// Input and output offsets of output element o (row-major over the kept
// dims).
__device__ __forceinline__ void reduce_bases(const ReduceDesc &d, int64_t o, int64_t &xb, int64_t &yo) {
  xb = 0;
  yo = 0;
  if (d.o32) {
    uint32_t rem = uint32_t(o);
    for (int k = d.keep_rank - 1; k >= 0; --k) {
      const uint32_t q = d.keep_div[k].div(rem);
      const int64_t c = int64_t(rem - q * d.keep_div[k].d);
      rem = q;
      xb += c * d.keep_xstride[k];
      yo += c * d.keep_ystride[k];
    }
    return;
  }
  int64_t rem = o;
  for (int k = d.keep_rank - 1; k >= 0; --k) {
    const int64_t c = rem % d.keep_dim[k];
    rem /= d.keep_dim[k];
    xb += c * d.keep_xstride[k];
    yo += c * d.keep_ystride[k];
  }
}

struct ReducePlan : NodePlan {
  ReduceDesc d;
  bool is_max = false;
  bool int8_in = false;
  float int8_factor = 1.0f;
  int64_t outputs = 0;
};

template <bool IS_MAX>
__global__ void reduce_kernel(float *__restrict__ y, const float *__restrict__ x, ReduceDesc d, int64_t outputs,
                              int64_t red_count) {
  for (int64_t o = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; o < outputs; o += int64_t(gridDim.x) * blockDim.x) {
    int64_t xb, yo;
    reduce_bases(d, o, xb, yo);
    float acc = IS_MAX ? -INFINITY : 0.0f;
    if (d.red_rank == 1) {
      // One reduced axis (adjacent reduced axes are merged at prepare): a
      // strided walk, sixteen loads in flight; the accumulation order stays
      // r = 0, 1, 2, ... as in the reference.
      const int64_t st = d.red_xstride[0];
      const float *p = x + xb;
      int64_t r = 0;
      for (; r + 16 <= red_count; r += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = p[(r + j) * st];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (IS_MAX)
            acc = v[j] > acc ? v[j] : acc;
          else
            acc += v[j] / d.denom;
        }
      }
      for (; r < red_count; ++r) {
        const float v = p[r * st];
        if (IS_MAX) {
          acc = v > acc ? v : acc;
        } else {
          acc += v / d.denom;
        }
      }
      y[yo] = acc;
      continue;
    }
    for (int64_t r = 0; r < red_count; ++r) {
      int64_t rr = r, xo = xb;
      for (int k = d.red_rank - 1; k >= 0; --k) {
        xo += (rr % d.red_dim[k]) * d.red_xstride[k];
        rr /= d.red_dim[k];
      }
      const float v = x[xo];
      if (IS_MAX) {
        if (v > acc) acc = v;
      } else {
        acc += v / d.denom;
      }
    }
    y[yo] = acc;
  }
}

__global__ void reduce_mean_i8_kernel(float *__restrict__ y, const int8_t *__restrict__ x, ReduceDesc d,
                                      int64_t outputs, int64_t red_count, float factor) {
  for (int64_t o = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; o < outputs; o += int64_t(gridDim.x) * blockDim.x) {
    int64_t xb, yo;
    reduce_bases(d, o, xb, yo);
    int32_t acc = 0;
    if (d.red_rank == 1) {
      // Integer sums are exact in any order: eight loads in flight.
      const int64_t st = d.red_xstride[0];
      const int8_t *p = x + xb;
      int64_t r = 0;
      for (; r + 8 <= red_count; r += 8) {
        int v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = p[(r + j) * st];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc += v[j];
      }
      for (; r < red_count; ++r) acc += p[r * st];
      y[yo] = __fmul_rn(float(acc), factor);
      continue;
    }
    for (int64_t r = 0; r < red_count; ++r) {
      int64_t rr = r, xo = xb;
      for (int k = d.red_rank - 1; k >= 0; --k) {
        xo += (rr % d.red_dim[k]) * d.red_xstride[k];
        rr /= d.red_dim[k];
      }
      acc += x[xo];
    }
    y[yo] = __fmul_rn(float(acc), factor);
  }
}

// ---------------- Softmax ----------------

// Softmax over any layouts (a channels-last rank-4 input, an output in
// another layout): one thread per row, the row's other coordinates walked
// in the output's physical order so neighbouring threads write
// neighbouring outputs.
struct SoftmaxView {
  int rank;                   // other (non-axis) dims
  int64_t dim[kMaxRank];      // in the output's physical order
  int64_t xs[kMaxRank], ys[kMaxRank];
  int64_t n, sxa, sya;        // axis extent and strides
};

struct SoftmaxPlan : NodePlan {
  int64_t outer = 1, dim = 1, inner = 1;
  bool view = false;
  SoftmaxView v;
};

__global__ void softmax_view_kernel(float *__restrict__ y, const float *__restrict__ x, SoftmaxView d, int64_t rows) {
  for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < rows; r += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = r, bx = 0, by = 0;
    for (int k = d.rank - 1; k >= 0; --k) {
      const int64_t c = rem % d.dim[k];
      rem /= d.dim[k];
      bx += c * d.xs[k];
      by += c * d.ys[k];
    }
    float m = -INFINITY;
    for (int64_t j = 0; j < d.n; ++j) m = fmaxf(m, x[bx + j * d.sxa]);
    float s = 0.0f;
    for (int64_t j = 0; j < d.n; ++j) {
      const float e = expf(x[bx + j * d.sxa] - m);
      y[by + j * d.sya] = e;
      s += e;
    }
    for (int64_t j = 0; j < d.n; ++j) y[by + j * d.sya] = y[by + j * d.sya] / s;
  }
}

__global__ void softmax_rows_kernel(float *__restrict__ y, const float *__restrict__ x, int64_t rows, int64_t dim) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t row = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; row < rows; row += warps) {
    const float *xr = x + row * dim;
    float *yr = y + row * dim;
    float m = -INFINITY;
    for (int64_t i = lane; i < dim; i += 32) m = fmaxf(m, xr[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
    for (int64_t i = lane; i < dim; i += 32) {
      const float e = expf(xr[i] - m);
      yr[i] = e;
      s += e;
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncwarp();
    for (int64_t i = lane; i < dim; i += 32) yr[i] = yr[i] / s;
  }
}

// Few long rows (a batch-1 classifier head): one 256-thread block per row,
// block-wide max and sum through shared memory.
constexpr int kSoftmaxBlock = 256;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float *sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  __syncthreads();  // sh is free (an earlier reduction has been read)
  if (lane == 0) sh[w] = v;
  __syncthreads();
  v = sh[0];
  for (int i = 1; i < kSoftmaxBlock / 32; ++i) v = is_max ? fmaxf(v, sh[i]) : v + sh[i];
  return v;
}

__global__ void __launch_bounds__(kSoftmaxBlock) softmax_row_block_kernel(float *__restrict__ y,
                                                                          const float *__restrict__ x, int64_t rows,
                                                                          int64_t dim) {
  __shared__ float sh[kSoftmaxBlock / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float *xr = x + row * dim;
    float *yr = y + row * dim;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < dim; i += kSoftmaxBlock) m = fmaxf(m, xr[i]);
    m = block_reduce(m, true, sh);
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < dim; i += kSoftmaxBlock) {
      const float e = expf(xr[i] - m);
      yr[i] = e;
      s += e;
    }
    s = block_reduce(s, false, sh);
    for (int64_t i = threadIdx.x; i < dim; i += kSoftmaxBlock) yr[i] = yr[i] / s;
  }
}

__global__ void softmax_strided_kernel(float *__restrict__ y, const float *__restrict__ x, int64_t outer, int64_t dim,
                                       int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t t = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t o = t / inner, in = t % inner;
    const float *xr = x + o * dim * inner + in;
    float *yr = y + o * dim * inner + in;
    float m = -INFINITY;
    for (int64_t d = 0; d < dim; ++d) m = fmaxf(m, xr[d * inner]);
    float s = 0.0f;
    for (int64_t d = 0; d < dim; ++d) {
      const float e = expf(xr[d * inner] - m);
      yr[d * inner] = e;
      s += e;
    }
    for (int64_t d = 0; d < dim; ++d) yr[d * inner] = yr[d * inner] / s;
  }
}

// ---------------- TopK ----------------

constexpr int kTopkMaxPow2 = 16384;

struct TopkPlan : NodePlan {
  int64_t outer = 1, dim = 1, inner = 1, k = 0;
  int largest = 1;
  int pow2 = 1;
  bool select = false;     // radix select + sort of k keys (k <= kSelectMax)
  bool smem_keys = true;   // select with the row's keys in shared memory (dim <= 16384)
  int sel_pow2 = 1;
  int64_t x_axis_stride = 1;
};

// Unsigned key whose order is the float order; -0 and +0 share a key so they
// tie (and fall back to the index) as they compare equal in the reference.
__device__ __forceinline__ uint32_t float_order_key(float v) {
  const uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void topk_kernel(float *__restrict__ values, float *__restrict__ indices, const float *__restrict__ x,
                            int64_t dim, int64_t inner, int64_t k, int largest, int pow2) {
  extern __shared__ unsigned long long keys[];
  const int64_t row = blockIdx.x;
  const int64_t o = row / inner, in = row % inner;
  const float *xr = x + o * dim * inner + in;
  for (int i = threadIdx.x; i < pow2; i += blockDim.x) {
    unsigned long long key = ~0ull;
    if (i < dim) {
      uint32_t hi = float_order_key(xr[int64_t(i) * inner]);
      if (largest) hi = ~hi;
      key = (static_cast<unsigned long long>(hi) << 32) | static_cast<uint32_t>(i);
    }
    keys[i] = key;
  }
  __syncthreads();
  for (int size = 2; size <= pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < pow2 / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const unsigned long long a = keys[lo], b = keys[hi];
        if ((a > b) == ascending) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    const unsigned long long key = keys[j];
    const uint32_t idx = static_cast<uint32_t>(key & 0xffffffffu);
    values[(o * k + j) * inner + in] = xr[int64_t(idx) * inner];
    indices[(o * k + j) * inner + in] = float(idx);
  }
}

// TopK by radix select, for k <= kSelectMax: the same (value, index) keys
// as topk_kernel (unique, so the k smallest keys are exactly the answer),
// the k-th smallest key found byte by byte from the top with 256-bin
// histograms over the keys that still share the chosen prefix (stopping as
// soon as the chosen bin holds exactly the keys still needed), then only
// the selected keys sorted (bitonic, next power of two >= k).
constexpr int kSelectMax = 2048;

// SMEM_KEYS: the row's keys are built once in shared memory (dim <= 16384);
// otherwise every pass recomputes them from the input in global memory.
template <bool SMEM_KEYS>
__global__ void __launch_bounds__(1024) topk_select_kernel(float *__restrict__ values, float *__restrict__ indices,
                                                           const float *__restrict__ x, int64_t dim, int64_t inner,
                                                           int k, int largest, int sel_pow2) {
  extern __shared__ unsigned long long keys[];  // dim keys (SMEM_KEYS)
  __shared__ unsigned long long sel[kSelectMax];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_bin, s_before, s_cnt, s_count;
  const int64_t row = blockIdx.x;
  const int64_t o = row / inner, in = row % inner;
  const float *xr = x + o * dim * inner + in;
  auto make_key = [&](int64_t i) {
    uint32_t hi = float_order_key(xr[i * inner]);
    if (largest) hi = ~hi;
    return (static_cast<unsigned long long>(hi) << 32) | static_cast<uint32_t>(i);
  };
  auto key_of = [&](int64_t i) { return SMEM_KEYS ? keys[i] : make_key(i); };
  if (SMEM_KEYS)
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) keys[i] = make_key(i);
  unsigned long long hi_mask = 0, hi_val = 0;  // top bits fixed so far
  uint32_t remaining = uint32_t(k);             // rank of the k-th key among the candidates
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
      const unsigned long long key = key_of(i);
      if ((key & hi_mask) == hi_val) atomicAdd(&hist[uint32_t(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // Warp 0: bin b with before(b) < remaining <= before(b) + hist[b].
      const int lane = threadIdx.x;
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[lane * 8 + j];
        tot += c[j];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      uint32_t before = incl - tot;
      if (before < remaining && remaining <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (before < remaining && remaining <= before + c[j]) {
            s_bin = uint32_t(lane * 8 + j);
            s_before = before;
            s_cnt = c[j];
          }
          before += c[j];
        }
      }
    }
    __syncthreads();
    remaining -= s_before;
    hi_mask |= 0xffull << shift;
    hi_val |= static_cast<unsigned long long>(s_bin) << shift;
    const bool done = s_cnt == remaining;  // the whole bin is selected
    __syncthreads();                       // everyone has read s_* before the next pass writes them
    if (done) break;
  }
  // Every key whose fixed top bits are <= the chosen prefix is selected: k keys.
  if (threadIdx.x == 0) s_count = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    const unsigned long long key = key_of(i);
    if ((key & hi_mask) <= hi_val) {
      const uint32_t pos = atomicAdd(&s_count, 1u);
      if (pos < uint32_t(kSelectMax)) sel[pos] = key;
    }
  }
  __syncthreads();
  for (int i = k + threadIdx.x; i < sel_pow2; i += blockDim.x) sel[i] = ~0ull;
  __syncthreads();
  for (int size = 2; size <= sel_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < sel_pow2 / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const unsigned long long a = sel[lo], b = sel[hi];
        if ((a > b) == ascending) {
          sel[lo] = b;
          sel[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const uint32_t idx = static_cast<uint32_t>(sel[j] & 0xffffffffu);
    values[(o * k + j) * inner + in] = xr[int64_t(idx) * inner];
    indices[(o * k + j) * inner + in] = float(idx);
  }
}

}  // namespace

int reduce_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 1 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  const int rank = tx.record->rank;
  int axes[kMaxRank];
  int naxes = 0;
  if (node->input_count > 1) {
    size_t n = 0;
    const float *v = host_weight_f32(ctx, node->inputs[1], &n);
    if (!v) return SPKV2_ERR_UNSUPPORTED;
    if (n > size_t(kMaxRank)) return -11;
    for (size_t i = 0; i < n; ++i) axes[naxes++] = int(v[i]) < 0 ? int(v[i]) + rank : int(v[i]);
  } else if (a.extra_count > 0) {
    if (a.extra_count > kMaxRank) return -11;
    for (int i = 0; i < a.extra_count; ++i) axes[naxes++] = a.extra[i] < 0 ? a.extra[i] + rank : a.extra[i];
  } else {
    for (int i = 0; i < rank; ++i) axes[naxes++] = i;
  }
  auto reduced = [&](int d) {
    for (int i = 0; i < naxes; ++i)
      if (axes[i] == d) return true;
    return false;
  };
  const View vx = make_view(tx), vy = make_view(ty);
  ReducePlan *p = new ReducePlan();
  ReduceDesc &d = p->d;
  memset(&d, 0, sizeof(d));
  p->is_max = node->op_type == SPKV2_OP_REDUCEMAX;
  p->int8_in = tx.record->dtype == SPKV2_DTYPE_INT8;
  if (ty.record->dtype != SPKV2_DTYPE_FP32 || (p->int8_in && p->is_max) ||
      (!p->int8_in && tx.record->dtype != SPKV2_DTYPE_FP32)) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }
  float denom = 1.0f;
  int yd = 0;
  for (int xd = 0; xd < rank; ++xd) {
    if (reduced(xd)) {
      d.red_dim[d.red_rank] = vx.dim[xd];
      d.red_xstride[d.red_rank] = vx.stride[xd];
      d.red_rank++;
      denom *= float(vx.dim[xd]);
      if (a.keepdims) yd++;
    } else {
      if (yd >= vy.rank) {
        delete p;
        return -11;
      }
      d.keep_dim[d.keep_rank] = vx.dim[xd];
      d.keep_xstride[d.keep_rank] = vx.stride[xd];
      d.keep_ystride[d.keep_rank] = vy.stride[yd];
      d.keep_rank++;
      yd++;
    }
  }
  d.denom = denom;
  // Adjacent reduced axes that are one strided run in memory (H, W of an
  // NHWC or NCHW tensor) merge into one axis: the row-major walk over them
  // visits the same elements in the same order.
  for (int k = d.red_rank - 2; k >= 0; --k) {
    if (d.red_xstride[k] == d.red_dim[k + 1] * d.red_xstride[k + 1]) {
      d.red_dim[k] *= d.red_dim[k + 1];
      d.red_xstride[k] = d.red_xstride[k + 1];
      for (int j = k + 1; j + 1 < d.red_rank; ++j) {
        d.red_dim[j] = d.red_dim[j + 1];
        d.red_xstride[j] = d.red_xstride[j + 1];
      }
      d.red_rank--;
    }
  }
  p->outputs = 1;
  for (int k = 0; k < d.keep_rank; ++k) p->outputs *= d.keep_dim[k];
  d.o32 = p->outputs < (int64_t(1) << 31) ? 1 : 0;
  for (int k = 0; k < d.keep_rank; ++k) d.keep_div[k] = FastDiv(uint32_t(d.o32 ? d.keep_dim[k] : 1));
  if (p->int8_in) {
    const float *sx = quant_scales(ctx, find_quant_param(ctx, node->inputs[0]));
    if (!sx) {
      delete p;
      return SPKV2_ERR_UNSUPPORTED;
    }
    p->int8_factor = sx[0] / denom;  // fp32 division on the host, one rounding
  }
  p->variant = p->int8_in ? "reduce_mean_int8" : (p->is_max ? "reduce_max" : "reduce_mean");
  set_node_plan(ctx, node, p);
  return 0;
}

int reduce_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  ReducePlan *p = node_plan<ReducePlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->outputs == 0) return 0;
  int64_t red = 1;
  for (int k = 0; k < p->d.red_rank; ++k) red *= p->d.red_dim[k];
  float *y = reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data);
  const void *x = ctx->tensors[node->inputs[0]].data;
  const int g = grid_for(p->outputs, 128);
  if (p->int8_in)
    reduce_mean_i8_kernel<<<g, 128, 0, ctx->stream>>>(y, static_cast<const int8_t *>(x), p->d, p->outputs, red,
                                                      p->int8_factor);
  else if (p->is_max)
    reduce_kernel<true><<<g, 128, 0, ctx->stream>>>(y, static_cast<const float *>(x), p->d, p->outputs, red);
  else
    reduce_kernel<false><<<g, 128, 0, ctx->stream>>>(y, static_cast<const float *>(x), p->d, p->outputs, red);
  return cuda_status(cudaGetLastError());
}

int softmax_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 1 || node->output_count < 1) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  const TensorState &ty = ctx->tensors[node->outputs[0]];
  if (tx.record->dtype != SPKV2_DTYPE_FP32 || ty.record->dtype != SPKV2_DTYPE_FP32) return SPKV2_ERR_UNSUPPORTED;
  const int rank = tx.record->rank;
  const int axis = a.axis < 0 ? a.axis + rank : a.axis;
  if (axis < 0 || axis >= rank || ty.record->rank != rank) return -11;
  SoftmaxPlan *p = new SoftmaxPlan();
  if (tx.layout != kRowMajor || ty.layout != kRowMajor) {
    const View vx = make_view(tx), vy = make_view(ty);
    int order[kMaxRank], n = 0;
    for (int i = 0; i < rank; ++i)
      if (i != axis) order[n++] = i;
    std::stable_sort(order, order + n, [&](int u, int w) { return vy.stride[u] > vy.stride[w]; });
    SoftmaxView &v = p->v;
    memset(&v, 0, sizeof(v));
    v.rank = n;
    for (int j = 0; j < n; ++j) {
      v.dim[j] = vy.dim[order[j]];
      v.xs[j] = vx.stride[order[j]];
      v.ys[j] = vy.stride[order[j]];
    }
    v.n = vy.dim[axis];
    v.sxa = vx.stride[axis];
    v.sya = vy.stride[axis];
    p->view = true;
    p->outer = vy.count() / std::max<int64_t>(v.n, 1);
    p->dim = v.n;
    p->variant = "softmax_view";
    set_node_plan(ctx, node, p);
    return 0;
  }
  for (int i = 0; i < axis; ++i) p->outer *= tx.record->shape[i];
  p->dim = tx.record->shape[axis];
  for (int i = axis + 1; i < rank; ++i) p->inner *= tx.record->shape[i];
  p->variant = p->inner == 1 ? "softmax_warp_rows" : "softmax_strided";
  set_node_plan(ctx, node, p);
  return 0;
}

int softmax_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  SoftmaxPlan *p = node_plan<SoftmaxPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  float *y = reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data);
  const float *x = reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data);
  if (p->outer * p->inner == 0 || p->dim == 0) return 0;
  if (p->view) {
    softmax_view_kernel<<<grid_for(p->outer, 128), 128, 0, ctx->stream>>>(y, x, p->v, p->outer);
    return cuda_status(cudaGetLastError());
  }
  if (p->inner == 1 && p->outer <= 256 && p->dim >= 512)
    softmax_row_block_kernel<<<int(p->outer), kSoftmaxBlock, 0, ctx->stream>>>(y, x, p->outer, p->dim);
  else if (p->inner == 1)
    softmax_rows_kernel<<<grid_for(p->outer * 32, 256), 256, 0, ctx->stream>>>(y, x, p->outer, p->dim);
  else
    softmax_strided_kernel<<<grid_for(p->outer * p->inner, 128), 128, 0, ctx->stream>>>(y, x, p->outer, p->dim,
                                                                                         p->inner);
  return cuda_status(cudaGetLastError());
}

int topk_prepare(Spkv2Context *ctx, const Spkv2NodeRecord *node, const Spkv2KernelSpecRecord *) {
  if (node->input_count < 2 || node->output_count < 2) return -3;
  Spkv2AttrRecord a;
  int rc = get_attr(ctx, node, &a);
  if (rc) return rc;
  const TensorState &tx = ctx->tensors[node->inputs[0]];
  if (tx.layout != kRowMajor || tx.record->dtype != SPKV2_DTYPE_FP32) return SPKV2_ERR_UNSUPPORTED;
  for (int i = 0; i < 2; ++i)
    if (ctx->tensors[node->outputs[i]].layout != kRowMajor) return SPKV2_ERR_UNSUPPORTED;
  size_t kn = 0;
  const float *kv = host_weight_f32(ctx, node->inputs[1], &kn);
  if (!kv || kn < 1) return SPKV2_ERR_UNSUPPORTED;
  const int rank = tx.record->rank;
  const int axis = a.axis < 0 ? a.axis + rank : a.axis;
  if (axis < 0 || axis >= rank) return -11;
  TopkPlan *p = new TopkPlan();
  for (int i = 0; i < axis; ++i) p->outer *= tx.record->shape[i];
  p->dim = tx.record->shape[axis];
  for (int i = axis + 1; i < rank; ++i) p->inner *= tx.record->shape[i];
  p->k = int64_t(size_t(kv[0]));
  if (p->k > p->dim) p->k = p->dim;
  p->largest = a.largest;
  p->pow2 = 1;
  while (p->pow2 < p->dim && p->pow2 <= kTopkMaxPow2) p->pow2 <<= 1;  // stops past the sort limit
  // Rows longer than the shared-memory sort take the radix select with keys
  // recomputed from global memory (k <= 2048); longer rows with a larger k
  // have no kernel.
  if (p->pow2 > kTopkMaxPow2 && (p->k > kSelectMax || p->dim > INT32_MAX)) {
    delete p;
    return SPKV2_ERR_UNSUPPORTED;
  }
  if (p->k <= kSelectMax && (p->pow2 > kTopkMaxPow2 || !getenv("SPKV2_TOPK_FULL_SORT"))) {
    p->select = true;
    p->smem_keys = p->pow2 <= kTopkMaxPow2;
    p->sel_pow2 = 1;
    while (p->sel_pow2 < p->k) p->sel_pow2 <<= 1;
    const size_t smem = p->smem_keys ? size_t(p->dim) * sizeof(unsigned long long) : 0;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(topk_select_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    p->variant = p->smem_keys ? "topk_radix_select" : "topk_radix_select_global";
  } else {
    const size_t smem = size_t(p->pow2) * sizeof(unsigned long long);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    p->variant = "topk_bitonic";
  }
  set_node_plan(ctx, node, p);
  return 0;
}

int topk_run(Spkv2Context *ctx, const Spkv2NodeRecord *node, void *) {
  TopkPlan *p = node_plan<TopkPlan>(ctx, node);
  if (!p) return SPKV2_ERR_NOT_PREPARED;
  if (p->k == 0 || p->dim == 0) return 0;
  const int64_t rows = p->outer * p->inner;
  if (rows == 0) return 0;
  float *vals = reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data);
  float *idx = reinterpret_cast<float *>(ctx->tensors[node->outputs[1]].data);
  const float *xin = reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data);
  if (p->select) {
    if (p->smem_keys)
      topk_select_kernel<true><<<unsigned(rows), 1024, size_t(p->dim) * sizeof(unsigned long long), ctx->stream>>>(
          vals, idx, xin, p->dim, p->inner, int(p->k), p->largest, p->sel_pow2);
    else
      topk_select_kernel<false><<<unsigned(rows), 1024, 0, ctx->stream>>>(vals, idx, xin, p->dim, p->inner,
                                                                         int(p->k), p->largest, p->sel_pow2);
    return cuda_status(cudaGetLastError());
  }
  const size_t smem = size_t(p->pow2) * sizeof(unsigned long long);
  topk_kernel<<<unsigned(rows), 1024, smem, ctx->stream>>>(
      reinterpret_cast<float *>(ctx->tensors[node->outputs[0]].data),
      reinterpret_cast<float *>(ctx->tensors[node->outputs[1]].data),
      reinterpret_cast<const float *>(ctx->tensors[node->inputs[0]].data), p->dim, p->inner, p->k, p->largest,
      p->pow2);
  return cuda_status(cudaGetLastError());
}

}  // namespace spkv2
