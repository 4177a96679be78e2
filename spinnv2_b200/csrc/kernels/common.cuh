// Shared device/host helpers for the B200 kernels.
//
// A `View` describes a tensor as its logical dims plus the PHYSICAL element
// stride of every logical dim, so one kernel serves row-major (NCHW) and
// channels-last (NHWC) storage.  Memory-bound kernels iterate over the
// output in its physical order (writes coalesced) and gather inputs through
// their strides; fast paths take over when all operands are contiguous and
// identically laid out.
#pragma once

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.h"

namespace spkv2 {

constexpr int kMaxRank = 8;

struct View {
  int rank = 0;
  int64_t dim[kMaxRank] = {};
  int64_t stride[kMaxRank] = {};
  int64_t count() const {
    int64_t n = 1;
    for (int i = 0; i < rank; ++i) n *= dim[i];
    return n;
  }
};

inline View make_view(const TensorState &t) {
  View v;
  const Spkv2TensorRecord *r = t.record;
  v.rank = r->rank;
  for (int i = 0; i < v.rank && i < kMaxRank; ++i) v.dim[i] = r->shape[i];
  if (t.layout == kNHWC && v.rank == 4) {
    const int64_t C = v.dim[1], H = v.dim[2], W = v.dim[3];
    v.stride[0] = H * W * C;
    v.stride[1] = 1;
    v.stride[2] = W * C;
    v.stride[3] = C;
  } else {
    int64_t s = 1;
    for (int i = v.rank - 1; i >= 0; --i) {
      v.stride[i] = s;
      s *= v.dim[i];
    }
  }
  return v;
}

inline bool is_rowmajor(const View &v) {
  int64_t s = 1;
  for (int i = v.rank - 1; i >= 0; --i) {
    if (v.dim[i] != 1 && v.stride[i] != s) return false;
    s *= v.dim[i];
  }
  return true;
}

// Iteration space over an output in physical order, with each operand's
// strides reordered to match.  Operand 0 is the output.
template <int NOPS>
struct IterSpace {
  int rank = 0;
  int64_t dim[kMaxRank] = {};
  int64_t stride[NOPS][kMaxRank] = {};
};

// Builds the physical-order iteration space of `out`; `ins` are broadcast to
// out's rank (right-aligned, size-1 dims get stride 0).
template <int NOPS>
inline IterSpace<NOPS> make_iter(const View &out, const View *ins, int nin) {
  IterSpace<NOPS> it;
  int order[kMaxRank];
  for (int i = 0; i < out.rank; ++i) order[i] = i;
  std::stable_sort(order, order + out.rank, [&](int a, int b) { return out.stride[a] > out.stride[b]; });
  it.rank = out.rank;
  for (int j = 0; j < out.rank; ++j) {
    const int d = order[j];
    it.dim[j] = out.dim[d];
    it.stride[0][j] = out.stride[d];
    for (int k = 0; k < nin && k + 1 < NOPS; ++k) {
      const View &in = ins[k];
      const int dd = d - (out.rank - in.rank);
      it.stride[k + 1][j] = (dd < 0 || in.dim[dd] == 1) ? 0 : in.stride[dd];
    }
  }
  return it;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Division by a run-time-invariant 32-bit divisor d >= 1 as a multiply-high
// and shifts (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994, round-up variant): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (t + ((n - t) >> 1)) >> (l - 1)
// where t = mulhi(m, n), for every 32-bit n; d = 1 is handled apart.
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div) {
    if (d <= 1) return;
    uint32_t l = 0;
    while ((uint64_t(1) << l) < d) ++l;
    m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
    s = l - 1;
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (d == 1) return n;
#ifdef __CUDA_ARCH__
    const uint32_t t = __umulhi(m, n);
#else
    const uint32_t t = uint32_t((uint64_t(m) * n) >> 32);
#endif
    return (t + ((n - t) >> 1)) >> s;
  }
};

// A small constant fp32 tensor (axes, k, slice bounds, constant indices)
// read from the package's host copy of the weights; nullptr if the tensor is
// not an fp32 weight inside the weight section.
inline const float *host_weight_f32(const Spkv2Context *ctx, uint32_t tid, size_t *count) {
  const Spkv2TensorRecord *r = ctx->tensors[tid].record;
  if (r->role != SPKV2_ROLE_WEIGHT || r->dtype != SPKV2_DTYPE_FP32) return nullptr;
  if (r->data_offset + r->size_bytes > ctx->weights_size) return nullptr;
  *count = elem_count(r);
  return reinterpret_cast<const float *>(ctx->weights + r->data_offset);
}

inline int grid_for(int64_t n, int threads) {
  int64_t blocks = ceil_div(n, threads);
  // Grid-stride beyond 148 SMs x 32 resident blocks.
  return int(std::min<int64_t>(std::max<int64_t>(blocks, 1), 148LL * 32));
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == 1) return v > 0.0f ? v : 0.0f;
  if (act == 2) return v / (1.0f + expf(-v));
  return v;
}

// apply_act over a register array, branching once: inside an element loop
// the compiler may if-convert the switch and evaluate the SiLU expf and
// divide for every element whatever `act` is.
template <int N>
__device__ __forceinline__ void apply_act_n(float (&v)[N], int act) {
  if (act == 1) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
  } else if (act == 2) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = v[j] / (1.0f + expf(-v[j]));
  }
}
__device__ __forceinline__ void apply_act32(float (&v)[32], int act) { apply_act_n<32>(v, act); }

// int8 requantisation rounding: round half to even, clamp to [lo, 127].
__device__ __forceinline__ int8_t sat_rne_i8(float v, int lo) {
  int q = __float2int_rn(v);
  q = q < lo ? lo : q;
  q = q > 127 ? 127 : q;
  return int8_t(q);
}

}  // namespace spkv2
