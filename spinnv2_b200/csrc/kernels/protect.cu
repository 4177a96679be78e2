// Device side of reliability protection plans (reference
// core/executor.c:400-498, range guard and DMR compare with reruns).
//
//   range scan  one pass over an fp32 tensor: the number of elements that are
//               non-finite or outside [lo, hi] (reference output_in_range),
//               and min / max over the elements that are not NaN (reference
//               record_output_range: its `<` / `>` updates skip NaNs, and a
//               NaN first element leaves both at NaN, which the host applies
//               from the first-element flag).
//   differ      whether two byte ranges differ (reference memcmp of the DMR
//               copies), as 32-bit words: protected tensors are fp32.
// Min / max travel as order-preserving unsigned keys so that plain integer
// atomics combine the per-warp results.  Both entry points synchronise the
// stream and hand the result to the host, which decides on reruns.
#include "common.cuh"

namespace spkv2 {

namespace {

// Order-preserving map of a non-NaN float onto uint32 (negative values
// reversed below the positives).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

inline float key_value(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

// out: [0] min key, [1] max key, [2] elements out of range, [3] any non-NaN
// element seen, [4] first element is NaN.
__global__ void range_scan_kernel(const float *__restrict__ x, uint64_t n, float lo, float hi, uint32_t *out) {
  uint32_t mn = 0xffffffffu, mx = 0u, bad = 0u, seen = 0u;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    if (!isfinite(v) || v < lo || v > hi) ++bad;
    if (!isnan(v)) {
      const uint32_t k = order_key(v);
      mn = k < mn ? k : mn;
      mx = k > mx ? k : mx;
      seen = 1u;
    }
    if (i == 0 && isnan(v)) out[4] = 1u;
  }
  mn = __reduce_min_sync(0xffffffffu, mn);
  mx = __reduce_max_sync(0xffffffffu, mx);
  bad = __reduce_add_sync(0xffffffffu, bad);
  seen = __reduce_or_sync(0xffffffffu, seen);
  if ((threadIdx.x & 31) == 0) {
    if (seen) {
      atomicMin(&out[0], mn);
      atomicMax(&out[1], mx);
      out[3] = 1u;
    }
    if (bad) atomicAdd(&out[2], bad);
  }
}

__global__ void words_differ_kernel(const uint32_t *__restrict__ a, const uint32_t *__restrict__ b, uint64_t n,
                                    uint32_t *out) {
  uint32_t d = 0u;
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += stride) d |= a[i] ^ b[i];
  d = __reduce_or_sync(0xffffffffu, d);
  if ((threadIdx.x & 31) == 0 && d) out[0] = 1u;
}

int read_back(uint32_t *d_out, uint32_t *h_out, int words, cudaStream_t stream) {
  int rc = cuda_status(cudaMemcpyAsync(h_out, d_out, sizeof(uint32_t) * words, cudaMemcpyDeviceToHost, stream));
  return rc ? rc : cuda_status(cudaStreamSynchronize(stream));
}

}  // namespace

int guard_range_scan(const float *x, uint64_t n, float lo, float hi, uint32_t *d_out, GuardRange *res,
                     cudaStream_t stream) {
  const uint32_t init[5] = {0xffffffffu, 0u, 0u, 0u, 0u};
  int rc = cuda_status(cudaMemcpyAsync(d_out, init, sizeof(init), cudaMemcpyHostToDevice, stream));
  if (rc) return rc;
  if (n > 0) {
    range_scan_kernel<<<grid_for(int64_t(n), 256), 256, 0, stream>>>(x, n, lo, hi, d_out);
    if ((rc = cuda_status(cudaGetLastError()))) return rc;
  }
  uint32_t h[5];
  if ((rc = read_back(d_out, h, 5, stream))) return rc;
  res->out_of_range = h[2];
  res->any = h[3] != 0;
  res->first_nan = h[4] != 0;
  res->min = h[3] ? key_value(h[0]) : 0.0f;
  res->max = h[3] ? key_value(h[1]) : 0.0f;
  return 0;
}

int guard_bytes_differ(const void *a, const void *b, uint64_t bytes, uint32_t *d_out, bool *differ,
                       cudaStream_t stream) {
  const uint32_t zero = 0u;
  int rc = cuda_status(cudaMemcpyAsync(d_out, &zero, sizeof(zero), cudaMemcpyHostToDevice, stream));
  if (rc) return rc;
  const uint64_t n = bytes / 4;
  if (n > 0) {
    words_differ_kernel<<<grid_for(int64_t(n), 256), 256, 0, stream>>>(static_cast<const uint32_t *>(a),
                                                                       static_cast<const uint32_t *>(b), n, d_out);
    if ((rc = cuda_status(cudaGetLastError()))) return rc;
  }
  uint32_t h = 0;
  if ((rc = read_back(d_out, &h, 1, stream))) return rc;
  *differ = h != 0;
  return 0;
}

}  // namespace spkv2
