// Diagnostic (not part of the runtime library): raw tcgen05.mma issue rate on
// this GPU.  One CTA per SM issues `iters` K steps of four M=128 x N MMAs
// (TF32: K=8 each, INT8: K=32 each) from fixed zeroed shared memory into one
// TMEM accumulator, then waits for them (bounded) and reports cycles per K
// step, MAC/cycle/SM and the aggregate rate.  These are the per-MMA costs the
// tile-width model in conv.h (pick_block_n) uses.
// Build and run on a B200:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -I spinnv2_b200/csrc/kernels -o /tmp/mma_rates spinnv2_b200/diag/mma_rates.cu && /tmp/mma_rates
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
#include "tcgen05.cuh"
using namespace spkv2::tc;

template <int N, int KIND, int NSTAGE>  // KIND 0 tf32, 1 i8
__global__ void __launch_bounds__(128, 1) mma_kernel(long long *cycles, int iters, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t done;
  __shared__ uint32_t tbase;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < NSTAGE * (16384 + N * 128) / 4; i += blockDim.x) reinterpret_cast<uint32_t *>(smem)[i] = 0;
  if (threadIdx.x == 0) { mbar_init(&done, 1); asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase)), "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before(); __syncthreads(); tc_fence_after();
  const uint32_t tmem = tbase;
  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = KIND == 0 ? ((1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (8u << 24))
                                         : ((2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (8u << 24));
    const long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
      uint8_t *st = smem + (i % NSTAGE) * (16384 + N * 128);
      const uint64_t da = smem_desc(st), db = smem_desc(st + 16384);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t step = uint64_t(kk * 32) >> 4;
        if (KIND == 0) mma_tf32(tmem, da + step, db + step, idesc, (i | kk) ? 1u : 0u);
        else mma_i8(tmem, da + step, db + step, idesc, (i | kk) ? 1u : 0u);
      }
    }
    mma_commit(&done);
    const long long tw = clock64();
    while (!mbar_try_wait(&done, 0) && clock64() - tw < kWaitCycles) {}
    cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before(); __syncthreads();
  if (warp == 0) { tc_fence_after(); asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)); }
}

template <int N, int KIND, int NSTAGE>
void run(const char *name, int iters) {
  long long *d; cudaMalloc(&d, 148 * 8);
  int *st; cudaMalloc(&st, 4);
  const int smem = NSTAGE * (16384 + N * 128) + 1024;
  cudaFuncSetAttribute(mma_kernel<N, KIND, NSTAGE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mma_kernel<N, KIND, NSTAGE><<<148, 128, smem>>>(d, iters, st);
  cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
  cudaEventRecord(a);
  mma_kernel<N, KIND, NSTAGE><<<148, 128, smem>>>(d, iters, st);
  cudaEventRecord(b); cudaEventSynchronize(b);
  float ms; cudaEventElapsedTime(&ms, a, b);
  long long h[148]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  double avg = 0; for (int i = 0; i < 148; ++i) avg += h[i]; avg /= 148;
  const double macs = double(iters) * 4 * 128 * N * (KIND == 0 ? 8 : 32);
  printf("%-22s N=%3d stages=%d: %.1f cycles/K-step(4 MMAs), %.0f MAC/cycle/SM, %.1f T(FL)OPS total (%s)\n", name, N, NSTAGE,
         avg / iters, macs / avg, 2.0 * macs * 148 / (ms * 1e-3) / 1e12, cudaGetErrorString(cudaGetLastError()));
  cudaFree(d); cudaFree(st);
}

int main() {
  run<64, 0, 1>("tf32", 20000);
  run<128, 0, 1>("tf32", 20000);
  run<256, 0, 1>("tf32", 20000);
  run<256, 0, 4>("tf32 4 stages", 20000);
  run<64, 1, 1>("i8", 20000);
  run<128, 1, 1>("i8", 20000);
  run<256, 1, 1>("i8", 20000);
  return 0;
}
