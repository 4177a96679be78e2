// Watchdog self-test: one block waits on an mbarrier that nothing arrives at,
// through the same bounded wait the tcgen05 kernels use, gives up after the
// given number of clock cycles, records its code in the context's status word
// and returns.  Nothing faults, traps or spins unbounded, so the context
// stays usable afterwards.
#include "common.cuh"
#include "tcgen05.cuh"

namespace spkv2 {

namespace {

using namespace tc;

constexpr int kProbeCode = 9;

__global__ void watchdog_probe_kernel(int *status, long long limit_cycles) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, &abort_flag, status, kProbeCode, limit_cycles);
  __syncthreads();
}

}  // namespace

int watchdog_probe(int *d_status, uint32_t wait_us, cudaStream_t s) {
  int dev = 0, khz = 1965000;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev);
  const long long cycles = (long long)(wait_us) * (long long)(khz) / 1000;
  watchdog_probe_kernel<<<1, 32, 0, s>>>(d_status, cycles);
  return cuda_status(cudaGetLastError());
}

}  // namespace spkv2
