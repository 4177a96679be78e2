// tcgen05 implicit-GEMM conv (sm_100a).  Filled in below the CUDA-core path.
#include "conv.h"

namespace spkv2 {

int conv_tc_prepare(ConvPlan &p, const void *w_raw_dev, cudaStream_t s) {
  (void)p;
  (void)w_raw_dev;
  (void)s;
  return SPKV2_ERR_UNSUPPORTED;
}

int conv_tc_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s) {
  (void)status;
  return conv_simt_launch(p, x, y, res, s);
}

}  // namespace spkv2
