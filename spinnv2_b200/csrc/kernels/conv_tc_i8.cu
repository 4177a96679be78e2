// tcgen05 kind::i8 implicit-GEMM convolution for sm_100a: int8 NHWC
// activations x int8 packed weights -> int32 accumulators in TMEM -> the
// requantising epilogue (or int32 output).
//
// Requantisation (one rounding per operation, no fused multiply-add):
//   a = acc + b_q[c]
//   v = fp32(a) * M[c]                     M[c] = fp32(s_x * s_w[c]) / s_y
//   v = v + fp32(r) * R                    fused residual r (int8), R = s_r / s_y
//   y = clamp(rne(v), Relu ? 0 : -128, 127)
// int32 output mode (int8 -> int32 conv): y = a.
//
// GEMM view as in conv_tc.cu: rows = output pixels, columns = output
// channels, K = (r, s, c) with c fastest; one K step = 128 int8 = 128 bytes,
// four MMAs of K = 32.  Persistent kernel, one CTA per SM, 320 threads:
//   warps 0-3  epilogue (TMEM lanes 32w..32w+31, double-buffered accumulator)
//   warps 4-7  A gathers (AMODE 1): 16-byte cp.async chunks (16 channels of
//              one tap, zero-fill for padding) straight into the operand
//              stage.  Each thread signals step it-(STAGES-1) (its own
//              copies landed: cp.async.wait_group, proxy fence, mbarrier
//              arrive) BEFORE it waits for the stage of step it to free up,
//              so the MMA never waits on that wait.
//   warp 8     TMA producer: weight panel B, and A in AMODE 2 (1x1 stride 1).
//   warp 9     TMEM allocation and the single-thread MMA issuer.
// Every wait is bounded; on timeout the CTA records a code in the status
// word and winds down.
#include <stdlib.h>
#include <string.h>

#include "conv.h"
#include "tcgen05.cuh"

namespace spkv2 {

namespace {

using namespace tc;

constexpr int kBM = 128;           // tile rows (pixels) = UMMA M
constexpr int kBK = 128;           // int8 elements (bytes) per K step
constexpr int kABytes = kBM * kBK;
constexpr int kThreads = 320;

struct I8Params {
  ConvGeo g;
  int Kpad, Npad, num_kb, n_tiles;
  int64_t tiles;
  int out_i32;  // 1: int32 output (acc + b_q), no requantisation
};

__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int BN, int STAGES, int AMODE>
__global__ void __launch_bounds__(kThreads, 1)
    conv_i8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                   const int8_t *__restrict__ x, const int32_t *__restrict__ bias_q,
                   const float *__restrict__ scale_m, const int8_t *__restrict__ res, void *__restrict__ y,
                   I8Params tp, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int B_BYTES = BN * kBK;
  constexpr int STAGE = kABytes + B_BYTES;
  constexpr int kCols = 2 * BN;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  __shared__ uint64_t raw_bar[STAGES], full_bar[STAGES], empty_bar[STAGES], accf_bar[2], acce_bar[2];
  __shared__ uint32_t tmem_base_holder;
  __shared__ volatile int abort_flag;

  const ConvGeo &g = tp.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&raw_bar[s], 1);     // TMA: B (and A in AMODE 2)
      mbar_init(&full_bar[s], 128);  // A gathers landed (AMODE 1)
      mbar_init(&empty_bar[s], 1);   // MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 128);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_holder;

  if (warp < 4) {
    // ------------------------------------------------------------ epilogue
    const int lo = g.act == 1 ? 0 : -128;
    const bool vec_out = g.ys[1] == 1 && (g.M % 16) == 0;
    const bool vec_res = g.has_res && g.rs[1] == 1 && (g.M % 16) == 0;
    const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
    int ti = 0;
    for (int64_t t = blockIdx.x; t < tp.tiles; t += gridDim.x, ++ti) {
      const int n0 = int(t % tp.n_tiles) * BN;
      const int64_t m0 = (t / tp.n_tiles) * kBM;
      const int ab = ti & 1;
      if (!mbar_wait(&accf_bar[ab], (ti >> 1) & 1, &abort_flag, status, 4)) break;
      tc_fence_after();
      const int64_t p = m0 + warp * 32 + lane;
      const bool pv = p < g.P;
      int n = 0, oh = 0, ow = 0;
      if (pv) {
        ow = int(p % g.OW);
        const int64_t q = p / g.OW;
        oh = int(q % g.OH);
        n = int(q / g.OH);
      }
      const int64_t ybase = int64_t(n) * g.ys[0] + int64_t(oh) * g.ys[2] + int64_t(ow) * g.ys[3];
      const int64_t rbase = int64_t(n) * g.rs[0] + int64_t(oh) * g.rs[2] + int64_t(ow) * g.rs[3];
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 32) {
        uint32_t acc[32];
        tmem_ld32(trow + uint32_t(ab * BN + cb), acc);
        if (cb + 32 >= BN) {
          tc_fence_before();
          mbar_arrive(&acce_bar[ab]);
        }
        const int c0 = n0 + cb;
        if (c0 >= g.M || !pv) continue;
        const int cn = min(32, g.M - c0);
        int32_t a[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int4 b = (g.has_bias && j < cn) ? __ldg(reinterpret_cast<const int4 *>(bias_q + c0 + j))
                                                : make_int4(0, 0, 0, 0);
          a[j] = int32_t(acc[j]) + b.x;
          a[j + 1] = int32_t(acc[j + 1]) + b.y;
          a[j + 2] = int32_t(acc[j + 2]) + b.z;
          a[j + 3] = int32_t(acc[j + 3]) + b.w;
        }
        if (tp.out_i32) {
          int32_t *y32 = static_cast<int32_t *>(y);
          if (cn == 32 && vec_out) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<int4 *>(y32 + ybase + c0 + j) = make_int4(a[j], a[j + 1], a[j + 2], a[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cn) y32[ybase + int64_t(c0 + j) * g.ys[1]] = a[j];
          }
          continue;
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 m = j < cn ? __ldg(reinterpret_cast<const float4 *>(scale_m + c0 + j)) : make_float4(0, 0, 0, 0);
          v[j] = __fmul_rn(float(a[j]), m.x);
          v[j + 1] = __fmul_rn(float(a[j + 1]), m.y);
          v[j + 2] = __fmul_rn(float(a[j + 2]), m.z);
          v[j + 3] = __fmul_rn(float(a[j + 3]), m.w);
        }
        if (g.has_res) {
          int8_t r[32];
          if (cn == 32 && vec_res) {
            *reinterpret_cast<int4 *>(r) = __ldg(reinterpret_cast<const int4 *>(res + rbase + c0));
            *reinterpret_cast<int4 *>(r + 16) = __ldg(reinterpret_cast<const int4 *>(res + rbase + c0 + 16));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = j < cn ? res[rbase + int64_t(c0 + j) * g.rs[1]] : int8_t(0);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __fmul_rn(float(r[j]), g.res_scale));
        }
        int8_t *y8 = static_cast<int8_t *>(y);
        if (cn == 32 && vec_out) {
          uint32_t w[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            w[j] = (uint32_t(sat_rne_i8(v[4 * j], lo)) & 0xffu) | ((uint32_t(sat_rne_i8(v[4 * j + 1], lo)) & 0xffu) << 8) |
                   ((uint32_t(sat_rne_i8(v[4 * j + 2], lo)) & 0xffu) << 16) |
                   ((uint32_t(sat_rne_i8(v[4 * j + 3], lo)) & 0xffu) << 24);
          *reinterpret_cast<uint4 *>(y8 + ybase + c0) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4 *>(y8 + ybase + c0 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < cn) y8[ybase + int64_t(c0 + j) * g.ys[1]] = int8_t(sat_rne_i8(v[j], lo));
        }
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ A gathers
    if constexpr (AMODE == 1) {
      const int at = tid - 128;
      const int chunk = at & 7, rsub = at >> 3;
      uint32_t it = 0;
      bool ok = true;
      // Step `pit`'s chunks of this thread have landed: publish them.
      auto publish = [&](uint32_t pit) {
        fence_proxy_async();
        mbar_arrive(&full_bar[pit % STAGES]);
      };
      for (int64_t t = blockIdx.x; t < tp.tiles && ok; t += gridDim.x) {
        const int64_t m0 = (t / tp.n_tiles) * kBM;
        int rn[8], rih[8], riw[8];
        bool rvalid[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t p = m0 + i * 16 + rsub;
          rvalid[i] = p < g.P;
          const int64_t pp = rvalid[i] ? p : 0;
          const int ow = int(pp % g.OW);
          const int64_t q = pp / g.OW;
          rih[i] = int(q % g.OH) * g.sh - g.ph;
          riw[i] = ow * g.sw - g.pw;
          rn[i] = int(q / g.OH);
        }
        for (int kb = 0; kb < tp.num_kb && ok; ++kb, ++it) {
          if (it >= uint32_t(STAGES - 1)) {
            cp_async_wait<STAGES - 2>();  // this thread's step it-(STAGES-1) landed
            publish(it - (STAGES - 1));
          }
          const int s = it % STAGES;
          ok = mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1, &abort_flag, status, 1);
          if (!ok) break;
          uint8_t *a_st = smem + s * STAGE;
          const int k0 = kb * kBK + chunk * 16;
          const bool kval = k0 < g.K;
          const int tap = k0 / g.Cg, c = k0 - tap * g.Cg;  // 16 channels of one tap (C % 16 == 0)
          const int r = tap / g.KW, sx = tap - r * g.KW;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int ih = rih[i] + r * g.dh, iw = riw[i] + sx * g.dw;
            const bool in = kval && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
            const int8_t *src = in ? x + ((int64_t(rn[i]) * g.H + ih) * g.W + iw) * g.C + c : x;
            cp_async16(a_st + swz_off(i * 16 + rsub, chunk), src, in ? 16u : 0u);
          }
          cp_async_commit();
        }
      }
      cp_async_wait<0>();
      if (ok) {
        const uint32_t first = it > uint32_t(STAGES - 1) ? it - (STAGES - 1) : 0;
        for (uint32_t pit = first; pit < it; ++pit) publish(pit);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t bytes = B_BYTES + (AMODE == 2 ? kABytes : 0);
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tp.tiles && ok; t += gridDim.x) {
        const int n0 = int(t % tp.n_tiles) * BN;
        const int64_t m0 = (t / tp.n_tiles) * kBM;
        for (int kb = 0; kb < tp.num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          ok = mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1, &abort_flag, status, 2);
          if (!ok) break;
          uint8_t *a_st = smem + s * STAGE;
          mbar_arrive_expect_tx(&raw_bar[s], bytes);
          tma_load_2d(a_st + kABytes, &wmap, kb * kBK, n0, &raw_bar[s]);
          if (AMODE == 2) tma_load_2d(a_st, &amap, kb * kBK, int(m0), &raw_bar[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
      uint32_t it = 0;
      int ti = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tp.tiles && ok; t += gridDim.x, ++ti) {
        const int ab = ti & 1;
        ok = mbar_wait(&acce_bar[ab], ((ti >> 1) & 1) ^ 1, &abort_flag, status, 7);
        if (!ok) break;
        tc_fence_after();
        const uint32_t dtm = tmem + uint32_t(ab * BN);
        for (int kb = 0; kb < tp.num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          ok = mbar_wait(&raw_bar[s], ph, &abort_flag, status, 3);
          if (ok && AMODE == 1) ok = mbar_wait(&full_bar[s], ph, &abort_flag, status, 3);
          if (!ok) break;
          tc_fence_after();
          uint8_t *a_st = smem + s * STAGE;
          const uint64_t da = smem_desc(a_st), db = smem_desc(a_st + kABytes);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t step = uint64_t(kk * 32) >> 4;  // 32 int8 = 32 bytes along K
            mma_i8(dtm, da + step, db + step, idesc, (kb == 0 && kk == 0) ? 0u : 1u);
          }
          mma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        mma_commit(&accf_bar[ab]);
      }
      // Every issued MMA must finish before TMEM is freed (also on abort).
      if (ti > 0) {
        const int last = (ti - 1) & 1;
        const long long t0 = clock64();
        while (!mbar_try_wait(&accf_bar[last], ((ti - 1) >> 1) & 1) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// [Npad][Kpad] int8, k = (r*KW + s)*C + c, zero padding, from OIHW int8.
__global__ void pack_i8_kernel(int8_t *__restrict__ dst, const int8_t *__restrict__ w, ConvGeo g, int Npad, int Kpad) {
  const int64_t total = int64_t(Npad) * Kpad;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / Kpad), k = int(i % Kpad);
    int8_t v = 0;
    if (m < g.M && k < g.K) {
      const int c = k % g.C, rs = k / g.C, s = rs % g.KW, r = rs / g.KW;
      v = w[((int64_t(m) * g.C + c) * g.KH + r) * g.KW + s];
    }
    dst[i] = v;
  }
}

constexpr int stages_of(int bn) { return bn == 256 ? 4 : bn == 128 ? 6 : 8; }

struct I8State {
  CUtensorMap wmap, amap;
  I8Params tp;
  int bn = 128, amode = 1, grid = 148;
  size_t smem = 0;
  bool set_attr_only = false;
  mutable const void *amap_base = nullptr;  // activation pointer the A map was encoded for
};

bool encode_a(const I8State &st, CUtensorMap *map, const void *x) {
  const ConvGeo &g = st.tp.g;
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, x, uint64_t(g.C), uint64_t(g.P), uint64_t(g.C), kBM);
}

template <int BN, int AMODE>
int launch_cfg(const I8State &st, const CUtensorMap &amap, const ConvPlan &p, const void *x, void *y, const void *res,
               int *status, cudaStream_t s) {
  auto kern = conv_i8_kernel<BN, stages_of(BN), AMODE>;
  if (st.set_attr_only)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st.smem)));
  kern<<<unsigned(st.grid), kThreads, st.smem, s>>>(st.wmap, amap, static_cast<const int8_t *>(x), p.bias_q,
                                                    p.scale_m, static_cast<const int8_t *>(res), y, st.tp, status);
  return cuda_status(cudaGetLastError());
}

template <int BN>
int launch_bn(const I8State &st, const CUtensorMap &amap, const ConvPlan &p, const void *x, void *y, const void *res,
              int *status, cudaStream_t s) {
  return st.amode == 2 ? launch_cfg<BN, 2>(st, amap, p, x, y, res, status, s)
                       : launch_cfg<BN, 1>(st, amap, p, x, y, res, status, s);
}

}  // namespace

// Eligible: int8 x / w, group 1, dense NHWC input with C % 16 == 0, 16-byte
// aligned activations, Cout >= 16.
int conv_tc_i8_prepare(ConvPlan &p, const void *w_dev, const void *x_dev, cudaStream_t s) {
  const ConvGeo &g = p.g;
  if ((p.mode != kConvI8 && p.mode != kConvI8ToI32) || g.groups != 1 || g.M < 16) return SPKV2_ERR_UNSUPPORTED;
  const bool nhwc_in = g.xs[1] == 1 && g.xs[3] == g.C && g.xs[2] == int64_t(g.W) * g.C;
  if (!nhwc_in || g.C % 16 != 0 || reinterpret_cast<uintptr_t>(x_dev) % 16 != 0) return SPKV2_ERR_UNSUPPORTED;
  if (!encode_fn()) return SPKV2_ERR_UNSUPPORTED;
  I8State *st = new I8State();
  memset(&st->wmap, 0, sizeof(st->wmap));
  memset(&st->amap, 0, sizeof(st->amap));
  int bn = g.M <= 32 ? 32 : g.M <= 64 ? 64 : g.M <= 128 ? 128 : 256;
  if (const char *e = getenv("SPKV2_TC_BN")) {
    const int v = atoi(e);
    if ((v == 32 || v == 64 || v == 128 || v == 256) && v <= std::max(32, int(ceil_div(g.M, 32) * 32))) bn = v;
  }
  st->bn = bn;
  st->amode = (g.KH == 1 && g.KW == 1 && g.sh == 1 && g.sw == 1 && g.ph == 0 && g.pw == 0) ? 2 : 1;
  I8Params &tp = st->tp;
  tp.g = g;
  tp.Kpad = int(ceil_div(g.K, kBK) * kBK);
  tp.Npad = int(ceil_div(g.M, bn) * bn);
  tp.num_kb = tp.Kpad / kBK;
  tp.n_tiles = tp.Npad / bn;
  tp.tiles = ceil_div(g.P, kBM) * tp.n_tiles;
  tp.out_i32 = p.mode == kConvI8ToI32 ? 1 : 0;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  st->grid = int(std::min<int64_t>(tp.tiles, sms));
  int8_t *wp = static_cast<int8_t *>(device_alloc(size_t(tp.Npad) * tp.Kpad));
  if (!wp) {
    delete st;
    return SPKV2_ERR_DEVICE_ALLOC;
  }
  pack_i8_kernel<<<grid_for(int64_t(tp.Npad) * tp.Kpad, 256), 256, 0, s>>>(wp, static_cast<const int8_t *>(w_dev), g,
                                                                         tp.Npad, tp.Kpad);
  int rc = cuda_status(cudaGetLastError());
  bool ok = rc == 0 && encode_2d(&st->wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wp, uint64_t(tp.Kpad),
                                 uint64_t(tp.Npad), uint64_t(tp.Kpad), uint32_t(bn));
  if (ok && st->amode == 2) {
    ok = encode_a(*st, &st->amap, x_dev);
    st->amap_base = x_dev;
  }
  if (!ok) {
    device_free(wp);
    delete st;
    return rc ? rc : SPKV2_ERR_UNSUPPORTED;
  }
  st->smem = size_t(stages_of(bn)) * (kABytes + bn * kBK) + 1024;
  p.w_tc = wp;
  p.tc_state = st;
  p.tc_i8 = true;
  p.tc_block_n = bn;
  p.tc_kpad = tp.Kpad;
  st->set_attr_only = true;
  rc = conv_tc_i8_launch(p, nullptr, nullptr, nullptr, nullptr, s);
  st->set_attr_only = false;
  if (rc) return rc;
  p.variant = std::string("tc_int8_bn") + std::to_string(bn) + (st->amode == 2 ? "_tma" : "_cpasync") +
              (tp.out_i32 ? "_i32out" : "");
  return 0;
}

void conv_tc_i8_release(void *state) { delete static_cast<I8State *>(state); }

int conv_tc_i8_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s) {
  const I8State &st = *static_cast<const I8State *>(p.tc_state);
  CUtensorMap amap = st.amap;
  if (st.amode == 2 && !st.set_attr_only && x != st.amap_base) {
    // The input was rebound to another device buffer since prepare.
    if (!encode_a(st, &amap, x)) return SPKV2_ERR_UNSUPPORTED;
  }
  switch (st.bn) {
    case 32: return launch_bn<32>(st, amap, p, x, y, res, status, s);
    case 64: return launch_bn<64>(st, amap, p, x, y, res, status, s);
    case 128: return launch_bn<128>(st, amap, p, x, y, res, status, s);
    default: return launch_bn<256>(st, amap, p, x, y, res, status, s);
  }
}

}  // namespace spkv2
