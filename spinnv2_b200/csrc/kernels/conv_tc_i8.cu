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
// four MMAs of K = 32.  Persistent kernel, one CTA per SM, 320 threads.
// A operand modes:
//   AMODE 3  im2col TMA (C % 128 == 0, square kernel): one tensor-map load
//            per K step brings 128 output pixels x 128 channels of one
//            filter tap, padding and image edges zero-filled by the TMA unit.
//   AMODE 5  im2col TMA for C == 64 (square kernel): a K step is two filter
//            taps, each loaded by its own im2col TMA (128 pixels x 64
//            channels, 64-byte swizzle) into one half of the A stage; the
//            MMAs read the halves through 64-byte-swizzle descriptors.  A tap
//            past the filter reads an image past the batch (zeros).
//   AMODE 2  tiled TMA (1x1, stride 1, no padding).
//   AMODE 1  cp.async gathers by warps 4-7 (C % 16 == 0), 16 channels of one
//            tap per 16-byte chunk, straight into the operand stage; each
//            thread publishes step it-(STAGES-1) (wait_group, proxy fence,
//            mbarrier arrive) before it waits for the stage of step it.
// Warp roles: epilogue warps 0-3 (AMODE 1), 0-7, or 0-15 for TMA-fed A with
// BN >= 128 (warps w, w+4, ... share TMEM lanes 32(w%4).. and split the
// tile's columns); then the TMA producer warp (weights, and A in the TMA
// modes) and the warp that allocates TMEM and issues the MMAs from one
// thread (warps 8 and 9 with 4 or 8 epilogue warps, 16 and 17 with 16).
// TMEM holds two accumulator buffers, so a tile's epilogue overlaps the
// next tile's MMAs.
// Epilogue with dense NHWC int8 output: each warp's 32 rows x CW columns go
// through a shared-memory tile: the residual tile (if any) is TMA-loaded
// into it, the requantised bytes overwrite it, and one TMA store writes it
// out.  With a residual the warp keeps two such tiles (RB = 2) and loads
// the residual of its NEXT tile while it requantises this one, so the
// residual's HBM latency is not paid once per tile (1x1 convs with K <= 128
// have little MMA work to hide it behind).  Other outputs (strided, int32)
// use per-thread stores.
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

struct I8Params {
  ConvGeo g;
  int Kpad, Npad, num_kb, n_tiles;
  int64_t tiles;
  int out_i32;  // 1: int32 output (acc + b_q), no requantisation
  int epi_tma;  // 1: NHWC int8 output (and residual) through TMA tiles
  // Tile and pixel coordinates in 32 bits by multiply-shift division (the
  // host keeps tiles and pixels below 2^31): a 64-bit division per tile and
  // pixel would cost each epilogue thread more instructions than a chunk of
  // requantisation.
  FastDiv nt_div, ow_div, oh_div;
};

// Output pixel p -> (n, oh, ow).
__device__ __forceinline__ void pixel_nhw_i8(const I8Params &tp, int64_t p, int &n, int &oh, int &ow) {
  const uint32_t q = tp.ow_div.div(uint32_t(p));
  ow = int(uint32_t(p) - q * uint32_t(tp.g.OW));
  const uint32_t r = tp.oh_div.div(q);
  oh = int(q - r * uint32_t(tp.g.OH));
  n = int(r);
}

__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Four requantised codes, a in the lowest byte: round to nearest even, then
// clamp to [lo, 127] (lo = 0 with Relu, else -128).  Relu is applied as
// max(v, 0) before rounding (the same code), the int8 saturation and the
// byte packing by cvt.pack.sat (two values per instruction: the first
// source lands in bits 15:8, the second in bits 7:0, the third operand's
// low half in bits 31:16).
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, int lo) {
  if (lo == 0) {
    a = fmaxf(a, 0.0f);
    b = fmaxf(b, 0.0f);
    c = fmaxf(c, 0.0f);
    d = fmaxf(d, 0.0f);
  }
  const int qa = __float2int_rn(a), qb = __float2int_rn(b), qc = __float2int_rn(c), qd = __float2int_rn(d);
  uint32_t hi, w;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(qd), "r"(qc), "r"(0));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(qb), "r"(qa), "r"(hi));
  return w;
}

// Epilogue warps: 4 with gathered A (warps 4-7 gather), else 8, or 16 for
// tiles of 128+ columns.  The requantising epilogue of a 1x1 conv with
// K <= 128 runs longer than the tile's MMAs and is bound by instruction
// latency; four warps per TMEM lane quarter (each with a quarter of the
// columns) keep more of it in flight.  The TMA producer and the MMA warp
// follow the epilogue (and gather) warps.
constexpr int epi_warps(int bn, int amode) { return amode == 1 ? 4 : bn >= 128 ? 16 : 8; }
constexpr int producer_warp(int bn, int amode) { return amode == 1 ? 8 : epi_warps(bn, amode); }
constexpr int threads_of(int bn, int amode) { return (producer_warp(bn, amode) + 2) * 32; }

template <int BN, int STAGES, int AMODE, int RB>
__global__ void __launch_bounds__(threads_of(BN, AMODE), 1)
    conv_i8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap ymap, const __grid_constant__ CUtensorMap rmap,
                   const int8_t *__restrict__ x, const int32_t *__restrict__ bias_q,
                   const float *__restrict__ scale_m, const int8_t *__restrict__ res, void *__restrict__ y,
                   I8Params tp, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int EPIW = epi_warps(BN, AMODE);
  constexpr int PROD_WARP = producer_warp(BN, AMODE), MMA_WARP = PROD_WARP + 1;
  constexpr int CW = BN * 4 / EPIW;  // columns (bytes) per epilogue warp
  constexpr int B_BYTES = BN * kBK;
  constexpr int STAGE = kABytes + B_BYTES;
  constexpr int kCols = 2 * BN;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  uint8_t *staging = smem + STAGES * STAGE;  // EPIW x RB x (32 rows x CW bytes)
  __shared__ uint64_t raw_bar[STAGES], full_bar[STAGES], empty_bar[STAGES], accf_bar[2], acce_bar[2];
  __shared__ uint64_t res_bar[EPIW * RB];
  __shared__ uint32_t tmem_base_holder;
  __shared__ volatile int abort_flag;

  const ConvGeo &g = tp.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&raw_bar[s], 1);     // TMA: B (and A in AMODE 2/3)
      mbar_init(&full_bar[s], 4);    // A gathers landed (AMODE 1): one arrival per A warp
      mbar_init(&empty_bar[s], 1);   // MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], EPIW);  // one arrival per epilogue warp
    }
    for (int w = 0; w < EPIW * RB; ++w) mbar_init(&res_bar[w], 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_holder;
  // Shared memory and TMEM only above; the next layer may start launching,
  // and this one waits here for the previous layer.
  pdl_launch_dependents();
  pdl_wait();

  if (warp < EPIW) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;            // TMEM lanes / tile rows 32q..32q+31
    const int col0 = (warp >> 2) * CW;       // first tile column of this warp
    const int lo = g.act == 1 ? 0 : -128;
    const bool vec_out = g.ys[1] == 1 && (g.M % 16) == 0;
    const bool vec_res = g.has_res && g.rs[1] == 1 && (g.M % 16) == 0;
    const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);
    const bool res_tma = tp.epi_tma && g.has_res;
    // Residual tile of tile tt into this warp's staging buffer b (lane 0);
    // issued[b] counts the loads into buffer b.
    int issued[RB] = {};
    auto load_res = [&](int64_t tt, int b) {
      const uint32_t tm = tp.nt_div.div(uint32_t(tt));
      const int tn0 = int(uint32_t(tt) - tm * uint32_t(tp.n_tiles)) * BN;
      const int64_t trow0 = int64_t(tm) * kBM + quarter * 32;
      mbar_arrive_expect_tx(&res_bar[warp * RB + b], 32 * CW);
      tma_load_2d(staging + (warp * RB + b) * (32 * CW), &rmap, tn0 + col0, int(trow0), &res_bar[warp * RB + b]);
      ++issued[b];
    };
    if (RB == 2 && res_tma && lane == 0 && int64_t(blockIdx.x) < tp.tiles) load_res(blockIdx.x, 0);
    __syncwarp();
    int ti = 0;
    bool failed = false;
    for (int64_t t = blockIdx.x; t < tp.tiles; t += gridDim.x, ++ti) {
      const uint32_t mt = tp.nt_div.div(uint32_t(t));
      const int n0 = int(uint32_t(t) - mt * uint32_t(tp.n_tiles)) * BN;
      const int64_t m0 = int64_t(mt) * kBM;
      const int64_t row0 = m0 + quarter * 32;  // first output pixel of this warp
      const int ab = ti & 1;
      const int rb = RB == 2 ? (ti & 1) : 0;  // staging buffer of this tile
      uint8_t *stile = staging + (warp * RB + rb) * (32 * CW);
      if (tp.epi_tma) {
        // A staging tile is free once the store that last used it has read
        // it (only the previous tile's store can still be pending); then a
        // residual load may start into it: this tile's (RB = 1) or the next
        // tile's, into the other buffer (RB = 2).
        if (lane == 0) {
          tma_store_wait_read0();
          if (res_tma && RB == 1) load_res(t, 0);
          if (res_tma && RB == 2 && t + gridDim.x < tp.tiles) load_res(t + gridDim.x, rb ^ 1);
        }
        __syncwarp();
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&accf_bar[ab], (ti >> 1) & 1, &abort_flag, status, 4))) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (res_tma &&
          !__all_sync(0xffffffffu, mbar_wait(&res_bar[warp * RB + rb], (RB == 2 ? (ti >> 1) : ti) & 1, &abort_flag, status, 6))) {
        failed = true;
        break;
      }
      const int64_t p = row0 + lane;
      const bool pv = p < g.P;
      int n = 0, oh = 0, ow = 0;
      if (pv) pixel_nhw_i8(tp, p, n, oh, ow);
      const int64_t ybase = int64_t(n) * g.ys[0] + int64_t(oh) * g.ys[2] + int64_t(ow) * g.ys[3];
      const int64_t rbase = int64_t(n) * g.rs[0] + int64_t(oh) * g.rs[2] + int64_t(ow) * g.rs[3];
#pragma unroll 1
      for (int cb = 0; cb < CW; cb += 32) {
        uint32_t acc[32];
        tmem_ld32(trow + uint32_t(ab * BN + col0 + cb), acc);
        if (cb + 32 >= CW) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[ab]);
        }
        const int c0 = n0 + col0 + cb;
        if (c0 >= g.M) continue;  // channel padding (warp-uniform)
        const int cn = min(32, g.M - c0);
        int32_t a[32];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int4 b = g.has_bias ? __ldg(reinterpret_cast<const int4 *>(bias_q + c0 + j)) : make_int4(0, 0, 0, 0);
          a[j] = int32_t(acc[j]) + b.x;
          a[j + 1] = int32_t(acc[j + 1]) + b.y;
          a[j + 2] = int32_t(acc[j + 2]) + b.z;
          a[j + 3] = int32_t(acc[j + 3]) + b.w;
        }
        if (tp.out_i32) {
          if (!pv) continue;
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
          const float4 m = __ldg(reinterpret_cast<const float4 *>(scale_m + c0 + j));
          v[j] = __fmul_rn(float(a[j]), m.x);
          v[j + 1] = __fmul_rn(float(a[j + 1]), m.y);
          v[j + 2] = __fmul_rn(float(a[j + 2]), m.z);
          v[j + 3] = __fmul_rn(float(a[j + 3]), m.w);
        }
        uint8_t *srow = stile + lane * CW + cb;  // this thread's 32 bytes of the staging tile
        if (g.has_res) {
          int8_t r[32];
          if (tp.epi_tma) {
            *reinterpret_cast<uint4 *>(r) = *reinterpret_cast<const uint4 *>(srow);
            *reinterpret_cast<uint4 *>(r + 16) = *reinterpret_cast<const uint4 *>(srow + 16);
          } else if (pv && cn == 32 && vec_res) {
            *reinterpret_cast<int4 *>(r) = __ldg(reinterpret_cast<const int4 *>(res + rbase + c0));
            *reinterpret_cast<int4 *>(r + 16) = __ldg(reinterpret_cast<const int4 *>(res + rbase + c0 + 16));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = (pv && j < cn) ? res[rbase + int64_t(c0 + j) * g.rs[1]] : int8_t(0);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __fmul_rn(float(r[j]), g.res_scale));
        }
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = pack4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3], lo);
        if (tp.epi_tma) {
          *reinterpret_cast<uint4 *>(srow) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4 *>(srow + 16) = make_uint4(w[4], w[5], w[6], w[7]);
        } else if (pv) {
          int8_t *y8 = static_cast<int8_t *>(y);
          if (cn == 32 && vec_out) {
            *reinterpret_cast<uint4 *>(y8 + ybase + c0) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4 *>(y8 + ybase + c0 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
            const int8_t *bytes = reinterpret_cast<const int8_t *>(w);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cn) y8[ybase + int64_t(c0 + j) * g.ys[1]] = bytes[j];
          }
        }
      }
      if (tp.epi_tma && !tp.out_i32) {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && row0 < g.P && n0 + col0 < g.M) tma_store_2d(&ymap, n0 + col0, int(row0), stile);
      }
    }
    if (failed && res_tma && lane == 0) {
      // Giving up: let this warp's residual loads that may still be in
      // flight land (bounded) before the CTA's shared memory goes away.
#pragma unroll
      for (int b = 0; b < RB; ++b) {
        if (issued[b] == 0) continue;
        const long long t0 = clock64();
        while (!mbar_try_wait(&res_bar[warp * RB + b], uint32_t(issued[b] - 1) & 1u) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
    if (tp.epi_tma && lane == 0) tma_store_wait_all();
  } else if (AMODE == 1 && warp < 8) {
    // ------------------------------------------------------------ A gathers
    if constexpr (AMODE == 1) {
      const int at = tid - 128;
      const int chunk = at & 7, rsub = at >> 3;
      uint32_t it = 0;
      bool ok = true;
      auto publish = [&](uint32_t pit) {  // the warp's chunks of step pit have landed
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_bar[pit % STAGES]);
      };
      for (int64_t t = blockIdx.x; t < tp.tiles && ok; t += gridDim.x) {
        const int64_t m0 = int64_t(tp.nt_div.div(uint32_t(t))) * kBM;
        int rn[8], rih[8], riw[8];
        bool rvalid[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t p = m0 + i * 16 + rsub;
          rvalid[i] = p < g.P;
          int ow, oh;
          pixel_nhw_i8(tp, rvalid[i] ? p : 0, rn[i], oh, ow);
          rih[i] = oh * g.sh - g.ph;
          riw[i] = ow * g.sw - g.pw;
        }
        for (int kb = 0; kb < tp.num_kb && ok; ++kb, ++it) {
          if (it >= uint32_t(STAGES - 1)) {
            cp_async_wait<STAGES - 2>();  // this thread's step it-(STAGES-1) landed
            publish(it - (STAGES - 1));
          }
          const int s = it % STAGES;
          ok = __all_sync(0xffffffffu, mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1, &abort_flag, status, 1));
          if (!ok) break;  // the warp leaves together
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
  } else if (warp == PROD_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t bytes = B_BYTES + (AMODE != 1 ? kABytes : 0);
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tp.tiles && ok; t += gridDim.x) {
        const uint32_t mt = tp.nt_div.div(uint32_t(t));
        const int n0 = int(uint32_t(t) - mt * uint32_t(tp.n_tiles)) * BN;
        const int64_t m0 = int64_t(mt) * kBM;
        int bw = 0, bh = 0, bn = 0;  // im2col base of the tile's first output pixel
        if (AMODE == 3 || AMODE == 5) {
          int ow, oh;
          pixel_nhw_i8(tp, m0, bn, oh, ow);
          bw = ow * g.sw - g.pw;
          bh = oh * g.sh - g.ph;
        }
        for (int kb = 0; kb < tp.num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          ok = mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1, &abort_flag, status, 2);
          if (!ok) break;
          uint8_t *a_st = smem + s * STAGE;
          mbar_arrive_expect_tx(&raw_bar[s], bytes);
          tma_load_2d(a_st + kABytes, &wmap, kb * kBK, n0, &raw_bar[s]);
          if (AMODE == 2) tma_load_2d(a_st, &amap, kb * kBK, int(m0), &raw_bar[s]);
          if (AMODE == 3) {
            const int k0 = kb * kBK;
            const int tap = k0 / g.C, c0 = k0 - tap * g.C;  // C % 128 == 0: one tap per K step
            const int r = tap / g.KW, sx = tap - r * g.KW;
            tma_load_im2col_4d(a_st, &amap, c0, bw, bh, bn, uint16_t(sx * g.dw), uint16_t(r * g.dh), &raw_bar[s]);
          }
          if (AMODE == 5) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int tap = 2 * kb + j;
              const bool real = tap < g.KH * g.KW;
              const int r = real ? tap / g.KW : 0, sx = real ? tap - r * g.KW : 0;
              tma_load_im2col_4d(a_st + j * (kABytes / 2), &amap, 0, bw, bh, real ? bn : g.N, uint16_t(sx * g.dw),
                                 uint16_t(r * g.dh), &raw_bar[s]);
            }
          }
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
      // One flat loop over this CTA's K steps (all its tiles) with the stage,
      // K-step and buffer positions kept as counters, so the issuing thread
      // spends little time between MMA batches.
      const int64_t my_tiles =
          int64_t(blockIdx.x) < tp.tiles ? (tp.tiles - 1 - int64_t(blockIdx.x)) / int64_t(gridDim.x) + 1 : 0;
      const uint32_t total = uint32_t(my_tiles) * uint32_t(tp.num_kb);
      const int num_kb = tp.num_kb;
      int ti = 0;                 // tiles handed to the epilogue
      uint32_t ab = 0, abph = 0;  // accumulator buffer and its phase parity
      uint32_t dtm = tmem;
      int kb = 0, s = 0;
      uint32_t ph = 0;
      for (uint32_t it = 0; it < total; ++it) {
        if (kb == 0) {
          if (!mbar_wait(&acce_bar[ab], abph ^ 1, &abort_flag, status, 7)) break;
          tc_fence_after();
          dtm = tmem + ab * uint32_t(BN);
        }
        if (!mbar_wait(&raw_bar[s], ph, &abort_flag, status, 3)) break;
        if (AMODE == 1 && !mbar_wait(&full_bar[s], ph, &abort_flag, status, 3)) break;
        tc_fence_after();
        uint8_t *a_st = smem + s * STAGE;
        const uint64_t da = smem_desc(a_st), db = smem_desc(a_st + kABytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t step = uint64_t(kk * 32) >> 4;  // 32 int8 = 32 bytes along K
          // AMODE 5: slices 0-1 in the first 64-byte-row half, 2-3 in the second.
          const uint64_t a = AMODE == 5 ? smem_desc_sw64(a_st + (kk >> 1) * (kABytes / 2)) + uint64_t((kk & 1) * 32 >> 4)
                                        : da + step;
          mma_i8(dtm, a, db + step, idesc, (kb | kk) ? 1u : 0u);
        }
        mma_commit(&empty_bar[s]);
        if (++kb == num_kb) {
          mma_commit(&accf_bar[ab]);
          ++ti;
          kb = 0;
          ab ^= 1u;
          if (ab == 0) abph ^= 1u;
        }
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
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
  if (warp == MMA_WARP) {
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

// Operand stages and shared memory per tile width and residual buffers.
constexpr int stages_of(int bn, int rb) { return bn == 256 ? (rb == 2 ? 3 : 4) : bn == 128 ? 6 : 8; }
constexpr size_t smem_of(int bn, int rb) {
  return size_t(stages_of(bn, rb)) * (kABytes + bn * kBK) + size_t(rb) * 128 * bn + 1024;
}

struct I8State {
  CUtensorMap wmap, amap, ymap, rmap;
  I8Params tp;
  int bn = 128, amode = 1, grid = 148;
  int rb = 1;  // epilogue staging buffers per warp (2: residual prefetch)
  size_t smem = 0;
  bool set_attr_only = false;
  const void *x_base = nullptr, *y_base = nullptr, *r_base = nullptr;  // pointers the maps were encoded for
};

int epi_cols(const I8State &st) { return st.bn * 4 / epi_warps(st.bn, st.amode); }

bool encode_a(const I8State &st, CUtensorMap *map, const void *x) {
  const ConvGeo &g = st.tp.g;
  if (st.amode == 3)
    return encode_im2col_nhwc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, x, g.N, g.H, g.W, g.C, g.KH, g.sh, g.ph, g.dh,
                              kBK, kBM);
  if (st.amode == 5)
    return encode_im2col_nhwc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, x, g.N, g.H, g.W, g.C, g.KH, g.sh, g.ph, g.dh,
                              64, kBM, CU_TENSOR_MAP_SWIZZLE_64B);
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, x, uint64_t(g.C), uint64_t(g.P), uint64_t(g.C), kBM);
}

bool encode_rows(const I8State &st, CUtensorMap *map, const void *base) {
  const ConvGeo &g = st.tp.g;
  return encode_2d_box(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, uint64_t(g.M), uint64_t(g.P), uint64_t(g.M),
                       uint32_t(epi_cols(st)), 32, CU_TENSOR_MAP_SWIZZLE_NONE);
}

struct Maps {
  CUtensorMap a, y, r;
};

template <int BN, int AMODE, int RB>
int launch_cfg(const I8State &st, const Maps &mp, const ConvPlan &p, const void *x, void *y, const void *res,
               int *status, cudaStream_t s) {
  auto kern = conv_i8_kernel<BN, stages_of(BN, RB), AMODE, RB>;
  if (st.set_attr_only)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st.smem)));
  return cuda_status(launch_kernel(kern, unsigned(st.grid), threads_of(BN, AMODE), st.smem, s, 1, st.wmap, mp.a,
                                   mp.y, mp.r,
                                   static_cast<const int8_t *>(x), p.bias_q, p.scale_m,
                                   static_cast<const int8_t *>(res), y, st.tp, status));
}

template <int BN>
int launch_bn(const I8State &st, const Maps &mp, const ConvPlan &p, const void *x, void *y, const void *res,
              int *status, cudaStream_t s) {
  if (st.rb == 2) {
    switch (st.amode) {
      case 5: return launch_cfg<BN, 5, 2>(st, mp, p, x, y, res, status, s);
      case 3: return launch_cfg<BN, 3, 2>(st, mp, p, x, y, res, status, s);
      case 2: return launch_cfg<BN, 2, 2>(st, mp, p, x, y, res, status, s);
      default: return launch_cfg<BN, 1, 2>(st, mp, p, x, y, res, status, s);
    }
  }
  switch (st.amode) {
    case 5: return launch_cfg<BN, 5, 1>(st, mp, p, x, y, res, status, s);
    case 3: return launch_cfg<BN, 3, 1>(st, mp, p, x, y, res, status, s);
    case 2: return launch_cfg<BN, 2, 1>(st, mp, p, x, y, res, status, s);
    default: return launch_cfg<BN, 1, 1>(st, mp, p, x, y, res, status, s);
  }
}

}  // namespace

// Eligible: int8 x / w, group 1, dense NHWC input with C % 16 == 0, 16-byte
// aligned activations, Cout >= 16.
int conv_tc_i8_prepare(ConvPlan &p, const void *w_dev, const void *x_dev, const void *y_dev, const void *r_dev,
                       cudaStream_t s) {
  const ConvGeo &g = p.g;
  if ((p.mode != kConvI8 && p.mode != kConvI8ToI32) || g.groups != 1 || g.M < 16) return SPKV2_ERR_UNSUPPORTED;
  const bool nhwc_in = g.xs[1] == 1 && g.xs[3] == g.C && g.xs[2] == int64_t(g.W) * g.C;
  if (!nhwc_in || g.C % 16 != 0 || reinterpret_cast<uintptr_t>(x_dev) % 16 != 0) return SPKV2_ERR_UNSUPPORTED;
  if (!encode_fn()) return SPKV2_ERR_UNSUPPORTED;
  I8State *st = new I8State();
  memset(&st->wmap, 0, sizeof(st->wmap));
  memset(&st->amap, 0, sizeof(st->amap));
  memset(&st->ymap, 0, sizeof(st->ymap));
  memset(&st->rmap, 0, sizeof(st->rmap));
  // The im2col maps walk window origins over the extent that bottom / right
  // padding equal to the top / left padding gives, and the row map assumes
  // the output extent is the input's: asymmetric padding takes the gathers.
  const bool square = g.KH == g.KW && g.sh == g.sw && g.ph == g.pw && g.dh == g.dw;
  const int span_w = g.W + 2 * g.pw - (g.KW - 1) * g.dw - 1, span_h = g.H + 2 * g.ph - (g.KH - 1) * g.dh - 1;
  const bool sym_extent = span_w >= 0 && span_h >= 0 && g.OW == span_w / g.sw + 1 && g.OH == span_h / g.sh + 1;
  if (g.KH == 1 && g.KW == 1 && g.sh == 1 && g.sw == 1 && g.ph == 0 && g.pw == 0 && g.OH == g.H && g.OW == g.W)
    st->amode = 2;
  else if (square && sym_extent && g.C % kBK == 0 && encode_im2col_fn())
    st->amode = 3;
  else if (square && sym_extent && g.C == 64 && encode_im2col_fn() && !getenv("SPKV2_I8_NO_IM2COL64"))
    st->amode = 5;
  else
    st->amode = 1;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Tile width from the wave / MMA-rate model; 4 epilogue warps (AMODE 1)
  // take at most 128 columns, 8 (AMODE 2/3) at least 64.
  int bn = pick_block_n(g.P, g.M, ceil_div(g.K, kBK), sms, st->amode == 1 ? 32 : 64, st->amode == 1 ? 128 : 256);
  if (const char *e = getenv("SPKV2_TC_BN")) {
    const int v = atoi(e);
    if ((v == 32 || v == 64 || v == 128 || v == 256) && v <= std::max(32, int(ceil_div(g.M, 32) * 32))) bn = v;
  }
  if (st->amode == 1 && bn == 256) bn = 128;  // 4 epilogue warps: at most 128 columns each
  if (st->amode != 1 && bn == 32) bn = 64;    // 8 epilogue warps: at least 32 columns each
  st->bn = bn;
  I8Params &tp = st->tp;
  tp.g = g;
  tp.Kpad = int(ceil_div(g.K, kBK) * kBK);
  tp.Npad = int(ceil_div(g.M, bn) * bn);
  tp.num_kb = tp.Kpad / kBK;
  tp.n_tiles = tp.Npad / bn;
  tp.tiles = ceil_div(g.P, kBM) * tp.n_tiles;
  tp.out_i32 = p.mode == kConvI8ToI32 ? 1 : 0;
  if (g.P >= (int64_t(1) << 31) || tp.tiles >= (int64_t(1) << 31)) {  // 32-bit coordinates
    delete st;
    return SPKV2_ERR_UNSUPPORTED;
  }
  tp.nt_div = FastDiv(uint32_t(tp.n_tiles));
  tp.ow_div = FastDiv(uint32_t(g.OW));
  tp.oh_div = FastDiv(uint32_t(g.OH));
  const bool nhwc_out = g.ys[1] == 1 && g.ys[3] == g.M && g.ys[2] == int64_t(g.OW) * g.M;
  const bool nhwc_res = !g.has_res || (g.rs[1] == 1 && g.rs[3] == g.M && g.rs[2] == int64_t(g.OW) * g.M);
  tp.epi_tma = (!tp.out_i32 && nhwc_out && nhwc_res && g.M % 16 == 0 &&
                reinterpret_cast<uintptr_t>(y_dev) % 16 == 0 && reinterpret_cast<uintptr_t>(r_dev) % 16 == 0)
                   ? 1
                   : 0;
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
  if (ok && st->amode != 1) ok = encode_a(*st, &st->amap, x_dev);
  if (ok && tp.epi_tma) ok = encode_rows(*st, &st->ymap, y_dev);
  if (ok && tp.epi_tma && g.has_res) ok = encode_rows(*st, &st->rmap, r_dev);
  st->x_base = x_dev;
  st->y_base = y_dev;
  st->r_base = r_dev;
  if (!ok) {
    device_free(wp);
    delete st;
    return rc ? rc : SPKV2_ERR_UNSUPPORTED;
  }
  st->rb = (tp.epi_tma && g.has_res && !getenv("SPKV2_I8_NO_RES_PREFETCH")) ? 2 : 1;
  st->smem = smem_of(bn, st->rb);
  p.w_tc = wp;
  p.tc_state = st;
  p.tc_i8 = true;
  p.tc_block_n = bn;
  p.tc_kpad = tp.Kpad;
  st->set_attr_only = true;
  rc = conv_tc_i8_launch(p, nullptr, nullptr, nullptr, nullptr, s);
  st->set_attr_only = false;
  if (rc) return rc;
  static const char *amodes[] = {"", "_cpasync", "_tma", "_im2col", "", "_im2col64"};
  p.variant = std::string("tc_int8_bn") + std::to_string(bn) + amodes[st->amode] + (tp.epi_tma ? "_tmastore" : "") +
              (st->rb == 2 ? "_resprefetch" : "") + (tp.out_i32 ? "_i32out" : "");
  return 0;
}

void conv_tc_i8_release(void *state) { delete static_cast<I8State *>(state); }

int conv_tc_i8_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s) {
  const I8State &st = *static_cast<const I8State *>(p.tc_state);
  // Tensor maps follow the tensors: one rebound to another device buffer
  // since prepare gets a freshly encoded map.
  Maps mp{st.amap, st.ymap, st.rmap};
  if (!st.set_attr_only) {
    if (st.amode != 1 && x != st.x_base && !encode_a(st, &mp.a, x)) return SPKV2_ERR_UNSUPPORTED;
    if (st.tp.epi_tma && y != st.y_base && !encode_rows(st, &mp.y, y)) return SPKV2_ERR_UNSUPPORTED;
    if (st.tp.epi_tma && p.g.has_res && res != st.r_base && !encode_rows(st, &mp.r, res)) return SPKV2_ERR_UNSUPPORTED;
  }
  switch (st.bn) {
    case 32: return launch_bn<32>(st, mp, p, x, y, res, status, s);
    case 64: return launch_bn<64>(st, mp, p, x, y, res, status, s);
    case 128: return launch_bn<128>(st, mp, p, x, y, res, status, s);
    default: return launch_bn<256>(st, mp, p, x, y, res, status, s);
  }
}

}  // namespace spkv2
