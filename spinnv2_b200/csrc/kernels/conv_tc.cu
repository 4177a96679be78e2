// tcgen05 implicit-GEMM convolution for sm_100a (fp32 activations, TF32
// tensor cores, 3xTF32 split for near-fp32 accuracy).
//
// GEMM view: rows = output pixels (n, oh, ow), columns = output channels,
// K = (r, s, c) with c fastest; A rows are the activation gathered on the
// fly (implicit im2col), B = packed weights [Cout_pad][K_pad] K-major.
//
// CTA tile: 128 pixels x BN channels, K step 32 fp32 (one 128-byte swizzle
// row).  Warp roles (192 threads):
//   warps 0-3  A operand, then the epilogue.  How A reaches shared memory:
//                AMODE 2 (1x1, stride 1, NHWC, C % 32 == 0): TMA tile load;
//                AMODE 1 (NHWC, C % 4 == 0): cp.async 16-byte gathers with
//                  zero-fill for padding, completion signalled on the stage
//                  mbarrier (many loads in flight per thread);
//                AMODE 0 (anything else, e.g. NCHW graph input, C = 3):
//                  per-element gathers through registers.
//              For AMODE 1/2 the same warps then convert the landed tile in
//              place, one stage behind the loads: TF32 hi = round-to-nearest,
//              lo = x - hi (3xTF32), written in the 128B-swizzled K-major
//              layout the MMA descriptors describe.
//              Epilogue: TMEM lanes 32w..32w+31 (= tile rows of warp w) ->
//              registers -> bias, residual, Relu/SiLU -> either a TMA store
//              staged through shared memory (NHWC outputs) or direct stores.
//   warp 4     TMA producer (one thread): weight panels (hi, and lo for
//              3xTF32) and, in AMODE 2, the A tile.  No multicast.
//   warp 5     TMEM allocation; one thread issues tcgen05.mma (M=128, N=BN,
//              K=8) into an fp32 TMEM accumulator and commits stage
//              releases to mbarriers.
// 3xTF32: acc += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi (three MMAs per K step).
// Every mbarrier wait is bounded (about a second of clock cycles); on timeout
// the CTA records a code in the context's status word and winds down.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "conv.h"

namespace spkv2 {

namespace {

constexpr int kBM = 128;          // tile rows (pixels) = UMMA M
constexpr int kBK = 32;           // fp32 elements per K step = 128 bytes
constexpr int kThreads = 192;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false on timeout or when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                          int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      if (status) atomicExch(status, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 16-byte async copy global -> shared; src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// Arrive on `bar` once all of this thread's prior cp.async copies landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128B-swizzled operand: SBO = 1024 B between 8-row groups,
// LBO = 16 B (unused for swizzled K-major), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
  const uint64_t addr = smem_u32(p);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// ---------------------------------------------------------------- kernel
struct TcParams {
  ConvGeo g;
  int Kpad;      // K rounded up to a multiple of 32
  int Npad;      // Cout rounded up to a multiple of BN
  int num_kb;    // Kpad / 32
};

template <int BN, bool SPLIT3>
struct StageBytes {
  static constexpr int A = kBM * 128;
  static constexpr int B = BN * 128;
  static constexpr int value = (SPLIT3 ? 2 : 1) * (A + B);
};

// Row / chunk mapping shared by the A loads and the conversion pass: thread t
// handles 16-byte chunk (t & 7) of rows i*16 + (t >> 3), i = 0..7.
__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <bool SPLIT3>
__device__ __forceinline__ void convert_stage(uint8_t *a_hi, uint8_t *a_lo, int tid) {
  const int chunk = tid & 7, rsub = tid >> 3;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t off = swz_off(i * 16 + rsub, chunk);
    const float4 v = *reinterpret_cast<const float4 *>(a_hi + off);
    float4 hi;
    hi.x = tf32_rna(v.x);
    hi.y = tf32_rna(v.y);
    hi.z = tf32_rna(v.z);
    hi.w = tf32_rna(v.w);
    *reinterpret_cast<float4 *>(a_hi + off) = hi;
    if (SPLIT3)
      *reinterpret_cast<float4 *>(a_lo + off) = make_float4(v.x - hi.x, v.y - hi.y, v.z - hi.z, v.w - hi.w);
  }
}

template <int BN, int STAGES, bool SPLIT3, int AMODE, bool EPI_TMA>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap ymap, const float *__restrict__ x,
                   const float *__restrict__ bias, const float *__restrict__ res, float *__restrict__ y, TcParams tp,
                   int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = StageBytes<BN, SPLIT3>::A;
  constexpr int B_BYTES = StageBytes<BN, SPLIT3>::B;
  constexpr int STAGE = StageBytes<BN, SPLIT3>::value;
  constexpr bool CONVERT = (AMODE == 1) || (AMODE == 2 && SPLIT3);
  __shared__ uint64_t raw_bar[STAGES], full_bar[STAGES], empty_bar[STAGES], done_bar;
  __shared__ uint32_t tmem_base_holder;
  __shared__ volatile int abort_flag;

  const ConvGeo &g = tp.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = tp.Npad / BN;
  const int n0 = (blockIdx.x % n_tiles) * BN;  // channel tile fastest: pixel tile shared in L2
  const int64_t m0 = int64_t(blockIdx.x / n_tiles) * kBM;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&raw_bar[s], AMODE == 2 ? 1 : 128 + 1);
      mbar_init(&full_bar[s], 128);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  constexpr uint32_t kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_holder;

  if (warp < 4) {
    // ------------------------------------------------------------ A operand
    const int chunk = tid & 7;
    const int rsub = tid >> 3;
    if (AMODE == 2) {
      if (CONVERT) {
        for (int kb = 0; kb < tp.num_kb; ++kb) {
          const int s = kb % STAGES;
          if (!mbar_wait(&raw_bar[s], (kb / STAGES) & 1, &abort_flag, status, 5)) break;
          uint8_t *a_hi = smem + s * STAGE;
          convert_stage<SPLIT3>(a_hi, a_hi + A_BYTES, tid);
          fence_proxy_async();
          mbar_arrive(&full_bar[s]);
        }
      }
    } else {
      int rn[8], rih[8], riw[8];
      bool rvalid[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t p = m0 + i * 16 + rsub;
        rvalid[i] = p < g.P;
        const int64_t pp = rvalid[i] ? p : 0;
        const int ow = int(pp % g.OW);
        const int64_t t = pp / g.OW;
        rih[i] = int(t % g.OH) * g.sh - g.ph;
        riw[i] = ow * g.sw - g.pw;
        rn[i] = int(t / g.OH);
      }
      bool ok = true;
      for (int kb = 0; kb < tp.num_kb && ok; ++kb) {
        const int s = kb % STAGES;
        ok = mbar_wait(&empty_bar[s], ((kb / STAGES) & 1) ^ 1, &abort_flag, status, 1);
        if (!ok) break;
        uint8_t *a_hi = smem + s * STAGE;
        const int k0 = kb * kBK + chunk * 4;
        if (AMODE == 1) {
          // The 4 channels of this chunk share one filter tap (C % 4 == 0).
          const bool kval = k0 < g.K;
          const int tap = k0 / g.Cg, c = k0 - tap * g.Cg;
          const int r = tap / g.KW, sx = tap - r * g.KW;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int ih = rih[i] + r * g.dh, iw = riw[i] + sx * g.dw;
            const bool in = kval && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
            const float *src = in ? x + ((int64_t(rn[i]) * g.H + ih) * g.W + iw) * g.C + c : x;
            cp_async16(a_hi + swz_off(i * 16 + rsub, chunk), src, in ? 16u : 0u);
          }
          cp_async_arrive(&raw_bar[s]);
          // Convert the previous stage while this one's copies are in flight.
          if (kb > 0) {
            const int ps = (kb - 1) % STAGES;
            ok = mbar_wait(&raw_bar[ps], ((kb - 1) / STAGES) & 1, &abort_flag, status, 6);
            if (!ok) break;
            uint8_t *p_hi = smem + ps * STAGE;
            convert_stage<SPLIT3>(p_hi, p_hi + A_BYTES, tid);
            fence_proxy_async();
            mbar_arrive(&full_bar[ps]);
          }
        } else {
          float4 v[8];
          int er[4], es[4], ec[4];
          bool ek[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = k0 + e;
            ek[e] = k < g.K;
            const int tap = k / g.Cg;
            ec[e] = k - tap * g.Cg;
            er[e] = tap / g.KW;
            es[e] = tap - er[e] * g.KW;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float f[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int ih = rih[i] + er[e] * g.dh, iw = riw[i] + es[e] * g.dw;
              const bool in = ek[e] && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
              f[e] = in ? __ldg(x + rn[i] * g.xs[0] + ec[e] * g.xs[1] + ih * g.xs[2] + iw * g.xs[3]) : 0.f;
            }
            v[i] = make_float4(f[0], f[1], f[2], f[3]);
          }
          uint8_t *a_lo = a_hi + A_BYTES;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t off = swz_off(i * 16 + rsub, chunk);
            float4 hi;
            hi.x = tf32_rna(v[i].x);
            hi.y = tf32_rna(v[i].y);
            hi.z = tf32_rna(v[i].z);
            hi.w = tf32_rna(v[i].w);
            *reinterpret_cast<float4 *>(a_hi + off) = hi;
            if (SPLIT3)
              *reinterpret_cast<float4 *>(a_lo + off) =
                  make_float4(v[i].x - hi.x, v[i].y - hi.y, v[i].z - hi.z, v[i].w - hi.w);
          }
          fence_proxy_async();
          mbar_arrive(&raw_bar[s]);
        }
      }
      if (AMODE == 1 && ok && tp.num_kb > 0) {
        const int kb = tp.num_kb - 1, ps = kb % STAGES;
        if (mbar_wait(&raw_bar[ps], (kb / STAGES) & 1, &abort_flag, status, 6)) {
          uint8_t *p_hi = smem + ps * STAGE;
          convert_stage<SPLIT3>(p_hi, p_hi + A_BYTES, tid);
          fence_proxy_async();
          mbar_arrive(&full_bar[ps]);
        }
      }
    }
    // ------------------------------------------------------------ epilogue
    if (mbar_wait(&done_bar, 0, &abort_flag, status, 4)) {
      tc_fence_after();
      const int row = warp * 32 + lane;
      const int64_t p = m0 + row;
      const bool pv = p < g.P;
      int n = 0, oh = 0, ow = 0;
      if (pv) {
        ow = int(p % g.OW);
        const int64_t t = p / g.OW;
        oh = int(t % g.OH);
        n = int(t / g.OH);
      }
      const int64_t ybase = int64_t(n) * g.ys[0] + int64_t(oh) * g.ys[2] + int64_t(ow) * g.ys[3];
      const int64_t rbase = int64_t(n) * g.rs[0] + int64_t(oh) * g.rs[2] + int64_t(ow) * g.rs[3];
      const bool rvec = g.rs[1] == 1 && (g.M % 4) == 0;
      // Staging for the TMA store: two 32x32 fp32 buffers per warp, reusing
      // the (now idle) operand stages.
      uint8_t *stage_buf = smem + warp * 8192;
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(cb), acc);
        const int c0 = n0 + cb;
        if (c0 >= g.M) continue;  // whole chunk in the channel padding (warp-uniform)
        float vals[32];
        const int cn = min(32, g.M - c0);
        if (cn == 32 && (!g.has_res || rvec)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 b = g.has_bias ? __ldg(reinterpret_cast<const float4 *>(bias + c0 + j)) : make_float4(0, 0, 0, 0);
            const float4 rr = (g.has_res && pv) ? __ldg(reinterpret_cast<const float4 *>(res + rbase + c0 + j))
                                                : make_float4(0, 0, 0, 0);
            vals[j] = apply_act(__uint_as_float(acc[j]) + b.x + rr.x, g.act);
            vals[j + 1] = apply_act(__uint_as_float(acc[j + 1]) + b.y + rr.y, g.act);
            vals[j + 2] = apply_act(__uint_as_float(acc[j + 2]) + b.z + rr.z, g.act);
            vals[j + 3] = apply_act(__uint_as_float(acc[j + 3]) + b.w + rr.w, g.act);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = __uint_as_float(acc[j]);
            if (j < cn) {
              const int c = c0 + j;
              if (g.has_bias) v += __ldg(bias + c);
              if (g.has_res && pv) v += __ldg(res + rbase + int64_t(c) * g.rs[1]);
              v = apply_act(v, g.act);
            }
            vals[j] = v;
          }
        }
        if (EPI_TMA) {
          uint8_t *buf = stage_buf + ((cb >> 5) & 1) * 4096;
          if (cb >= 64 && lane == 0) tma_store_wait_read1();  // the buffer's previous store has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4 *>(buf + swz_off(lane, j)) =
                make_float4(vals[4 * j], vals[4 * j + 1], vals[4 * j + 2], vals[4 * j + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0 && m0 + warp * 32 < g.P) tma_store_2d(&ymap, c0, int(m0 + warp * 32), buf);
        } else if (pv) {
          if (cn == 32 && g.ys[1] == 1 && (g.M % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4 *>(y + ybase + c0 + j) =
                  make_float4(vals[j], vals[j + 1], vals[j + 2], vals[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cn) y[ybase + int64_t(c0 + j) * g.ys[1]] = vals[j];
          }
        }
      }
      if (EPI_TMA && lane == 0) tma_store_wait_all();
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t bytes = (SPLIT3 ? 2 : 1) * B_BYTES + (AMODE == 2 ? A_BYTES : 0);
      for (int kb = 0; kb < tp.num_kb; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(&empty_bar[s], ((kb / STAGES) & 1) ^ 1, &abort_flag, status, 2)) break;
        uint8_t *a_hi = smem + s * STAGE;
        uint8_t *b_hi = a_hi + (SPLIT3 ? 2 : 1) * A_BYTES;
        mbar_arrive_expect_tx(&raw_bar[s], bytes);
        tma_load_2d(b_hi, &wmap, kb * kBK, n0, &raw_bar[s]);
        if (SPLIT3) tma_load_2d(b_hi + B_BYTES, &wmap, kb * kBK, tp.Npad + n0, &raw_bar[s]);
        if (AMODE == 2) tma_load_2d(a_hi, &amap, kb * kBK, int(m0), &raw_bar[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
      for (int kb = 0; kb < tp.num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(CONVERT ? &full_bar[s] : &raw_bar[s], ph, &abort_flag, status, 3)) break;
        tc_fence_after();
        uint8_t *a_hi = smem + s * STAGE;
        uint8_t *a_lo = a_hi + A_BYTES;
        uint8_t *b_hi = a_hi + (SPLIT3 ? 2 : 1) * A_BYTES;
        uint8_t *b_lo = b_hi + B_BYTES;
        const uint64_t dah = smem_desc(a_hi), dbh = smem_desc(b_hi);
        const uint64_t dal = smem_desc(a_lo), dbl = smem_desc(b_lo);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t step = uint64_t(kk * 32) >> 4;  // 8 tf32 = 32 bytes along K
          const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
          if (SPLIT3) {
            mma_tf32(tmem, dal + step, dbh + step, idesc, first);
            mma_tf32(tmem, dah + step, dbl + step, idesc, 1u);
            mma_tf32(tmem, dah + step, dbh + step, idesc, 1u);
          } else {
            mma_tf32(tmem, dah + step, dbh + step, idesc, first);
          }
        }
        mma_commit(&empty_bar[s]);
      }
      mma_commit(&done_bar);
      // MMAs must be complete before TMEM is freed, also on the abort path.
      const long long t0 = clock64();
      while (!mbar_try_wait(&done_bar, 0) && clock64() - t0 < kWaitCycles) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- weights
// [part][Npad][Kpad], k = (r*KW + s)*Cg + c; part 0 = TF32(rna) of w,
// part 1 = w - part 0 (3xTF32 only); zero padding.
__global__ void pack_tc_kernel(float *__restrict__ dst, const float *__restrict__ w, ConvGeo g, int Npad, int Kpad,
                               int split3) {
  const int64_t total = int64_t(Npad) * Kpad;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / Kpad), k = int(i % Kpad);
    float v = 0.f;
    if (m < g.M && k < g.K) {
      const int c = k % g.Cg, rs = k / g.Cg, s = rs % g.KW, r = rs / g.KW;
      v = w[((int64_t(m) * g.Cg + c) * g.KH + r) * g.KW + s];
    }
    const float hi = tf32_rna(v);
    dst[i] = hi;
    if (split3) dst[total + i] = v - hi;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D fp32 tensor map, 128-byte swizzle: dims {inner, outer}, row pitch in
// elements, box {32, box_rows}.
bool encode_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer, uint64_t pitch, uint32_t box_rows) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch * sizeof(float)};
  const cuuint32_t box[2] = {uint32_t(kBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct TcState {
  CUtensorMap wmap, amap, ymap;
  TcParams tp;
  int bn = 128;
  int stages = 2;
  bool split3 = true;
  int amode = 0;
  bool epi_tma = false;
  size_t smem = 0;
  bool set_attr_only = false;  // dispatch only sets the kernel's smem attribute
};

template <int BN, int STAGES, bool SPLIT3, int AMODE, bool EPI>
int launch_cfg(const TcState &st, const float *x, float *y, const float *bias, const float *res, int *status,
               cudaStream_t s) {
  auto kern = conv_tc_kernel<BN, STAGES, SPLIT3, AMODE, EPI>;
  if (st.set_attr_only)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st.smem)));
  const int64_t mt = ceil_div(st.tp.g.P, kBM);
  const int64_t blocks = mt * (st.tp.Npad / BN);
  if (blocks > 0x7fffffffLL) return SPKV2_ERR_UNSUPPORTED;
  kern<<<unsigned(blocks), kThreads, st.smem, s>>>(st.wmap, st.amap, st.ymap, x, bias, res, y, st.tp, status);
  return cuda_status(cudaGetLastError());
}

template <int BN, int STAGES, bool SPLIT3>
int launch_modes(const TcState &st, const float *x, float *y, const float *bias, const float *res, int *status,
                 cudaStream_t s) {
  if (st.epi_tma) {
    switch (st.amode) {
      case 2: return launch_cfg<BN, STAGES, SPLIT3, 2, true>(st, x, y, bias, res, status, s);
      case 1: return launch_cfg<BN, STAGES, SPLIT3, 1, true>(st, x, y, bias, res, status, s);
      default: return launch_cfg<BN, STAGES, SPLIT3, 0, true>(st, x, y, bias, res, status, s);
    }
  }
  switch (st.amode) {
    case 2: return launch_cfg<BN, STAGES, SPLIT3, 2, false>(st, x, y, bias, res, status, s);
    case 1: return launch_cfg<BN, STAGES, SPLIT3, 1, false>(st, x, y, bias, res, status, s);
    default: return launch_cfg<BN, STAGES, SPLIT3, 0, false>(st, x, y, bias, res, status, s);
  }
}

int stages_for(int bn, bool split3) {
  const int stage = (split3 ? 2 : 1) * (kBM * 128 + bn * 128);
  return std::min(4, (200 * 1024) / stage);
}

}  // namespace

// Eligible: fp32 in and out, group 1, Cout >= 16, 3xTF32 or TF32 math.
int conv_tc_prepare(ConvPlan &p, const void *w_raw_dev, const void *x_dev, const void *y_dev, cudaStream_t s) {
  const ConvGeo &g = p.g;
  if (p.mode != kConvF32 || g.groups != 1 || g.M < 16) return SPKV2_ERR_UNSUPPORTED;
  if (p.math != SPKV2_CUDA_MATH_3XTF32 && p.math != SPKV2_CUDA_MATH_TF32) return SPKV2_ERR_UNSUPPORTED;
  if (!encode_fn()) return SPKV2_ERR_UNSUPPORTED;
  TcState *st = new TcState();
  memset(&st->wmap, 0, sizeof(st->wmap));
  memset(&st->amap, 0, sizeof(st->amap));
  memset(&st->ymap, 0, sizeof(st->ymap));
  st->split3 = p.math == SPKV2_CUDA_MATH_3XTF32;
  int bn = g.M <= 32 ? 32 : g.M <= 64 ? 64 : 128;
  if (!st->split3 && g.M >= 256) bn = 256;
  if (const char *e = getenv("SPKV2_TC_BN")) {
    const int v = atoi(e);
    if ((v == 32 || v == 64 || v == 128 || v == 256) && v <= std::max(32, int(ceil_div(g.M, 32) * 32))) bn = v;
  }
  st->bn = bn;
  st->stages = stages_for(bn, st->split3);
  const bool nhwc_in = g.xs[1] == 1 && g.xs[3] == g.C && g.xs[2] == int64_t(g.W) * g.C;
  const bool c32 = g.C % 32 == 0;
  if (nhwc_in && c32 && g.KH == 1 && g.KW == 1 && g.sh == 1 && g.sw == 1 && g.ph == 0 && g.pw == 0 &&
      reinterpret_cast<uintptr_t>(x_dev) % 16 == 0)
    st->amode = 2;
  else if (nhwc_in && g.C % 4 == 0 && reinterpret_cast<uintptr_t>(x_dev) % 16 == 0)
    st->amode = 1;
  else
    st->amode = 0;
  const bool nhwc_out = g.ys[1] == 1 && g.ys[3] == g.M && g.ys[2] == int64_t(g.OW) * g.M;
  st->epi_tma = nhwc_out && g.M % 4 == 0 && reinterpret_cast<uintptr_t>(y_dev) % 16 == 0;
  TcParams &tp = st->tp;
  tp.g = g;
  tp.Kpad = int(ceil_div(g.K, kBK) * kBK);
  tp.Npad = int(ceil_div(g.M, bn) * bn);
  tp.num_kb = tp.Kpad / kBK;
  const int parts = st->split3 ? 2 : 1;
  float *wtc = static_cast<float *>(device_alloc(size_t(parts) * tp.Npad * tp.Kpad * sizeof(float)));
  if (!wtc) {
    delete st;
    return SPKV2_ERR_DEVICE_ALLOC;
  }
  pack_tc_kernel<<<grid_for(int64_t(tp.Npad) * tp.Kpad, 256), 256, 0, s>>>(wtc, static_cast<const float *>(w_raw_dev),
                                                                           g, tp.Npad, tp.Kpad, st->split3 ? 1 : 0);
  int rc = cuda_status(cudaGetLastError());
  bool ok = rc == 0 && encode_2d(&st->wmap, wtc, uint64_t(tp.Kpad), uint64_t(parts) * tp.Npad, uint64_t(tp.Kpad), uint32_t(bn));
  if (ok && st->amode == 2) ok = encode_2d(&st->amap, x_dev, uint64_t(g.C), uint64_t(g.P), uint64_t(g.C), kBM);
  if (ok && st->epi_tma) ok = encode_2d(&st->ymap, y_dev, uint64_t(g.M), uint64_t(g.P), uint64_t(g.M), 32);
  if (!ok) {
    device_free(wtc);
    delete st;
    return rc ? rc : SPKV2_ERR_UNSUPPORTED;
  }
  st->smem = size_t(st->stages) * size_t(parts) * (kBM * 128 + bn * 128) + 1024;
  // At most one CTA per SM: TMEM (<= 256 columns) is never contended.
  st->smem = std::max<size_t>(st->smem, 120 * 1024);
  p.w_tc = wtc;
  p.tc_state = st;
  p.tc_block_n = bn;
  p.tc_kpad = tp.Kpad;
  st->set_attr_only = true;
  rc = conv_tc_launch(p, nullptr, nullptr, nullptr, nullptr, s);
  st->set_attr_only = false;
  if (rc) return rc;
  static const char *amodes[] = {"gather", "cpasync", "tma"};
  p.variant = std::string(st->split3 ? "tc_3xtf32" : "tc_tf32") + "_bn" + std::to_string(bn) + "_" +
              amodes[st->amode] + (st->epi_tma ? "_tmastore" : "");
  return 0;
}

void conv_tc_release(void *state) { delete static_cast<TcState *>(state); }

int conv_tc_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s) {
  const TcState &st = *static_cast<const TcState *>(p.tc_state);
  const float *xf = static_cast<const float *>(x);
  float *yf = static_cast<float *>(y);
  const float *rf = static_cast<const float *>(res);
  const float *bias = p.bias_f;
  if (st.split3) {
    switch (st.bn) {
      case 32: return launch_modes<32, 4, true>(st, xf, yf, bias, rf, status, s);
      case 64: return launch_modes<64, 4, true>(st, xf, yf, bias, rf, status, s);
      case 256: return launch_modes<256, 2, true>(st, xf, yf, bias, rf, status, s);
      default: return launch_modes<128, 3, true>(st, xf, yf, bias, rf, status, s);
    }
  }
  switch (st.bn) {
    case 32: return launch_modes<32, 4, false>(st, xf, yf, bias, rf, status, s);
    case 64: return launch_modes<64, 4, false>(st, xf, yf, bias, rf, status, s);
    case 256: return launch_modes<256, 4, false>(st, xf, yf, bias, rf, status, s);
    default: return launch_modes<128, 4, false>(st, xf, yf, bias, rf, status, s);
  }
}

}  // namespace spkv2
