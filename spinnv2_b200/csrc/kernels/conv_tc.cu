// tcgen05 implicit-GEMM convolution for sm_100a (fp32 activations, TF32
// tensor cores, 3xTF32 split for near-fp32 accuracy).
//
// GEMM view: rows = output pixels (n, oh, ow), columns = output channels,
// K = (r, s, c) with c fastest; A rows are gathered from the activation
// (implicit im2col), B = packed weights [Cout_pad][K_pad] K-major.
//
// CTA tile: 128 pixels x BN channels, K step 32 fp32 (one 128-byte swizzle
// row).  Warp roles (192 threads):
//   warps 0-3  A producers: each thread gathers 16-byte chunks of 8 rows
//              (8 threads cover one 128-byte row: coalesced), converts to
//              TF32 (hi = round-to-nearest TF32, lo = x - hi), stores them in
//              the 128B-swizzled K-major layout, then run the epilogue
//              (TMEM lanes 32w..32w+31 = tile rows of warp w).
//   warp 4     B producer: one thread issues TMA loads (no multicast) of the
//              weight panels (hi, and lo for 3xTF32).
//   warp 5     MMA issuer: allocates TMEM, one thread issues tcgen05.mma
//              (M=128, N=BN, K=8 per instruction) into an fp32 TMEM
//              accumulator and commits stage releases; frees TMEM at the end.
// 3xTF32: acc += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi (three MMAs per K step).
// Pipelines use mbarriers; every wait is bounded (about a second of clock
// cycles) and on timeout the CTA records an error in the context status word
// and winds down without further waits on the failed barrier.
#include <cuda.h>
#include <cudaTypedefs.h>
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
  int split3;    // 1: 3xTF32, 0: TF32
};

// Shared memory per stage: A_hi, [A_lo], B_hi, [B_lo]; each 1024-aligned.
template <int BN, bool SPLIT3>
struct StageBytes {
  static constexpr int A = kBM * 128;
  static constexpr int B = BN * 128;
  static constexpr int value = (SPLIT3 ? 2 : 1) * (A + B);
};

// AVEC: activation NHWC with C % 4 == 0 (16-byte chunk gathers); otherwise
// per-element gathers through the generic strides.
template <int BN, int STAGES, bool SPLIT3, bool AVEC>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const float *__restrict__ x,
                   const float *__restrict__ bias, const float *__restrict__ res, float *__restrict__ y, TcParams tp,
                   int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = StageBytes<BN, SPLIT3>::A;
  constexpr int B_BYTES = StageBytes<BN, SPLIT3>::B;
  constexpr int STAGE = StageBytes<BN, SPLIT3>::value;
  __shared__ uint64_t full_bar[STAGES], empty_bar[STAGES], done_bar;
  __shared__ uint32_t tmem_base_holder;
  __shared__ volatile int abort_flag;

  const ConvGeo &g = tp.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = tp.Npad / BN;
  const int n0 = (blockIdx.x % n_tiles) * BN;  // channel tile fastest: pixel tile shared in L2
  const int64_t m0 = int64_t(blockIdx.x / n_tiles) * kBM;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 128 + 1);
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
    // ------------------------------------------------------------ A producer
    const int chunk = tid & 7;   // 16-byte chunk of the 128-byte row
    const int rsub = tid >> 3;   // 0..15: row within a group of 16
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
    for (int kb = 0; kb < tp.num_kb; ++kb) {
      const int s = kb % STAGES;
      const uint32_t ph = (kb / STAGES) & 1;
      if (!mbar_wait(&empty_bar[s], ph ^ 1, &abort_flag, status, 1)) break;
      uint8_t *a_hi = smem + s * STAGE;
      uint8_t *a_lo = a_hi + A_BYTES;
      float4 v[8];
      const int k0 = kb * kBK + chunk * 4;
      if (AVEC) {
        // The 4 channels of this chunk share one filter tap (C % 4 == 0).
        const bool kval = k0 < g.K;
        const int tap = k0 / g.Cg, c = k0 - tap * g.Cg;
        const int r = tap / g.KW, sx = tap - r * g.KW;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int ih = rih[i] + r * g.dh, iw = riw[i] + sx * g.dw;
          const bool ok = kval && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
          v[i] = ok ? __ldg(reinterpret_cast<const float4 *>(x + ((int64_t(rn[i]) * g.H + ih) * g.W + iw) * g.C + c))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      } else {
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
            const bool ok = ek[e] && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
            f[e] = ok ? __ldg(x + rn[i] * g.xs[0] + ec[e] * g.xs[1] + ih * g.xs[2] + iw * g.xs[3]) : 0.f;
          }
          v[i] = make_float4(f[0], f[1], f[2], f[3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int row = i * 16 + rsub;
        const uint32_t off = row * 128 + ((chunk ^ (row & 7)) << 4);
        float4 hi, lo;
        hi.x = tf32_rna(v[i].x);
        hi.y = tf32_rna(v[i].y);
        hi.z = tf32_rna(v[i].z);
        hi.w = tf32_rna(v[i].w);
        *reinterpret_cast<float4 *>(a_hi + off) = hi;
        if (SPLIT3) {
          lo.x = v[i].x - hi.x;
          lo.y = v[i].y - hi.y;
          lo.z = v[i].z - hi.z;
          lo.w = v[i].w - hi.w;
          *reinterpret_cast<float4 *>(a_lo + off) = lo;
        }
      }
      fence_proxy_async();
      mbar_arrive(&full_bar[s]);
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
      const bool yvec = g.ys[1] == 1 && (g.M % 4) == 0;
      const bool rvec = g.rs[1] == 1 && (g.M % 4) == 0;
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 32) {
        uint32_t acc[32];
        tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(cb), acc);
        const int c0 = n0 + cb;
        if (!pv || c0 >= g.M) continue;
        float vals[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] = __uint_as_float(acc[j]);
        const int cn = min(32, g.M - c0);
        if (cn == 32 && yvec && (!g.has_res || rvec)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 b = g.has_bias ? __ldg(reinterpret_cast<const float4 *>(bias + c0 + j)) : make_float4(0, 0, 0, 0);
            float4 rr = g.has_res ? __ldg(reinterpret_cast<const float4 *>(res + rbase + c0 + j))
                                  : make_float4(0, 0, 0, 0);
            float4 o;
            o.x = apply_act(vals[j] + b.x + rr.x, g.act);
            o.y = apply_act(vals[j + 1] + b.y + rr.y, g.act);
            o.z = apply_act(vals[j + 2] + b.z + rr.z, g.act);
            o.w = apply_act(vals[j + 3] + b.w + rr.w, g.act);
            *reinterpret_cast<float4 *>(y + ybase + c0 + j) = o;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < cn) {
              const int c = c0 + j;
              float v = vals[j];
              if (g.has_bias) v += __ldg(bias + c);
              if (g.has_res) v += __ldg(res + rbase + int64_t(c) * g.rs[1]);
              y[ybase + int64_t(c) * g.ys[1]] = apply_act(v, g.act);
            }
          }
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ B producer (TMA)
    if (lane == 0) {
      for (int kb = 0; kb < tp.num_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, &abort_flag, status, 2)) break;
        uint8_t *b_hi = smem + s * STAGE + (SPLIT3 ? 2 : 1) * A_BYTES;
        mbar_arrive_expect_tx(&full_bar[s], (SPLIT3 ? 2 : 1) * B_BYTES);
        tma_load_2d(b_hi, &wmap, kb * kBK, n0, &full_bar[s]);
        if (SPLIT3) tma_load_2d(b_hi + B_BYTES, &wmap, kb * kBK, tp.Npad + n0, &full_bar[s]);
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
      bool ok = true;
      for (int kb = 0; kb < tp.num_kb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        ok = mbar_wait(&full_bar[s], ph, &abort_flag, status, 3);
        if (!ok) break;
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

struct TcState {
  CUtensorMap map;
  TcParams tp;
  int bn = 128;
  int stages = 2;
  bool split3 = true;
  bool avec = true;
  size_t smem = 0;
  bool set_attr_only = false;  // dispatch only sets the kernel's smem attribute
};

template <int BN, int STAGES, bool SPLIT3, bool AVEC>
int launch_cfg(const TcState &st, const float *x, float *y, const float *bias, const float *res, int *status,
               cudaStream_t s) {
  auto kern = conv_tc_kernel<BN, STAGES, SPLIT3, AVEC>;
  if (st.set_attr_only)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st.smem)));
  const int64_t mt = ceil_div(st.tp.g.P, kBM);
  const int64_t blocks = mt * (st.tp.Npad / BN);
  if (blocks > 0x7fffffffLL) return SPKV2_ERR_UNSUPPORTED;
  kern<<<unsigned(blocks), kThreads, st.smem, s>>>(st.map, x, bias, res, y, st.tp, status);
  return cuda_status(cudaGetLastError());
}

template <int BN, int STAGES, bool SPLIT3>
int launch_avec(const TcState &st, const float *x, float *y, const float *bias, const float *res, int *status,
                cudaStream_t s) {
  return st.avec ? launch_cfg<BN, STAGES, SPLIT3, true>(st, x, y, bias, res, status, s)
                 : launch_cfg<BN, STAGES, SPLIT3, false>(st, x, y, bias, res, status, s);
}

}  // namespace

// Eligible: fp32 in/out, group 1, output channels >= 16.  Tile width BN is
// the smallest of {32, 64, 128, 256}... covering Cout, capped at 128 (256 for
// Cout >= 512 in TF32 mode).
int conv_tc_prepare(ConvPlan &p, const void *w_raw_dev, cudaStream_t s) {
  const ConvGeo &g = p.g;
  if (p.mode != kConvF32 || g.groups != 1 || g.M < 16) return SPKV2_ERR_UNSUPPORTED;
  if (p.math != SPKV2_CUDA_MATH_3XTF32 && p.math != SPKV2_CUDA_MATH_TF32) return SPKV2_ERR_UNSUPPORTED;
  if (!encode_fn()) return SPKV2_ERR_UNSUPPORTED;
  TcState *st = new TcState();
  st->split3 = p.math == SPKV2_CUDA_MATH_3XTF32;
  st->bn = g.M <= 32 ? 32 : g.M <= 64 ? 64 : 128;
  st->stages = st->split3 ? (st->bn == 128 ? 3 : 4) : 4;
  st->avec = g.xs[1] == 1 && g.C % 4 == 0;
  TcParams &tp = st->tp;
  tp.g = g;
  tp.Kpad = int(ceil_div(g.K, kBK) * kBK);
  tp.Npad = int(ceil_div(g.M, st->bn) * st->bn);
  tp.num_kb = tp.Kpad / kBK;
  tp.split3 = st->split3 ? 1 : 0;
  const int parts = st->split3 ? 2 : 1;
  const size_t wbytes = size_t(parts) * tp.Npad * tp.Kpad * sizeof(float);
  float *wtc = static_cast<float *>(device_alloc(wbytes));
  if (!wtc) {
    delete st;
    return SPKV2_ERR_DEVICE_ALLOC;
  }
  pack_tc_kernel<<<grid_for(int64_t(tp.Npad) * tp.Kpad, 256), 256, 0, s>>>(wtc, static_cast<const float *>(w_raw_dev),
                                                                           g, tp.Npad, tp.Kpad, tp.split3);
  int rc = cuda_status(cudaGetLastError());
  if (rc) {
    device_free(wtc);
    delete st;
    return rc;
  }
  // Weight panel tensor map: dims {Kpad, parts*Npad}, box {32, BN}, 128B swizzle.
  const cuuint64_t dims[2] = {cuuint64_t(tp.Kpad), cuuint64_t(parts) * cuuint64_t(tp.Npad)};
  const cuuint64_t strides[1] = {cuuint64_t(tp.Kpad) * sizeof(float)};
  const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(st->bn)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult cr = encode_fn()(&st->map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, wtc, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) {
    device_free(wtc);
    delete st;
    return SPKV2_ERR_UNSUPPORTED;
  }
  const int stage_bytes = parts * (kBM * 128 + st->bn * 128);
  st->smem = size_t(st->stages) * stage_bytes + 1024;
  // Keep at most two CTAs per SM so their TMEM allocations (<= 256 columns
  // each) always fit in the 512 columns.
  st->smem = std::max<size_t>(st->smem, 80 * 1024);
  p.w_tc = wtc;
  p.tc_state = st;
  // Opt the chosen kernel into its dynamic shared memory on this device.
  st->set_attr_only = true;
  rc = conv_tc_launch(p, nullptr, nullptr, nullptr, nullptr, s);
  st->set_attr_only = false;
  if (rc) return rc;
  p.tc_block_n = st->bn;
  p.tc_kpad = tp.Kpad;
  p.variant = std::string(st->split3 ? "tc_3xtf32" : "tc_tf32") + "_bn" + std::to_string(st->bn) +
              (st->avec ? "_vec" : "_gather");
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
      case 32: return launch_avec<32, 4, true>(st, xf, yf, bias, rf, status, s);
      case 64: return launch_avec<64, 4, true>(st, xf, yf, bias, rf, status, s);
      default: return launch_avec<128, 3, true>(st, xf, yf, bias, rf, status, s);
    }
  }
  switch (st.bn) {
    case 32: return launch_avec<32, 4, false>(st, xf, yf, bias, rf, status, s);
    case 64: return launch_avec<64, 4, false>(st, xf, yf, bias, rf, status, s);
    default: return launch_avec<128, 4, false>(st, xf, yf, bias, rf, status, s);
  }
}

}  // namespace spkv2
