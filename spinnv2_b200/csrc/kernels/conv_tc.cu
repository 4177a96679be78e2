// tcgen05 implicit-GEMM convolution for sm_100a (fp32 activations, TF32
// tensor cores, 3xTF32 split for near-fp32 accuracy).  Also serves Gemm as a
// 1x1 convolution over [M,1,1,K].
//
// GEMM view: rows = output pixels (n, oh, ow), columns = output channels,
// K = (r, s, c) with c fastest; A rows are the activation gathered on the
// fly (implicit im2col), B = packed weights [Cout_pad][K_pad] K-major.
//
// Persistent kernel: one CTA per SM walks output tiles (128 pixels x BN
// channels) in a static round-robin.  Warp roles (480 threads):
//   warps 0-7   epilogue: warps w and w+4 read TMEM lanes 32(w%4).. (tile
//               rows) and split the tile's columns -> registers -> bias,
//               residual (prefetched into L2 when the tile starts), Relu /
//               SiLU -> TMA store staged through shared memory (NHWC
//               outputs) or direct stores.  TMEM holds two accumulator
//               buffers, so the epilogue overlaps the next tile's mainloop.
//   warps 8-11  A operand.  AMODE 2 (1x1, stride 1, C % 32 == 0, output
//               extent = input extent): the tile arrives by a tiled TMA load;
//               AMODE 3 (other square convs, C % 32 == 0, the output extent
//               of equal top / bottom and left / right padding): by an im2col
//               TMA load (128 output pixels x 32 channels of one filter tap,
//               padding zero-filled by the TMA unit); AMODE 5 (C % 16 == 0,
//               space-to-depth first convs, any padding: window corners from
//               the output extent): two 16-channel 64-byte im2col columns per
//               K step; AMODE 4 (4-channel inputs, as AMODE 3's extent): eight
//               16-byte im2col columns per K step in an unswizzled
//               core-matrix layout.  The
//               tile lands straight in the operand stage; for 3xTF32 these
//               warps add its low part.  AMODE 1 (any other conv): each
//               thread gathers its 16-byte chunks with cp.async (zero-fill
//               for padding) into a landing ring of LAND slots, LAND-1 K
//               steps ahead of the MMA, and later copies ITS OWN chunks into
//               the operand stage, so a per-thread cp.async.wait_group is the
//               only synchronisation the landing needs.
//               TF32 split: the tensor core reads fp32 operands as TF32 by
//               dropping the low 13 mantissa bits, so the raw tile is the
//               high part and lo = x - trunc_tf32(x) is exact in fp32 (half
//               the shared-memory traffic of writing a rounded high part).
//   warp 12     TMA producer (one thread): weight panels (hi, and lo for
//               3xTF32).  No multicast.
//   warp 13     TMEM allocation; one thread issues tcgen05.mma (M=128, N=BN,
//               K=8) and commits stage releases and finished accumulators.
//   warp 14     TMA producer (one thread) of the A tile in the TMA A modes
//               (2-5): the weight and activation loads of a stage are issued
//               by two threads, measured on B200: neutral on the ResNet-101
//               3xTF32 step, +2 % TF32 mode and detector bs64.
// 3xTF32: acc += A_lo*B_hi + A_hi*B_lo + A_hi*B_hi (three MMAs per K step).
// The tensor core's fp32 accumulation truncates, which over long K chains
// biases the sum (the error grows linearly with K).  In 3xTF32 mode each
// group of `group` K steps therefore accumulates into its own TMEM buffer,
// and the epilogue warps add each finished partial into a third TMEM region
// of running sums with round-to-nearest fp32 adds ("promotion"), so the MMA
// of the next group overlaps the add of this one.
// Inputs that are not dense NHWC with C % 4 == 0 (a network's NCHW graph
// input, C = 3) are first re-laid out into a plan-owned NHWC buffer with C
// rounded up to 4.
// Every mbarrier wait is bounded (about a second of clock cycles); on timeout
// the CTA records a code in the context's status word and winds down.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "conv.h"
#include "tcgen05.cuh"

namespace spkv2 {

namespace {

using namespace tc;

constexpr int kBM = 128;          // tile rows (pixels) = UMMA M
constexpr int kBK = 32;           // fp32 elements per K step = 128 bytes
constexpr int kABytes = kBM * 128;
constexpr int kThreads = 480;               // 8 epilogue + 4 A-operand + weight TMA + MMA + A TMA warps
constexpr int kEpiWarps = 8;
constexpr int kStagingBytes = kEpiWarps * 4096;  // epilogue: one 32x32 fp32 tile per warp

// ---------------------------------------------------------------- kernel
struct TcParams {
  ConvGeo g;       // GEMM-side geometry (C may be the padded channel count)
  int Kpad;        // K rounded up to a multiple of 32
  int Npad;        // rows per weight-panel part (Cout rounded up to a multiple of BN, or the stored panel's)
  int num_kb;      // Kpad / 32
  int n_tiles;     // ceil(Cout / BN)
  int64_t tiles;   // m_tiles * n_tiles
  int group;       // K steps per TMEM partial when promoting (3xTF32)
  int out_i8;      // quantise the output: y = clamp(rne(act(v) * (1 / s_y)), -128, 127)
  int res_tma;     // residual tiles arrive by TMA in the epilogue staging tile (NHWC residual, TMA store)
  int64_t dp_tiles;  // tiles walked whole, round-robin over the CTAs (all tiles without stream-K)
  int64_t sk_units;  // stream-K: K steps of tiles dp_tiles.. spread evenly over CTAs 0..sk_ctas-1 (0: off)
  int sk_ctas;       // CTAs sharing the stream-K units (fewer CTAs: fewer segments per tile to add up)
  int sk_park_all;   // split-K: every segment parks its partial; conv_tc_reduce_kernel finishes all tiles
  int p32;           // output pixel count < 2^31: pixel coordinates by 32-bit multiply-shift divisions
  FastDiv ow_div, oh_div;
  FastDiv nt_div, u_div, g_div, nk_div;  // n_tiles, sk_units, sk_ctas, num_kb (stream-K / split-K schedule)
};

// Epilogue activation over a register array (one branch per call).  SiLU
// as v / (1 + e^-v) with the fast exponential and divide intrinsics: a few
// ulp from the correctly rounded quotient, far inside the fp32 output
// tolerance, and a third of the instructions of expf and an IEEE divide.
template <int N>
__device__ __forceinline__ void epi_act(float (&v)[N], int act) {
  if (act == 1) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
  } else if (act == 2) {
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] = __fdividef(v[j], 1.0f + __expf(-v[j]));
  }
}

// Output pixel p -> (n, oh, ow).
__device__ __forceinline__ void pixel_nhw(const TcParams &tp, int64_t p, int &n, int &oh, int &ow) {
  if (tp.p32) {
    const uint32_t q = tp.ow_div.div(uint32_t(p));
    ow = int(uint32_t(p) - q * uint32_t(tp.g.OW));
    const uint32_t r = tp.oh_div.div(q);
    oh = int(q - r * uint32_t(tp.g.OH));
    n = int(r);
  } else {
    ow = int(p % tp.g.OW);
    const int64_t q = p / tp.g.OW;
    oh = int(q % tp.g.OH);
    n = int(q / tp.g.OH);
  }
}

// One unit of a CTA's work: K steps [kb0, kb1) of output tile `tile`.  A
// stream-K tile whose K steps are spread over several CTAs has nseg > 1
// segments, of which this CTA's is number `seg`; its partial sums go to this
// CTA's workspace slot `slot` (0: the first segment of its share, 1: the
// last) and the epilogue warp that arrives last adds all of them.
struct Seg {
  int64_t tile;
  int kb0, kb1;
  int nseg, seg;
  int tt;  // index among the stream-K tiles
  int slot;
};

// The static schedule every role of a CTA walks in the same order: whole
// tiles tile0, tile0 + tstep, ... below dp_tiles, then this CTA's contiguous
// share [u0, u1) of the remaining tiles' K steps (unit u = K step u % nk of
// stream-K tile u / nk), cut at tile boundaries; only CTAs below sk_ctas
// take a share.  SK = false compiles the whole-tile schedule only (kernels
// that never use stream-K).
template <bool SK>
struct WorkIter {
  int64_t t, tstep, dp_tiles;
  int64_t u, u0, u1, U;
  int nk, G, b;
  // The stream-K arithmetic is 32-bit with the host's multiply-shift
  // divisors (the host keeps U * G below 2^31): it runs in every role
  // before the first load or MMA of the kernel.
  FastDiv u_div, g_div, nk_div;
  __device__ WorkIter(const TcParams &tp, int64_t tile0, int64_t step, int cta, int grid)
      : t(tile0), tstep(step), dp_tiles(SK ? tp.dp_tiles : tp.tiles), U(SK ? tp.sk_units : 0), nk(tp.num_kb),
        G(SK && tp.sk_units ? tp.sk_ctas : grid), b(cta), u_div(tp.u_div), g_div(tp.g_div), nk_div(tp.nk_div) {
    u0 = U ? (b < G ? int64_t(start_of(b)) : U) : 0;
    u1 = U ? (b < G ? int64_t(start_of(b + 1)) : U) : 0;
    u = u0;
  }
  __device__ int64_t start_of(int64_t cta) const { return g_div.div(uint32_t(cta) * uint32_t(U)); }
  // CTA whose share holds unit v.
  __device__ int64_t owner(int64_t v) const { return u_div.div((uint32_t(v) + 1) * uint32_t(G) - 1); }
  // Workspace slot in which CTA `cta` keeps its segment of stream-K tile tt.
  __device__ int slot_of(int64_t cta, int64_t tt) const { return start_of(cta) >= tt * nk ? 0 : 1; }
  // K steps of this CTA's whole schedule.
  __device__ uint32_t total_steps() const {
    const int64_t mine = t < dp_tiles ? int64_t(uint32_t(dp_tiles - 1 - t) / uint32_t(tstep)) + 1 : 0;
    return uint32_t(mine * nk + (u1 - u0));
  }
  __device__ bool next(Seg &s) {
    if (t < dp_tiles) {
      s.tile = t;
      s.kb0 = 0;
      s.kb1 = nk;
      s.nseg = 1;
      s.seg = s.tt = s.slot = 0;
      t += tstep;
      return true;
    }
    if (!SK || u >= u1) return false;
    const int64_t tt = nk_div.div(uint32_t(u));
    s.tt = int(tt);
    s.tile = dp_tiles + tt;
    s.kb0 = int(u - tt * nk);
    s.kb1 = int(s.kb0 + u1 - u < nk ? s.kb0 + u1 - u : nk);
    s.slot = u == u0 ? 0 : 1;
    u += s.kb1 - s.kb0;
    if (s.kb0 == 0 && s.kb1 == nk) {
      s.nseg = 1;
      s.seg = 0;
    } else {
      const int64_t blo = owner(tt * nk);
      s.nseg = int(owner(tt * nk + nk - 1) - blo + 1);
      s.seg = int(b - blo);
    }
    return true;
  }
};

// A-low-in-TMEM variant (single-CTA 3xTF32, BN = 128, TMA-fed A): the A
// warps write A's low part into a TMEM ring (one 32-column slot per stage)
// instead of shared memory and the A_lo * B_hi MMAs read A from TMEM.  The
// stage shrinks to [A hi][B hi][B lo] (48 KB), so four stages fit instead of
// three.  Two accumulator buffers (promotion every few K steps leaves the
// epilogue a group's time per add) free the TMEM for the ring.  Narrow tiles
// keep A's low part in shared memory: measured on B200 with the ring at BN =
// 64 / 32 (6 / 8 stages), the detector's 3x3 16-channel convs took 375
// instead of 335 us and ResNet-50 INT8 bs256 (its fp32 BN = 64 first conv)
// dropped from 57.7k to 55.6k img/s.
constexpr bool alo_tmem(int bn, bool split3, int amode, bool pair) {
  return split3 && !pair && bn == 128 && (amode == 2 || amode == 3 || amode == 5);
}

// One pipeline stage: [A (hi)][A lo (3xTF32)][B hi][B lo (3xTF32)], or
// [A hi][B hi][B lo] when A's low part lives in TMEM.
constexpr int stage_bytes(int brows, bool split3, bool alo = false) {
  return alo ? kABytes + 2 * brows * 128 : (split3 ? 2 : 1) * (kABytes + brows * 128);
}

// TMEM accumulator buffers the MMA rotates through.  3xTF32 hands a partial
// buffer to the epilogue every `group` K steps to be added into the fp32
// sums; with three buffers the epilogue has two groups' time to do it before
// the MMA needs the buffer again.  TF32 hands off once per tile (two buffers:
// tile t's epilogue overlaps tile t+1's MMAs).
template <int BN, bool SPLIT3, bool ALO = false, int STAGES = 0>
struct AccLayout {
  static constexpr int nbuf = ALO ? 2 : SPLIT3 && 4 * BN <= 512 ? 3 : 2;
  static constexpr int sum_col = nbuf * BN;                     // promoted sums (3xTF32)
  static constexpr int alo_col = sum_col + (SPLIT3 ? BN : 0);  // A low-part ring (ALO)
  static constexpr int cols = alo_col + (ALO ? 32 * STAGES : 0);
};

// Row / chunk mapping shared by the A loads and the conversion pass: thread t
// (0..127) handles 16-byte chunk (t & 7) of rows i*16 + (t >> 3), i = 0..7.
__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
  return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// The tensor core reads an fp32 operand of kind::tf32 as TF32 by dropping
// the low 13 mantissa bits.  So a raw fp32 tile is its own high part, and the
// 3xTF32 low part is lo = x - trunc_tf32(x), exact in fp32.  Thread t handles
// its chunks of the tile at `src`: copies them to dst_hi unless src == dst_hi,
// and for 3xTF32 writes the low parts to dst_lo.
template <bool SPLIT3>
__device__ __forceinline__ void convert_tile(const uint8_t *src, uint8_t *dst_hi, uint8_t *dst_lo, int t) {
  const int chunk = t & 7, rsub = t >> 3;
  const bool copy = src != dst_hi;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t off = swz_off(i * 16 + rsub, chunk);
    const float4 v = *reinterpret_cast<const float4 *>(src + off);
    if (copy) *reinterpret_cast<float4 *>(dst_hi + off) = v;
    if (SPLIT3) {
      const float hx = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
      const float hy = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
      const float hz = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
      const float hw = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
      *reinterpret_cast<float4 *>(dst_lo + off) = make_float4(v.x - hx, v.y - hy, v.z - hz, v.w - hw);
    }
  }
}

template <int BN, int STAGES, int LAND, bool SPLIT3, int AMODE, bool EPI_TMA, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap ymap, const __grid_constant__ CUtensorMap rmap,
                   const float *__restrict__ x,
                   const float *__restrict__ bias, const float *__restrict__ res, float *__restrict__ y, TcParams tp,
                   float *__restrict__ sk_ws, int *__restrict__ sk_cnt, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // PAIR: 2-SM tiles.  The two CTAs of a cluster share one M = 256 x N = BN
  // MMA issued by CTA 0; each holds its 128 rows of A and BN/2 rows of B.
  static_assert(!PAIR || (AMODE == 2 || AMODE == 3), "CTA pairs take TMA-fed A operands");
  constexpr int BROWS = PAIR ? BN / 2 : BN;  // weight rows held by this CTA
  constexpr int TILE_ROWS = PAIR ? 2 * kBM : kBM;
  constexpr int B_BYTES = BROWS * 128;
  constexpr bool ALO = alo_tmem(BN, SPLIT3, AMODE, PAIR);
  constexpr int STAGE = stage_bytes(BROWS, SPLIT3, ALO);
  // Stream-K (a tail past the last full wave, or split-K over all tiles)
  // exists in single-CTA kernels.
  constexpr bool SK = !PAIR;
  using Iter = WorkIter<SK>;
  constexpr int B_OFF = (SPLIT3 && !ALO ? 2 : 1) * kABytes;  // B hi within a stage
  // The A warps hand the stage to the MMA (full_bar) whenever they touch it:
  // for gathers (copied from the landing ring), for 3xTF32 (low parts) and,
  // in a CTA pair, to tell the leader that this CTA's operands have landed.
  // Otherwise TF32 TMA tiles go to the tensor core as loaded.
  constexpr bool CONVERT = (AMODE == 1) || SPLIT3;
  constexpr bool SEP_A = AMODE != 1;  // a second TMA thread (warp 14) loads the A tiles
  constexpr bool RELAY = CONVERT || PAIR;
  // TMEM: the accumulator buffers + the promoted sums for 3xTF32, rounded
  // up to a power of two >= 32 columns.
  using Acc = AccLayout<BN, SPLIT3, ALO, STAGES>;
  constexpr int NBUF = Acc::nbuf;
  constexpr int kCols = Acc::cols;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128 : kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "accumulators exceed TMEM");
  uint8_t *land = smem + STAGES * STAGE;    // AMODE 1 landing ring
  uint8_t *staging = land + LAND * kABytes;  // epilogue TMA-store staging
  __shared__ uint64_t raw_bar[STAGES], full_bar[STAGES], empty_bar[STAGES], accf_bar[NBUF], acce_bar[NBUF];
  __shared__ uint64_t res_bar[kEpiWarps];  // residual tile landed in the warp's staging tile
  __shared__ uint32_t tmem_base_holder;
  __shared__ volatile int abort_flag;

  const ConvGeo &g = tp.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;                    // 0 = leader of the pair
  const int64_t tile0 = PAIR ? int64_t(cluster_id_x()) : int64_t(blockIdx.x);
  const int64_t tstep = PAIR ? int64_t(cluster_count_x()) : int64_t(gridDim.x);
  // Barriers completed by the other CTA of a pair are waited on with
  // acquire at cluster scope.
  auto wait_any = [&](uint64_t *bar, uint32_t parity, int code) {
    return PAIR ? mbar_wait_cluster(bar, parity, &abort_flag, status, code)
                : mbar_wait(bar, parity, &abort_flag, status, code);
  };
  // Arrivals that the leader's MMA thread waits for come from both CTAs.
  auto arrive_leader = [&](uint64_t *bar) {
    if (PAIR)
      mbar_arrive_rank(bar, 0);
    else
      mbar_arrive(bar);
  };

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&raw_bar[s], SEP_A ? 2 : 1);         // TMA producers' arrive.expect_tx (+ transaction bytes)
      mbar_init(&full_bar[s], PAIR ? 8 : 4);         // one arrival per A warp (of both CTAs of a pair)
      mbar_init(&empty_bar[s], 1);                   // MMA commit
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], kEpiWarps * (PAIR ? 2 : 1));  // one arrival per epilogue warp
    }
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&res_bar[w], 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 13) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&tmem_base_holder)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&tmem_base_holder)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // both CTAs' barriers exist before any remote arrival
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_holder;
  // Everything above touches only this CTA's shared memory and TMEM; the
  // next layer may start launching now, and this one waits here for the
  // previous layer's outputs (and for its reads of buffers this one writes).
  pdl_launch_dependents();
  pdl_wait();

  if (warp < kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // Warps w and w+4 read TMEM lanes 32(w%4).. (tile rows) and split the
    // tile's columns; with BN = 32 warps 4-7 only hand the buffers back.
    const int quarter = warp & 3;
    const int ncol = BN >= 64 ? BN / 2 : (warp < 4 ? BN : 0);
    const int col0 = BN >= 64 ? (warp >> 2) * (BN / 2) : 0;
    uint8_t *stage_buf = staging + warp * 4096;
    const bool rvec = g.rs[1] == 1 && (g.M % 4) == 0;
    uint32_t sc = 0;  // TMA-store chunks issued by this warp
    uint32_t rc = 0;  // residual tiles loaded by this warp
    const bool res_tma = EPI_TMA && tp.res_tma && g.has_res;
    uint32_t gi = 0;  // accumulator hand-offs consumed (one per K group)
    const uint32_t trow = tmem + (uint32_t(quarter * 32) << 16);  // this warp's TMEM lanes
    const uint32_t tsum = trow + uint32_t(Acc::sum_col);            // promoted sums (3xTF32)
    float4 *const ws4 = reinterpret_cast<float4 *>(sk_ws);
    Iter wi(tp, tile0, tstep, int(blockIdx.x), int(gridDim.x));
    Seg sg;
    while (wi.next(sg)) {
      const int64_t t = sg.tile;
      const int ngroups = (sg.kb1 - sg.kb0 + tp.group - 1) / tp.group;
      const uint32_t mt = tp.nt_div.div(uint32_t(t));  // tile row, column (tiles < 2^31)
      const int n0 = int(uint32_t(t) - mt * uint32_t(tp.n_tiles)) * BN;
      const int64_t m0 = int64_t(mt) * TILE_ROWS + rank * kBM;
      const int row = quarter * 32 + lane;
      const int64_t p = m0 + row;
      const bool pv = p < g.P;
      int n = 0, oh = 0, ow = 0;
      if (pv) pixel_nhw(tp, p, n, oh, ow);
      const int64_t ybase = int64_t(n) * g.ys[0] + int64_t(oh) * g.ys[2] + int64_t(ow) * g.ys[3];
      const int64_t rbase = int64_t(n) * g.rs[0] + int64_t(oh) * g.rs[2] + int64_t(ow) * g.rs[3];
      if (g.has_res && pv && rvec) {
        // Pull this row's residual into L2 while the MMAs run.
        for (int j = 0; j < ncol && n0 + col0 + j < g.M; j += 32)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(res + rbase + n0 + col0 + j));
      }
      // All K groups but the last: add the group's partial into the sums
      // (round-to-nearest fp32 adds) and hand the partial buffer back.
      bool failed = false;
      for (int gidx = 0; gidx + 1 < ngroups; ++gidx, ++gi) {
        const int pb = int(gi % NBUF);
        if (!__all_sync(0xffffffffu, wait_any(&accf_bar[pb], (gi / NBUF) & 1, 4))) {
          failed = true;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cb = col0; cb < col0 + ncol; cb += 32) {
          uint32_t part[32];
          tmem_ld32(trow + uint32_t(pb * BN + cb), part);
          if (gidx > 0) {
            uint32_t sum[32];
            tmem_ld32(tsum + uint32_t(cb), sum);
#pragma unroll
            for (int j = 0; j < 32; ++j) part[j] = __float_as_uint(__uint_as_float(part[j]) + __uint_as_float(sum[j]));
          }
          tmem_st32(tsum + uint32_t(cb), part);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&acce_bar[pb]);
      }
      if (failed) break;
      const int ab = int(gi % NBUF);
      if (!__all_sync(0xffffffffu, wait_any(&accf_bar[ab], (gi / NBUF) & 1, 4))) break;
      tc_fence_after();
      // Bias, residual, activation and store of accumulator columns
      // cb..cb+31 of this thread's row.
      auto store_chunk = [&](int cb, const uint32_t(&acc)[32]) {
        const int c0 = n0 + cb;
        if (c0 >= g.M) return;  // channel padding (warp-uniform)
        float vals[32];
        const int cn = min(32, g.M - c0);
        if (res_tma) {
          // (acc + bias) + residual, the residual read from the staging tile
          // its TMA load filled (rows past the end of the tensor read zeros).
          if (!__all_sync(0xffffffffu, mbar_wait(&res_bar[warp], rc & 1, &abort_flag, status, 6))) return;
          ++rc;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 b = g.has_bias ? __ldg(reinterpret_cast<const float4 *>(bias + c0 + j)) : make_float4(0, 0, 0, 0);
            const float4 rr = *reinterpret_cast<const float4 *>(stage_buf + swz_off(lane, j / 4));
            vals[j] = __uint_as_float(acc[j]) + b.x + rr.x;
            vals[j + 1] = __uint_as_float(acc[j + 1]) + b.y + rr.y;
            vals[j + 2] = __uint_as_float(acc[j + 2]) + b.z + rr.z;
            vals[j + 3] = __uint_as_float(acc[j + 3]) + b.w + rr.w;
          }
        } else if ((cn & 3) == 0 && (!g.has_res || rvec)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const bool in = j < cn;  // a narrow tile's padding columns load nothing
            const float4 b = g.has_bias && in ? __ldg(reinterpret_cast<const float4 *>(bias + c0 + j))
                                              : make_float4(0, 0, 0, 0);
            const float4 rr = (g.has_res && pv && in) ? __ldg(reinterpret_cast<const float4 *>(res + rbase + c0 + j))
                                                      : make_float4(0, 0, 0, 0);
            vals[j] = __uint_as_float(acc[j]) + b.x + rr.x;
            vals[j + 1] = __uint_as_float(acc[j + 1]) + b.y + rr.y;
            vals[j + 2] = __uint_as_float(acc[j + 2]) + b.z + rr.z;
            vals[j + 3] = __uint_as_float(acc[j + 3]) + b.w + rr.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = __uint_as_float(acc[j]);
            if (j < cn) {
              const int c = c0 + j;
              if (g.has_bias) v += __ldg(bias + c);
              if (g.has_res && pv) v += __ldg(res + rbase + int64_t(c) * g.rs[1]);
            }
            vals[j] = v;
          }
        }
        // Activation, one uniform branch per chunk; a narrow tile's padding
        // columns (cn <= 16) are skipped.
        if (cn > 16) {
          epi_act<32>(vals, g.act);
        } else {
          epi_act<16>(reinterpret_cast<float(&)[16]>(vals), g.act);
        }
        if (tp.out_i8) {
          // fp32 conv with an int8 output (the first conv of an INT8 network).
          if (!pv) return;
          int8_t *y8 = reinterpret_cast<int8_t *>(y);
          if (cn == 32 && g.ys[1] == 1 && (g.M % 16) == 0) {
            uint32_t w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint32_t b = 0;
#pragma unroll
              for (int e = 0; e < 4; ++e)
                b |= (uint32_t(sat_rne_i8(__fmul_rn(vals[4 * j + e], g.out_scale_inv), -128)) & 0xffu) << (8 * e);
              w[j] = b;
            }
            *reinterpret_cast<uint4 *>(y8 + ybase + c0) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4 *>(y8 + ybase + c0 + 16) = make_uint4(w[4], w[5], w[6], w[7]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cn) y8[ybase + int64_t(c0 + j) * g.ys[1]] = int8_t(sat_rne_i8(__fmul_rn(vals[j], g.out_scale_inv), -128));
          }
          return;
        }
        if (EPI_TMA) {
          uint8_t *buf = stage_buf;
          if (!res_tma && sc >= 1 && lane == 0) tma_store_wait_read0();  // the previous store has read the tile
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4 *>(buf + swz_off(lane, j)) =
                make_float4(vals[4 * j], vals[4 * j + 1], vals[4 * j + 2], vals[4 * j + 3]);
          fence_proxy_async();
          __syncwarp();
          if (lane == 0 && m0 + quarter * 32 < g.P) tma_store_2d(&ymap, c0, int(m0 + quarter * 32), buf);
          ++sc;
        } else if (pv) {
          if (g.ys[1] == 1 && (g.M % 4) == 0 && (cn & 3) == 0) {
            // NHWC rows of 4-aligned channel counts: 16-byte stores (a
            // narrow tile stores only its cn real columns).
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              if (j < cn)
                *reinterpret_cast<float4 *>(y + ybase + c0 + j) =
                    make_float4(vals[j], vals[j + 1], vals[j + 2], vals[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cn) y[ybase + int64_t(c0 + j) * g.ys[1]] = vals[j];
          }
        }
      };
      // Start chunk cb's residual tile into the staging tile (free once the
      // previous chunk's store has read it); the TMEM reads and the bias
      // overlap its flight.
      auto issue_res = [&](int cb) {
        if (res_tma && n0 + cb < g.M) {
          if (lane == 0) {
            if (sc >= 1) tma_store_wait_read0();
            mbar_arrive_expect_tx(&res_bar[warp], 4096);
            tma_load_2d(stage_buf, &rmap, n0 + cb, int(m0 + quarter * 32), &res_bar[warp]);
          }
          __syncwarp();
        }
      };
      // Last K group: partial (+ sums) of columns cb..cb+31; the buffer goes
      // back to the MMA once the warp's last chunk is read.
      auto read_acc = [&](int cb, uint32_t(&acc)[32]) {
        tmem_ld32(trow + uint32_t(ab * BN + cb), acc);
        if (ngroups > 1) {
          uint32_t sum[32];
          tmem_ld32(tsum + uint32_t(cb), sum);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __float_as_uint(__uint_as_float(acc[j]) + __uint_as_float(sum[j]));
        }
        if (cb + 32 >= col0 + ncol) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_leader(&acce_bar[ab]);
          ++gi;
        }
      };
      if (ncol == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(&acce_bar[ab]);
        ++gi;
        continue;
      }
      bool finish = true;
      int64_t blo = 0;
      if (SK && (sg.nseg > 1 || tp.sk_park_all)) {
        // Stream-K segment: park this warp's part of the tile in the CTA's
        // workspace slot ([chunk][4-column group][row] float4s, so a warp's
        // stores are contiguous) and count the arrival; the segment's last
        // warp to arrive adds all segments in segment order (the same sum
        // whichever CTA finishes last) and finishes the tile below.
        float4 *mine = ws4 + size_t(blockIdx.x * 2 + sg.slot) * (BN * 32);
#pragma unroll 1
        for (int cb = col0; cb < col0 + ncol; cb += 32) {
          uint32_t acc[32];
          read_acc(cb, acc);
          if (pv) {  // rows past the last pixel are never read back
#pragma unroll
            for (int q = 0; q < 8; ++q)
              __stcg(&mine[((cb >> 5) * 8 + q) * 128 + row],
                     make_float4(__uint_as_float(acc[4 * q]), __uint_as_float(acc[4 * q + 1]),
                                 __uint_as_float(acc[4 * q + 2]), __uint_as_float(acc[4 * q + 3])));
          }
        }
        if (tp.sk_park_all) continue;  // the reduce kernel finishes every tile
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          int *cnt = &sk_cnt[int64_t(sg.tt) * kEpiWarps + warp];
          last = atomicAdd(cnt, 1) == sg.nseg - 1;
          if (last) atomicExch(cnt, 0);  // ready for the next launch
        }
        finish = __shfl_sync(0xffffffffu, last, 0) != 0;
        if (finish) __threadfence();
        blo = wi.owner(int64_t(sg.tt) * tp.num_kb);
      }
      if (!finish) continue;
      // Bias, residual, activation -> store, chunk by chunk.
#pragma unroll 1
      for (int cb = col0; cb < col0 + ncol; cb += 32) {
        issue_res(cb);
        uint32_t acc[32];
        if (!SK || sg.nseg == 1) {
          read_acc(cb, acc);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = 0u;  // +0.0f
#pragma unroll 1
          for (int j = 0; j < sg.nseg; ++j) {
            const float4 *src = ws4 + size_t((blo + j) * 2 + wi.slot_of(blo + j, sg.tt)) * (BN * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 f = __ldcg(&src[((cb >> 5) * 8 + q) * 128 + row]);
              acc[4 * q] = __float_as_uint(__uint_as_float(acc[4 * q]) + f.x);
              acc[4 * q + 1] = __float_as_uint(__uint_as_float(acc[4 * q + 1]) + f.y);
              acc[4 * q + 2] = __float_as_uint(__uint_as_float(acc[4 * q + 2]) + f.z);
              acc[4 * q + 3] = __float_as_uint(__uint_as_float(acc[4 * q + 3]) + f.w);
            }
          }
        }
        store_chunk(cb, acc);
      }
    }
    if (EPI_TMA && lane == 0) tma_store_wait_all();
  } else if (warp < kEpiWarps + 4) {
    // ------------------------------------------------------------ A operand
    const int at = tid - 32 * kEpiWarps;
    uint32_t it = 0;  // global K-step counter
    bool ok = true;
    if constexpr (AMODE != 1) {
      if (RELAY) {  // 3xTF32: the low parts of the TMA-landed tile; pairs: tell the leader
        const uint32_t total = Iter(tp, tile0, tstep, int(blockIdx.x), int(gridDim.x)).total_steps();
        for (; it < total; ++it) {
          const int s = it % STAGES;
          const bool landed = mbar_wait(&raw_bar[s], (it / STAGES) & 1, &abort_flag, status, 5);
          if (!__all_sync(0xffffffffu, landed)) break;  // the warp leaves together
          uint8_t *a_hi = smem + s * STAGE;
          if constexpr (ALO) {
            // Row r = this warp's TMEM lane quarter + lane: its 32 K values
            // (eight swizzled 16-byte chunks) -> low parts -> TMEM slot s.
            const int r = (warp & 3) * 32 + lane;
            uint32_t lo[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              // AMODE 5: K elements 0-15 in the first 64-byte-swizzled half
              // (16-byte chunk cc of row r at r * 64 + (cc ^ (r / 2 % 4)) * 16),
              // 16-31 in the second.
              const uint32_t off = AMODE == 5 ? uint32_t((c >> 2) * (kABytes / 2) + r * 64 + (((c & 3) ^ ((r >> 1) & 3)) << 4))
                                              : swz_off(r, c);
              const float4 v = *reinterpret_cast<const float4 *>(a_hi + off);
              lo[4 * c] = __float_as_uint(v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u));
              lo[4 * c + 1] = __float_as_uint(v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u));
              lo[4 * c + 2] = __float_as_uint(v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u));
              lo[4 * c + 3] = __float_as_uint(v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
            }
            tmem_st32(tmem + (uint32_t((warp & 3) * 32) << 16) + uint32_t(Acc::alo_col + s * 32), lo);
            tmem_wait_st();
            tc_fence_before();
          } else {
            if (SPLIT3) convert_tile<SPLIT3>(a_hi, a_hi, a_hi + kABytes, at);
            fence_proxy_async();
          }
          // One arrival per warp (each mbarrier arrival is a shared-memory
          // read-modify-write the barrier serialises): every lane's writes
          // are fenced above and ordered before lane 0's arrival here.
          __syncwarp();
          if (lane == 0) arrive_leader(&full_bar[s]);
        }
      }
    } else {
      const int chunk = at & 7;
      const int rsub = at >> 3;
      // Converts K step `pit` from its landing slot into its operand stage
      // once the MMA has released that stage.
      auto finish = [&](uint32_t pit) -> bool {
        const int s = pit % STAGES;
        const bool freed = mbar_wait(&empty_bar[s], ((pit / STAGES) & 1) ^ 1, &abort_flag, status, 1);
        if (!__all_sync(0xffffffffu, freed)) return false;
        uint8_t *a_hi = smem + s * STAGE;
        convert_tile<SPLIT3>(land + (pit % LAND) * kABytes, a_hi, a_hi + kABytes, at);
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_bar[s]);
        return true;
      };
      Iter wi(tp, tile0, tstep, int(blockIdx.x), int(gridDim.x));
      Seg sg;
      while (ok && wi.next(sg)) {
        const int64_t m0 = int64_t(tp.nt_div.div(uint32_t(sg.tile))) * kBM;
        int rn[8], rih[8], riw[8];
        bool rvalid[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int64_t p = m0 + i * 16 + rsub;
          rvalid[i] = p < g.P;
          int ow, oh;
          pixel_nhw(tp, rvalid[i] ? p : 0, rn[i], oh, ow);
          rih[i] = oh * g.sh - g.ph;
          riw[i] = ow * g.sw - g.pw;
        }
        for (int kb = sg.kb0; kb < sg.kb1 && ok; ++kb, ++it) {
          // Gather K step `it` into landing slot it % LAND.  That slot's
          // previous step (it - LAND) was converted one iteration ago by this
          // same thread, which reads only the chunks it loads.
          uint8_t *slot = land + (it % LAND) * kABytes;
          const int k0 = kb * kBK + chunk * 4;
          const bool kval = k0 < g.K;
          const int tap = k0 / g.Cg, c = k0 - tap * g.Cg;  // 4 channels of one tap (C % 4 == 0)
          const int r = tap / g.KW, sx = tap - r * g.KW;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int ih = rih[i] + r * g.dh, iw = riw[i] + sx * g.dw;
            const bool in = kval && rvalid[i] && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
            const float *src = in ? x + ((int64_t(rn[i]) * g.H + ih) * g.W + iw) * g.C + c : x;
            cp_async16(slot + swz_off(i * 16 + rsub, chunk), src, in ? 16u : 0u);
          }
          cp_async_commit();
          if (it >= uint32_t(LAND - 1)) {
            cp_async_wait<LAND - 1>();  // step it-(LAND-1) has landed
            ok = finish(it - (LAND - 1));
          }
        }
      }
      cp_async_wait<0>();  // nothing of ours in flight past this point
      if (ok) {
        const uint32_t first = it > uint32_t(LAND - 1) ? it - (LAND - 1) : 0;
        for (uint32_t pit = first; pit < it && ok; ++pit) ok = finish(pit);
      }
    }
  } else if (warp == kEpiWarps + 4 || warp == kEpiWarps + 6) {
    // ------------------------------------------------------------ TMA producers
    // Warp 12 loads the weight panels; in the TMA A modes warp 14 loads the A
    // tile of the same stage, so the loads of one stage do not queue behind
    // each other in one issuing thread (every instruction between a stage
    // becoming free and its loads lengthens the K step).
    const bool a_role = warp == kEpiWarps + 6;
    if (lane == 0 && (!a_role || SEP_A)) {
      const uint32_t bytes = a_role ? uint32_t(kABytes) : uint32_t((SPLIT3 ? 2 : 1) * B_BYTES);
      uint32_t it = 0;
      bool ok = true;
      Iter wi(tp, tile0, tstep, int(blockIdx.x), int(gridDim.x));
      Seg sg;
      while (ok && wi.next(sg)) {
        const int64_t t = sg.tile;
        const uint32_t mt = tp.nt_div.div(uint32_t(t));  // tile row, column (tiles < 2^31)
        const int n0 = int(uint32_t(t) - mt * uint32_t(tp.n_tiles)) * BN;
        const int64_t m0 = int64_t(mt) * TILE_ROWS + rank * kBM;
        const int brow = n0 + int(rank) * BROWS;  // first weight row this CTA loads
        int bw = 0, bh = 0, bn = 0;  // im2col base of the tile's first output pixel
        if (a_role && (AMODE == 3 || AMODE == 4 || AMODE == 5)) {
          int ow, oh;
          pixel_nhw(tp, m0, bn, oh, ow);
          bw = ow * g.sw - g.pw;
          bh = oh * g.sh - g.ph;
        }
        // AMODE 3 position of K step kb (C % 32 == 0: one filter tap per K
        // step), AMODE 5 position of its first 16-channel half, advanced
        // incrementally so no division sits between the stage becoming free
        // and the loads (two divisions per K step there cost the fp32 first
        // convs 13 % on B200).
        int c0 = 0, sx = 0, r = 0;
        if (a_role && (AMODE == 3 || AMODE == 5)) {
          const int k0 = sg.kb0 * kBK, tap = k0 / g.C;
          c0 = k0 - tap * g.C;
          r = tap / g.KW;
          sx = tap - r * g.KW;
        }
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint16_t woff = uint16_t(sx * g.dw), hoff = uint16_t(r * g.dh);
          ok = wait_any(&empty_bar[s], ((it / STAGES) & 1) ^ 1, 2);
          if (!ok) break;
          uint8_t *a_hi = smem + s * STAGE;
          uint8_t *b_hi = a_hi + B_OFF;
          mbar_arrive_expect_tx(&raw_bar[s], bytes);
          if (!a_role) {
            tma_load_2d(b_hi, &wmap, kb * kBK, brow, &raw_bar[s]);
            if (SPLIT3) tma_load_2d(b_hi + B_BYTES, &wmap, kb * kBK, tp.Npad + brow, &raw_bar[s]);
            continue;
          }
          if (AMODE == 2) tma_load_2d(a_hi, &amap, kb * kBK, int(m0), &raw_bar[s]);
          if (AMODE == 3) {
            tma_load_im2col_4d(a_hi, &amap, c0, bw, bh, bn, woff, hoff, &raw_bar[s]);
            if ((c0 += kBK) == g.C) {
              c0 = 0;
              if (++sx == g.KW) {
                sx = 0;
                ++r;
              }
            }
          }
          if (AMODE == 5) {
            // C % 16 == 0 (16 for space-to-depth inputs): each K step is two
            // 16-channel halves, k = 32 kb + 16 j, each a 128 pixel x 64 byte
            // im2col column of filter tap k / C at channel k % C in its own
            // 64-byte-swizzled half of the A tile; a half past the filter
            // reads an image past the batch (zeros).
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const bool real = r < g.KH;
              tma_load_im2col_4d(a_hi + j * (kABytes / 2), &amap, real ? c0 : 0, bw, bh, real ? bn : g.N,
                                 uint16_t(real ? sx * g.dw : 0), uint16_t(real ? r * g.dh : 0), &raw_bar[s]);
              if ((c0 += 16) == g.C) {
                c0 = 0;
                if (++sx == g.KW) {
                  sx = 0;
                  ++r;
                }
              }
            }
          }
          if (AMODE == 4) {
            // C == 4: eight taps per K step, one 128 pixel x 16 byte column
            // each; taps past the filter read an image past the batch (zeros).
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              const int tap = kb * 8 + j;
              const bool real = tap < g.KH * g.KW;
              const int r = real ? tap / g.KW : 0, sx = real ? tap - r * g.KW : 0;
              tma_load_im2col_4d(a_hi + j * 2048, &amap, 0, bw, bh, real ? bn : g.N, uint16_t(sx * g.dw),
                                 uint16_t(r * g.dh), &raw_bar[s]);
            }
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    // (in a CTA pair only the leader issues; the peer's warp just frees TMEM)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) |
                                 (uint32_t(TILE_ROWS >> 4) << 24);
      // The CTA's K steps (all its tiles and stream-K segments) as runs of
      // plain steps between accumulator hand-offs, with the stage, segment
      // and group positions kept as counters: measured with in-kernel clock
      // traces, every instruction the issuing thread executes between MMA
      // batches leaves the tensor pipe idle, so the inner loop holds only
      // the barrier test, the MMAs and the stage release.
      // Segment lengths only: whole tiles (nk steps), then this CTA's
      // stream-K share cut at tile boundaries (32-bit: units < 2^31).
      const Iter wi(tp, tile0, tstep, int(blockIdx.x), int(gridDim.x));
      const uint32_t total = wi.total_steps();
      const uint32_t nk = uint32_t(tp.num_kb);
      uint32_t dp_left = total - uint32_t(wi.u1 - wi.u0);  // steps of whole tiles
      uint32_t u = uint32_t(wi.u0);
      const uint32_t uend = uint32_t(wi.u1);
      int seg_left = 0;  // K steps left in the current segment
      uint32_t gi = 0;            // accumulator hand-offs issued (one per K group)
      uint32_t ab = 0, abph = 0;  // accumulator buffer and its phase parity
      int gk = 0;              // K step within its group
      int s = 0;               // stage
      uint32_t ph = 0;         // stage phase parity
      // Waits of this thread test the barrier first (one instruction when
      // the phase completed long ago, the common case); a pair's barriers
      // take the cluster-scope acquire.
      auto wait_fast = [&](uint64_t *bar, uint32_t parity, int code) {
        return PAIR ? mbar_wait_cluster(bar, parity, &abort_flag, status, code)
                    : mbar_wait_fast(bar, parity, &abort_flag, status, code);
      };
      // Stage 0's operand descriptors.  AMODE 4 A tiles are unswizzled
      // 4-channel columns: core matrices of 8 pixels x 16 bytes, 2 KB apart
      // along K, 128 B apart along M; AMODE 5 A tiles are two 64-byte-swizzled
      // halves.
      auto a_base_desc = [&](const uint8_t *p) -> uint64_t {
        return AMODE == 4 ? smem_desc_noswz(p, 2048, 128) : AMODE == 5 ? smem_desc_sw64(p) : smem_desc(p);
      };
      const uint64_t dah0 = a_base_desc(smem), dal0 = a_base_desc(smem + kABytes);
      const uint64_t dbh0 = smem_desc(smem + B_OFF), dbl0 = smem_desc(smem + B_OFF + B_BYTES);
      bool ok = true;
      for (uint32_t it = 0; ok && it < total;) {
        if (seg_left == 0) {
          if (dp_left > 0) {
            seg_left = int(nk);
            dp_left -= nk;
          } else {
            const uint32_t r = nk - u % nk;
            seg_left = int(r < uend - u ? r : uend - u);
            u += uint32_t(seg_left);
          }
        }
        if (gk == 0) {
          if (!wait_fast(&acce_bar[ab], abph ^ 1, 7)) break;
          tc_fence_after();
        }
        const uint32_t dtm = tmem + ab * uint32_t(BN);
        // A run of K steps up to the next hand-off (end of the K group or of
        // the segment): nothing but waits, MMAs and stage releases.
        const int run = min(tp.group - gk, seg_left);
        for (int r = 0; r < run; ++r) {
          // B (and, in AMODE 2/3/4, A) lands by TMA on raw_bar; a converted
          // (or, in a pair, relayed) stage is signalled on full_bar, after
          // the A warps saw raw_bar themselves.  (AMODE 1: the A warps gather
          // A and do not see raw_bar, so both are waited on here.)
          // This stage's descriptors: stage 0's plus the stage offset (the
          // 14-bit address field is linear in the shared-memory address),
          // computed before the waits so nothing but the fence sits between
          // the stage becoming ready and its MMAs.
          const uint64_t soff = uint64_t(s) * uint64_t(STAGE >> 4);
          const uint64_t dbh = dbh0 + soff, dbl = dbl0 + soff, dah = dah0 + soff, dal = dal0 + soff;
          if (!(AMODE != 1 && RELAY) && !mbar_wait_fast(&raw_bar[s], ph, &abort_flag, status, 3)) {
            ok = false;
            break;
          }
          if (RELAY && !wait_fast(&full_bar[s], ph, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int gstep = gk + r;  // the group's first K step overwrites the accumulator
          // Operand descriptors of K slice kk (8 tf32 = 32 bytes along K).
          // AMODE 4: two 2 KB core-matrix columns per slice; AMODE 5: slices
          // 0-1 in the first 64-byte-swizzled half, 2-3 in the second.
          auto a_desc = [&](uint64_t d, int kk) -> uint64_t {
            return AMODE == 5   ? d + uint64_t((kk >> 1) * (kABytes / 2 / 16) + (kk & 1) * 2)
                   : AMODE == 4 ? d + (uint64_t(kk * 4096) >> 4)
                                : d + (uint64_t(kk * 32) >> 4);
          };
          // 3xTF32 issues the step's 12 MMAs pass by pass (A_lo*B_hi over the
          // four K slices, then A_hi*B_lo, then A_hi*B_hi), so consecutive
          // MMAs read different K slices.  Measured with a probe kernel on
          // the B200 (148 CTAs, one issuing thread each): 1259 cycles per
          // step when the three MMAs of one slice are issued back to back,
          // 937 cycles pass by pass (768 ideal).
#pragma unroll
          for (int pass = 0; pass < (SPLIT3 ? 3 : 1); ++pass) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bstep = uint64_t(kk * 32) >> 4;
              const uint64_t db = (SPLIT3 && pass == 1 ? dbl : dbh) + bstep;
              const uint32_t acc = (pass | gstep | kk) ? 1u : 0u;
              if (SPLIT3 && pass == 0 && ALO) {
                // A_lo from TMEM: slot s, columns kk*8.. (one 32-bit column per K element).
                mma_tf32_ta(dtm, tmem + uint32_t(Acc::alo_col + s * 32 + kk * 8), db, idesc, acc);
              } else {
                const uint64_t da = SPLIT3 && pass == 0 ? a_desc(dal, kk) : a_desc(dah, kk);
                if (PAIR)
                  mma_tf32_pair(dtm, da, db, idesc, acc);
                else
                  mma_tf32(dtm, da, db, idesc, acc);
              }
            }
          }
          if (PAIR)
            mma_commit_pair(&empty_bar[s]);  // frees the stage in both CTAs
          else
            mma_commit(&empty_bar[s]);
          s = s + 1 == STAGES ? 0 : s + 1;
          ph ^= s == 0 ? 1u : 0u;
        }
        if (!ok) break;
        it += uint32_t(run);
        gk += run;
        seg_left -= run;
        if (gk == tp.group || seg_left == 0) {
          if (PAIR)
            mma_commit_pair(&accf_bar[ab]);
          else
            mma_commit(&accf_bar[ab]);
          ++gi;
          gk = 0;
          if (++ab == uint32_t(NBUF)) {
            ab = 0;
            abph ^= 1u;
          }
        }
      }
      // Every issued MMA must finish before TMEM is freed (also on abort):
      // a bounded wait on the last accumulator hand-off.
      if (gi > 0) {
        const int last = int((gi - 1) % NBUF);
        const long long t0 = clock64();
        while (!mbar_try_wait(&accf_bar[last], ((gi - 1) / NBUF) & 1) && clock64() - t0 < kWaitCycles) {
        }
      }
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync();  // the leader's MMAs read the peer's shared memory until here
  else
    __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- split-K
// Finishes a split-K launch (sk_park_all): every CTA parked the partial sums
// of its K range of one or two tiles in its two workspace slots
// ([chunk][4-column group][row] float4s).  Per output element the tile's
// segments are added in segment order (CTA order, so the result does not
// depend on which CTA finished first), then bias, residual and activation
// are applied as in the conv epilogue: y = act((sum + b) + r).  One thread
// per (tile row, 4 output channels); consecutive threads take consecutive
// rows, so the workspace reads are coalesced 16-byte loads.
template <int BN>
__global__ void __launch_bounds__(256) conv_tc_reduce_kernel(const float4 *__restrict__ ws,
                                                             const float *__restrict__ bias,
                                                             const float *__restrict__ res, float *__restrict__ y,
                                                             TcParams tp) {
  pdl_launch_dependents();
  pdl_wait();  // the conv launch's partials are complete and visible
  const ConvGeo &g = tp.g;
  // 32-bit index arithmetic with multiply-shift divisions (split-K runs only
  // for a few tiles: the host keeps every product below 2^31).
  const uint32_t U = uint32_t(tp.sk_units), G = uint32_t(tp.sk_ctas);
  const uint32_t nk = uint32_t(tp.num_kb), n_tiles = uint32_t(tp.n_tiles);
  constexpr uint32_t kGroups = BN / 4;
  const uint32_t total = uint32_t(tp.tiles) * kBM * kGroups;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t row = i % kBM;
    const uint32_t rest = i / kBM;
    const uint32_t cg = rest % kGroups;
    const uint32_t tt = rest / kGroups;
    const uint32_t mt = tp.nt_div.div(tt);
    const int64_t p = int64_t(mt) * kBM + row;
    const int c0 = int(tt - mt * n_tiles) * BN + int(cg) * 4;
    if (p >= g.P || c0 >= g.M) continue;
    // CTAs whose shares hold the tile's first and last K steps (the
    // WorkIter owner / start arithmetic).
    const uint32_t v0 = tt * nk, v1 = v0 + nk - 1;
    const uint32_t blo = tp.u_div.div((v0 + 1) * G - 1), bhi = tp.u_div.div((v1 + 1) * G - 1);
    const uint32_t idx = cg * 128 + row;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    // Sixteen segments' loads in flight at a time, added in segment order.
    for (uint32_t j0 = blo; j0 <= bhi; j0 += 16) {
      float4 f[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t j = j0 + k;
        const uint32_t slot = tp.g_div.div(j * U) >= v0 ? 0 : 1;
        f[k] = j <= bhi ? __ldcg(&ws[size_t(j * 2 + slot) * (BN * 32) + idx]) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        if (j0 + k <= bhi) {
          a.x += f[k].x;
          a.y += f[k].y;
          a.z += f[k].z;
          a.w += f[k].w;
        }
      }
    }
    int n, oh, ow;
    pixel_nhw(tp, p, n, oh, ow);
    const int64_t ybase = int64_t(n) * g.ys[0] + int64_t(oh) * g.ys[2] + int64_t(ow) * g.ys[3];
    const int64_t rbase = int64_t(n) * g.rs[0] + int64_t(oh) * g.rs[2] + int64_t(ow) * g.rs[3];
    float v[4] = {a.x, a.y, a.z, a.w};
    const int cn = g.M - c0 < 4 ? g.M - c0 : 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (e < cn) {
        const int c = c0 + e;
        if (g.has_bias) v[e] += __ldg(bias + c);
        if (g.has_res) v[e] += __ldg(res + rbase + int64_t(c) * g.rs[1]);
        v[e] = apply_act(v[e], g.act);
      }
    }
    if (cn == 4 && g.ys[1] == 1 && ((ybase + c0) & 3) == 0) {
      *reinterpret_cast<float4 *>(y + ybase + c0) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < cn) y[ybase + int64_t(c0 + e) * g.ys[1]] = v[e];
    }
  }
}

// ---------------------------------------------------------------- weights
// [part][Npad][Kpad] with k = (r*KW + s)*Cg + c over the GEMM channel count
// Cg (which may be padded above the weight's Cw); part 0 = TF32(rna) of w,
// part 1 = w - part 0 (3xTF32 only); zero padding.  w_kn: the weights are a
// [K][Cout] matrix (Gemm B with transB = 0) instead of OIHW.  packed_kw > 0:
// row-packed input (see pack_rows_kernel), k = r*32 + s*4 + c for the
// original kernel width packed_kw.  s2d_k > 0: space-to-depth input (see
// to_s2d_kernel) of a stride-2 conv with an s2d_k x s2d_k kernel and
// padding parity s2d_podd; k = tap*16 + (sh*2 + sw)*4 + c over the g.KH x
// g.KW taps (a, b) of the transformed stride-1 conv, holding the original
// tap (2a + sh - s2d_podd, 2b + sw - s2d_podd) (zero outside the kernel).
__global__ void pack_tc_kernel(float *__restrict__ dst, const float *__restrict__ w, ConvGeo g, int Cw, int Npad,
                               int Kpad, int split3, int w_kn, int packed_kw, int s2d_k, int s2d_podd) {
  const int64_t total = int64_t(Npad) * Kpad;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / Kpad), k = int(i % Kpad);
    float v = 0.f;
    if (m < g.M && k < g.K) {
      if (s2d_k > 0) {
        const int tap = k >> 4, ch = k & 15, c = ch & 3;
        const int r = 2 * (tap / g.KW) + (ch >> 3) - s2d_podd, sx = 2 * (tap % g.KW) + ((ch >> 2) & 1) - s2d_podd;
        if (c < Cw && r >= 0 && r < s2d_k && sx >= 0 && sx < s2d_k)
          v = w[((int64_t(m) * Cw + c) * s2d_k + r) * s2d_k + sx];
      } else if (packed_kw > 0) {
        const int r = k / 32, j = k % 32, s = j / 4, c = j % 4;
        if (s < packed_kw && c < Cw) v = w[((int64_t(m) * Cw + c) * g.KH + r) * packed_kw + s];
      } else {
        const int c = k % g.Cg, rs = k / g.Cg, s = rs % g.KW, r = rs / g.KW;
        if (c < Cw) v = w_kn ? w[int64_t(c) * g.M + m] : w[((int64_t(m) * Cw + c) * g.KH + r) * g.KW + s];
      }
    }
    const float hi = tf32_rna(v);
    dst[i] = hi;
    if (split3) dst[total + i] = v - hi;
  }
}

// TC_PANEL_F32X2 panel [2][npad][kpad] (k = (r*KW + s)*C + c) -> OIHW
// weights, w = part0 + part1 (exact: part1 is the fp32 remainder).
__global__ void unpack_panel_kernel(float *__restrict__ oihw, const float *__restrict__ panel, ConvGeo g, int npad,
                                    int kpad) {
  const int64_t total = int64_t(g.M) * g.K;
  const int64_t part = int64_t(npad) * kpad;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / g.K), rem = int(i % g.K);  // OIHW order: rem = (c*KH + r)*KW + s
    const int sx = rem % g.KW, r = (rem / g.KW) % g.KH, c = rem / (g.KW * g.KH);
    const int64_t k = (int64_t(r) * g.KW + sx) * g.Cg + c;
    oihw[i] = panel[int64_t(m) * kpad + k] + panel[part + int64_t(m) * kpad + k];
  }
}

// Row packing for convs with few input channels (C <= 4, 4 * KW <= 32; a
// network's first conv): dst[n][h][ow][s*4 + c] = x[n][c][h][ow*sw - pw + s]
// for s < KW and c < C, zero elsewhere (padding, and the 32 - 4*KW tail), so
// one 128-byte packed pixel holds a whole filter row for output column ow and
// the conv becomes a KH x 1 conv over the packed tensor (stride sh x 1,
// padding ph x 0).  One thread per (n, h, ow, 4-float group).
__global__ void pack_rows_kernel(float *__restrict__ dst, const float *__restrict__ x, int N, int C, int H, int W,
                                 int OW, int KW, int sw, int pw, int64_t xs0, int64_t xs1, int64_t xs2, int64_t xs3) {
  const int64_t total = int64_t(N) * H * OW * 8;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int s = int(i & 7);
    const int64_t pix = i >> 3;  // (n, h, ow)
    const int ow = int(pix % OW);
    const int h = int((pix / OW) % H);
    const int n = int(pix / (int64_t(OW) * H));
    const int iw = ow * sw - pw + s;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (s < KW && iw >= 0 && iw < W) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < C) v[c] = x[n * xs0 + c * xs1 + h * xs2 + iw * xs3];
    }
    *reinterpret_cast<float4 *>(dst + pix * 32 + s * 4) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Space-to-depth by 2 of a few-channel input (C <= 4, any 4-D strides xs)
// for a stride-2 conv: dst[n][i][j][(sh*2 + sw)*4 + c] = x[n][c][2i + sh][2j
// + sw], zero past the image and for c >= C, so the conv becomes a stride-1
// conv over 16 channels (64 bytes per pixel).  One thread per (n, i, j,
// sub-pixel): one 16-byte store.
__global__ void to_s2d_kernel(float *__restrict__ dst, const float *__restrict__ x, int N, int C, int H, int W,
                              int H2, int W2, int64_t xs0, int64_t xs1, int64_t xs2, int64_t xs3) {
  const int64_t total = int64_t(N) * H2 * W2 * 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int sub = int(i & 3);
    const int64_t pix = i >> 2;  // (n, i, j)
    const int j = int(pix % W2);
    const int ii = int((pix / W2) % H2);
    const int n = int(pix / (int64_t(W2) * H2));
    const int h = 2 * ii + (sub >> 1), w = 2 * j + (sub & 1);
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (h < H && w < W) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < C) v[c] = x[n * xs0 + c * xs1 + h * xs2 + w * xs3];
    }
    *reinterpret_cast<float4 *>(dst + pix * 16 + sub * 4) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Any 4-D fp32 view (strides xs) -> dense NHWC with C4 >= C channels
// (zero-filled); one thread per (pixel, 4-channel group), so for an NCHW
// source the loads coalesce along pixels and the stores are 16 bytes.
__global__ void to_nhwc4_kernel(float *__restrict__ dst, const float *__restrict__ x, int N, int C, int H, int W,
                                int C4, int64_t xs0, int64_t xs1, int64_t xs2, int64_t xs3) {
  const int G = C4 / 4;
  const int64_t total = int64_t(N) * H * W * G;
  const int64_t HW = int64_t(H) * W;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t pix = i % (int64_t(N) * HW);
    const int grp = int(i / (int64_t(N) * HW));
    const int w = int(pix % W);
    const int h = int((pix / W) % H);
    const int n = int(pix / HW);
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = grp * 4 + e;
      v[e] = c < C ? x[n * xs0 + c * xs1 + h * xs2 + w * xs3] : 0.f;
    }
    *reinterpret_cast<float4 *>(dst + pix * C4 + grp * 4) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Pipeline shape per (BN, split, A mode): operand stages and landing slots,
// sized so stages + landing ring + epilogue staging fit in 227 KB.
struct PipeShape {
  int stages, land;
};
// In a CTA pair each CTA holds BN/2 weight rows, so its stages are those of
// a BN/2-wide single-CTA tile.
// With A's low part in TMEM (BN = 128) a stage is [A hi][B hi][B lo], 48 KB:
// four stages (the ring takes 32 TMEM columns per stage).
constexpr PipeShape pipe_shape(int bn, bool split3, int amode, bool pair = false) {
  const int b = pair ? bn / 2 : bn;  // weight rows per CTA
  return amode != 1 ? (split3 ? (alo_tmem(bn, split3, amode, pair) ? PipeShape{b == 128 ? 4 : b == 64 ? 6 : 8, 0}
                                                                   : PipeShape{b == 256 ? 2 : b == 128 ? 3 : 4, 0})
                              : PipeShape{b == 256 ? 4 : 6, 0})
                    : (split3 ? PipeShape{b == 256 ? 1 : b == 128 ? 2 : 3, b == 128 ? 4 : 3}
                              : PipeShape{b == 256 ? 3 : 4, b == 256 ? 3 : 4});
}

size_t smem_bytes(int bn, bool split3, int amode, bool pair) {
  const PipeShape ps = pipe_shape(bn, split3, amode, pair);
  const int brows = pair ? bn / 2 : bn;
  return size_t(ps.stages) * size_t(stage_bytes(brows, split3, alo_tmem(bn, split3, amode, pair))) +
         size_t(ps.land) * kABytes + kStagingBytes + 1024;
}

// Clusters of two CTAs with this kernel's shared memory can be scheduled.
bool cluster_launch_ok(int dev) {
  int ok = 0;
  return cudaDeviceGetAttribute(&ok, cudaDevAttrClusterLaunch, dev) == cudaSuccess && ok;
}

struct TcState {
  CUtensorMap wmap, amap, ymap, rmap;
  TcParams tp;
  int bn = 128;
  bool split3 = true;
  int amode = 1;
  bool pair = false;  // 2-SM tiles (cluster of 2, cta_group::2 MMA)
  bool epi_tma = false;
  size_t smem = 0;
  int grid = 148;
  bool set_attr_only = false;  // dispatch only sets the kernel's smem attribute
  float *staged_x = nullptr;   // NHWC4 (or row-packed) copy of an input that needs relayout
  bool packed_rows = false;    // staged_x is row-packed (pack_rows_kernel)
  bool s2d = false;            // staged_x is space-to-depth by 2 (to_s2d_kernel), AMODE 5
  ConvGeo src;                 // geometry of the original input (relayout source)
  const void *amap_base = nullptr, *ymap_base = nullptr, *rmap_base = nullptr;  // pointers the maps were encoded for
  int *sk_cnt = nullptr;   // stream-K arrival counters [stream-K tiles][epilogue warps]
  size_t sk_cnt_bytes = 0;
  size_t sk_ws_bytes = 0;  // workspace the launch needs for partial tiles (two slots per CTA)
  ~TcState() {
    device_free(staged_x);
    device_free(sk_cnt);
  }
};

bool encode_a(const TcState &st, CUtensorMap *map, const void *x) {
  const ConvGeo &g = st.tp.g;
  if (st.amode == 3)
    return encode_im2col_nhwc2(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, g.N, g.H, g.W, g.C, g.KH, g.KW, g.sh, g.sw,
                               g.ph, g.pw, g.dh, g.dw, kBK, kBM);
  if (st.amode == 4)
    return encode_im2col_nhwc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, g.N, g.H, g.W, 4, g.KH, g.sh, g.ph, g.dh, 4,
                              kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st.amode == 5) {
    // 16-channel (64-byte) boxes, 64-byte swizzle; window origins from
    // (-pw, -ph) to the last output pixel's, (OW - 1) * sw - pw (and H).
    const int lower[2] = {-g.pw, -g.ph};
    const int upper[2] = {(g.OW - 1) * g.sw - g.pw - (g.W - 1), (g.OH - 1) * g.sh - g.ph - (g.H - 1)};
    return encode_im2col_corners(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, g.N, g.H, g.W, g.C, lower, upper, g.sw,
                                 g.sh, 16, kBM, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, uint64_t(g.C), uint64_t(g.P), uint64_t(g.C), kBM);
}

bool encode_y(const TcState &st, CUtensorMap *map, const void *y) {
  const ConvGeo &g = st.tp.g;
  return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, uint64_t(g.M), uint64_t(g.P), uint64_t(g.M), 32);
}

struct Maps {
  CUtensorMap a, y, r;
};

template <int BN, bool SPLIT3, int AMODE, bool EPI, bool PAIR = false>
int launch_cfg(const TcState &st, const Maps &mp, const float *x, float *y, const float *bias, const float *res,
               float *sk_ws, int *status, cudaStream_t s) {
  constexpr PipeShape ps = pipe_shape(BN, SPLIT3, AMODE, PAIR);
  auto kern = conv_tc_kernel<BN, ps.stages, ps.land, SPLIT3, AMODE, EPI, PAIR>;
  if (st.set_attr_only)
    return cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(st.smem)));
  return cuda_status(launch_kernel(kern, unsigned(st.grid), kThreads, st.smem, s, PAIR ? 2 : 1, st.wmap, mp.a, mp.y,
                                   mp.r, x, bias, res, y, st.tp, sk_ws, st.sk_cnt, status));
}

template <int BN, bool SPLIT3>
int launch_modes(const TcState &st, const Maps &mp, const float *x, float *y, const float *bias, const float *res,
                 float *w, int *status, cudaStream_t s) {
  if constexpr (BN >= 128) {
    if (st.pair) {
      if (st.epi_tma)
        return st.amode == 3 ? launch_cfg<BN, SPLIT3, 3, true, true>(st, mp, x, y, bias, res, w, status, s)
                             : launch_cfg<BN, SPLIT3, 2, true, true>(st, mp, x, y, bias, res, w, status, s);
      return st.amode == 3 ? launch_cfg<BN, SPLIT3, 3, false, true>(st, mp, x, y, bias, res, w, status, s)
                           : launch_cfg<BN, SPLIT3, 2, false, true>(st, mp, x, y, bias, res, w, status, s);
    }
  }
  if (st.epi_tma) {
    switch (st.amode) {
      case 5: return launch_cfg<BN, SPLIT3, 5, true>(st, mp, x, y, bias, res, w, status, s);
      case 4: return launch_cfg<BN, SPLIT3, 4, true>(st, mp, x, y, bias, res, w, status, s);
      case 3: return launch_cfg<BN, SPLIT3, 3, true>(st, mp, x, y, bias, res, w, status, s);
      case 2: return launch_cfg<BN, SPLIT3, 2, true>(st, mp, x, y, bias, res, w, status, s);
      default: return launch_cfg<BN, SPLIT3, 1, true>(st, mp, x, y, bias, res, w, status, s);
    }
  }
  switch (st.amode) {
    case 5: return launch_cfg<BN, SPLIT3, 5, false>(st, mp, x, y, bias, res, w, status, s);
    case 4: return launch_cfg<BN, SPLIT3, 4, false>(st, mp, x, y, bias, res, w, status, s);
    case 3: return launch_cfg<BN, SPLIT3, 3, false>(st, mp, x, y, bias, res, w, status, s);
    case 2: return launch_cfg<BN, SPLIT3, 2, false>(st, mp, x, y, bias, res, w, status, s);
    default: return launch_cfg<BN, SPLIT3, 1, false>(st, mp, x, y, bias, res, w, status, s);
  }
}

}  // namespace

// Eligible: fp32 in and out, group 1, 3xTF32 or TF32 math.  Narrow outputs
// (Cout < 32, e.g. a detector's 4-channel box head) run in one 32-column
// tile with direct stores.
int conv_tc_prepare_ex(ConvPlan &p, const void *w_raw_dev, const void *x_dev, const void *y_dev, bool w_kn,
                       cudaStream_t s, const void *r_dev, const float *panel, int panel_npad) {
  const ConvGeo &g0 = p.g;
  if ((p.mode != kConvF32 && p.mode != kConvF32ToI8) || g0.groups != 1 || g0.M < 1) return SPKV2_ERR_UNSUPPORTED;
  if (p.math != SPKV2_CUDA_MATH_3XTF32 && p.math != SPKV2_CUDA_MATH_TF32) return SPKV2_ERR_UNSUPPORTED;
  if (!encode_fn()) return SPKV2_ERR_UNSUPPORTED;
  TcState *st = new TcState();
  memset(&st->wmap, 0, sizeof(st->wmap));
  memset(&st->amap, 0, sizeof(st->amap));
  memset(&st->ymap, 0, sizeof(st->ymap));
  memset(&st->rmap, 0, sizeof(st->rmap));
  st->src = g0;
  ConvGeo g = g0;
  const bool nhwc_in = g.xs[1] == 1 && g.xs[3] == g.C && g.xs[2] == int64_t(g.W) * g.C;
  const bool aligned_in = reinterpret_cast<uintptr_t>(x_dev) % 16 == 0;
  // Row packing pays for wide filters (a 7x7 first conv: ResNet-50 INT8 bs256
  // 55.5k img/s packed vs 46.2k re-laid out); a 3x3 first conv is faster
  // re-laid out to 4 channels and read by 4-channel im2col TMA (detector bs64
  // 4215 vs 4083 img/s).  The packed row holds KW adjacent pixels, so only
  // for convs without horizontal dilation.
  const bool row_pack = !(nhwc_in && g.C % 4 == 0 && aligned_in) && g.C <= 4 && 4 * g.KW <= 32 && g.KW >= 5 &&
                        g.dw == 1 && encode_im2col_fn() && !getenv("SPKV2_TC_NO_ROWPACK");
  // Space-to-depth for stride-2 few-channel convs (a network's first conv):
  // pixel (i, j) of the staged input holds the 2 x 2 input pixels (2i.., 2j..)
  // x 4 channels, so the conv becomes a stride-1 k' x k' conv over 16
  // channels, k' = (k - 1 + p % 2) / 2 + 1, padding ceil(p / 2) at the top and
  // left, read by two-tap im2col TMA (64 bytes per tap).  The staged input is
  // the size of a 4-channel copy (no per-tap inflation as in row packing).
  const bool s2d = g.C <= 4 && g.sh == 2 && g.sw == 2 && g.KH == g.KW && g.ph == g.pw && g.dh == 1 && g.dw == 1 &&
                   g.KH >= 2 && encode_im2col_fn() && !getenv("SPKV2_TC_NO_S2D");
  if (s2d) {
    const int H2 = int(ceil_div(g.H, 2)), W2 = int(ceil_div(g.W, 2));
    const int k2 = (g.KH - 1 + (g.ph & 1)) / 2 + 1, pad = (g.ph + 1) / 2;
    st->staged_x = static_cast<float *>(device_alloc(size_t(g.N) * H2 * W2 * 16 * sizeof(float) + 256));
    if (!st->staged_x) {
      delete st;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    st->s2d = true;
    g.C = g.Cg = 16;
    g.H = H2;
    g.W = W2;
    g.KH = g.KW = k2;
    g.sh = g.sw = 1;
    g.ph = g.pw = pad;
    g.K = k2 * k2 * 16;
    g.xs[0] = int64_t(H2) * W2 * 16;
    g.xs[1] = 1;
    g.xs[2] = int64_t(W2) * 16;
    g.xs[3] = 16;
    x_dev = st->staged_x;
    p.launches = 2;
  } else if (row_pack) {
    // Few-channel input: pack each filter row's KW x 4 channels into one
    // 128-byte pixel; the GEMM side becomes a KH x 1 conv over 32 channels.
    st->staged_x = static_cast<float *>(device_alloc(size_t(g.N) * g.H * g.OW * 32 * sizeof(float) + 256));
    if (!st->staged_x) {
      delete st;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    st->packed_rows = true;
    g.C = g.Cg = 32;
    g.W = g.OW;
    g.KW = 1;
    g.sw = 1;
    g.pw = 0;
    g.dw = 1;
    g.K = g.KH * 32;
    g.xs[0] = int64_t(g.H) * g.W * 32;
    g.xs[1] = 1;
    g.xs[2] = int64_t(g.W) * 32;
    g.xs[3] = 32;
    x_dev = st->staged_x;
    p.launches = 2;
  } else if (!(nhwc_in && g.C % 4 == 0 && aligned_in)) {
    // Re-lay the input out as dense NHWC with C rounded up to 4.
    const int C4 = int(ceil_div(g.C, 4) * 4);
    st->staged_x = static_cast<float *>(device_alloc(size_t(g.N) * g.H * g.W * C4 * sizeof(float) + 256));
    if (!st->staged_x) {
      delete st;
      return SPKV2_ERR_DEVICE_ALLOC;
    }
    g.C = g.Cg = C4;
    g.K = g.KH * g.KW * C4;
    g.xs[0] = int64_t(g.H) * g.W * C4;
    g.xs[1] = 1;
    g.xs[2] = int64_t(g.W) * C4;
    g.xs[3] = C4;
    x_dev = st->staged_x;
    p.launches = 2;
  }
  if (panel && (st->packed_rows || st->s2d || g.Cg != g0.Cg || w_kn)) {
    // The stored panel's K order is over the original channels.
    delete st;
    return SPKV2_ERR_UNSUPPORTED;
  }
  st->split3 = p.math == SPKV2_CUDA_MATH_3XTF32;
  // A operand: tiled TMA for 1x1 stride-1 convs, im2col TMA for other
  // square convs with C % 32 == 0, cp.async gathers otherwise.  The
  // one-column im2col maps (AMODE 3, 4) walk window origins from (-pw, -ph)
  // over the extent that bottom / right padding equal to the top / left
  // padding gives, and the row map (AMODE 2) assumes the output extent is
  // the input's: a conv whose output extent says otherwise (asymmetric
  // padding) takes the two-column map, whose corners follow the output
  // extent, or the gathers.
  const bool square = g.KH == g.KW && g.sh == g.sw && g.ph == g.pw && g.dh == g.dw;
  const int span_w = g.W + 2 * g.pw - (g.KW - 1) * g.dw - 1, span_h = g.H + 2 * g.ph - (g.KH - 1) * g.dh - 1;
  const bool sym_extent = span_w >= 0 && span_h >= 0 && g.OW == span_w / g.sw + 1 && g.OH == span_h / g.sh + 1;
  const bool im2col_ok = encode_im2col_fn() && !getenv("SPKV2_TC_NO_IM2COL");
  if (st->s2d)
    st->amode = 5;
  else if (g.C % 4 == 0 && g.C >= 32 && g.KH == 1 && g.KW == 1 && g.sh == 1 && g.sw == 1 && g.ph == 0 && g.pw == 0 &&
           g.OH == g.H && g.OW == g.W)
    st->amode = 2;  // [P][C] rows; a last K step past C reads zeros (outside the tensor)
  else if (g.C % 32 == 0 && (square || st->packed_rows) && sym_extent && im2col_ok)
    st->amode = 3;
  else if (g.C % 16 == 0 && im2col_ok)
    st->amode = 5;  // C % 16 == 0: two 64-byte (16-channel) im2col columns per K step
  else if (g.C == 4 && square && sym_extent && im2col_ok)
    st->amode = 4;  // 4-channel (re-laid-out) inputs: eight 16-byte im2col columns per K step
  else
    st->amode = 1;
  // Tile width from the wave / MMA-rate model.  3xTF32 stays at <= 128: two
  // partial buffers plus the promoted sums take 3 x BN TMEM columns, and TMEM
  // has 512.
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int bn = pick_block_n(g.P, g.M, ceil_div(g.K, kBK), sms, 32, st->split3 ? 128 : 256);
  if (const char *e = getenv("SPKV2_TC_BN")) {
    const int v = atoi(e);
    if ((v == 32 || v == 64 || v == 128 || v == 256) && v <= std::max(32, int(ceil_div(g.M, 32) * 32))) bn = v;
  }
  if (st->split3 && bn == 256) bn = 128;
  // 2-SM tiles (opt-in, SPKV2_TC_PAIR=1) for TMA-fed convs wide enough to
  // fill the pairs: each CTA streams half of the weight panel (TF32 pairs use
  // N = 256 when Cout >= 256).  Measured on B200 they are slower than single
  // tiles at ResNet shapes: the stage hand-off from the peer CTA to the
  // leader lengthens each K step more than the halved weight traffic saves.
  {
    const char *e = getenv("SPKV2_TC_PAIR");
    const bool allow = e && e[0] == '1';
    const int pbn = st->split3 ? 128 : (g.M >= 256 ? 256 : 128);
    if (allow && (st->amode == 2 || st->amode == 3) && g.M >= 128 && cluster_launch_ok(dev)) {
      st->pair = true;
      bn = pbn;
    }
  }
  // Split-K over every tile (small batches): when the tiles fill at most
  // half of the SMs, G CTAs (up to one per SM, at least two K steps each)
  // take even shares of all tiles' K steps, park their partial sums, and
  // conv_tc_reduce_kernel adds each tile's segments in order and finishes
  // it, in parallel over the whole tile instead of one CTA per tile.  The
  // widest tile that Cout fills (fewer partial sums to add).
  int ska_g = 0;
  if (!st->pair && p.mode == kConvF32 && !getenv("SPKV2_TC_NO_STREAMK") && !getenv("SPKV2_TC_NO_SPLITK")) {
    const int wide = st->split3 ? 128 : 256;
    int bw = 32;
    while (bw < wide && bw < g.M) bw *= 2;
    const int64_t t = ceil_div(g.P, kBM) * ceil_div(g.M, bw);
    const int64_t units = t * ceil_div(g.K, kBK);
    // At least `min_steps` K steps per CTA (SPKV2_TC_SPLITK_MIN_STEPS, default
    // 4): fewer CTAs mean fewer partial sums to add up.  Measured on
    // ResNet-101 bs1 (p50 through spkv2_run): 2 -> 1.61 ms, 4 -> 1.57 ms,
    // 8 -> 1.60 ms; without split-K 1.67 ms.
    int min_steps = 4;
    if (const char *e = getenv("SPKV2_TC_SPLITK_MIN_STEPS")) min_steps = std::max(1, atoi(e));
    const int64_t gsk = std::min<int64_t>(sms, units / min_steps);
    // (units * G < 2^31: the reduce kernel's 32-bit index arithmetic.)
    if (2 * t <= sms && gsk >= 2 * t && units * sms < (int64_t(1) << 31)) {
      bn = bw;
      ska_g = int(gsk);
    }
  }
  st->bn = bn;
  const bool nhwc_out = g.ys[1] == 1 && g.ys[3] == g.M && g.ys[2] == int64_t(g.OW) * g.M;
  st->epi_tma = p.mode == kConvF32 && nhwc_out && g.M % 4 == 0 && g.M >= 32 &&
                reinterpret_cast<uintptr_t>(y_dev) % 16 == 0;
  TcParams &tp = st->tp;
  tp.g = g;
  tp.Kpad = int(ceil_div(g.K, kBK) * kBK);
  tp.Npad = panel ? panel_npad : int(ceil_div(g.M, bn) * bn);  // rows per panel part
  tp.num_kb = tp.Kpad / kBK;
  tp.n_tiles = int(ceil_div(g.M, bn));
  tp.tiles = ceil_div(g.P, st->pair ? 2 * kBM : kBM) * tp.n_tiles;  // pair tiles have 256 rows
  // 3xTF32 promotes every `group` K steps; TF32 hands off once per tile.
  tp.out_i8 = p.mode == kConvF32ToI8 ? 1 : 0;
  const bool nhwc_res = g.has_res && g.rs[1] == 1 && g.rs[3] == g.M && g.rs[2] == int64_t(g.OW) * g.M;
  tp.res_tma = (st->epi_tma && nhwc_res && reinterpret_cast<uintptr_t>(r_dev) % 16 == 0) ? 1 : 0;
  tp.group = tp.num_kb;
  tp.p32 = g.P < (int64_t(1) << 31) ? 1 : 0;
  tp.ow_div = FastDiv(uint32_t(g.OW));
  tp.oh_div = FastDiv(uint32_t(g.OH));
  if (st->split3) {
    // Promotion interval: each add of a group into the running sums costs
    // the epilogue warps TMEM round trips, and the truncating accumulation
    // inside a group grows with its length.  Measured on ResNet-101 (B200,
    // logits of O(10-100)): the worst logit uses 16 / 23 / 38 / 114 % of its
    // element-wise fp32 tolerance (1e-3 + 1e-4 |ref|) at intervals 4 / 8 /
    // 16 / whole K, for 8.80k / 9.24k / 9.38k / 9.50k img/s at batch 64;
    // 8 keeps a 4x margin.
    tp.group = 8;
    if (const char *e = getenv("SPKV2_TC_PROMOTE_GROUP")) tp.group = std::max(1, atoi(e));
  }
  st->grid = st->pair ? 2 * int(std::min<int64_t>(tp.tiles, sms / 2)) : int(std::min<int64_t>(tp.tiles, sms));
  // A pre-packed panel always holds both parts (TF32 reads part 0 only).
  const int parts = panel ? 2 : st->split3 ? 2 : 1;
  float *wtc = panel ? const_cast<float *>(panel)
                     : static_cast<float *>(device_alloc(size_t(parts) * tp.Npad * tp.Kpad * sizeof(float)));
  if (!wtc) {
    delete st;
    return SPKV2_ERR_DEVICE_ALLOC;
  }
  if (!panel)
    pack_tc_kernel<<<grid_for(int64_t(tp.Npad) * tp.Kpad, 256), 256, 0, s>>>(
        wtc, static_cast<const float *>(w_raw_dev), g, g0.Cg, tp.Npad, tp.Kpad, st->split3 ? 1 : 0, w_kn ? 1 : 0,
        st->packed_rows ? g0.KW : 0, st->s2d ? g0.KH : 0, g0.ph & 1);
  int rc = cuda_status(cudaGetLastError());
  bool ok = rc == 0 && encode_2d(&st->wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, wtc, uint64_t(tp.Kpad),
                                 uint64_t(parts) * tp.Npad, uint64_t(tp.Kpad), uint32_t(st->pair ? bn / 2 : bn));
  if (ok && st->amode != 1) ok = encode_a(*st, &st->amap, x_dev);
  if (ok && st->epi_tma) ok = encode_y(*st, &st->ymap, y_dev);
  if (ok && tp.res_tma) ok = encode_y(*st, &st->rmap, r_dev);  // same geometry as the output
  // Stream-K for the tiles past the last full wave when that shortens the
  // critical path (each CTA gets an even share of their K steps; a tile
  // split across CTAs is finished by the last epilogue warp to arrive).
  // 3xTF32 only: measured on B200, TF32 main loops are short enough that
  // writing and re-reading the partial tiles costs more than it saves
  // (ResNet-101 bs64 TF32 with the same model applied: 15.2k -> 13.5k img/s).
  tp.dp_tiles = tp.tiles;
  tp.sk_units = 0;
  tp.sk_ctas = sms;
  tp.sk_park_all = 0;
  if (ok && ska_g > 0) {
    tp.dp_tiles = 0;
    tp.sk_units = tp.tiles * tp.num_kb;
    tp.sk_ctas = ska_g;
    tp.sk_park_all = 1;
    st->grid = ska_g;
    st->sk_ws_bytes = size_t(ska_g) * 2 * size_t(bn) * kBM * sizeof(float);
    p.launches += 1;  // conv_tc_reduce_kernel
  } else if (ok && st->split3 && !st->pair && !getenv("SPKV2_TC_NO_STREAMK")) {
    // Critical path in K steps: whole rounds, then the CTA's share of the
    // tail, then the fix-up, which adds up the tile's segments (about
    // Gs / tail + 1 of them) one L2 round trip per segment and 32-column
    // chunk (about a K step per segment), plus a fixed cost for parking the
    // partial and counting the arrival.  The number of CTAs Gs that share
    // the tail trades the share against the segment count: a few tiles over
    // all 148 SMs (batch 1) would leave each tile ~40 segments to add up.
    const int64_t nk = tp.num_kb, rounds = tp.tiles / sms, tail = tp.tiles % sms;
    const double dp_steps = double(rounds + (tail ? 1 : 0)) * nk;
    constexpr double kFixPerSeg = 1.0, kFixBase = 2.0;
    double best = 0.9 * dp_steps;
    int best_g = 0;
    for (int64_t segs = 2; tail > 0 && segs <= 64; ++segs) {
      const int64_t gs = std::min<int64_t>(sms, tail * segs);
      const double share = ceil(double(tail * nk) / double(gs));
      const double nseg = ceil(double(gs) / double(tail)) + 1.0;
      const double cost = double(rounds) * nk + share + kFixBase + kFixPerSeg * nseg;
      if (share >= 1 && cost < best) {
        best = cost;
        best_g = int(gs);
      }
      if (gs == sms) break;
    }
    if (const char *e = getenv("SPKV2_TC_SK_CTAS")) best_g = tail > 0 ? std::min(sms, std::max(1, atoi(e))) : 0;
    if (best_g > 0 && tail * nk * sms < (int64_t(1) << 31)) {  // 32-bit schedule arithmetic
      tp.dp_tiles = rounds * sms;
      tp.sk_units = tail * nk;
      tp.sk_ctas = best_g;
      st->grid = sms;
      st->sk_cnt_bytes = size_t(tail) * kEpiWarps * sizeof(int);
      st->sk_cnt = static_cast<int *>(device_alloc(st->sk_cnt_bytes));
      ok = st->sk_cnt && cudaMemsetAsync(st->sk_cnt, 0, st->sk_cnt_bytes, s) == cudaSuccess;
      st->sk_ws_bytes = size_t(sms) * 2 * size_t(bn) * kBM * sizeof(float);
    }
  }
  tp.nk_div = FastDiv(uint32_t(tp.num_kb));
  tp.nt_div = FastDiv(uint32_t(tp.n_tiles));
  if (tp.tiles >= (int64_t(1) << 31)) ok = false;  // 32-bit tile arithmetic
  if (tp.sk_units) {
    tp.u_div = FastDiv(uint32_t(tp.sk_units));
    tp.g_div = FastDiv(uint32_t(tp.sk_ctas));
  }
  st->rmap_base = r_dev;
  st->amap_base = x_dev;
  st->ymap_base = y_dev;
  if (!ok) {
    if (!panel) device_free(wtc);
    delete st;
    return rc ? rc : SPKV2_ERR_UNSUPPORTED;
  }
  st->smem = smem_bytes(bn, st->split3, st->amode, st->pair);
  p.w_tc = wtc;
  p.w_tc_borrowed = panel != nullptr;
  p.tc_state = st;
  p.tc_block_n = bn;
  p.tc_kpad = tp.Kpad;
  st->set_attr_only = true;
  rc = conv_tc_launch(p, nullptr, nullptr, nullptr, nullptr, s, nullptr);
  st->set_attr_only = false;
  if (rc) return rc;
  p.variant = std::string(st->split3 ? "tc_3xtf32" : "tc_tf32") + (st->pair ? "_pair" : "") +
              (tp.sk_park_all ? "_splitk" : tp.sk_units ? "_sk" : "") + "_bn" + std::to_string(bn) +
              (st->amode == 5   ? "_im2col2tap"
               : st->amode == 4 ? "_im2col4"
               : st->amode == 3 ? "_im2col"
               : st->amode == 2 ? "_tma"
                                : "_cpasync") +
              (st->epi_tma ? "_tmastore" : "") +
              (st->s2d ? "_s2d" : st->packed_rows ? "_rowpack" : st->staged_x ? "_relayout" : "") +
              (panel ? "_prepacked" : "");
  return 0;
}

int conv_tc_prepare(ConvPlan &p, const void *w_raw_dev, const void *x_dev, const void *y_dev, const void *r_dev,
                    cudaStream_t s) {
  return conv_tc_prepare_ex(p, w_raw_dev, x_dev, y_dev, false, s, r_dev);
}

int conv_unpack_panel(float *oihw, const float *panel, const ConvGeo &g, int npad, int kpad, cudaStream_t s) {
  unpack_panel_kernel<<<grid_for(int64_t(g.M) * g.K, 256), 256, 0, s>>>(oihw, panel, g, npad, kpad);
  return cuda_status(cudaGetLastError());
}

void conv_tc_release(void *state) { delete static_cast<TcState *>(state); }

size_t conv_tc_sk_workspace_bytes(const ConvPlan &p) {
  return p.tc_state ? static_cast<const TcState *>(p.tc_state)->sk_ws_bytes : 0;
}

void *conv_tc_sk_counters(const ConvPlan &p, size_t *bytes) {
  const TcState *st = static_cast<const TcState *>(p.tc_state);
  *bytes = st ? st->sk_cnt_bytes : 0;
  return st ? st->sk_cnt : nullptr;
}

int conv_tc_launch(const ConvPlan &p, const void *x, void *y, const void *res, int *status, cudaStream_t s,
                   float *sk_ws) {
  const TcState &st = *static_cast<const TcState *>(p.tc_state);
  if (st.sk_ws_bytes && !sk_ws && !st.set_attr_only) return SPKV2_ERR_UNSUPPORTED;  // stream-K needs its workspace
  const float *xf = static_cast<const float *>(x);
  if (st.staged_x && !st.set_attr_only) {
    const ConvGeo &o = st.src;
    if (st.s2d) {
      const ConvGeo &t = st.tp.g;
      const int64_t total = int64_t(o.N) * t.H * t.W * 4;
      to_s2d_kernel<<<grid_for(total, 256), 256, 0, s>>>(st.staged_x, xf, o.N, o.C, o.H, o.W, t.H, t.W, o.xs[0],
                                                         o.xs[1], o.xs[2], o.xs[3]);
    } else if (st.packed_rows) {
      const int64_t total = int64_t(o.N) * o.H * o.OW * 8;
      pack_rows_kernel<<<grid_for(total, 256), 256, 0, s>>>(st.staged_x, xf, o.N, o.C, o.H, o.W, o.OW, o.KW, o.sw,
                                                           o.pw, o.xs[0], o.xs[1], o.xs[2], o.xs[3]);
    } else {
      const int C4 = st.tp.g.C;
      const int64_t total = int64_t(o.N) * o.H * o.W * (C4 / 4);
      to_nhwc4_kernel<<<grid_for(total, 256), 256, 0, s>>>(st.staged_x, xf, o.N, o.C, o.H, o.W, C4, o.xs[0], o.xs[1],
                                                          o.xs[2], o.xs[3]);
    }
    int rc = cuda_status(cudaGetLastError());
    if (rc) return rc;
    xf = st.staged_x;
  }
  float *yf = static_cast<float *>(y);
  const float *rf = static_cast<const float *>(res);
  const float *bias = p.bias_f;
  // Tensor maps follow the tensors: a graph input or output rebound to
  // another device buffer since prepare gets freshly encoded maps.
  Maps mp{st.amap, st.ymap, st.rmap};
  if (!st.set_attr_only) {
    if (st.amode != 1 && !st.staged_x && xf != st.amap_base && !encode_a(st, &mp.a, xf)) return SPKV2_ERR_UNSUPPORTED;
    if (st.epi_tma && yf != st.ymap_base && !encode_y(st, &mp.y, yf)) return SPKV2_ERR_UNSUPPORTED;
    if (st.tp.res_tma && rf != st.rmap_base && !encode_y(st, &mp.r, rf)) return SPKV2_ERR_UNSUPPORTED;
  }
  int rc = 0;
  if (st.split3) {
    switch (st.bn) {
      case 32: rc = launch_modes<32, true>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
      case 64: rc = launch_modes<64, true>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
      default: rc = launch_modes<128, true>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
    }
  } else {
    switch (st.bn) {
      case 32: rc = launch_modes<32, false>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
      case 64: rc = launch_modes<64, false>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
      case 256: rc = launch_modes<256, false>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
      default: rc = launch_modes<128, false>(st, mp, xf, yf, bias, rf, sk_ws, status, s); break;
    }
  }
  if (rc || !st.tp.sk_park_all || st.set_attr_only) return rc;
  // Split-K: add the parked segments and finish every tile.
  const float4 *ws = reinterpret_cast<const float4 *>(sk_ws);
  const int64_t threads = st.tp.tiles * kBM * (st.bn / 4);
  const unsigned blocks = unsigned(std::min<int64_t>(ceil_div(threads, 256), 148LL * 8));
  switch (st.bn) {
    case 32: return cuda_status(launch_kernel(conv_tc_reduce_kernel<32>, blocks, 256, 0, s, 1, ws, bias, rf, yf, st.tp));
    case 64: return cuda_status(launch_kernel(conv_tc_reduce_kernel<64>, blocks, 256, 0, s, 1, ws, bias, rf, yf, st.tp));
    case 256: return cuda_status(launch_kernel(conv_tc_reduce_kernel<256>, blocks, 256, 0, s, 1, ws, bias, rf, yf, st.tp));
    default: return cuda_status(launch_kernel(conv_tc_reduce_kernel<128>, blocks, 256, 0, s, 1, ws, bias, rf, yf, st.tp));
  }
}

}  // namespace spkv2
