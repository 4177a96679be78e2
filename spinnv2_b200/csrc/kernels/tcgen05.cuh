// tcgen05 / TMA / mbarrier building blocks shared by the implicit-GEMM
// kernels (conv_tc.cu: TF32 / 3xTF32, conv_tc_i8.cu: kind::i8), as inline
// PTX for sm_100a.  No cluster multicast anywhere: every TMA load targets the
// issuing CTA's own shared memory from this GPU's global memory.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

namespace spkv2 {
namespace tc {

constexpr long long kWaitCycles = 2000000000LL;  // bounded waits: ~1 s at 1.9 GHz

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

// One bounded probe: the thread is suspended (not spinning, so it takes no
// issue slots from the warps doing work) until the phase completes or about
// a millisecond passes.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: true if the phase with this parity has completed.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false on timeout (after `limit` clock cycles; the first
// role to give up records `code` in the status word) or when another role
// already aborted.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                                int code, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      if (status) atomicExch(status, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                          int code) {
  return mbar_wait_limit(bar, parity, abort_flag, status, code, kWaitCycles);
}

// The same bounded wait with a non-blocking test first: the common case of
// a phase that completed long ago costs one instruction.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                               int code) {
  return mbar_test(bar, parity) || mbar_wait_limit(bar, parity, abort_flag, status, code, kWaitCycles);
}

// Programmatic dependent launch: let the stream's next kernel begin
// launching, and wait until the previous kernel has completed with its
// writes visible.  Both are no-ops when the launch did not allow it.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// im2col load of a 4-D NHWC tensor map: `pixels x channels` box starting at
// base position {c, w, h, n}, shifted by the filter tap {w_off, h_off}.
__device__ __forceinline__ void tma_load_im2col_4d(void *dst, const CUtensorMap *map, int c, int w, int h, int n,
                                                   uint16_t w_off, uint16_t h_off, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c), "r"(w), "r"(h), "r"(n), "r"(smem_u32(bar)), "h"(w_off),
      "h"(h_off)
      : "memory");
}

__device__ __forceinline__ void tma_store_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

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
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128B-swizzled operand: SBO = 1024 B between 8-row groups,
// LBO = 16 B (unused for swizzled K-major), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(const void *p) {
  const uint64_t addr = smem_u32(p);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// K-major, 64B-swizzled operand (rows of 64 bytes): SBO = 512 B between
// 8-row groups, layout type 4 (64-byte swizzle); the tile must start on a
// 512-byte boundary.
__device__ __forceinline__ uint64_t smem_desc_sw64(const void *p) {
  const uint64_t addr = smem_u32(p);
  return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | (uint64_t(512 >> 4) << 32) | (1ull << 46) | (4ull << 61);
}

// K-major operand without swizzle, in 8-row x 16-byte core matrices: `lbo`
// bytes between core matrices along K, `sbo` bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc_noswz(const void *p, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = smem_u32(p);
  return ((addr & 0x3FFFFull) >> 4) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) | (uint64_t((sbo >> 4) & 0x3FFF) << 32) |
         (1ull << 46);
}

// A operand from TMEM (lane = row, one 32-bit column per K element).
__device__ __forceinline__ void mma_tf32_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
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

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// ---------------------------------------------------------------- CTA pairs
// 2-SM (cta_group::2) tiles: two CTAs of a cluster share one M = 256 MMA;
// CTA 0 (the leader) issues it, each CTA holds its 128 rows of A and half of
// B at the same shared-memory offsets, and each CTA's TMEM holds its rows of
// the accumulator.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// All threads of both CTAs: barrier across the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on the mbarrier at the same offset in cluster CTA `rank` (release at
// cluster scope, so this thread's earlier shared-memory writes, made visible
// to the async proxy by a proxy fence, are ordered before the arrival).
__device__ __forceinline__ void mbar_arrive_rank(uint64_t *bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// Bounded probe with acquire at cluster scope (for barriers that receive
// arrivals from the peer CTA).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                                  int *status, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      if (status) atomicExch(status, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                              uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive (once the issuing thread's earlier MMAs complete) on the mbarrier at
// this offset in both CTAs of the pair.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}

// ---------------------------------------------------------------- host side
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D tensor map with 128-byte swizzle: dims {inner, outer} in elements of
// `elem_bytes`, row pitch in elements, box {128 bytes, box_rows}.  Elements
// outside the dims read as zero.
inline bool encode_2d(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void *base,
                      uint64_t inner, uint64_t outer, uint64_t pitch, uint32_t box_rows) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch * elem_bytes};
  const cuuint32_t box[2] = {128u / elem_bytes, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D tensor map with an explicit box and swizzle mode (inner box in
// elements).
inline bool encode_2d_box(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void *base,
                          uint64_t inner, uint64_t outer, uint64_t pitch, uint32_t box_inner, uint32_t box_rows,
                          CUtensorMapSwizzle swizzle) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch * elem_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode_fn()(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  }
  return fn;
}

// im2col map of a dense NHWC tensor [N][H][W][C] for a square conv (kernel k,
// stride s, pad p, dilation d): the bounding box of filter-window origins
// runs from -p to (dim - 1) + p - (k - 1) * d in W and H, traversed with
// step s; rows of `channels` elements (128 bytes with the default 128-byte
// swizzle; 16 bytes per pixel, unswizzled, for 4-channel inputs).
// General form: kernel kh x kw, stride sh x sw, padding ph x pw, dilation
// dh x dw (corner and stride arrays in the tensor's dimension order, W
// before H).
inline bool encode_im2col_nhwc2(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void *base,
                                int N, int H, int W, int C, int kh, int kw, int sh, int sw, int ph, int pw, int dh,
                                int dw, uint32_t channels, uint32_t pixels,
                                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (!encode_im2col_fn()) return false;
  const cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(N)};
  const cuuint64_t strides[3] = {cuuint64_t(C) * elem_bytes, cuuint64_t(W) * C * elem_bytes,
                                 cuuint64_t(H) * W * C * elem_bytes};
  const int lower[2] = {-pw, -ph};
  const int upper[2] = {pw - (kw - 1) * dw, ph - (kh - 1) * dh};
  const cuuint32_t estr[4] = {1, cuuint32_t(sw), cuuint32_t(sh), 1};
  return encode_im2col_fn()(map, dtype, 4, const_cast<void *>(base), dims, strides, lower, upper, channels, pixels,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// im2col map of a dense NHWC tensor with explicit window-origin corners
// (lower[0] / upper[0] along W, [1] along H: origins run from lower to
// dim - 1 + upper) and traversal strides sw x sh.
inline bool encode_im2col_corners(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void *base,
                                  int N, int H, int W, int C, const int lower[2], const int upper[2], int sw, int sh,
                                  uint32_t channels, uint32_t pixels, CUtensorMapSwizzle swizzle) {
  if (!encode_im2col_fn()) return false;
  const cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(N)};
  const cuuint64_t strides[3] = {cuuint64_t(C) * elem_bytes, cuuint64_t(W) * C * elem_bytes,
                                 cuuint64_t(H) * W * C * elem_bytes};
  const cuuint32_t estr[4] = {1, cuuint32_t(sw), cuuint32_t(sh), 1};
  return encode_im2col_fn()(map, dtype, 4, const_cast<void *>(base), dims, strides, lower, upper, channels, pixels,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool encode_im2col_nhwc(CUtensorMap *map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void *base,
                               int N, int H, int W, int C, int k, int s, int p, int d, uint32_t channels,
                               uint32_t pixels, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (!encode_im2col_fn()) return false;
  const cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(N)};
  const cuuint64_t strides[3] = {cuuint64_t(C) * elem_bytes, cuuint64_t(W) * C * elem_bytes,
                                 cuuint64_t(H) * W * C * elem_bytes};
  const int lower[2] = {-p, -p};
  const int upper[2] = {p - (k - 1) * d, p - (k - 1) * d};
  const cuuint32_t estr[4] = {1, cuuint32_t(s), cuuint32_t(s), 1};
  return encode_im2col_fn()(map, dtype, 4, const_cast<void *>(base), dims, strides, lower, upper, channels, pixels,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- launches
// Launch with programmatic stream serialisation (the kernel's prologue may
// overlap the previous kernel's tail; the kernel calls pdl_wait() before its
// first global access) unless SPKV2_NO_PDL is set; optionally as clusters of
// `cluster` CTAs.
inline bool pdl_enabled() {
  static const bool on = getenv("SPKV2_NO_PDL") == nullptr;
  return on;
}

template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kern)(Params...), unsigned grid, unsigned block, size_t smem, cudaStream_t s,
                          int cluster, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = unsigned(cluster);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

}  // namespace tc
}  // namespace spkv2
