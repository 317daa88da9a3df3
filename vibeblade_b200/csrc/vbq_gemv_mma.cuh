// vbq_gemv_mma.cuh -- device helpers shared by the integer tensor-core GEMV kernels
// (vbq_gemv_mma.cu: batch 1..4, vbq_gemv_wide.cu: batch 8 / 16): ldmatrix, the u8 x s8
// m16n8k32 MMA, 2-D TMA loads, thread-block cluster primitives and hinted mbarrier waits.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "vbq_common.cuh"

namespace vbq {
namespace gmma {

// fixed point: |v| < 2^(e + 1) <=> |n| < 2^22 with n = rint(v * 2^(21 - e))
constexpr float kMagic = 12582912.f;  // 1.5 * 2^23
constexpr int kExpMin = -100, kExpMax = 100;

// 32 rows x 16 bytes (lane L gives the address of row L) as the m16n8k32 8-bit A fragment:
// r0 / r1 = rows 4t .. 4t + 3 of byte column g / g + 8, r2 / r3 = rows 16 + 4t .. (g = lane / 4,
// t = lane % 4); byte-granular transpose, so the codes need no permute after the load
__device__ __forceinline__ void ldmatrix_a8_trans(uint32_t saddr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(saddr));
}
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// ---- thread-block cluster: one cluster = the K-splits of one tile, leader = split 0 ----
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_u32(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// whole-cluster barrier, every thread of every CTA (release / acquire)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// fp32 load from another CTA's shared memory (a shared::cluster address from mapa)
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
// 16 bytes into another CTA's shared memory; the bytes complete on its mbarrier
__device__ __forceinline__ void st_async_v4(uint32_t remote, float4 v, uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(remote), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar)
      : "memory");
}

// mbarrier wait that lets the hardware park the warp until the phase completes (up to
// kSuspendNs per try), bounded by `budget` SM cycles overall
constexpr uint32_t kSuspendNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_hinted(uint32_t bar, uint32_t parity, long long budget) {
  if (mbar_try_wait_hint(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_hint(bar, parity)) {
    if (clock64() - t0 > budget) return false;
  }
  return true;
}

__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }
// 1 / s for a power of two s = 2^k with |k| <= 126 (exact: the exponent field is negated)
__device__ __forceinline__ float inv_pow2(float s) { return __uint_as_float(0x7f000000u - __float_as_uint(s)); }

// ---- host: the weight operand's tensor map ---------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The GEMV kernels' weight map: the K x RB bytes as a 2-D u16 array, boxes of `pitch` bytes x
// `rows` rows, L2 256-byte promotion.  The map depends only on these arguments, so each
// host thread keeps the last few it encoded (encoding is a driver call of about a
// microsecond, on every decode launch otherwise).  Returns false when encoding fails.
inline bool weight_map(EncodeTiledFn enc, const void* w, int64_t K, int64_t RB, int pitch, int rows,
                       CUtensorMap* out) {
  struct Entry {
    CUtensorMap map;
    const void* w;
    int64_t K, RB;
    int pitch, rows;
    bool valid;
  };
  thread_local Entry cache[8] = {};
  const uintptr_t key = (reinterpret_cast<uintptr_t>(w) >> 8) ^ (uintptr_t)K ^ ((uintptr_t)RB << 4) ^
                        ((uintptr_t)pitch << 12) ^ (uintptr_t)rows;
  Entry& e = cache[(key ^ (key >> 3) ^ (key >> 6)) & 7];
  if (e.valid && e.w == w && e.K == K && e.RB == RB && e.pitch == pitch && e.rows == rows) {
    *out = e.map;
    return true;
  }
  cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)RB};
  cuuint32_t box[2] = {(cuuint32_t)(pitch / 2), (cuuint32_t)rows};
  cuuint32_t es[2] = {1, 1};
  e.valid = false;
  if (enc(&e.map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  e.w = w, e.K = K, e.RB = RB, e.pitch = pitch, e.rows = rows, e.valid = true;
  *out = e.map;
  return true;
}

}  // namespace gmma
}  // namespace vbq
