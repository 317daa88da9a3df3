// vbq_gemv_half.cuh -- device helpers of the fp16 tensor-core GEMV kernel
// (vbq_gemv_half.cu): packed fp16 arithmetic on code words, the f16 m16n8k16 MMA, and the
// consumer warps' named barrier with its OR vote.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace vbq {
namespace ghalf {

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t lop_nib(uint32_t r, uint32_t mask) {
  return (r & mask) | 0x64006400u;  // one LOP3
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// consumer warps only (named barrier 1, 256 threads)
__device__ __forceinline__ void bar_sync_c() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool bar_or_c(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

}  // namespace ghalf
}  // namespace vbq
