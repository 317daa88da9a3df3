// vbq_common.cuh -- shared device helpers for the sm_100a k-quant kernels.
//
// Block formats (kevin046/VibeBlade cpp/include/ggml_types.h:109-141):
//   Q4_K 144 B: fp16 d @0, fp16 dmin @2, 12 B packed 6-bit scales/mins @4, 128 B nibbles @16
//   Q6_K 210 B: ql[128] @0, qh[64] @128, int8 scales[16] @192, fp16 d @208
//   Q8_0  34 B: fp16 d @0, int8 qs[32] @2 (GGUF block)
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace vbq {

constexpr int kF32 = 0;
constexpr int kF16 = 1;
constexpr int kQ4_0 = 2;
constexpr int kQ4_1 = 3;
constexpr int kQ5_0 = 6;
constexpr int kQ5_1 = 7;
constexpr int kQ8_0 = 8;
constexpr int kQ2_K = 10;
constexpr int kQ3_K = 11;
constexpr int kQ4_K = 12;
constexpr int kQ5_K = 13;
constexpr int kQ6_K = 14;
constexpr int kQ8_K = 15;
constexpr int kBF16 = 30;

template <int QT> struct Fmt;
template <> struct Fmt<kQ4_K> { static constexpr int kValues = 256, kBytes = 144; };
template <> struct Fmt<kQ6_K> { static constexpr int kValues = 256, kBytes = 210; };
template <> struct Fmt<kQ8_0> { static constexpr int kValues = 32, kBytes = 34; };
// the other block types of the reference's dispatcher (cpp/include/ggml_types.h:52-71,
// :82-168), read by the dequant kernel and the generic GEMV only
template <> struct Fmt<kQ4_0> { static constexpr int kValues = 32, kBytes = 18; };
template <> struct Fmt<kQ4_1> { static constexpr int kValues = 32, kBytes = 20; };
template <> struct Fmt<kQ5_0> { static constexpr int kValues = 32, kBytes = 22; };
template <> struct Fmt<kQ5_1> { static constexpr int kValues = 32, kBytes = 24; };
template <> struct Fmt<kQ2_K> { static constexpr int kValues = 256, kBytes = 84; };
template <> struct Fmt<kQ3_K> { static constexpr int kValues = 256, kBytes = 110; };
template <> struct Fmt<kQ5_K> { static constexpr int kValues = 256, kBytes = 176; };
template <> struct Fmt<kQ8_K> { static constexpr int kValues = 256, kBytes = 292; };
// unquantized weights (small GGUF tensors such as the MoE router): one value per "block"
template <> struct Fmt<kF32> { static constexpr int kValues = 1, kBytes = 4; };
template <> struct Fmt<kF16> { static constexpr int kValues = 1, kBytes = 2; };
template <> struct Fmt<kBF16> { static constexpr int kValues = 1, kBytes = 2; };

// Bytes holding one 256-value column tile of a row: one Q4_K / Q6_K block, or eight
// Q8_0 blocks.
template <int QT> struct Tile {
  static constexpr int kBytes = Fmt<QT>::kBytes * (256 / Fmt<QT>::kValues);
};

// fp16 -> fp32 with the reference's rounding (cpp/src/fp16_compat.cpp:13-35): exact
// for normals, zeros, inf; fp16 subnormals come out at twice their IEEE value, which
// the reference's k-quant dequantizers inherit.  Used for Q4_K d/dmin and Q6_K d.
__device__ __forceinline__ float f16_ref(uint32_t h) {
  float f = __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
  return ((h & 0x7c00u) == 0u) ? f * 2.0f : f;
}

// Exact IEEE fp16 -> fp32 (the Q8_0 scale; cpp/src/cuda_kernels.cu:731).
__device__ __forceinline__ float f16_ieee(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// (float)u for 0 <= u < 2^23, exactly, without an integer-to-float conversion: u in the
// mantissa of 2^23, then 2^23 subtracted (both steps exact).  The conversion unit runs at a
// fraction of the FP32 rate, the OR and FADD at the full rate.
__device__ __forceinline__ float u2f(uint32_t u) {
  return __fsub_rn(__uint_as_float(0x4b000000u | u), 8388608.0f);
}
// (float)((int)u - OFF) the same way, for 0 <= u < 2^23 and 0 <= OFF < 2^23.
template <int OFF>
__device__ __forceinline__ float u2f_minus(uint32_t u) {
  return __fsub_rn(__uint_as_float(0x4b000000u | u), 8388608.0f + (float)OFF);
}
// (float)(int8_t)b for the byte b (the low 8 bits of b).
__device__ __forceinline__ float s8f(uint32_t b) { return u2f_minus<128>((b & 0xffu) ^ 0x80u); }

// nan -> 0, +-inf -> +-65504, then clip to +-65504 (vibeblade/moe.py:472-473)
__device__ __forceinline__ float sanitize(float v) {
  if (v != v) return 0.0f;
  return fminf(fmaxf(v, -65504.0f), 65504.0f);
}
// x * sigmoid(x) = x / (1 + e^-x), the reference's two-sided form (vibeblade/moe.py:36-50)
// written without its branch: for the sanitised inputs (|x| <= 65504) e^-x is +inf only
// where x < -88, and the quotient is then -0, as in the two-sided form.  expf is the full-
// precision exponential; __fdividef is within 2 ulp for every denominator here (>= 1).
// Branch-free, so a warp whose inputs have both signs does not run both halves.
__device__ __forceinline__ float silu_ref(float x) { return __fdividef(x, 1.0f + expf(-x)); }
// One SwiGLU value, silu(g) * u of the sanitised inputs (the FFN's gate and up,
// cpp/src/fast_model.cpp:946-953; the same arithmetic as vbq_swiglu).
__device__ __forceinline__ float swiglu1(float g, float u) { return silu_ref(sanitize(g)) * sanitize(u); }

// Input of a fused GEMV: x[b, k] itself, or, with SWIGLU, silu(gu[b, k]) * gu[b, K + k]
// where x points at a [batch, 2K] buffer holding a gate | up matmul's output (the down
// projection's input, computed where it is read instead of in a pass of its own).
template <bool SWIGLU>
__device__ __forceinline__ float gemv_x(const float* __restrict__ x, int64_t b, int64_t K, int64_t k) {
  if constexpr (SWIGLU) {
    const float* r = x + b * 2 * K;
    return swiglu1(__ldg(r + k), __ldg(r + K + k));
  } else {
    return __ldg(x + b * K + k);
  }
}

// Output epilogue of the GEMV kernels: y[b, n] = acc + bias[n] + res[b, n], each term only
// when its pointer is set (the reference adds the Q/K/V biases after its GEMVs,
// cpp/src/fast_model.cpp:659-668, and the residual after o and down, :813-824, :990-998).
// res is [batch, N] like y and may be y itself (read before the write, same thread).
struct Epi {
  const float* bias;
  const float* res;
};
__device__ __forceinline__ float epi_apply(const Epi& e, float v, int64_t b, int64_t N, int64_t n) {
  if (e.bias) v += __ldg(e.bias + n);
  if (e.res) v += e.res[b * N + n];
  return v;
}

// Q4_K sub-block scale and min (get_scale_min_k4, cpp/src/dequant.cpp:258-266).
// s0/s1/s2 are scale bytes 0-3, 4-7, 8-11 as little-endian words.
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2,
                                              int& sc, int& mn) {
  if (j < 4) {
    sc = (int)(byte_of(s0, j) & 63u);
    mn = (int)(byte_of(s1, j) & 63u);
  } else {
    const int i = j - 4;
    sc = (int)((byte_of(s2, i) & 0xfu) | ((byte_of(s0, i) >> 6) << 4));
    mn = (int)((byte_of(s2, i) >> 4) | ((byte_of(s1, i) >> 6) << 4));
  }
}

// Branch-free form of q4k_scale_min for a sub-block index fixed per thread: the
// selector/shift/mask recipe is computed once (Q4kScaleRecipe(j)) and applied per row.
struct Q4kScaleRecipe {
  bool hi;        // j >= 4
  int pa, ma;     // low part: (A >> pa) & ma, A = hi ? s2 : s0 (scale) / s2 : s1 (min)
  int pb;         // high 2 bits: (s0 >> pb) & 0x30 (scale) / (s1 >> pb) & 0x30 (min)
  int mb;         // 0x30 when hi, else 0
  __device__ __forceinline__ explicit Q4kScaleRecipe(int j) {
    hi = j >= 4;
    const int i = hi ? j - 4 : j;
    pa = 8 * i;
    ma = hi ? 0x0f : 0x3f;
    pb = 8 * i + 2;  // bits 8i+6..8i+7 shifted down to 4..5
    mb = hi ? 0x30 : 0;
  }
  __device__ __forceinline__ void apply(uint32_t s0, uint32_t s1, uint32_t s2, int& sc,
                                        int& mn) const {
    const uint32_t As = hi ? s2 : s0;
    const uint32_t Am = hi ? (s2 >> 4) : s1;
    sc = (int)(((As >> pa) & (uint32_t)ma) | ((s0 >> pb) & (uint32_t)mb));
    mn = (int)(((Am >> pa) & (uint32_t)ma) | ((s1 >> pb) & (uint32_t)mb));
  }
};

// Read 4 bytes at a 2-byte-aligned shared/global address as one little-endian word.
// Only aligned words that hold at least one of the 4 bytes are touched, so the read
// never leaves the pages the data lives on.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 3u) * 8u;
  const uint32_t lo = q[0];
  return sh ? __funnelshift_r(lo, q[1], sh) : lo;
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return (uint32_t)*reinterpret_cast<const uint16_t*>(p);
}

// cp.async (Ampere-style asynchronous global->shared copies), used by the GEMV
// pipeline: no mbarrier, so no wait on the device can outlive its group.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---- mbarrier + bulk-copy (TMA, non-tensor) helpers --------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint32_t bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued before has landed (the arrival
// was counted in the barrier's init count).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// Bulk global -> shared copy (16-byte aligned addresses, size a multiple of 16) that
// reports its bytes to `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of `bar` with the given parity, giving up after `budget` SM clock
// cycles (returns false then).  Every device-side wait in this library is bounded.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long budget) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > budget) return false;
  }
  return true;
}

// ~2 s at the B200's 1.965 GHz boost clock.
constexpr long long kWaitBudgetCycles = 4000000000LL;

// Status bits a kernel raises in its file's device status word.
constexpr unsigned kStatusTimeout = 1u;

}  // namespace vbq
