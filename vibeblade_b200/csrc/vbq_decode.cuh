// vbq_decode.cuh -- one lane's 8 consecutive values of a 256-value unit of a weight row.
//
// A unit is 256 consecutive values of one row: one Q4_K / Q6_K block, eight Q8_0 blocks,
// or 256 F32 / F16 / BF16 values; lane l produces values 8 l .. 8 l + 7.  Values are the
// reference's dequantized fp32 values bit for bit (cpp/src/dequant.cpp:268-301, :359-402,
// :407-411; the GGUF Q8_0 block of cpp/src/cuda_kernels.cu:718-735): every product and
// difference the reference rounds separately is rounded separately here.  Used by the
// dequant kernel and the generic GEMV.
#pragma once
#include "vbq_common.cuh"

namespace vbq {

template <int QT>
__device__ __forceinline__ void decode8(const uint8_t* __restrict__ tile, int lane, float v[8]);

// Q4_K: lane covers values 8*lane..8*lane+7 -> sub-block s = lane/4, nibble half s&1,
// qs bytes 32*(s/2) + 8*(lane%4) .. +7.
template <>
__device__ __forceinline__ void decode8<kQ4_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const float d = f16_ref(ld_u16(blk));
  const float dmin = f16_ref(ld_u16(blk + 2));
  const uint32_t s0 = ld_u32_a2(blk + 4), s1 = ld_u32_a2(blk + 8), s2 = ld_u32_a2(blk + 12);
  const int s = lane >> 2;
  int sc, mn;
  q4k_scale_min(s, s0, s1, s2, sc, mn);
  const float dl = __fmul_rn(d, (float)sc);
  const float ml = __fmul_rn(dmin, (float)mn);
  const uint8_t* q = blk + 16 + 32 * (s >> 1) + 8 * (lane & 3);
  const uint32_t w0 = ld_u32_a2(q), w1 = ld_u32_a2(q + 4);
  const int hs = (s & 1) * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = i < 4 ? w0 : w1;
    const uint32_t nib = (w >> (8 * (i & 3) + hs)) & 0xfu;
    v[i] = __fsub_rn(__fmul_rn(dl, (float)nib), ml);
  }
}

// Q6_K (reference layout): value i -> ql nibble i&1 of byte i>>1, qh field i&3 of byte
// i>>2, int8 scale i>>4, out = (d*scale)*(q-32).  Lane: ql bytes 4*lane..+3, qh bytes
// 2*lane..+1, scale 192 + lane/2.
template <>
__device__ __forceinline__ void decode8<kQ6_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const float d = f16_ref(ld_u16(blk + 208));
  const int sc = (int)(int8_t)blk[192 + (lane >> 1)];
  const float ds = __fmul_rn(d, (float)sc);
  const uint32_t ql = ld_u32_a2(blk + 4 * lane);
  const uint32_t qh = ld_u16(blk + 128 + 2 * lane);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int lo = (int)((ql >> (4 * i)) & 0xfu);
    const int hi = (int)((qh >> (2 * i)) & 0x3u);
    v[i] = __fmul_rn(ds, (float)((lo | (hi << 4)) - 32));
  }
}

// Q8_0 (GGUF block, fp16 d): the 256-value unit spans blocks lane/4, values 8*(lane%4)..
template <>
__device__ __forceinline__ void decode8<kQ8_0>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* blk = unit + 34 * (lane >> 2);
  const float d = f16_ieee(ld_u16(blk));
  const uint8_t* q = blk + 2 + 8 * (lane & 3);
  const uint32_t w0 = ld_u32_a2(q), w1 = ld_u32_a2(q + 4);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t w = i < 4 ? w0 : w1;
    const int qv = (int)(int8_t)(uint8_t)(w >> (8 * (i & 3)));
    v[i] = __fmul_rn((float)qv, d);
  }
}

// F32 rows: the values as stored (memcpy in the reference's dequantize_row).
template <>
__device__ __forceinline__ void decode8<kF32>(const uint8_t* __restrict__ unit, int lane,
                                              float v[8]) {
  const uint8_t* p = unit + 32 * lane;
  if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 16);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(ld_u16(p + 4 * i) | (ld_u16(p + 4 * i + 2) << 16));
  }
}

// F16 rows: the reference's f16_to_f32 (fp16 subnormals doubled, cpp/src/fp16_compat.cpp).
template <>
__device__ __forceinline__ void decode8<kF16>(const uint8_t* __restrict__ unit, int lane,
                                              float v[8]) {
  const uint8_t* p = unit + 16 * lane;
  if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = f16_ref(w[i] & 0xffffu);
      v[2 * i + 1] = f16_ref(w[i] >> 16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = f16_ref(ld_u16(p + 2 * i));
  }
}

// BF16 rows: the top half of an fp32 (bf16_to_f32, cpp/include/ggml_types.h:175-180).
template <>
__device__ __forceinline__ void decode8<kBF16>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* p = unit + 16 * lane;
  if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(ld_u16(p + 2 * i) << 16);
  }
}

// The first `cnt` (< 8) values of the lane, for the ragged end of an unquantized row (the
// rest read as 0); nothing past the row is touched.
template <int QT>
__device__ __forceinline__ void decode_tail(const uint8_t* __restrict__ unit, int lane, int cnt,
                                            float v[8]) {
  static_assert(Fmt<QT>::kValues == 1, "ragged lanes exist only for unquantized rows");
  constexpr int E = Fmt<QT>::kBytes;
  const uint8_t* p = unit + 8 * E * lane;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float f = 0.f;
    if (i < cnt) {
      if constexpr (QT == kF32) f = __uint_as_float(ld_u16(p + 4 * i) | (ld_u16(p + 4 * i + 2) << 16));
      else if constexpr (QT == kF16) f = f16_ref(ld_u16(p + 2 * i));
      else f = __uint_as_float(ld_u16(p + 2 * i) << 16);
    }
    v[i] = f;
  }
}

}  // namespace vbq
