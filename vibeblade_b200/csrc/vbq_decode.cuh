// vbq_decode.cuh -- one lane's 8 consecutive values of a 256-value unit of a weight row.
//
// A unit is 256 consecutive values of one row: one block of a 256-value type (Q2_K, Q3_K,
// Q4_K, Q5_K, Q6_K, Q8_K), eight blocks of a 32-value type (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0),
// or 256 F32 / F16 / BF16 values; lane l produces values 8 l .. 8 l + 7.  Values are the
// reference's dequantized fp32 values bit for bit (cpp/src/dequant.cpp:23-93, :128-245,
// :268-301, :317-402, :407-411; the GGUF Q8_0 block of cpp/src/cuda_kernels.cu:718-735):
// every product and sum the reference rounds separately is rounded separately here.  Used
// by the dequant kernel and the generic GEMV.
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

// ---- the other block types of the reference's dispatcher ----
// Blocks sit at 2-byte-aligned offsets (every block size is even), so 16-bit fields are
// read directly and 4-byte runs with ld_u32_a2.  Small integers become floats through
// u2f / s8f (exact, at the FP32 rate).

// Q4_0, 18 B (cpp/src/dequant.cpp:23-35): d @0, qs @2; value i of a block is nibble i&1 of
// qs[i>>1], so the lane's 8 values (block lane/4, values 8(lane&3)..) are the 8 nibbles of
// one 4-byte word, lowest first; out = (q - 8) * d.
template <>
__device__ __forceinline__ void decode8<kQ4_0>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* blk = unit + 18 * (lane >> 2);
  const float d = f16_ref(ld_u16(blk));
  const uint32_t w = ld_u32_a2(blk + 2 + 4 * (lane & 3));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(u2f_minus<8>((w >> (4 * i)) & 0xfu), d);
}

// Q4_1, 20 B (:40-53): d @0, m @2, qs @4; out = d * q + m.
template <>
__device__ __forceinline__ void decode8<kQ4_1>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* blk = unit + 20 * (lane >> 2);
  const float d = f16_ref(ld_u16(blk)), m = f16_ref(ld_u16(blk + 2));
  const uint32_t w = ld_u32_a2(blk + 4 + 4 * (lane & 3));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(__fmul_rn(d, u2f((w >> (4 * i)) & 0xfu)), m);
}

// Q5_0, 22 B (:58-73): d @0, qh @2 (bit i = fifth bit of value i), qs @6; out = (q - 16) * d.
template <>
__device__ __forceinline__ void decode8<kQ5_0>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* blk = unit + 22 * (lane >> 2);
  const float d = f16_ref(ld_u16(blk));
  const uint32_t hb = ld_u32_a2(blk + 2) >> (8 * (lane & 3));
  const uint32_t w = ld_u32_a2(blk + 6 + 4 * (lane & 3));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t q = ((w >> (4 * i)) & 0xfu) | (((hb >> i) & 1u) << 4);
    v[i] = __fmul_rn(u2f_minus<16>(q), d);
  }
}

// Q5_1, 24 B (:78-93): d @0, m @2, qh @4, qs @8; out = d * q + m.
template <>
__device__ __forceinline__ void decode8<kQ5_1>(const uint8_t* __restrict__ unit, int lane,
                                               float v[8]) {
  const uint8_t* blk = unit + 24 * (lane >> 2);
  const float d = f16_ref(ld_u16(blk)), m = f16_ref(ld_u16(blk + 2));
  const uint32_t hb = ld_u32_a2(blk + 4) >> (8 * (lane & 3));
  const uint32_t w = ld_u32_a2(blk + 8 + 4 * (lane & 3));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t q = ((w >> (4 * i)) & 0xfu) | (((hb >> i) & 1u) << 4);
    v[i] = __fadd_rn(__fmul_rn(d, u2f(q)), m);
  }
}

// Q2_K, 84 B (:128-150): scales[16] @0, qs[64] @16, d @80, dmin @82.  The lane's values
// are half (lane&1) of sub-block lane/2; the reference reads value l of a sub-block from
// bits 2(l&3) of qs[4s + l/8], so the lane's 8 codes come from one byte, each twice;
// out = (d * (scale & 15)) * q + dmin (the reference adds dmin itself).
template <>
__device__ __forceinline__ void decode8<kQ2_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const int s = lane >> 1;
  const float d = f16_ref(ld_u16(blk + 80)), mn = f16_ref(ld_u16(blk + 82));
  const float dl = __fmul_rn(d, u2f(blk[s] & 0xfu));
  const uint32_t q = blk[16 + 4 * s + (lane & 1)];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(__fmul_rn(dl, u2f((q >> (2 * (i & 3))) & 3u)), mn);
}

// Q3_K scale of sub-block j (get_scale_min_k3, :155-166; its min is unused).
__device__ __forceinline__ int q3k_scale(const uint8_t* __restrict__ sc, int j) {
  if (j < 4) return sc[j] & 63;
  if (j < 8) return sc[j + 4] & 63;
  return (sc[j - 4] >> 4) & 63;
}

// Q3_K, 110 B (:168-218): hmask[32] @0, qs[64] @32, scales[12] @96, d @108.  The lane's
// values: chunk c = lane/8 of 64, quarter t = (lane/2)&3, half (lane&1) of its 16; codes
// from one byte, qs[16c + 4t + (lane&1)], each twice (bits 2(l&3)); the high bit of value l
// is bit 4c + 2t of hmask[l], and 0 once that shift reaches 8 (the reference shifts a
// byte); out = (d * scale(4c + t)) * (q + 8 h).
template <>
__device__ __forceinline__ void decode8<kQ3_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const int c = lane >> 3, t = (lane >> 1) & 3, sh = 4 * c + 2 * t;
  const float d = f16_ref(ld_u16(blk + 108));
  const float dt = __fmul_rn(d, u2f((uint32_t)q3k_scale(blk + 96, 4 * c + t)));
  const uint32_t q = blk[32 + 16 * c + 4 * t + (lane & 1)];
  const uint8_t* hm = blk + 8 * (lane & 1);
  const uint32_t h0 = ld_u32_a2(hm), h1 = ld_u32_a2(hm + 4);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t hbyte = byte_of(i < 4 ? h0 : h1, i & 3);
    const uint32_t h = sh < 8 ? (hbyte >> sh) & 1u : 0u;
    v[i] = __fmul_rn(dt, u2f(((q >> (2 * (i & 3))) & 3u) + 8u * h));
  }
}

// Q5_K, 176 B (:307-354): d @0, dmin @2, scales[12] @4 (the Q4_K packing), qh[32] @16,
// qs[128] @48.  The reference advances its qh pointer 32 bytes per 64-value chunk, as it
// does qs, so chunk c reads its fifth bits from bytes 16 + 32c.. (qs bytes from chunk 1 on),
// bit 7 for the chunk's first 32 values and bit 3 for the second.  The lane's values: chunk
// c = lane/8, half (lane/4)&1, offset l0 = 8(lane&3); out = (d*sc)*q - dmin*m.
template <>
__device__ __forceinline__ void decode8<kQ5_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const int c = lane >> 3, half = (lane >> 2) & 1, l0 = 8 * (lane & 3);
  const float d = f16_ref(ld_u16(blk)), dmin = f16_ref(ld_u16(blk + 2));
  const uint32_t s0 = ld_u32_a2(blk + 4), s1 = ld_u32_a2(blk + 8), s2 = ld_u32_a2(blk + 12);
  int sc, mn;
  q4k_scale_min(2 * c + half, s0, s1, s2, sc, mn);
  const float d1 = __fmul_rn(d, u2f((uint32_t)sc)), m1 = __fmul_rn(dmin, u2f((uint32_t)mn));
  const uint8_t* qp = blk + 48 + 32 * c + l0;
  const uint8_t* hp = blk + 16 + 32 * c + l0;
  const uint32_t q0 = ld_u32_a2(qp), q1 = ld_u32_a2(qp + 4);
  const uint32_t g0 = ld_u32_a2(hp), g1 = ld_u32_a2(hp + 4);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t qb = byte_of(i < 4 ? q0 : q1, i & 3), hb = byte_of(i < 4 ? g0 : g1, i & 3);
    const uint32_t q = half ? ((qb >> 4) | (((hb >> 3) & 1u) << 4)) : ((qb & 0xfu) | (((hb >> 7) & 1u) << 4));
    v[i] = __fsub_rn(__fmul_rn(d1, u2f(q)), m1);
  }
}

// Q8_K, 292 B (:226-245): d (fp32) @0, then eight 33-byte sub-blocks at 4 + 33s, each 32
// int8 codes and an int8 scale; out = q * (d * scale).  Sub-blocks start at odd offsets,
// so the codes are read bytewise.
template <>
__device__ __forceinline__ void decode8<kQ8_K>(const uint8_t* __restrict__ blk, int lane,
                                               float v[8]) {
  const float d = __uint_as_float(ld_u16(blk) | (ld_u16(blk + 2) << 16));
  const uint8_t* sub = blk + 4 + 33 * (lane >> 2);
  const float ds = __fmul_rn(d, s8f(sub[32]));
  const uint8_t* q = sub + 8 * (lane & 3);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(s8f(q[i]), ds);
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
