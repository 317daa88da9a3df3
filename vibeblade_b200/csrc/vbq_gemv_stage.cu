// vbq_gemv_stage.cu -- fused dequant-GEMV for the reference dispatcher's other block types
// (Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, Q8_K), streamed through shared memory.
//
//   y[b, n] = sum_k x[b, k] * deq(W)[k, n]  (+ bias[n]) (+ res[b, n])
//
// (cpp/src/dequant.cpp:739-780 with the dequantizers of :23-245, :317-354).  The generic
// kernel (vbq_gemv_any.cu) reads each lane's bytes straight from global memory with a few
// rows in flight per warp, too few bytes in flight to keep HBM busy; this kernel keeps a
// ring of row stages in flight per warp instead.
//
// Decomposition: a CTA owns C 256-column units of the output (C = 2 for Q3_K, whose
// 110-byte unit is not a whole number of 4-byte words; 1 otherwise), a K-slice and a group
// of up to 4 batch rows.  Each of its 8 warps streams a contiguous share of the slice's rows
// through a ring of its own in shared memory (3-8 stages of 8 rows), with 16-byte
// cp.async of the granules that cover each row's chunk, so the loop has no CTA-wide
// barrier; all but one of the ring's stages are issued before the dependency wait on the
// previous grid (weights do not depend on it).  After that wait the slice's activations
// (B x kslice fp32) are loaded into shared memory once, so no row waits on a global load.
// Lane l takes values 8 l .. 8 l + 7 of each unit of a row from shared memory and adds
// their products with x[b, k] in fp32, reassociated as (x * d) * q + x * m (Dot<QT>
// below), which takes a third of the instructions of dequantizing each value first (the
// dequant kernel keeps the reference's values bit for bit; the GEMV's bar is 1e-3).  The
// warps then add their sums in warp order, the K-slices of a column group (one
// thread-block cluster) in split order at the cluster leader, which writes y.
// Deterministic, no scratch, no atomics, no waits beyond the cp.async groups and barriers
// of the CTA and its cluster.
//
// Requirements (checked by the launcher, which otherwise leaves the call to the generic
// kernel): N a multiple of C * 256, row_bytes 4-byte and w 16-byte aligned, K * row_bytes
// a multiple of 16, the rings and the slice's activations within 200 KB of shared memory.
#include <cuda_runtime.h>

#include "vbq_common.cuh"
#include "vbq_decode.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {
namespace gstage {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kWRows = 8;       // rows per stage of a warp's ring
constexpr int kMaxBatch = 4;    // batch rows per CTA
constexpr int kMaxSplit = 8;    // portable cluster size

template <int QT> struct Cfg {
  static constexpr int kUnit = Tile<QT>::kBytes;                // bytes of one 256-value unit
  static constexpr int kC = (kUnit % 4 == 0) ? 1 : 2;           // units per CTA
  static constexpr int kChunk = kC * kUnit;                     // bytes of a row the CTA reads
  static_assert(kChunk % 4 == 0, "a row chunk must be whole 4-byte words");
  // a row's chunk starts 4-byte aligned; the 16-byte granules that cover it, at most
  static constexpr int kGran = (kChunk + 12 + 15) / 16;
  static constexpr int kPitch = 16 * kGran;                     // a row's place in a stage
  static constexpr int kStage = kWRows * kPitch;
  // stages per warp ring: about 80 KB of rings per CTA, 3 to 8 stages (measured on B200 at
  // 4096 x 14336, batch 1: 8 rows a stage and ~64-80 KB beat 4 rows and 41-78 KB, and
  // larger rings cost Q8_K its second CTA per SM)
  static constexpr int kRingRaw = 81920 / (kWarps * kStage);
  static constexpr int kRing = kRingRaw < 3 ? 3 : (kRingRaw > 8 ? 8 : kRingRaw);
  static constexpr int kWarpRing = kRing * kStage;              // one warp's ring
  static constexpr int kRingBytes = kWarps * kWarpRing;
  // after the loop the same memory holds [warp][b][C * 256] sums and the CTA's [b][C * 256]
  static constexpr int kRedBytes = (kWarps + 1) * kMaxBatch * kC * 256 * 4;
};

// ---- one lane's share of one row: values 8 lane .. 8 lane + 7 of a 256-value unit ----
// The GEMV does not need the dequantized values themselves (the dequant kernel produces
// those bit for bit), only their products with x; it adds them reassociated, as
//   x * (d * q + m) = (x * d) * q + x * m,
// with x * d formed once per row and lane, the codes turned into floats by byte permutes
// into the mantissa of 2^23 (exact), fp32x2 FMAs into acc[b][j] (values 2j and 2j + 1) and
// the lane's offset terms x * m (one block, or one sub-block, per lane) summed apart in
// off[b].  The unit's bytes are in shared memory.

// 2^23 + byte j of x, as a float (exact)
__device__ __forceinline__ float bf(uint32_t x, int j) {
  return __uint_as_float(__byte_perm(x, 0x4b000000u, 0x7540u + (uint32_t)j));
}
__device__ __forceinline__ uint32_t s_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}
__device__ __forceinline__ uint32_t s_u32(const uint8_t* p) {  // 4-byte aligned
  return *reinterpret_cast<const uint32_t*>(p);
}
// 4 bytes at any offset
__device__ __forceinline__ uint32_t s_u32_any(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  return __funnelshift_r(q[0], q[1], (uint32_t)(a & 3u) * 8u);
}
// f[j] = bytes (2j, 2j+1) of the value bytes e0 (values 0-3) and e1 (4-7), minus `base`
__device__ __forceinline__ void pairs_from_bytes(uint32_t e0, uint32_t e1, float base, float2 (&f)[4]) {
  const float2 c = make_float2(base, base);
  f[0] = __fadd2_rn(make_float2(bf(e0, 0), bf(e0, 1)), c);
  f[1] = __fadd2_rn(make_float2(bf(e0, 2), bf(e0, 3)), c);
  f[2] = __fadd2_rn(make_float2(bf(e1, 0), bf(e1, 1)), c);
  f[3] = __fadd2_rn(make_float2(bf(e1, 2), bf(e1, 3)), c);
}
// f[j] = (byte j of lo, byte j of hi) minus `base`: the nibble layout of the 32-value
// types, where a byte holds values 2i (low nibble) and 2i + 1 (high)
__device__ __forceinline__ void pairs_lo_hi(uint32_t lo, uint32_t hi, float base, float2 (&f)[4]) {
  const float2 c = make_float2(base, base);
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = __fadd2_rn(make_float2(bf(lo, j), bf(hi, j)), c);
}
template <int B>
__device__ __forceinline__ void fma_rows(const float2 (&f)[4], const float (&s)[B], float2 (&acc)[B][4]) {
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float2 s2 = make_float2(s[b], s[b]);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[b][j] = __ffma2_rn(f[j], s2, acc[b][j]);
  }
}

constexpr float k2p23 = 8388608.0f;

template <int QT> struct Dot;

// Q4_0 (cpp/src/dequant.cpp:23-35): (q - 8) * d
template <> struct Dot<kQ4_0> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* unit, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&)[B], const uint2*) {
    const uint8_t* blk = unit + 18 * (lane >> 2);
    const float d = f16_ref(s_u16(blk));
    const uint32_t w = ld_u32_a2(blk + 2 + 4 * (lane & 3));
    float2 f[4];
    pairs_lo_hi(w & 0x0f0f0f0fu, (w >> 4) & 0x0f0f0f0fu, -(k2p23 + 8.f), f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) s[b] = x[b] * d;
    fma_rows<B>(f, s, acc);
  }
};

// Q4_1 (:40-53): d * q + m
template <> struct Dot<kQ4_1> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* unit, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&off)[B], const uint2*) {
    const uint8_t* blk = unit + 20 * (lane >> 2);
    const uint32_t dm = s_u32(blk);
    const float d = f16_ref(dm & 0xffffu), m = f16_ref(dm >> 16);
    const uint32_t w = s_u32(blk + 4 + 4 * (lane & 3));
    float2 f[4];
    pairs_lo_hi(w & 0x0f0f0f0fu, (w >> 4) & 0x0f0f0f0fu, -k2p23, f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      s[b] = x[b] * d;
      off[b] = fmaf(x[b], m, off[b]);
    }
    fma_rows<B>(f, s, acc);
  }
};

// Q5_0 (:58-73): (q - 16) * d, fifth bits in qh; lut[h] spreads the 8 fifth bits of a lane
// to bit 4 of the bytes of its (lo, hi) nibble words
template <> struct Dot<kQ5_0> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* unit, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&)[B], const uint2* lut) {
    const uint8_t* blk = unit + 22 * (lane >> 2);
    const float d = f16_ref(s_u16(blk));
    const uint32_t hb = (ld_u32_a2(blk + 2) >> (8 * (lane & 3))) & 0xffu;
    const uint32_t w = ld_u32_a2(blk + 6 + 4 * (lane & 3));
    const uint2 h = lut[hb];
    float2 f[4];
    pairs_lo_hi((w & 0x0f0f0f0fu) | h.x, ((w >> 4) & 0x0f0f0f0fu) | h.y, -(k2p23 + 16.f), f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) s[b] = x[b] * d;
    fma_rows<B>(f, s, acc);
  }
};

// Q5_1 (:78-93): d * q + m
template <> struct Dot<kQ5_1> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* unit, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&off)[B], const uint2* lut) {
    const uint8_t* blk = unit + 24 * (lane >> 2);
    const uint32_t dm = s_u32(blk);
    const float d = f16_ref(dm & 0xffffu), m = f16_ref(dm >> 16);
    const uint32_t hb = (s_u32(blk + 4) >> (8 * (lane & 3))) & 0xffu;
    const uint32_t w = s_u32(blk + 8 + 4 * (lane & 3));
    const uint2 h = lut[hb];
    float2 f[4];
    pairs_lo_hi((w & 0x0f0f0f0fu) | h.x, ((w >> 4) & 0x0f0f0f0fu) | h.y, -k2p23, f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      s[b] = x[b] * d;
      off[b] = fmaf(x[b], m, off[b]);
    }
    fma_rows<B>(f, s, acc);
  }
};

// Q2_K (:128-150): (d * (scale & 15)) * q + dmin; the lane's 8 values take the 4 codes of
// one byte twice (values i and i + 4 share a code)
template <> struct Dot<kQ2_K> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* blk, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&off)[B], const uint2*) {
    const int sb = lane >> 1;
    const uint32_t dd = s_u32(blk + 80);
    const float d = f16_ref(dd & 0xffffu), dmin = f16_ref(dd >> 16);
    const float dl = __fmul_rn(d, u2f(blk[sb] & 0xfu));
    const uint32_t q = blk[16 + 4 * sb + (lane & 1)];
    const float2 f01 = make_float2(u2f(q & 3u), u2f((q >> 2) & 3u));
    const float2 f23 = make_float2(u2f((q >> 4) & 3u), u2f(q >> 6));
    const float2 f[4] = {f01, f23, f01, f23};
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      s[b] = x[b] * dl;
      off[b] = fmaf(x[b], dmin, off[b]);
    }
    fma_rows<B>(f, s, acc);
  }
};

// Q3_K (:168-218): (d * scale) * (q + 8 h); 4 codes of one byte (each twice) plus the high
// bits of hmask bytes l0 .. l0 + 7, bit 4c + 2t (0 from a shift of 8 on)
template <> struct Dot<kQ3_K> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* blk, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&)[B], const uint2*) {
    const int c = lane >> 3, t = (lane >> 1) & 3, sh = 4 * c + 2 * t, j = 4 * c + t;
    const float d = f16_ref(s_u16(blk + 108));
    // get_scale_min_k3's scale of sub-block j without a branch (lanes hold different j):
    // byte j (j < 4), j + 4 (j < 8) or j - 4 (its high nibble) of the 12 scale bytes
    const int sidx = j < 4 ? j : (j < 8 ? j + 4 : j - 4);
    const uint32_t sb = blk[96 + sidx];
    const uint32_t scale = j < 8 ? (sb & 63u) : (sb >> 4);
    const float dt = __fmul_rn(d, u2f(scale));
    const uint32_t q = blk[32 + 16 * c + 4 * t + (lane & 1)];
    const uint32_t qrep = (q & 3u) | ((q & 0x0cu) << 6) | ((q & 0x30u) << 12) | ((q & 0xc0u) << 18);
    const uint8_t* hm = blk + 8 * (lane & 1);
    // high bits: bit sh of each hmask byte, none once sh reaches 8 (masked, not branched)
    const uint32_t keep = sh < 8 ? 0x01010101u : 0u;
    const uint32_t m0 = ((ld_u32_a2(hm) >> (sh & 7)) & keep) << 3;
    const uint32_t m1 = ((ld_u32_a2(hm + 4) >> (sh & 7)) & keep) << 3;
    float2 f[4];
    pairs_from_bytes(qrep + m0, qrep + m1, -k2p23, f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) s[b] = x[b] * dt;
    fma_rows<B>(f, s, acc);
  }
};

// Q5_K (:307-354): (d * sc) * q - dmin * m; chunk c reads its fifth bits from bytes
// 16 + 32c + l (bit 7 for the chunk's first half, bit 3 for its second)
template <> struct Dot<kQ5_K> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* blk, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&off)[B], const uint2*) {
    const int c = lane >> 3, half = (lane >> 2) & 1, l0 = 8 * (lane & 3);
    const uint32_t dd = s_u32(blk);
    const float d = f16_ref(dd & 0xffffu), dmin = f16_ref(dd >> 16);
    int sc, mn;  // sub-block 2c + half differs across the warp: the branch-free unpacking
    Q4kScaleRecipe(2 * c + half).apply(s_u32(blk + 4), s_u32(blk + 8), s_u32(blk + 12), sc, mn);
    const float d1 = __fmul_rn(d, u2f((uint32_t)sc)), m1 = __fmul_rn(dmin, u2f((uint32_t)mn));
    const uint8_t* qp = blk + 48 + 32 * c + l0;
    const uint8_t* hp = blk + 16 + 32 * c + l0;
    const uint32_t qsh = 4u * (uint32_t)half, hsh = 7u - 4u * (uint32_t)half;
    const uint32_t e0 = ((s_u32(qp) >> qsh) & 0x0f0f0f0fu) | (((s_u32(hp) >> hsh) & 0x01010101u) << 4);
    const uint32_t e1 = ((s_u32(qp + 4) >> qsh) & 0x0f0f0f0fu) | (((s_u32(hp + 4) >> hsh) & 0x01010101u) << 4);
    float2 f[4];
    pairs_from_bytes(e0, e1, -k2p23, f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      s[b] = x[b] * d1;
      off[b] = fmaf(-x[b], m1, off[b]);
    }
    fma_rows<B>(f, s, acc);
  }
};

// Q8_K (:226-245): q * (d * scale), int8 codes of 33-byte sub-blocks at odd offsets
template <> struct Dot<kQ8_K> {
  template <int B>
  __device__ __forceinline__ static void row(const uint8_t* blk, int lane, const float (&x)[B],
                                             float2 (&acc)[B][4], float (&)[B], const uint2*) {
    const float d = __uint_as_float(s_u32(blk));
    const uint8_t* sub = blk + 4 + 33 * (lane >> 2);
    const float ds = __fmul_rn(d, s8f(sub[32]));
    const uint8_t* q = sub + 8 * (lane & 3);
    float2 f[4];
    pairs_from_bytes(s_u32_any(q) ^ 0x80808080u, s_u32_any(q + 4) ^ 0x80808080u, -(k2p23 + 128.f), f);
    float s[B];
#pragma unroll
    for (int b = 0; b < B; ++b) s[b] = x[b] * ds;
    fma_rows<B>(f, s, acc);
  }
};

// the fifth-bit spread table of Q5_0 / Q5_1: entry h sets bit 4 of byte i of .x when bit 2i
// of h is set (values 0, 2, 4, 6) and of byte i of .y for bit 2i + 1 (values 1, 3, 5, 7)
template <int QT> struct UsesLut { static constexpr bool value = QT == kQ5_0 || QT == kQ5_1; };
// its place in shared memory: after the ring and the slice's activations, 16-byte aligned
__host__ __device__ __forceinline__ int lut_offset(int ring_bytes, int batch_rows, int kslice) {
  return (ring_bytes + batch_rows * kslice * 4 + 15) & ~15;
}
__device__ __forceinline__ uint2 fifth_bit_entry(uint32_t h) {
  uint2 e = make_uint2(0u, 0u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    e.x |= ((h >> (2 * i)) & 1u) << (8 * i + 4);
    e.y |= ((h >> (2 * i + 1)) & 1u) << (8 * i + 4);
  }
  return e;
}

// Copy rows [row0, row0 + rows) of the CTA's column chunk into a warp's stage: each row
// as the 16-byte granules that cover its chunk (its start rounded down to 16 bytes), one
// granule per lane at a time.  Rows keep their 4-byte offset inside the first granule.
template <int QT>
__device__ __forceinline__ void issue_rows(uint8_t* stage, const uint8_t* __restrict__ w, int64_t RB,
                                           int64_t col0, int row0, int rows, int lane) {
  using C = Cfg<QT>;
  for (int g = lane; g < rows * C::kGran; g += 32) {
    const int r = g / C::kGran, c = g - r * C::kGran;
    const int64_t start = (int64_t)(row0 + r) * RB + col0;
    const int o = (int)(start & 15);
    if (16 * c < o + C::kChunk) cp_async16(stage + r * C::kPitch + 16 * c, w + (start - o) + 16 * c);
  }
}

template <int QT, int B, bool SWIGLU>
__global__ void __launch_bounds__(kThreads)
gemv_stage_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w, float* y, Epi epi,
                  int K, int N, int64_t RB, int batch, int kslice) {
  using C = Cfg<QT>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  x += (int64_t)blockIdx.z * B * (SWIGLU ? 2 * (int64_t)K : (int64_t)K);
  y += (int64_t)blockIdx.z * B * N;
  if (epi.res) epi.res += (int64_t)blockIdx.z * B * N;
  batch = batch - (int)blockIdx.z * B < B ? batch - (int)blockIdx.z * B : B;
  const int64_t col0 = (int64_t)grp * C::kChunk;  // byte offset of the CTA's chunk in a row
  const int k0 = split * kslice;
  const int k1 = (k0 + kslice < K) ? k0 + kslice : K;
  const int nk = k1 - k0;
  // this warp's rows: a contiguous share of the slice, in stages of kWRows
  const int per = (nk + kWarps - 1) / kWarps;
  const int wr0 = k0 + min(nk, warp * per);
  const int wr1 = k0 + min(nk, (warp + 1) * per);
  const int nst = (wr1 - wr0 + kWRows - 1) / kWRows;
  uint8_t* const ring = smem + warp * C::kWarpRing;
  // a row's offset inside its first granule, (k * RB + col0) mod 16, from RB and col0 mod 16
  const uint32_t rb16 = (uint32_t)(RB & 15), c16 = (uint32_t)(col0 & 15);

  // prologue: the first kRing - 1 stages (weights only) before the dependency wait
#pragma unroll 1
  for (int s = 0; s < C::kRing - 1; ++s) {
    if (s < nst) {
      const int r0 = wr0 + s * kWRows;
      issue_rows<QT>(ring + s * C::kStage, w, RB, col0, r0, min(kWRows, wr1 - r0), lane);
    }
    cp_async_commit();
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x / res come from the previous grid

  // the slice's activations into shared memory, [b][k - k0], all loads issued before any
  // store (one round trip), read back per row without a global-memory wait
  float* const xs = reinterpret_cast<float*>(smem + C::kRingBytes);
#pragma unroll
  for (int b = 0; b < B; ++b) {
#pragma unroll 8
    for (int i = threadIdx.x; i < nk; i += kThreads)
      xs[b * nk + i] = (b < batch) ? gemv_x<SWIGLU>(x, b, K, k0 + i) : 0.f;
  }
  uint2* const lut = reinterpret_cast<uint2*>(smem + lut_offset(C::kRingBytes, B, kslice));
  if constexpr (UsesLut<QT>::value) lut[threadIdx.x] = fifth_bit_entry(threadIdx.x);
  __syncthreads();

  float2 acc[C::kC][B][4];
  float off[C::kC][B];
#pragma unroll
  for (int u = 0; u < C::kC; ++u)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      off[u][b] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[u][b][j] = make_float2(0.f, 0.f);
    }

  // the warp's own ring: no CTA-wide barrier in the loop
#pragma unroll 1
  for (int s = 0; s < nst; ++s) {
    cp_async_wait<C::kRing - 2>();
    __syncwarp();  // stage s has landed for every lane; stage s - 1 is consumed
    {
      const int sn = s + C::kRing - 1;  // refill the slot of stage s - 1
      if (sn < nst) {
        const int r0 = wr0 + sn * kWRows;
        issue_rows<QT>(ring + (sn % C::kRing) * C::kStage, w, RB, col0, r0, min(kWRows, wr1 - r0), lane);
      }
      cp_async_commit();
    }
    const uint8_t* stage = ring + (s % C::kRing) * C::kStage;
    const int kb = wr0 + s * kWRows;  // the stage's first row
    if (kb + kWRows <= wr1) {
      // a full stage: no per-row test, so the rows' shared-memory reads overlap
      float xv[kWRows][B];
#pragma unroll
      for (int r = 0; r < kWRows; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) xv[r][b] = xs[b * nk + (kb + r - k0)];
#pragma unroll
      for (int r = 0; r < kWRows; ++r) {
        const uint8_t* row = stage + r * C::kPitch + (int)(((uint32_t)(kb + r) * rb16 + c16) & 15u);
#pragma unroll
        for (int u = 0; u < C::kC; ++u)
          Dot<QT>::template row<B>(row + u * C::kUnit, lane, xv[r], acc[u], off[u], lut);
      }
    } else {
#pragma unroll 1
      for (int r = 0; r < wr1 - kb; ++r) {
        float xv[B];
#pragma unroll
        for (int b = 0; b < B; ++b) xv[b] = xs[b * nk + (kb + r - k0)];
        const uint8_t* row = stage + r * C::kPitch + (int)(((uint32_t)(kb + r) * rb16 + c16) & 15u);
#pragma unroll
        for (int u = 0; u < C::kC; ++u)
          Dot<QT>::template row<B>(row + u * C::kUnit, lane, xv, acc[u], off[u], lut);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // every copy has landed and every warp is done with its ring

  // ---- warps -> CTA sums (warp order) ----
  constexpr int kW = C::kC * 256;                                  // columns of the CTA
  float* red = reinterpret_cast<float*>(smem);                   // [warp][b][kW]
  float* cta_sum = red + kWarps * kMaxBatch * kW;                // [b][kW]
#pragma unroll
  for (int u = 0; u < C::kC; ++u)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float4* dst = reinterpret_cast<float4*>(red + (warp * kMaxBatch + b) * kW + u * 256 + 8 * lane);
      const float o = off[u][b];
      dst[0] = make_float4(acc[u][b][0].x + o, acc[u][b][0].y + o, acc[u][b][1].x + o, acc[u][b][1].y + o);
      dst[1] = make_float4(acc[u][b][2].x + o, acc[u][b][2].y + o, acc[u][b][3].x + o, acc[u][b][3].y + o);
    }
  __syncthreads();
  const int c = threadIdx.x;  // column of a unit this thread sums
#pragma unroll
  for (int u = 0; u < C::kC; ++u) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < kWarps; ++q) sum += red[(q * kMaxBatch + b) * kW + u * 256 + c];
      cta_sum[b * kW + u * 256 + c] = sum;
    }
  }
  // ---- K-slices -> the cluster leader (split order), then the output ----
  if (S > 1) gmma::cluster_sync_all();  // every CTA's sums are in its shared memory
  else __syncthreads();
  if (split == 0) {
    const uint32_t local = smem_u32(cta_sum);
#pragma unroll
    for (int u = 0; u < C::kC; ++u) {
      const int64_t n = ((int64_t)grp * C::kC + u) * 256 + c;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= batch) break;
        const int idx = b * C::kC * 256 + u * 256 + c;
        float sum = cta_sum[idx];
        for (int r = 1; r < S; ++r) sum += gmma::ld_cluster_f32(gmma::mapa_u32(local + (uint32_t)(idx * 4), (uint32_t)r));
        y[(int64_t)b * N + n] = epi_apply(epi, sum, b, N, n);
      }
    }
  }
  if (S > 1) gmma::cluster_sync_all();  // the leader's remote reads are done before exit
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// shared memory beyond which a call is left to the generic kernel (a K-slice's activations
// take B * kslice * 4 bytes beside the ring)
constexpr int kSmemCap = 200 * 1024;

template <int QT, int B, bool SW>
static cudaError_t launch_t(const float* x, const void* w, float* y, Epi epi, int64_t K, int64_t N,
                            int64_t RB, int batch, cudaStream_t st) {
  using C = Cfg<QT>;
  auto kern = gemv_stage_kernel<QT, B, SW>;
  static DeviceOnce configured;
  static DeviceSlots occupancy;  // resident CTAs per SM at a typical size, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads,
                                                      C::kRingBytes + B * 1024 * 4);
    if (e != cudaSuccess) return e;
    occupancy.set(dev, per_sm < 1 ? 1 : per_sm);
    configured.mark(dev);
  }
  const int groups = (int)(N / (256 * C::kC));
  const int zg = (batch + B - 1) / B;
  // splits: fill the resident CTA slots once (one wave), every warp of a split at least
  // one stage of rows
  constexpr int64_t kMinRows = (int64_t)kWarps * kWRows;
  const int64_t slots = (int64_t)occupancy.get(dev) * sm_count();
  int64_t S = slots / ((int64_t)groups * zg);
  const int64_t max_by_rows = (K + kMinRows - 1) / kMinRows;
  if (S > max_by_rows) S = max_by_rows;
  if (S > kMaxSplit) S = kMaxSplit;
  if (S < 1) S = 1;
  int64_t kslice = (K + S - 1) / S;
  kslice = (kslice + kMinRows - 1) / kMinRows * kMinRows;
  S = (K + kslice - 1) / kslice;
  if (S < 1) S = 1;
  int64_t smem = UsesLut<QT>::value ? lut_offset(C::kRingBytes, B, (int)kslice) + 256 * 8
                                    : C::kRingBytes + (int64_t)B * kslice * 4;
  if (smem < C::kRedBytes) smem = C::kRedBytes;
  if (smem > kSmemCap) return cudaErrorNotSupported;  // the caller uses the generic kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)groups, (unsigned)S, (unsigned)zg);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)S;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = S > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, x, static_cast<const uint8_t*>(w), y, epi, (int)K, (int)N, RB,
                            batch, (int)kslice);
}

template <int QT, bool SW>
static cudaError_t launch_b(const float* x, const void* w, float* y, Epi epi, int64_t K, int64_t N,
                            int64_t RB, int batch, cudaStream_t st) {
  if (batch <= 1) return launch_t<QT, 1, SW>(x, w, y, epi, K, N, RB, batch, st);
  if (batch <= 2) return launch_t<QT, 2, SW>(x, w, y, epi, K, N, RB, batch, st);
  return launch_t<QT, 4, SW>(x, w, y, epi, K, N, RB, batch, st);
}

template <int QT>
static cudaError_t launch_q(const float* x, const void* w, float* y, int64_t K, int64_t N, int64_t RB,
                            int batch, cudaStream_t st, const GemvFuse& f) {
  const Epi epi{f.bias, f.res};
  return f.swiglu_x ? launch_b<QT, true>(x, w, y, epi, K, N, RB, batch, st)
                    : launch_b<QT, false>(x, w, y, epi, K, N, RB, batch, st);
}

// N whole column groups; rows 4-byte aligned and w 16-byte aligned (granules start at
// 16-byte boundaries); K * RB a multiple of 16, so the granule that holds a matrix's last
// byte ends with it.
template <int QT>
static bool takes(int64_t K, int64_t N, int64_t RB, const void* w) {
  return N % (256 * Cfg<QT>::kC) == 0 && RB % 4 == 0 && (K * RB) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
}

}  // namespace gstage

bool gemv_stage_takes(int qtype, int64_t K, int64_t N, int64_t row_bytes, const void* w) {
  switch (qtype) {
    case kQ4_0: return gstage::takes<kQ4_0>(K, N, row_bytes, w);
    case kQ4_1: return gstage::takes<kQ4_1>(K, N, row_bytes, w);
    case kQ5_0: return gstage::takes<kQ5_0>(K, N, row_bytes, w);
    case kQ5_1: return gstage::takes<kQ5_1>(K, N, row_bytes, w);
    case kQ2_K: return gstage::takes<kQ2_K>(K, N, row_bytes, w);
    case kQ3_K: return gstage::takes<kQ3_K>(K, N, row_bytes, w);
    case kQ5_K: return gstage::takes<kQ5_K>(K, N, row_bytes, w);
    case kQ8_K: return gstage::takes<kQ8_K>(K, N, row_bytes, w);
    default: return false;
  }
}

cudaError_t launch_gemv_stage(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                              int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (batch < 1 || K < 1 || N < 1 || K > INT32_MAX || N > INT32_MAX) return cudaErrorInvalidValue;
  if ((batch + gstage::kMaxBatch - 1) / gstage::kMaxBatch > 65535) return cudaErrorInvalidValue;
  if (!gemv_stage_takes(qtype, K, N, row_bytes, w)) return cudaErrorInvalidValue;
  switch (qtype) {
    case kQ4_0: return gstage::launch_q<kQ4_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ4_1: return gstage::launch_q<kQ4_1>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_0: return gstage::launch_q<kQ5_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_1: return gstage::launch_q<kQ5_1>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ2_K: return gstage::launch_q<kQ2_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ3_K: return gstage::launch_q<kQ3_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_K: return gstage::launch_q<kQ5_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ8_K: return gstage::launch_q<kQ8_K>(x, w, y, K, N, row_bytes, batch, st, f);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vbq
