// vbq_gemv.cu -- fused dequant-GEMV for decode (batch 1..16) on sm_100a.
//
// Computes y[b, n] = sum_k x[b, k] * deq(W)[k, n] for W laid out like the reference's
// gemv_dequant (cpp/src/dequant.cpp:739-780): K rows, quant blocks along N.  The
// reference dequantizes each row into scratch and runs an axpy on one core; here the
// matrix streams through HBM once.
//
// Decomposition
//   * A CTA owns one 256-value column tile (one Q4_K / Q6_K block, or eight Q8_0 blocks,
//     per row) and a K-slice.  The grid is one wave (two CTAs per SM), so the split S over
//     K follows from the tile count.  Each CTA writes its tile's partial sums to the
//     caller's scratch; the CTA that finishes a tile last (atomic counter) adds the S
//     partials in split order and writes y -- deterministic -- and resets the counter,
//     leaving the scratch ready for the next call.
//   * Threads read their units (one row x VPT columns: the block header and the thread's
//     quant bytes) straight from global memory into registers, a few units ahead of the
//     math (software pipelining), with no shared-memory staging, barriers or waits in the
//     main loop: the weight stream is a plain coalesced load stream.  Shared memory is
//     kept small because it is carved out of the L1 the stream passes through.
//   * Launched with programmatic dependent launch: a GEMV queued behind another starts on
//     the SMs the previous one frees and streams its first weights before it waits for
//     the previous grid, which hides most of the launch gap and the split-K tail.
//   * A thread owns VPT output columns of the tile for B batch rows.  Integer work stays
//     off the half-rate ALU pipe where possible: one LOP3 turns two Q4_K nibbles (or two
//     Q8_0 bytes) into the fp16 pair (1024+q, 1024+q'), an exact integer that converts to
//     fp32 on the FMA pipe; Q6_K's 6-bit values are masked into the top mantissa bits of
//     the float 1 + u/64.  acc += (x * scale) * (offset + q) runs on packed fp32x2 FMAs;
//     the constant part (offset x scale, plus the Q4_K min term) is kept per sub-block and
//     subtracted from the accumulators every few rows, so the running sums never carry a
//     large offset.
//   Accuracy: fp32 products and sums throughout (max-norm relative error ~1e-5).
#include <cstdlib>

#include "vbq_common.cuh"
#include <atomic>

#include "vbq_internal.h"

namespace vbq {

// Sticky error bits raised by kernels of this file (kStatusTimeout: a bounded wait gave
// up).  The GEMV's main loop has no waits; the word is kept for the status API.
__device__ unsigned g_gemv_status = 0;

template <int QT, int B, int VPT>
struct GemvCfg {
  static constexpr int kThreads = 256;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kTPR = 256 / VPT;             // threads sharing one row's tile
  static constexpr int kRowLanes = kThreads / kTPR;  // rows the CTA works on side by side
  static constexpr int kTileBytes = Tile<QT>::kBytes;  // 144 / 210 / 272
  static constexpr int kUnroll = (B == 1 && QT != kQ8_0) ? 3 : 2;  // units in flight per thread
  static constexpr int kMinBlocks = (B <= 2) ? 2 : 1;  // CTAs per SM the registers allow
  static constexpr int kSets = kRowLanes;            // partial-sum sets per CTA
  // The reduction stages at most kRound sets (1 KB each) at a time: shared memory stays
  // small because it is carved out of the L1 cache the weight stream runs through (a
  // 64 KB carve-out measured ~1.6x slower streaming).
  static constexpr int kRound = kSets < 16 ? kSets : 16;
  // set stride 256 + kTPR floats: the 32 lanes of a warp store to 32 different banks
  static constexpr int kSetStride = 256 + kTPR;
  static constexpr int kRedBytes = kRound * kSetStride * 4;
  static constexpr int kOutBytes = B * 256 * 4;
  static constexpr int kSmem = kRedBytes + kOutBytes;
  static constexpr int kFlushEvery = 8;  // rows per thread between offset flushes
  static_assert(kTPR <= 32 && 32 % kTPR == 0, "a row's tile must fit in one warp");
  static_assert(kSets % kRound == 0, "reduction rounds");
};

__device__ __forceinline__ float fbits(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Nibbles at bits 0-3 and 16-19 of w -> (1024 + n0, 1024 + n1) as fp32, exact: one LOP3
// builds the fp16 pair (exponent of 1024, nibble in the low mantissa bits) and the pair
// converts on the FMA pipe.
__device__ __forceinline__ float2 h2f2(uint32_t w) {
  const uint32_t h = (w & 0x000f000fu) | 0x64006400u;
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// Bytes at bits 0-7 and 16-23 of w -> (1024 + b0, 1024 + b1) as fp32, exact.
__device__ __forceinline__ float2 h2f2_byte(uint32_t w) {
  const uint32_t h = (w & 0x00ff00ffu) | 0x64006400u;
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// Small non-negative integer v (< 2^23) times d, exactly as d * (float)v rounds: the float
// 2^23 + v is built with one OR and the FMA computes d*(2^23+v) - d*2^23 with one rounding.
__device__ __forceinline__ float mul_small(float d, float d_2p23, uint32_t v) {
  return fmaf(d, __uint_as_float(0x4b000000u | v), -d_2p23);
}

// ---------------------------------------------------------------------------------
// Per-type row math.  A thread owns VPT columns of the 256-value tile; acc[b][p] holds
// two values (packed for fma.rn.f32x2) and corr[b][g] the offset of value group g.
// col_of(c, t) maps value t of thread-chunk c to its column in the tile.
// ---------------------------------------------------------------------------------
template <int QT, int B, int VPT>
struct RowMath;

// Q4_K.  A thread owns bytes [32g+bo, 32g+bo+VPT/2) of the block's qs: their low
// nibbles are columns 64g+bo+t (sub-block 2g), their high nibbles 64g+32+bo+t
// (sub-block 2g+1).  Pair p of the accumulators holds bytes (j, j+2) of word w of the
// span: p = 2w + j (low nibbles) and kBPT/2 + 2w + j (high nibbles).
template <int B, int VPT>
struct RowMath<kQ4_K, B, VPT> {
  static constexpr int kBPT = VPT / 2;   // qs bytes per thread
  static constexpr int kGroups = 2;      // [0] low-nibble sub-block, [1] high
  static constexpr int kP = VPT / 2;     // float2 accumulators per batch row
  __device__ __forceinline__ static void cols(int c, int& g, int& bo) {
    constexpr int tpg = 32 / kBPT;       // threads per 64-value group
    g = c / tpg;
    bo = (c % tpg) * kBPT;
  }
  __device__ __forceinline__ static int col_of(int c, int t) {
    int g, bo;
    cols(c, g, bo);
    const int p = t >> 1, e = t & 1;
    const bool high = p >= kBPT / 2;
    const int q = high ? p - kBPT / 2 : p;
    return 64 * g + (high ? 32 : 0) + bo + 4 * (q >> 1) + (q & 1) + 2 * e;
  }
  __device__ __forceinline__ static int group_of(int t) { return (t >> 1) < kBPT / 2 ? 0 : 1; }

  // Raw bytes of one (row, thread-chunk) unit: the 16-byte block header and the thread's
  // qs bytes, loaded straight from global memory (header through L1: the 4 threads of a
  // row share it; qs streamed past L1).
  struct Frag {
    uint4 h;
    uint32_t w[kBPT / 4];
  };
  __device__ __forceinline__ static void load(Frag& f, const uint8_t* __restrict__ rp, int c) {
    int g, bo;
    cols(c, g, bo);
    f.h = __ldg(reinterpret_cast<const uint4*>(rp));
    const uint8_t* qp = rp + 16 + 32 * g + bo;
    if constexpr (kBPT >= 16) {
#pragma unroll
      for (int i = 0; i < kBPT / 16; ++i) {
        const uint4 t = __ldcs(reinterpret_cast<const uint4*>(qp) + i);
        f.w[4 * i] = t.x; f.w[4 * i + 1] = t.y; f.w[4 * i + 2] = t.z; f.w[4 * i + 3] = t.w;
      }
    } else if constexpr (kBPT == 8) {
      const uint2 t = __ldcs(reinterpret_cast<const uint2*>(qp));
      f.w[0] = t.x; f.w[1] = t.y;
    } else {
      f.w[0] = __ldcs(reinterpret_cast<const unsigned*>(qp));
    }
  }

  // Sub-block scales and mins of the thread's group g: scale/min pairs (2g, 2g+1) as
  // 16-bit lanes of one word each, unpacked SIMD-within-a-register.
  __device__ __forceinline__ static void scales(const uint4& h, int g, uint32_t& sc, uint32_t& mn) {
    const int sh = 16 * (g & 1);
    if (g < 2) {  // get_scale_min_k4, j < 4: low 6 bits of bytes j (scales) and j+4 (mins)
      sc = (h.y >> sh) & 0x3f3fu;
      mn = (h.z >> sh) & 0x3f3fu;
    } else {      // j >= 4: low/high nibble of byte j+4, top 2 bits of bytes j-4 / j
      sc = ((h.w >> sh) & 0x0f0fu) | ((h.y >> (sh + 2)) & 0x3030u);
      mn = ((h.w >> (sh + 4)) & 0x0f0fu) | ((h.z >> (sh + 2)) & 0x3030u);
    }
  }

  __device__ __forceinline__ static void run(const Frag& f, const float* xv, int c,
                                             float2 (&acc)[B][kP], float (&corr)[B][kGroups]) {
    int g, bo;
    cols(c, g, bo);
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&f.h.x));
    // the reference's fp16 conversion doubles subnormals (cpp/src/fp16_compat.cpp:13-35)
    const float d = ((f.h.x & 0x7c00u) == 0u) ? 2.0f * dd.x : dd.x;
    const float dmin = ((f.h.x & 0x7c000000u) == 0u) ? 2.0f * dd.y : dd.y;
    uint32_t sc, mn;
    scales(f.h, g, sc, mn);
    const float d23 = d * 8388608.0f, m23 = dmin * 8388608.0f;
    const float s_lo = mul_small(d, d23, sc & 0xffu);
    const float s_hi = mul_small(d, d23, sc >> 8);
    const float c_lo = fmaf(1024.0f, s_lo, mul_small(dmin, m23, mn & 0xffu));
    const float c_hi = fmaf(1024.0f, s_hi, mul_small(dmin, m23, mn >> 8));
    float alo[B], ahi[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      alo[b] = xv[b] * s_lo;
      ahi[b] = xv[b] * s_hi;
      corr[b][0] = fmaf(xv[b], c_lo, corr[b][0]);
      corr[b][1] = fmaf(xv[b], c_hi, corr[b][1]);
    }
#pragma unroll
    for (int wi = 0; wi < kBPT / 4; ++wi) {
      const float2 lo02 = h2f2(f.w[wi]);
      const float2 hi02 = h2f2(f.w[wi] >> 4);
      const float2 lo13 = h2f2(f.w[wi] >> 8);
      const float2 hi13 = h2f2(f.w[wi] >> 12);
      const int pl = 2 * wi, ph = kBPT / 2 + 2 * wi;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float2 al = f2(alo[b], alo[b]), ah = f2(ahi[b], ahi[b]);
        acc[b][pl] = __ffma2_rn(lo02, al, acc[b][pl]);
        acc[b][pl + 1] = __ffma2_rn(lo13, al, acc[b][pl + 1]);
        acc[b][ph] = __ffma2_rn(hi02, ah, acc[b][ph]);
        acc[b][ph + 1] = __ffma2_rn(hi13, ah, acc[b][ph + 1]);
      }
    }
  }
};

// Q6_K (reference layout): u = lo | hi<<4 in 0..63 as the float 1 + u/64 (bits 17-22);
// int8 scale per 16 values.  A thread owns VPT consecutive columns.
template <int B, int VPT>
struct RowMath<kQ6_K, B, VPT> {
  static constexpr int kGroups = VPT >= 16 ? VPT / 16 : 1;
  static constexpr int kP = VPT / 2;
  __device__ __forceinline__ static int col_of(int c, int t) { return c * VPT + t; }
  __device__ __forceinline__ static int group_of(int t) { return t >> 4; }

  // Q6_K blocks sit at 2-byte alignment; the unit's bytes are read with aligned 32-bit
  // loads inside run(), so the fragment is just the block's address.
  struct Frag {
    const uint8_t* p;
  };
  __device__ __forceinline__ static void load(Frag& f, const uint8_t* __restrict__ rp, int) {
    f.p = rp;
  }
  __device__ __forceinline__ static void run(const Frag& f, const float* xv, int c,
                                             float2 (&acc)[B][kP], float (&corr)[B][kGroups]) {
    const uint8_t* __restrict__ bp = f.p;
    const int v0 = c * VPT;
    const float d = f16_ref(ld_u16(bp + 208));
    uint32_t ql[VPT / 8];
#pragma unroll
    for (int i = 0; i < VPT / 8; ++i) ql[i] = ld_u32_a2(bp + (v0 >> 1) + 4 * i);
    uint32_t qh[(VPT + 15) / 16];
    if constexpr (VPT >= 16) {
#pragma unroll
      for (int i = 0; i < VPT / 16; ++i) qh[i] = ld_u32_a2(bp + 128 + (v0 >> 2) + 4 * i);
    } else {
      qh[0] = ld_u16(bp + 128 + (v0 >> 2));
    }
    float a[kGroups][B];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
      const int sc = (int)(int8_t)bp[192 + (v0 >> 4) + g];
      const float ds64 = d * (float)(64 * sc);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        a[g][b] = xv[b] * ds64;
        corr[b][g] = fmaf(1.5f, a[g][b], corr[b][g]);
      }
    }
#pragma unroll
    for (int p = 0; p < VPT / 2; ++p) {
      float fv[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = 2 * p + e;
        const uint32_t lq = ql[t >> 3], hq = qh[t >> 4];
        const int sl = 17 - 4 * (t & 7), sh = 21 - 2 * (t & 15);
        const uint32_t lo = sl >= 0 ? (lq << sl) : (lq >> -sl);
        const uint32_t hi = sh >= 0 ? (hq << sh) : (hq >> -sh);
        fv[e] = fbits((lo & 0x001e0000u) | (hi & 0x00600000u) | 0x3f800000u);
      }
      const int g = (2 * p) >> 4;
#pragma unroll
      for (int b = 0; b < B; ++b)
        acc[b][p] = __ffma2_rn(f2(fv[0], fv[1]), f2(a[g][b], a[g][b]), acc[b][p]);
    }
  }
};

// Q8_0 (GGUF block): u = q + 128 in 0..255 as 1024 + u (fp16 pair per LOP3, exact).
// Pair p = 2w + j of a block holds columns (4w + j, 4w + j + 2).
template <int B, int VPT>
struct RowMath<kQ8_0, B, VPT> {
  static constexpr int kBlocks = VPT >= 32 ? VPT / 32 : 1;
  static constexpr int kGroups = kBlocks;
  static constexpr int kP = VPT / 2;
  static constexpr int kVB = VPT >= 32 ? 32 : VPT;  // values per block handled
  __device__ __forceinline__ static int col_of(int c, int t) {
    const int blk = t / kVB, tt = t % kVB;
    const int p = tt >> 1, e = tt & 1;
    return c * VPT + blk * kVB + 4 * (p >> 1) + (p & 1) + 2 * e;
  }
  __device__ __forceinline__ static int group_of(int t) { return t / kVB; }

  // VPT >= 32: the thread's kBlocks blocks are contiguous (34 bytes each, 2-byte
  // aligned) and are read as the aligned 32-bit words covering them.  VPT < 32: the
  // block's fp16 scale plus the thread's VPT quant bytes.  Realigned in registers.
  static constexpr int kSpanBytes = VPT >= 32 ? kBlocks * 34 : VPT;
  static constexpr int kWords = (kSpanBytes + 2 + 3) / 4;
  struct Frag {
    uint32_t w[kWords];
    uint32_t sh;     // span misalignment * 8 (0 or 16)
    uint32_t dbits;  // fp16 scale (VPT < 32 only)
  };
  __device__ __forceinline__ static void load(Frag& f, const uint8_t* __restrict__ rp, int c) {
    const int v0 = c * VPT;
    const uint8_t* bp = rp + 34 * (v0 >> 5);
    const uint8_t* sp = bp;
    if constexpr (VPT < 32) {
      f.dbits = __ldg(reinterpret_cast<const unsigned short*>(bp));
      sp = bp + 2 + (v0 & 31);
    } else {
      f.dbits = 0;
    }
    const uintptr_t a = reinterpret_cast<uintptr_t>(sp);
    const unsigned* q = reinterpret_cast<const unsigned*>(a & ~uintptr_t(3));
    f.sh = (uint32_t)(a & 3u) * 8u;
    // the last word is only read when it holds data (misaligned span)
    const int nw = f.sh ? kWords : (kSpanBytes + 3) / 4;
#pragma unroll
    for (int i = 0; i < kWords; ++i) f.w[i] = (i < nw) ? __ldcs(q + i) : 0u;
  }
  // 4 bytes at an even byte offset of the span
  __device__ __forceinline__ static uint32_t word(const Frag& f, int byte_off) {
    const int i = byte_off >> 2;
    const uint32_t sh = f.sh + (uint32_t)(byte_off & 3) * 8u;  // 0, 16 or 32
    if (sh == 0) return f.w[i];
    if (sh == 32) return f.w[i + 1];
    return __funnelshift_r(f.w[i], f.w[i + 1], sh);
  }
  __device__ __forceinline__ static void run(const Frag& f, const float* xv, int c,
                                             float2 (&acc)[B][kP], float (&corr)[B][kGroups]) {
#pragma unroll
    for (int blk = 0; blk < kBlocks; ++blk) {
      const int base = VPT >= 32 ? blk * 34 : 0;  // block start inside the span
      const uint32_t dbits = VPT >= 32 ? (word(f, base) & 0xffffu) : f.dbits;
      const float d = f16_ieee(dbits);
      float a[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        a[b] = xv[b] * d;
        corr[b][blk] = fmaf(1152.0f, a[b], corr[b][blk]);
      }
#pragma unroll
      for (int wi = 0; wi < kVB / 4; ++wi) {
        const int off = VPT >= 32 ? base + 2 + 4 * wi : 4 * wi;
        const uint32_t ww = word(f, off) ^ 0x80808080u;
        const float2 f02 = h2f2_byte(ww);
        const float2 f13 = h2f2_byte(ww >> 8);
        const int p = (blk * kVB) / 2 + 2 * wi;
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const float2 ab = f2(a[b], a[b]);
          acc[b][p] = __ffma2_rn(f02, ab, acc[b][p]);
          acc[b][p + 1] = __ffma2_rn(f13, ab, acc[b][p + 1]);
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------------

template <int QT, int B, int VPT, bool SWIGLU>
__global__ void __launch_bounds__(256, GemvCfg<QT, B, VPT>::kMinBlocks) gemv_kernel(const float* __restrict__ x,
                                                   const uint8_t* __restrict__ w,
                                                   float* y, int64_t K, int64_t N,
                                                   int64_t RB, int64_t kslice, int batch,
                                                   float* __restrict__ partials,
                                                   unsigned* __restrict__ counters, Epi epi) {
  using C = GemvCfg<QT, B, VPT>;
  using M = RowMath<QT, B, VPT>;
  using Frag = typename M::Frag;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int s_last;

  const int64_t tile = blockIdx.x;
  const int split = blockIdx.y;
  const int S = gridDim.y;
  const int64_t k0 = (int64_t)split * kslice;
  const int64_t k1 = (k0 + kslice < K) ? k0 + kslice : K;

  const int tid = threadIdx.x;
  const int c = tid % C::kTPR;   // column chunk of the tile
  const int rl = tid / C::kTPR;  // row lane of the CTA
  // rows of this thread: k0 + rl + i * kRowLanes
  const int64_t span = k1 - k0;
  const int nrows = span > rl ? (int)((span - rl + C::kRowLanes - 1) / C::kRowLanes) : 0;

  float2 acc[B][M::kP];
  float corr[B][M::kGroups];
#pragma unroll
  for (int b = 0; b < B; ++b) {
#pragma unroll
    for (int p = 0; p < M::kP; ++p) acc[b][p] = f2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < M::kGroups; ++g) corr[b][g] = 0.f;
  }
  auto flush = [&]() {
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
      for (int p = 0; p < M::kP; ++p) {
        acc[b][p].x -= corr[b][M::group_of(2 * p)];
        acc[b][p].y -= corr[b][M::group_of(2 * p + 1)];
      }
#pragma unroll
      for (int g = 0; g < M::kGroups; ++g) corr[b][g] = 0.f;
    }
  };

  const uint8_t* wrow = w + (k0 + rl) * RB + tile * C::kTileBytes;  // this thread's first row
  const int64_t wstep = (int64_t)C::kRowLanes * RB;
  const int64_t kx0 = k0 + rl;  // this thread's first row (the x index)

  // Programmatic dependent launch: let the next kernel in the stream start filling SMs as
  // this grid drains, and stream the first weight units before waiting for the previous
  // grid (weights never depend on it; x, y and the scratch may).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Software pipeline: kUnroll units in flight; a unit's slot is refilled right after use.
  Frag f[C::kUnroll];
  float xs[C::kUnroll][B];
#pragma unroll
  for (int u = 0; u < C::kUnroll; ++u)
    if (u < nrows) M::load(f[u], wrow + u * wstep, c);
  asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
  for (int u = 0; u < C::kUnroll; ++u) {
    if (u < nrows) {
#pragma unroll
      for (int b = 0; b < B; ++b)
        xs[u][b] = (b < batch) ? gemv_x<SWIGLU>(x, b, K, kx0 + u * C::kRowLanes) : 0.f;
    }
  }
  int since_flush = 0;
  for (int i = 0; i < nrows; i += C::kUnroll) {
#pragma unroll
    for (int u = 0; u < C::kUnroll; ++u) {
      if (i + u < nrows) {
        const Frag cur = f[u];
        float xv[B];
#pragma unroll
        for (int b = 0; b < B; ++b) xv[b] = xs[u][b];
        const int nx = i + u + C::kUnroll;
        if (nx < nrows) {
          M::load(f[u], wrow + nx * wstep, c);
#pragma unroll
          for (int b = 0; b < B; ++b)
            xs[u][b] = (b < batch) ? gemv_x<SWIGLU>(x, b, K, kx0 + (int64_t)nx * C::kRowLanes) : 0.f;
        }
        M::run(cur, xv, c, acc, corr);
      }
    }
    since_flush += C::kUnroll;
    if (since_flush >= C::kFlushEvery) {
      flush();
      since_flush = 0;
    }
  }
  flush();

  // ---- reduce all partial-sum sets of the CTA into outbuf[B][256] (set order fixed) ----
  // Set rl stores value t of thread-chunk c at [rl][t * kTPR + c] (bank-conflict free with
  // the padded set stride); thread tid then owns slot (t, c) = (tid / kTPR, tid % kTPR)
  // and adds it over the sets, reading consecutive words.
  float* red = reinterpret_cast<float*>(smem);
  float* outbuf = reinterpret_cast<float*>(smem + C::kRedBytes);
  const int my_t = tid / C::kTPR, my_c = tid % C::kTPR;
  const int my_col = M::col_of(my_c, my_t);
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float sum = 0.f;
#pragma unroll 1
    for (int r0 = 0; r0 < C::kSets; r0 += C::kRound) {
      if (rl >= r0 && rl < r0 + C::kRound) {
        float* dst = red + (rl - r0) * C::kSetStride + c;
#pragma unroll
        for (int p = 0; p < M::kP; ++p) {
          dst[(2 * p) * C::kTPR] = acc[b][p].x;
          dst[(2 * p + 1) * C::kTPR] = acc[b][p].y;
        }
      }
      __syncthreads();
      float part[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains: short dependency path
#pragma unroll
      for (int s2 = 0; s2 < C::kRound; ++s2) part[s2 & 3] += red[s2 * C::kSetStride + tid];
      sum += (part[0] + part[1]) + (part[2] + part[3]);
      __syncthreads();
    }
    outbuf[b * 256 + my_col] = sum;
  }
  __syncthreads();

  const int E = batch * 256;
  if (S == 1) {
    for (int e = tid; e < E; e += C::kThreads)
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = epi_apply(epi, outbuf[e], e >> 8, N, tile * 256 + (e & 255));
    return;
  }

  // ---- split-K: publish this CTA's partial; the last CTA of the tile adds them up ----
  for (int e = tid; e < E; e += C::kThreads)
    partials[((int64_t)split * batch + (e >> 8)) * N + tile * 256 + (e & 255)] = outbuf[e];
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&counters[tile], 1u) == (unsigned)(S - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = tid; e < E; e += C::kThreads) {
    const int b = e >> 8, n = e & 255;
    float sum = 0.f;
    for (int sp = 0; sp < S; ++sp)
      sum += __ldcg(partials + ((int64_t)sp * batch + b) * N + tile * 256 + n);
    y[(int64_t)b * N + tile * 256 + n] = epi_apply(epi, sum, b, N, tile * 256 + n);
  }
  if (tid == 0) counters[tile] = 0u;  // leave the scratch ready for the next call
}

// ---------------------------------------------------------------------------------
// Launch planning: one wave of CTAs (two per SM), split-K factor from the tile count.
// ---------------------------------------------------------------------------------
constexpr int kGemvMinRows = 64, kGemvMaxSplit = 64;

// SM count per device ordinal (atomic cache: first calls may come from several threads)
int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int gemv_split_override() {
  // tuning override, read once (thread-safe static initialisation)
  static const int v = [] {
    const char* env = getenv("VBQ_GEMV_SPLIT");
    const int e = env ? atoi(env) : 0;
    return (e >= 1 && e <= kGemvMaxSplit) ? e : 0;
  }();
  return v;
}

// VBQ_GEMV_SCALAR=1 routes Q4_K, Q6_K and Q8_0 to the scalar kernel (comparison runs).
static bool scalar_override() {
  static const bool v = [] {
    const char* env = getenv("VBQ_GEMV_SCALAR");
    return env && atoi(env) == 1;
  }();
  return v;
}

GemvPlan plan_gemv(int64_t K, int64_t N, int batch, int qtype) {
  GemvPlan p{};
  if (!scalar_override() && ((qtype == kQ4_K && gemv_mma_fits(K, N, batch)) ||
                             (qtype == kQ6_K && gemv_q6_fits(K, N, batch)) ||
                             (qtype == kQ8_0 && gemv_q8_fits(K, N, batch)))) {
    p.splits = 1;  // chosen at launch; the splits reduce in a cluster, without scratch
    p.kslice = K;
    return p;
  }
  const int64_t tiles = N / 256;
  const int64_t slots = (batch <= 2 ? 2LL : 1LL) * sm_count();  // one wave (kMinBlocks)
  int64_t S = tiles > 0 ? slots / tiles : 1;
  const int64_t s_rows = (K + kGemvMinRows - 1) / kGemvMinRows;  // >= 64 rows per CTA
  if (S > s_rows) S = s_rows;
  if (S > kGemvMaxSplit) S = kGemvMaxSplit;
  if (S < 1) S = 1;
  if (gemv_split_override()) S = gemv_split_override();
  // K-slices of whole 128-row stages (the tensor-core kernel's stage height)
  int64_t kslice = (K + S - 1) / S;
  kslice = (kslice + 127) / 128 * 128;
  S = (K + kslice - 1) / kslice;
  if (S < 1) S = 1;
  p.splits = (int)S;
  p.kslice = kslice;
  p.counter_bytes = S > 1 ? ((tiles * 4 + 255) / 256) * 256 : 0;
  p.scratch_bytes = S > 1 ? (size_t)p.counter_bytes + (size_t)S * batch * N * sizeof(float) : 0;
  return p;
}

template <int QT, int B, int VPT, bool SW>
static cudaError_t launch_gemv_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, const GemvPlan& plan, void* scratch,
                                 cudaStream_t st, Epi epi) {
  using C = GemvCfg<QT, B, VPT>;
  auto kern = gemv_kernel<QT, B, VPT, SW>;
  static DeviceOnce configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    // keep shared memory to what two CTAs need; the rest stays L1 for the weight stream
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 25);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  unsigned* counters = static_cast<unsigned*>(scratch);
  float* partials = plan.splits > 1
                        ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + plan.counter_bytes)
                        : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)plan.splits, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, x, static_cast<const uint8_t*>(w), y, K, N, RB,
                            plan.kslice, batch, partials, counters, epi);
}

template <int QT, bool SW>
static cudaError_t launch_gemv_q(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, const GemvPlan& p, void* scratch,
                                 cudaStream_t st, Epi e) {
  if (batch <= 1) {
    if constexpr (QT == kQ8_0) return launch_gemv_t<QT, 1, 32, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
    else return launch_gemv_t<QT, 1, 64, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
  }
  if (batch <= 2) return launch_gemv_t<QT, 2, 32, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
  if (batch <= 4) return launch_gemv_t<QT, 4, 16, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
  if (batch <= 8) return launch_gemv_t<QT, 8, 8, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
  return launch_gemv_t<QT, 16, 8, SW>(x, w, y, K, N, RB, batch, p, scratch, st, e);
}

template <int QT>
static cudaError_t launch_gemv_f(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, const GemvPlan& p, void* scratch,
                                 cudaStream_t st, const GemvFuse& f) {
  const Epi e{f.bias, f.res};
  return f.swiglu_x ? launch_gemv_q<QT, true>(x, w, y, K, N, RB, batch, p, scratch, st, e)
                    : launch_gemv_q<QT, false>(x, w, y, K, N, RB, batch, p, scratch, st, e);
}

cudaError_t launch_gemv(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                        int64_t row_bytes, int batch, const GemvPlan& plan, void* scratch,
                        cudaStream_t st, const GemvFuse& f) {
  if (N % 256 != 0 || batch < 1 || batch > 16) return cudaErrorNotSupported;
  switch (qtype) {
    case kQ4_K:
      if (!scalar_override() && gemv_mma_fits(K, N, batch))
        return launch_gemv_mma_q4k(x, w, y, K, N, row_bytes, batch, st, f);
      return launch_gemv_f<kQ4_K>(x, w, y, K, N, row_bytes, batch, plan, scratch, st, f);
    case kQ6_K:
      if (!scalar_override() && gemv_q6_fits(K, N, batch))
        return launch_gemv_q6_mma(x, w, y, K, N, row_bytes, batch, st, f);
      return launch_gemv_f<kQ6_K>(x, w, y, K, N, row_bytes, batch, plan, scratch, st, f);
    case kQ8_0:
      if (!scalar_override() && gemv_q8_fits(K, N, batch))
        return launch_gemv_q8_mma(x, w, y, K, N, row_bytes, batch, st, f);
      return launch_gemv_f<kQ8_0>(x, w, y, K, N, row_bytes, batch, plan, scratch, st, f);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemv_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
