// vbq_gemv_q6.cu -- Q6_K dequant-GEMV on the integer tensor cores (decode, batch 1).
//
//   y[n] = sum_k x[k] * deq(W)[k, n],   deq(W)[k, n] = (d[k] * sc[k, s]) * (u[k, n] - 32)
//
// with the reference's Q6_K block (cpp/src/dequant.cpp:359-402): 256 values in 210 bytes,
// ql[128] @0 (value i: nibble i & 1 of byte i >> 1), qh[64] @128 (value i: 2-bit field
// i & 3 of byte i >> 2), int8 scales[16] @192 (s = i >> 4), fp16 d @208; u = lo | hi << 4.
// Regrouped as
//   y[n] = sum_k u[k, n] * v[k, s]  -  32 * sum_k v[k, s],   v = x * (d * sc),
// the first term runs on mma.sync m16n8k32 (u8 x s8 -> s32), two instructions per 1024
// weights, the second in fp32 on the side:
//   * A (16 columns x 32 rows): the 6-bit codes u as exact u8.  A pair p of ql bytes
//     (2p, 2p + 1) holds values 4p .. 4p + 3 and shares qh byte p.  M-tile row g of a
//     16-byte ql chunk is the pair's even byte, row g + 8 its odd byte; the low-nibble
//     MMA takes values 4p and 4p + 2, the high-nibble MMA 4p + 1 and 4p + 3.  Each lane
//     loads its fragment bytes itself (a 16-bit load of its pair per row, an 8-bit load
//     of its qh byte per row): Q6_K blocks are only 2-byte aligned in a row, so the rows
//     cannot go through ldmatrix without first being copied to aligned addresses.  Four
//     PRMTs turn four rows' pairs into the even- and odd-byte registers, three PRMTs the
//     qh bytes, and one LOP3 per register merges nibble and high bits.
//   * B (32 rows x 8): v as a 22-bit fixed-point integer n on a power-of-two scale per
//     warp, in three signed byte digits (the 1.5 * 2^23 magic, as in vbq_gemv_mma.cu).
//     A chunk covers two 16-column sub-blocks (pairs 8c .. 8c + 3 and 8c + 4 .. 8c + 7),
//     so B columns 0-2 hold the digits of the first sub-block's v and 4-6 the second's;
//     columns 3 and 7 are all ones, so the MMA also yields sum u, and the digit offset
//     comes off in int32.  Every B column is used.
//   * The s32 accumulators run across the CTA's stages; a stage whose |v| outgrows the
//     scale, or whose sampled |v| all sit 16x below it, moves the sums to fp32 and sets
//     the scale again (warp-uniform; rare on ordinary activations).
// Accuracy: each v is rounded to 2^-20 of the warp's largest |v| in the stage that set the
// scale (headroom 2-4x), products and sums exact, fp32 at the end.  A non-finite v marks
// the warp's 128 outputs NaN.
//
// Decomposition: a CTA owns one 256-column tile (one block per row) and every S-th 128-row
// stage of the matrix; the S splits of a tile form one thread-block cluster and add up in
// split 0's shared memory (st.async), as in vbq_gemv_mma.cu.
// Staging: a row pitch RB = 210 N / 256 is only 2-byte aligned, but rows k = c + 8i of one
// class c lie 8 RB apart, a multiple of 16 bytes.  So each class has its own 2-D tensor
// map (base: the row-c start rounded down to 16 bytes; x in bytes), and a stage is eight
// TMA boxes of 16 rows x 224 bytes, the 16-byte-aligned window that holds the tile's block
// in each row (the block sits at byte o = its address mod 16 of the window, the same o for
// the whole class).  Per-row bulk copies (128 per stage) measured 2.6x slower than the
// scalar kernel: the copy engine's cost per request dominates.  The maps end at each row's
// last byte and at K, so the boxes zero-fill past the matrix.
// Stage row r sits at (r mod 8) x 3584 + 224 (r / 8).  The MMA's reduction index k of a
// warp (rows 32q .. 32q + 31) maps to stage row 32q + 8t + 4h + j for k = 16h + 4t + j, so
// the four rows of one fragment load (t = 0..3) sit 224 bytes apart in one box: distinct
// 32-byte bank windows, and every 16-bit fragment load is one wavefront.
// Warps: eight per CTA, two CTAs per SM (128 registers a thread), each warp 32 rows x 128
// columns of a stage: the B table for its rows, then 4 x 2 MMAs.  There is no producer
// warp: a 3-slot ring per CTA, the first stages issued at the start, and the last warp to
// finish a slot (a shared counter) refills it with the stage three further on.  The ALU
// pipe bounds the kernel (code building and byte packing; the tensor pipe is ~8 % busy), so
// fragment rows are packed with multiply-adds on the FMA pipe.  Waits are bounded.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "vbq_common.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up).
__device__ unsigned g_gemv_q6_status = 0;

namespace gq6 {

using gmma::kMagic;
using gmma::kExpMin;
using gmma::kExpMax;
using gmma::pow2f;
using gmma::inv_pow2;
using gmma::mma_u8s8;
using gmma::mbar_wait_hinted;
using gmma::cluster_arrive;
using gmma::cluster_wait;
using gmma::cluster_rank;
using gmma::mapa_u32;
using gmma::st_async_v4;

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * kConsumers;  // no producer warp: the last warp through a slot refills it
constexpr int kRows = 16 * kConsumers;  // rows per stage
constexpr int kBlock = 210;             // bytes of one Q6_K block
constexpr int kWin = 224;               // loaded window per row (covers o + 210, o <= 14)
constexpr int kBoxRows = kRows / 8;     // rows of one class in a stage
constexpr int kBoxBytes = kBoxRows * kWin;  // 3584 = 28 x 128: boxes stay 128-byte aligned
// stage row r: box r mod 8, row r / 8 of the box
__host__ __device__ constexpr int line_off(int r) { return (r & 7) * kBoxBytes + kWin * (r >> 3); }
constexpr int kStageBytes = 8 * kBoxBytes;  // 28672
// B table per warp: [4 chunks][8 columns][32 rows] s8, rows ordered so that lane (g, t)'s
// two fragment words are adjacent (one 8-byte load at byte 8t of column g); chunk stride
// 288 B keeps the table stores of the four chunks on different banks.
constexpr int kColStride = 32;
constexpr int kChunkStride = 288;
constexpr int kTblBytes = 4 * kChunkStride;

// the eight class maps (a grid constant: 1 KB of kernel parameters)
struct ClassMaps {
  CUtensorMap m[8];
};

constexpr int kMaxStages = 6;
struct Bars {
  uint64_t full[kMaxStages];
  uint64_t red;               // the cluster leader's: the other splits' partial sums have landed
  unsigned done[kMaxStages];  // warps through the slot's current stage
  int abort;
  int issued;                 // stages whose boxes have been issued
};
static_assert(sizeof(Bars) <= 128, "barrier block");
constexpr int kMaxSplit = 16;

// Per batch size.  Batch 1: two CTAs per SM (126 registers) with a 3-slot ring each.
// Batch 2 and 4: more sets of accumulators and tables need more registers, so one CTA per
// SM with a 6- / 5-slot ring (batch 4 at 255 registers spills ~130 bytes).  Shared memory: the ring, one B table per warp and batch row, the
// barriers, and the cluster leader's receive slots (sized at launch).
template <int BATCH>
struct Cfg {
  static constexpr int kStages = BATCH == 1 ? 3 : (BATCH == 2 ? 6 : 5);
  static constexpr int kMinBlocks = BATCH == 1 ? 2 : 1;
  static constexpr int kSmemCap = (BATCH == 1 ? 113 : 227) * 1024;
  static constexpr int kTblOff = kStages * kStageBytes;
  static constexpr int kBarOff = kTblOff + kConsumers * BATCH * kTblBytes;
  static constexpr int kRecvOff = kBarOff + 128;
  static constexpr int kSmemBase = kRecvOff + 128;  // + alignment slack
  static_assert(kStages <= kMaxStages, "barrier block");
  // per-warp outputs and the CTA's sum reuse the ring after the main loop
  static_assert(kConsumers * BATCH * 128 * 4 + BATCH * 256 * 4 <= kStages * kStageBytes,
                "reduction buffer inside the ring");
};

// 16- / 8-bit shared loads at a 32-bit shared address, zero-extended
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
// atomic add on a shared word with acquire-release ordering at CTA scope; returns the old value
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old) : "r"(smem_u32(p)), "r"(v) : "memory");
  return old;
}
// a * m + b on the FMA pipe (packing disjoint bit fields without the ALU pipe)
__device__ __forceinline__ uint32_t mad_u32(uint32_t a, uint32_t m, uint32_t b) {
  uint32_t d;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(m), "r"(b));
  return d;
}

// batch: rows of x and y present (1 .. BATCH)
template <int BATCH, bool SWIGLU>
__global__ void __launch_bounds__(kThreads, Cfg<BATCH>::kMinBlocks)
gemv_q6_kernel(const __grid_constant__ ClassMaps maps, const float* __restrict__ x, float* y,
               int K, int N, int64_t RB, int batch, Epi epi) {
  using C = Cfg<BATCH>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte aligned: TMA box destinations
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  Bars& bars = *reinterpret_cast<Bars*>(smem + C::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 128-row stages split, split + S, split + 2S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  // Offset of a row's block in its 16-byte window: (k RB + 210 tile) mod 16 (w is 16-byte
  // aligned).  Stages start at multiples of 128 rows, so it depends only on the row's
  // place r in the stage.
  const int rb15 = (int)(RB & 15), t15 = (tile * kBlock) & 15;
  auto off_of = [&](int r) { return (r * rb15 + t15) & 15; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      bars.done[s] = 0u;
    }
    mbar_init(smem_u32(&bars.red), 1);
    bars.abort = 0;
    bars.issued = nst < kStages ? nst : kStages;
    mbar_fence_init();
  }
  __syncthreads();
  if (S > 1) cluster_arrive();  // barriers initialised; waited for before any remote store
  // Programmatic dependent launch: weights are streamed before waiting for the previous
  // grid (they never depend on it), x, y and the cluster exchange only after.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_q6_status, kStatusTimeout);
  };

  // flushed fp32 sums [batch row][chunk][low / high nibbles] of the lane's MMA row (g for
  // t even, g + 8 for t odd), the sums of v for the lane's two table sub-blocks per batch
  // row, non-finite flags (bit b)
  float fac[BATCH][4][2];
  float2 sv[BATCH];
#pragma unroll
  for (int b = 0; b < BATCH; ++b) {
#pragma unroll
    for (int c = 0; c < 4; ++c) fac[b][c][0] = fac[b][c][1] = 0.f;
    sv[b] = make_float2(0.f, 0.f);
  }
  unsigned nonfin = 0u;

  // Stage loads: class c's box at x = the window of the tile's block in map c, y = the
  // stage's first row of the class; classes without rows (K < 8) have no map and load
  // nothing.  One warp issues a stage: lane 0 sets the byte count, lanes 0 .. 7 a box each.
  const int n_cls = K < 8 ? K : 8;
  const int xw = ((((int)(RB & 15) * (lane & 7)) & 15) + tile * kBlock) & ~15;
  auto load_stage = [&](int sidx, int slot) {
    const uint32_t fb = smem_u32(&bars.full[slot]);
    if (lane == 0) mbar_arrive_expect_tx(fb, (uint32_t)(n_cls * kBoxBytes));
    __syncwarp();
    if (lane < n_cls)
      gmma::tma_load_2d(smem_u32(smem + slot * kStageBytes + lane * kBoxBytes), &maps.m[lane], xw,
                        (split + S * sidx) * kBoxRows, fb);
  };
  // the first stages: weights never depend on the previous grid
  if (warp == 0)
    for (int s = 0; s < kStages && s < nst; ++s) load_stage(s, s);

  {
    // warp: columns 128 gp .. + 127 and rows rw .. rw + 31 of each stage
    const int gp = warp & 1, rw = 32 * (warp >> 1);
    const int g = lane >> 2, t = lane & 3;   // MMA fragment role
    const int m = lane & 7, cc = lane >> 3;  // table role: rows 4m .. 4m + 3, chunk cc
    // the warp's B tables, one per batch row
    uint8_t* tbl = smem + C::kTblOff + warp * BATCH * kTblBytes;
    for (int i = lane; i < BATCH * 4 * 2 * 8; i += 32) {  // all-ones columns 3 and 7 of each chunk
      const int w8 = i & 7, c2 = (i >> 3) & 1, ch = (i >> 4) & 3, tb = i >> 6;
      reinterpret_cast<uint32_t*>(tbl + tb * kTblBytes + ch * kChunkStride + (3 + 4 * c2) * kColStride)[w8] =
          0x01010101u;
    }
    // Fragment loads, k = 4t + j (j < 4) and 16 + 4t + (j - 4): warp rows 8t + j and
    // 8t + 4 + (j - 4); the pair of m-tile row g in chunk c is 8c + g, its ql bytes at
    // o + 64 gp + 2 (8c + g), its qh byte at o + 128 + 32 gp + 8c + g.  The offsets are the
    // same in every stage; a row's qh byte sits qh_d bytes after its ql pair.  Above batch
    // 2, where registers are short, the qh (and scale) addresses are formed from that
    // distance; below, they are kept (measured 2 % faster at batch 1).
    int ql_off[8], qh_off[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = rw + 8 * t + j;
      ql_off[j] = line_off(r) + off_of(r) + 64 * gp + 2 * g;
      qh_off[j] = ql_off[j] + 128 - 32 * gp - g;
    }
    const uint32_t qh_d = (uint32_t)(128 - 32 * gp - g);
    // table rows k = 4m + j: warp rows 8 (m & 3) + 4 (m >> 2) + j (consecutive); d at o + 208,
    // the scale pair (sub-blocks 8 gp + 2 cc, + 1) at o + 192 + 8 gp + 2 cc
    const int trow = rw + 8 * (m & 3) + 4 * (m >> 2);
    int d_off[4], sc_off[4];
    const int sc_d = 8 * gp + 2 * cc - 16;  // the scale pair, relative to d
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = trow + j;
      d_off[j] = line_off(r) + off_of(r) + 208;
      sc_off[j] = d_off[j] + sc_d;
    }
    // the lane's table words: chunk cc, k = 4m .. 4m + 3 (byte 8 (m & 3) + 4 (m >> 2) of a
    // column); its B fragments: column g, k = 4t .. 4t + 3 and 16 + 4t .. 16 + 4t + 3
    uint8_t* const tcol = tbl + cc * kChunkStride + 8 * (m & 3) + 4 * (m >> 2);
    const uint8_t* const tfrag = tbl + g * kColStride + 8 * t;
    __syncwarp();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    int acc[BATCH][4][2][4];  // [batch row][chunk][low / high nibbles][fragment]
    float scale[BATCH];       // powers of two; the step of v is 1 / scale
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      scale[b] = 1.f;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[b][c][h][0] = acc[b][c][h][1] = acc[b][c][h][2] = acc[b][c][h][3] = 0;
    }
    // bit b: batch row b's scale may come down (a present row whose scale was not set from
    // an all-zero stage)
    uint32_t down_ok = 0u;
    // s32 sums -> fp32.  Lanes t even hold digits 0, 1 of their sub-block, lanes t odd digit
    // 2 and the code sum S.  With the top digit centred (d2 - 64 per code) the pair's parts
    // are (a0 + 256 a1) and (65536 (a2 - 64 S) + 32896 S): the int32 difference is exact and
    // the fp32 terms stay within 2^-20 of the result.
    auto flush = [&]() {
      const int odd = t & 1;
      const float c1 = odd ? 65536.f : 1.f, c2 = odd ? 32896.f : 256.f;
      const int cen = odd ? 64 : 0;
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const float sb = inv_pow2(scale[b]);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int* a = acc[b][c][h];
            const float p0 = fmaf(c2, (float)a[1], c1 * (float)(a[0] - cen * a[1]));
            const float p1 = fmaf(c2, (float)a[3], c1 * (float)(a[2] - cen * a[3]));
            // the pair's halves: lane t even keeps row g, lane t odd row g + 8
            const float mine = odd ? p1 : p0, other = odd ? p0 : p1;
            const float sum = mine + __shfl_xor_sync(0xffffffffu, other, 1);
            fac[b][c][h] = fmaf(sum, sb, fac[b][c][h]);
            a[0] = a[1] = a[2] = a[3] = 0;
          }
      }
    };

    // x of the lane's table rows, two stages ahead (one above batch 2, where registers
    // are short)
    constexpr int kAhead = BATCH > 2 ? 1 : 2;
    int kx = split * kRows + trow;
    const int kstep = S * kRows;
    auto load_x = [&](int k, float (&xv)[BATCH][4]) {
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[b][j] = (b < batch && k + j < K) ? gemv_x<SWIGLU>(x, b, K, k + j) : 0.f;
    };
    float xn[BATCH][4], xnn[BATCH][4];
    load_x(kx, xn);
    if constexpr (kAhead == 2) {
      kx += kstep;
      load_x(kx, xnn);
    }
#pragma unroll 1
    for (int it = 0; it < nst; ++it) {
      const int u = it % kStages;
      const uint32_t par = (uint32_t)(it / kStages) & 1u;
      float xv[BATCH][4];
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          xv[b][j] = xn[b][j];
          if constexpr (kAhead == 2) xn[b][j] = xnn[b][j];
        }
      kx += kstep;
      if constexpr (kAhead == 2) load_x(kx, xnn);  // rows of the stage after next (zero past K)
      else load_x(kx, xn);                         // rows of the next stage
      if (!__all_sync(0xffffffffu, mbar_wait_hinted(smem_u32(&bars.full[u]), par, kWaitBudgetCycles))) {
        if (lane == 0) give_up();
        break;
      }
      const uint8_t* st = smem + u * kStageBytes;
      const int krow = (split + S * it) * kRows + trow;  // the lane's first table row
      // ---- v = x * (d * sc) of rows trow + j, sub-blocks (2 cc, 2 cc + 1) of the warp ----
      float2 v[BATCH][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t dh = *reinterpret_cast<const uint16_t*>(st + d_off[j]);
        const int so = BATCH > 2 ? d_off[j] + sc_d : sc_off[j];
        const uint32_t sp = (uint32_t)*reinterpret_cast<const uint16_t*>(st + so) ^ 0x8080u;
        // the int8 scales as floats: byte ^ 0x80 into the 2^23 magic, minus 2^23 + 128 (exact)
        const float2 sc = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(sp, 0x4b000000u, 0x7650)),
                                                 __uint_as_float(__byte_perm(sp, 0x4b000000u, 0x7651))),
                                     make_float2(-8388736.f, -8388736.f));
        const float d = f16_ref(dh);
        // d * sc is the reference's fp32 scale (exact product); rows past K are zero-filled
        const float2 dl = __fmul2_rn(make_float2(d, d), sc);
        const bool live = krow + j < K;
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          v[b][j] = live ? __fmul2_rn(make_float2(xv[b][j], xv[b][j]), dl) : make_float2(0.f, 0.f);
          sv[b] = __fadd2_rn(sv[b], v[b][j]);
        }
      }
      // v on the current scale: 1.5 * 2^23 + n in the float, in range exactly when the float
      // keeps the exponent of 2^23 (|n| < 2^22); NaN, inf and overflow leave it
      uint32_t wd[BATCH][4][2];
      uint32_t out = 0u, small = 0u;
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          wd[b][j][0] = __float_as_uint(fmaf(v[b][j].x, scale[b], kMagic));
          wd[b][j][1] = __float_as_uint(fmaf(v[b][j].y, scale[b], kMagic));
          out |= (wd[b][j][0] ^ 0x4b000000u) | (wd[b][j][1] ^ 0x4b000000u);
        }
        // the shrink test: one sampled value per lane and batch row, |n| < 2^16 <=>
        // w - (1.5 * 2^23 - 2^16) below 2^17 (an out-of-range word fails it and rescales
        // through `out` anyway)
        small |= (wd[b][0][0] - 0x4b3f0000u < 0x20000u) ? (1u << b) : 0u;
      }
      const bool shrink = __reduce_and_sync(0xffffffffu, small & down_ok) != 0u;
      if (__any_sync(0xffffffffu, out >= (1u << 23)) || shrink || it == 0) {
        // rare (and the first stage): flag non-finite values, move the sums to fp32, then
        // scale each batch row to 2-4x the warp's largest finite |v| and encode again.  The
        // max ignores NaN and is capped so that huge values do not rescale every stage.
        if (it > 0) flush();
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          float sum = 0.f, mx = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sum += fabsf(v[b][j].x) + fabsf(v[b][j].y);
            mx = fmaxf(mx, fmaxf(fabsf(v[b][j].x), fabsf(v[b][j].y)));
          }
          nonfin |= (sum < 0x1p100f) ? 0u : (1u << b);  // NaN / inf propagate
          mx = fminf(mx, 0x1p99f);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          int e = (int)((__float_as_uint(mx) >> 23) & 0xffu) - 127 + 1;
          e = e < kExpMin ? kExpMin : (e > kExpMax ? kExpMax : e);
          scale[b] = pow2f(21 - e);
          down_ok = (b < batch && e > kExpMin) ? (down_ok | (1u << b)) : (down_ok & ~(1u << b));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            wd[b][j][0] = __float_as_uint(fmaf(v[b][j].x, scale[b], kMagic));
            wd[b][j][1] = __float_as_uint(fmaf(v[b][j].y, scale[b], kMagic));
          }
        }
      }
      // ---- B tables: three signed digits of n, four rows per word, per sub-block ----
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t a0 = wd[b][0][h], a1 = wd[b][1][h], a2 = wd[b][2][h], a3 = wd[b][3][h];
          const uint32_t t01 = __byte_perm(a0, a1, 0x5140), t23 = __byte_perm(a2, a3, 0x5140);
          const uint32_t u01 = __byte_perm(a0, a1, 0x0062), u23 = __byte_perm(a2, a3, 0x0062);
          uint8_t* col = tcol + b * kTblBytes + 4 * h * kColStride;
          *reinterpret_cast<uint32_t*>(col) = __byte_perm(t01, t23, 0x5410) ^ 0x80808080u;
          *reinterpret_cast<uint32_t*>(col + kColStride) = __byte_perm(t01, t23, 0x7632) ^ 0x80808080u;
          *reinterpret_cast<uint32_t*>(col + 2 * kColStride) = __byte_perm(u01, u23, 0x5410);
        }
      __syncwarp();
      // ---- 4 chunks of 8 pairs x 32 rows: low- and high-nibble MMAs ----
      // the fragment rows' shared addresses in this stage (chunk c adds 16c / 8c)
      uint32_t qa[8], ha[8];
      const uint32_t stb = smem_u32(st);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        qa[j] = stb + (uint32_t)ql_off[j];
        ha[j] = BATCH > 2 ? qa[j] + qh_d : stb + (uint32_t)qh_off[j];
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ev[2], od[2], hq[2];  // [rows 4t.. / 16 + 4t..]: even bytes, odd bytes, qh
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t q[4], hb[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            q[j] = lds_u16(qa[4 * hh + j] + 16u * c);
            hb[j] = lds_u8(ha[4 * hh + j] + 8u * c);
          }
          // rows j = 0..3 of the pair (even byte, odd byte) and of the qh byte, packed by
          // multiply-adds; two PRMTs split even and odd bytes
          const uint32_t p01 = mad_u32(q[1], 65536u, q[0]), p23 = mad_u32(q[3], 65536u, q[2]);
          ev[hh] = __byte_perm(p01, p23, 0x6420);
          od[hh] = __byte_perm(p01, p23, 0x7531);
          hq[hh] = mad_u32(mad_u32(hb[3], 256u, hb[2]), 65536u, mad_u32(hb[1], 256u, hb[0]));
        }
        // codes u = nibble | field << 4 (u8 0..63).  f02 holds fields 0 / 2 at bits 0-1 / 4-5
        // of each byte, f13 fields 1 / 3; the masks keep each byte's bits 6-7 zero.
        // (right shifts as mul.hi on the FMA pipe measured 5 % slower than these)
        uint32_t alo[4], ahi[4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t f02 = hq[hh] & 0x33333333u, f13 = (hq[hh] >> 2) & 0x33333333u;
          alo[2 * hh] = (ev[hh] & 0x0f0f0f0fu) | ((f02 * 16u) & 0xf0f0f0f0u);      // value 4p
          alo[2 * hh + 1] = (od[hh] & 0x0f0f0f0fu) | (f02 & 0xf0f0f0f0u);         // value 4p + 2
          ahi[2 * hh] = ((ev[hh] >> 4) & 0x0f0f0f0fu) | ((f13 * 16u) & 0xf0f0f0f0u);  // 4p + 1
          ahi[2 * hh + 1] = ((od[hh] >> 4) & 0x0f0f0f0fu) | (f13 & 0xf0f0f0f0u);     // 4p + 3
        }
        // fragment order: a0 row g k 0-15, a1 row g + 8, a2 row g k 16-31, a3 row g + 8;
        // one A for every batch row
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const uint2 bf = *reinterpret_cast<const uint2*>(tfrag + b * kTblBytes + c * kChunkStride);
          mma_u8s8(acc[b][c][0], alo[0], alo[1], alo[2], alo[3], bf.x, bf.y);
          mma_u8s8(acc[b][c][1], ahi[0], ahi[1], ahi[2], ahi[3], bf.x, bf.y);
        }
      }
      __syncwarp();  // table and stage reads done
      // the last warp through slot u refills it with stage it + kStages: the warps' reads
      // of the slot come before their count (the __syncwarp above, then a release), the
      // count before the refill (acquire), and the proxy fence orders them before the
      // asynchronous copy
      unsigned last = 0u;
      if (lane == 0) last = atom_add_acq_rel(&bars.done[u], 1u) == (unsigned)(kConsumers - 1);
      if (__shfl_sync(0xffffffffu, last, 0)) {
        if (lane == 0) bars.done[u] = 0u;
        if (it + kStages < nst) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          load_stage(it + kStages, u);
          if (lane == 0) atomicMax(&bars.issued, it + kStages + 1);
        }
      }
    }
    flush();
    // sums of v over the lane's group (lanes 8 cc .. 8 cc + 7); flags over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      if (o < 8) {
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          sv[b].x += __shfl_xor_sync(0xffffffffu, sv[b].x, o);
          sv[b].y += __shfl_xor_sync(0xffffffffu, sv[b].y, o);
        }
      }
      nonfin |= __shfl_xor_sync(0xffffffffu, nonfin, o);
    }
  }

  // ---- per-warp outputs -> shared memory (the stage ring, now idle) ----
  __syncthreads();
  if (*abort_flag) {
    // a wait gave up: boxes may still be landing in the ring; they land (bounded) first
    if (threadIdx.x == 0) {
      const int is = bars.issued;
      for (int j = is > kStages ? is - kStages : 0; j < is; ++j)
        mbar_wait_bounded(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    __syncthreads();
  }
  float* red = reinterpret_cast<float*>(smem);  // [warp][batch row][the warp's 128 columns]
  {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        // sums of v of chunk c's sub-blocks sit in lanes 8c .. 8c + 7
        const float sx = __shfl_sync(0xffffffffu, sv[b].x, 8 * c);
        const float sy = __shfl_sync(0xffffffffu, sv[b].y, 8 * c);
        // lanes whose MMA rows (pairs 8c + g: sub-block g >> 2) met the B columns of that
        // sub-block (t >> 1) hold outputs: row g (t even) / g + 8 (t odd) of the chunk,
        // i.e. values 32c + 4g + 2 (t & 1) + h
        if ((t >> 1) == (g >> 2) && b < batch) {
          const float off = 32.f * ((g >> 2) ? sy : sx);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            red[(warp * BATCH + b) * 128 + 32 * c + 4 * g + 2 * (t & 1) + h] =
                ((nonfin >> b) & 1u) ? __int_as_float(0x7fc00000) : fac[b][c][h] - off;
        }
      }
  }
  __syncthreads();

  // ---- sum the warps in order: this CTA's partial y, [batch row][256] ----
  const int E = batch * 256;
  float* outbuf = red + kConsumers * BATCH * 128;  // after the per-warp slots, still in the ring
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, half = (e >> 7) & 1, cl = e & 127;
    float v = 0.f;
    for (int w2 = half; w2 < kConsumers; w2 += 2) v += red[(w2 * BATCH + b) * 128 + cl];  // this half's warps
    outbuf[e] = v;
  }
  __syncthreads();

  if (S == 1) {
    for (int e = threadIdx.x; e < E; e += kThreads) {
      const int b = e >> 8, n = tile * 256 + (e & 255);
      y[(int64_t)b * N + n] = epi_apply(epi, outbuf[e], b, N, n);
    }
    return;
  }
  // ---- split-K inside the cluster: splits 1 .. S-1 push their partials into the leader's
  // slots (st.async, counted on its barrier) and exit; the leader adds them in split order
  cluster_wait();  // every CTA of the cluster has initialised its barriers
  const uint32_t rank = cluster_rank();
  float* recv = reinterpret_cast<float*>(smem + C::kRecvOff);
  if (rank != 0) {
    const uint32_t dst = mapa_u32(smem_u32(recv + (rank - 1) * E), 0u);
    const uint32_t bar = mapa_u32(smem_u32(&bars.red), 0u);
    for (int e4 = threadIdx.x; e4 < E / 4; e4 += kThreads)
      st_async_v4(dst + 16u * (uint32_t)e4, reinterpret_cast<const float4*>(outbuf)[e4], bar);
    return;
  }
  if (threadIdx.x == 0) mbar_arrive_expect_tx(smem_u32(&bars.red), (uint32_t)((S - 1) * E * 4));
  if (!mbar_wait_bounded(smem_u32(&bars.red), 0, kWaitBudgetCycles) && threadIdx.x == 0) give_up();
  for (int e = threadIdx.x; e < E; e += kThreads) {
    float sum = outbuf[e];
    for (int sp = 1; sp < S; ++sp) sum += recv[(sp - 1) * E + e];
    const int b = e >> 8, n = tile * 256 + (e & 255);
    y[(int64_t)b * N + n] = epi_apply(epi, sum, b, N, n);
  }
}

}  // namespace gq6

// ---- host side -----------------------------------------------------------------------

static gmma::EncodeTiledFn encode_fn_q6() {
  static gmma::EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<gmma::EncodeTiledFn>(p);
  });
  return fn;
}

// The eight class maps of a K x RB Q6_K matrix at w (16-byte aligned): map c covers rows
// c, c + 8, ... as a u8 array of (RB + delta_c) bytes per row, 8 RB apart, from the row-c
// start rounded down to 16 bytes (delta_c = c RB mod 16 bytes before it); boxes of 224 bytes
// x 16 rows.  Each host thread keeps the last few sets it encoded.  Returns false when
// encoding fails.
static bool class_maps(gmma::EncodeTiledFn enc, const void* w, int64_t K, int64_t RB, gq6::ClassMaps* out) {
  struct Entry {
    gq6::ClassMaps maps;
    const void* w;
    int64_t K, RB;
    bool valid;
  };
  thread_local Entry cache[4] = {};
  const uintptr_t key = (reinterpret_cast<uintptr_t>(w) >> 8) ^ (uintptr_t)K ^ ((uintptr_t)RB << 3);
  Entry& e = cache[(key ^ (key >> 5)) & 3];
  if (e.valid && e.w == w && e.K == K && e.RB == RB) {
    *out = e.maps;
    return true;
  }
  e.valid = false;
  for (int c = 0; c < 8; ++c) {
    if (c >= K) {  // no rows in this class: never loaded
      memset(&e.maps.m[c], 0, sizeof(CUtensorMap));
      continue;
    }
    const uintptr_t start = reinterpret_cast<uintptr_t>(w) + (uintptr_t)(c * RB);
    const uintptr_t base = start & ~uintptr_t(15);
    cuuint64_t dims[2] = {(cuuint64_t)(RB + (int64_t)(start - base)), (cuuint64_t)((K - c + 7) / 8)};
    cuuint64_t strides[1] = {(cuuint64_t)(8 * RB)};
    cuuint32_t box[2] = {(cuuint32_t)gq6::kWin, (cuuint32_t)gq6::kBoxRows};
    cuuint32_t es[2] = {1, 1};
    if (enc(&e.maps.m[c], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, reinterpret_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  e.w = w, e.K = K, e.RB = RB, e.valid = true;
  *out = e.maps;
  return true;
}

// Splits per tile: one wave (Cfg::kMinBlocks CTAs per SM) when the tiles fit in it, with
// room for every tile's cluster at once and 25 % to spare (cudaOccupancyMaxActiveClusters,
// cached per shape); two splits past half a wave of tiles; at most 16 (one cluster) and
// the leader's receive slots (batch KB per split) inside the shared-memory budget.
template <int BATCH, bool SW>
static int choose_splits_q6(int64_t K, int64_t N, int batch) {
  using namespace gq6;
  using C = Cfg<BATCH>;
  const int tiles = (int)(N / 256);
  const int64_t tot_st = (K + kRows - 1) / kRows;
  const int slots = C::kMinBlocks * sm_count();
  int S = tiles > 0 ? slots / tiles : 1;
  // More tiles than half the slots: two splits, unless one already fills 85 % of a wave.
  // Each SM runs its CTAs at a fixed rate (the ALU pipe bounds the kernel), so CTAs half as
  // long even out the SMs' loads and shorten the last wave.  Measured (us, K = 4096, one /
  // two splits): 192 tiles 52.2 / 44.6, 256 tiles 52.2 / 54.9, 400 tiles 83.7 / 81.8,
  // 501 tiles 101.6 / 97.9, 593 tiles 128.9 / 120.8.
  if (S < 2) S = (tiles <= slots && tiles * 100 >= 85 * slots) ? 1 : 2;
  if (S > kMaxSplit) S = kMaxSplit;
  if (S > tot_st) S = (int)tot_st;
  if (S < 1) S = 1;
  const int slot_bytes = batch * 1024;
  if (gemv_split_override()) {
    S = gemv_split_override() > kMaxSplit ? kMaxSplit : gemv_split_override();
    if (S > tot_st) S = (int)tot_st;
    while (S > 1 && C::kSmemBase + (S - 1) * slot_bytes > C::kSmemCap) --S;
    return S;
  }
  while (S > 1 && C::kSmemBase + (S - 1) * slot_bytes > C::kSmemCap) --S;
  if ((int64_t)tiles * S > slots) return S;  // several waves by design: pairs place anywhere
  struct Entry { int64_t tiles; int batch, s_in, s_out; };
  static Entry cache[32];
  static int n_cache = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_cache; ++i)
    if (cache[i].tiles == tiles && cache[i].batch == batch && cache[i].s_in == S) return cache[i].s_out;
  const int s_in = S;
  for (; S > 1; --S) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)S, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBase + (S - 1) * slot_bytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, gq6::gemv_q6_kernel<BATCH, SW>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      active = 0;
    }
    if (active * 4 >= tiles * 5) break;
  }
  if (n_cache < 32) cache[n_cache++] = Entry{tiles, batch, s_in, S};
  return S;
}

template <int BATCH, bool SW>
static cudaError_t launch_q6_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t RB, int batch, cudaStream_t st, Epi epi) {
  using namespace gq6;
  using C = Cfg<BATCH>;
  auto enc = encode_fn_q6();
  if (!enc) return cudaErrorNotSupported;
  ClassMaps maps;
  if (!class_maps(enc, w, K, RB, &maps)) return cudaErrorInvalidValue;
  auto kern = gemv_q6_kernel<BATCH, SW>;
  static DeviceOnce configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemCap);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  const int S = choose_splits_q6<BATCH, SW>(K, N, batch);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemBase + (S - 1) * batch * 1024;
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
  return cudaLaunchKernelEx(&cfg, kern, maps, x, y, (int)K, (int)N, RB, batch, epi);
}

// Whether the tensor-core Q6_K kernel takes this call: batch 1 to 16 (groups of 4 above 4),
// whole 256-column tiles, and K up to 2^17 (the s32 sums hold at most K / 4 x 32 terms below 64 x 128 in
// magnitude, well inside 2^31).  The weights must be 16-byte aligned (the C ABI requires it).
constexpr int64_t kQ6MaxK = 131072;
bool gemv_q6_fits(int64_t K, int64_t N, int batch) {
  return batch >= 1 && batch <= 16 && K >= 1 && K <= kQ6MaxK && N % 256 == 0 && N > 0;
}

// Up to 4 batch rows in one launch.
static cudaError_t launch_q6_rows(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                  int64_t row_bytes, int batch, cudaStream_t st, bool sw, Epi epi) {
  if (batch == 1)
    return sw ? launch_q6_t<1, true>(x, w, y, K, N, row_bytes, 1, st, epi)
              : launch_q6_t<1, false>(x, w, y, K, N, row_bytes, 1, st, epi);
  // batch 3-4 on the 4-row form: measured against two 2-row launches (the weights streamed
  // twice) at batch 4, 4096 x 128256 239 vs 323 us, 14336 x 4096 39.7 vs 52.5 us
  if (batch > 2)
    return sw ? launch_q6_t<4, true>(x, w, y, K, N, row_bytes, batch, st, epi)
              : launch_q6_t<4, false>(x, w, y, K, N, row_bytes, batch, st, epi);
  return sw ? launch_q6_t<2, true>(x, w, y, K, N, row_bytes, batch, st, epi)
            : launch_q6_t<2, false>(x, w, y, K, N, row_bytes, batch, st, epi);
}

// Batch 5-16 as consecutive launches over groups of 4 rows (each streams the weights again).
cudaError_t launch_gemv_q6_mma(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_q6_fits(K, N, batch) || (reinterpret_cast<uintptr_t>(w) & 15u) != 0 ||
      row_bytes != (N / 256) * gq6::kBlock)
    return cudaErrorNotSupported;
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int b0 = 0; b0 < batch; b0 += 4) {
    const int nb = batch - b0 < 4 ? batch - b0 : 4;
    const Epi epi{f.bias, f.res ? f.res + (int64_t)b0 * N : nullptr};
    cudaError_t e = launch_q6_rows(x + (int64_t)b0 * xrow, w, y + (int64_t)b0 * N, K, N, row_bytes, nb, st,
                                   f.swiglu_x, epi);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t gemv_q6_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_q6_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_q6_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
