// vbq_gemv_mma.cu -- Q4_K dequant-GEMV on the integer tensor cores (decode, batch 1..4).
//
//   y[b, n] = sum_k x[b, k] * deq(W)[k, n],  deq(W)[k, n] = dl[k, s] * q[k, n] - ml[k, s]
//
// (cpp/src/dequant.cpp:268-301, :739-780; s = the 32-column sub-block of n).  Regrouped as
//   y[b, n] = sum_k q[k, n] * v[b, k, s]  -  sum_k x[b, k] * ml[k, s],   v = x * dl,
// the first term runs on mma.sync m16n8k32 (u8 x s8 -> s32), two instructions per 1024
// weights:
//   * A (16 columns x 32 rows): the 4-bit codes as exact u8.  ldmatrix.trans of four
//     8-row matrices hands each lane the bytes of rows (2t, 2t+1) of two adjacent byte
//     columns from each matrix; one PRMT per register gathers four rows of one byte
//     column, one LOP keeps the low nibbles (q) or the high nibbles in place (16 q).
//   * B (32 rows x 8): v as a 22-bit fixed-point integer n on a power-of-two scale per warp
//     and batch row, in three signed byte digits.  One FFMA with the 1.5 * 2^23 magic puts
//     n + 2^22 in the float mantissa, one XOR turns its two low bytes into signed digits
//     (the top byte is already 0..127), one PRMT per digit packs two rows.  The digits sum
//     to n + 4161408; column 3 (7) of B is all ones, so the MMA also yields sum q, and the
//     offset comes off exactly in 64-bit integers.
//   * The s32 accumulators run across the CTA's stages (exact integer sums).  A stage
//     whose |v| outgrows the scale (rare; warp-uniform) first moves the sums so far to
//     fp32 and raises the scale.  The min term is summed in fp32 on the side.
// Accuracy: each v is rounded to 2^-19 of the warp's largest |v| for its batch row (headroom
// 4-8x), products and sums are exact, fp32 at the end.  A v that is not finite (or beyond
// 2^100) marks its batch row and sub-block, whose outputs are then NaN.
//
// Decomposition: a CTA owns one 256-column tile (one Q4_K block per row) and every S-th
// 128-row stage of the matrix (stages split, split + S, ...), so each CTA samples the
// whole row range; its partial sums go to the caller's scratch and the CTA finishing a
// tile last adds the S partials in split order (deterministic) and resets the tile's
// counter.  Warp 8 TMA-loads the stages (144 B per row) into a 4-deep ring; warps 0-7 each
// take 32 rows x 128 columns of a stage: the B table for their rows, then 4 x 2 MMAs per
// column set.  Each lane reads its two rows of x from global memory a stage ahead.  Waits
// are bounded.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up); each
// translation unit keeps its own word (no relocatable device code).
__device__ unsigned g_gemv_mma_status = 0;


namespace gmma {

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 16 * kConsumers;   // rows per stage
constexpr int kPitch = 144;              // one Q4_K block per row
constexpr int kStageBytes = kRows * kPitch;  // 18432
constexpr int kStages = 4;
// B table per warp and column set: [4 local sub-blocks][8 columns][32 rows] s8.  Column
// stride 48 B: the fragment loads (word 12 g + t) hit 32 different banks; sub-block stride
// 416 B: the row-pair stores of the two lane halves land 16 banks apart.
constexpr int kColStride = 48;
constexpr int kSbStride = 416;
constexpr int kTblBytes = 4 * kSbStride;  // 1664
constexpr int kRedBytes = kConsumers * 4 * 128 * 4 + 4 * 256 * 4;  // per-warp outputs + CTA sum
// fixed point: |v| < 2^(e + 1) <=> |n| < 2^22 with n = rint(v * 2^(21 - e))
constexpr float kMagic = 12582912.f;       // 1.5 * 2^23
constexpr long long kDigitOffset = 4161408;  // sum of the digits minus n
constexpr int kExpMin = -100, kExpMax = 100;

struct Bars {
  uint64_t full[kStages], empty[kStages];
  int abort;
};
constexpr int kTblOff = kStages * kStageBytes;
constexpr int kRedOff = 0;  // the per-warp outputs reuse the stage ring afterwards
static_assert(kRedBytes <= kStages * kStageBytes, "reduction buffer inside the ring");
template <int NSET> struct Lay {
  static constexpr int kBarOff = kTblOff + kConsumers * NSET * kTblBytes;
  static constexpr int kSmem = kBarOff + 128 + 128;  // + alignment slack
};

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t saddr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
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
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// |v| as the rescale test sees it: values past 2^100, inf and NaN count as 0 (they are
// flagged instead)
__device__ __forceinline__ float mag(float v) {
  const float a = fabsf(v);
  return a < 0x1p100f ? a : 0.f;
}

template <int BATCH>
__global__ void __launch_bounds__(kThreads, BATCH <= 2 ? 2 : 1)
gemv_mma_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ x,
                float* __restrict__ y, int K, int N, int batch, float* __restrict__ partials,
                unsigned* __restrict__ counters) {
  constexpr int NSET = BATCH <= 2 ? 1 : 2;  // B column sets: two batch rows per set
  extern __shared__ uint8_t smem_raw[];
  // 128-byte aligned: TMA destinations and ldmatrix rows
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  using L = Lay<NSET>;
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 128-row stages split, split + S, split + 2S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto stage = [&](int s) { return smem + s * kStageBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), kConsumers);
    }
    bars.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  // Programmatic dependent launch: the next kernel may start filling SMs as this grid
  // drains; weights are streamed before waiting for the previous grid (they never depend
  // on it), x, y and the scratch only after.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_mma_status, kStatusTimeout);
  };

  // flushed fp32 sums [set][chunk][low / high nibbles][row g / g + 8], min-term sums
  // [batch][low / high sub-block], non-finite flags (bit 2 b + h)
  float fac[NSET][4][2][2];
  float mins[BATCH][2];
  unsigned nonfin = 0u;
#pragma unroll
  for (int z = 0; z < NSET; ++z)
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) fac[z][c][h][0] = fac[z][c][h][1] = 0.f;
#pragma unroll
  for (int b = 0; b < BATCH; ++b) mins[b][0] = mins[b][1] = 0.f;

  if (warp == kConsumers) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int it = 0;
      for (; it < nst && !*abort_flag; ++it) {
        const int s = it % kStages;
        if (it == kStages) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (!mbar_wait_bounded(smem_u32(&bars.empty[s]), ((it / kStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full[s]);
        mbar_arrive_expect_tx(fb, kStageBytes);
        tma_load_2d(smem_u32(stage(s)), &tmap_w, tile * (kPitch / 2), (split + S * it) * kRows, fb);
      }
      // every issued stage lands before the CTA may exit
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait_bounded(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    const int gp = warp & 1;          // this warp's columns 128 gp .. + 127
    const int rw = 32 * (warp >> 1);  // and its 32 rows of each stage
    // table role: rows rw + 2 rp, + 1 and local group gl (sub-blocks 2 q, 2 q + 1 of the tile)
    const int rp = lane & 15, gl = lane >> 4, q = 2 * gp + gl;
    // MMA k index of row 2 rp: rows 8 i + 2 t' + e of matrix i sit at k = 16 (i >> 1) +
    // 4 t' + 2 (i & 1) + e
    const int kap0 = 16 * (rp >> 3) + 4 * (rp & 3) + 2 * ((rp >> 2) & 1);
    const int g = lane >> 2, t = lane & 3;  // MMA fragment role
    uint8_t* tbl = smem + kTblOff + warp * NSET * kTblBytes;
    for (int i = lane; i < NSET * kTblBytes / 4; i += 32) reinterpret_cast<uint32_t*>(tbl)[i] = 0u;
    __syncwarp();
    for (int i = lane; i < NSET * 4 * 2 * 8; i += 32) {  // all-ones columns 3 and 7
      const int w8 = i & 7, c2 = (i >> 3) & 1, sb = (i >> 4) & 3, z = i >> 6;
      reinterpret_cast<uint32_t*>(tbl + z * kTblBytes + sb * kSbStride + (3 + 4 * c2) * kColStride)[w8] =
          0x01010101u;
    }
    __syncwarp();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int row0 = rw + 2 * rp;  // stage row of this lane's first row
    auto load_x = [&](int it, float2 (&xv)[BATCH]) {
      const int k = (split + S * it) * kRows + row0;
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const float* xb = x + (int64_t)b * K;
        xv[b].x = (b < batch && k < K) ? __ldg(xb + k) : 0.f;
        xv[b].y = (b < batch && k + 1 < K) ? __ldg(xb + k + 1) : 0.f;
      }
    };
    int acc[NSET][4][2][4];  // [set][chunk][low / high nibbles][fragment]
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[z][c][h][0] = acc[z][c][h][1] = acc[z][c][h][2] = acc[z][c][h][3] = 0;
    float scale[BATCH], step[BATCH], bound[BATCH];
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      scale[b] = 1.f;
      step[b] = 1.f;
      bound[b] = 0.f;  // the first stage sets the scale
    }
    // s32 sums -> fp32: lanes t even hold digits 0, 1 of batch row 2z + t/2, lanes t odd
    // digit 2 and the code sum of the same row; each pair adds its halves in 64 bits
    auto flush = [&]() {
#pragma unroll
      for (int z = 0; z < NSET; ++z) {
        const float sb = (t >> 1) ? ((2 * z + 1 < BATCH) ? step[(2 * z + 1) % BATCH] : 0.f) : step[(2 * z) % BATCH];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int* a = acc[z][c][h];
            long long p0, p1;
            if (t & 1) {
              p0 = 65536LL * a[0] - kDigitOffset * a[1];
              p1 = 65536LL * a[2] - kDigitOffset * a[3];
            } else {
              p0 = (long long)a[0] + 256LL * a[1];
              p1 = (long long)a[2] + 256LL * a[3];
            }
            p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
            p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
            const float f = h ? sb * 0.0625f : sb;  // high nibbles entered as 16 q
            fac[z][c][h][0] = fmaf((float)p0, f, fac[z][c][h][0]);
            fac[z][c][h][1] = fmaf((float)p1, f, fac[z][c][h][1]);
            a[0] = a[1] = a[2] = a[3] = 0;
          }
      }
    };

    float2 xn[BATCH];
    if (nst > 0) load_x(0, xn);
    // ldmatrix: lane L gives row rw + L (matrix L >> 3, row L & 7) of the warp's qs bytes
    const uint32_t lm_lane = (uint32_t)((rw + lane) * kPitch + 16 + 64 * gp);
    for (int it = 0; it < nst; ++it) {
      if (*abort_flag) break;
      float2 xv[BATCH];
#pragma unroll
      for (int b = 0; b < BATCH; ++b) xv[b] = xn[b];
      if (it + 1 < nst) load_x(it + 1, xn);  // a stage ahead
      const int s = it % kStages;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars.full[s]), (it / kStages) & 1,
                                                      kWaitBudgetCycles))) {
        if (lane == 0) give_up();
        break;
      }
      const uint8_t* st = stage(s);
      // ---- scales of the lane's two rows (get_scale_min_k4, cpp/src/dequant.cpp:258-266,
      // four sub-blocks per word) ----
      const uint4 h0 = *reinterpret_cast<const uint4*>(st + row0 * kPitch);
      const uint4 h1 = *reinterpret_cast<const uint4*>(st + (row0 + 1) * kPitch);
      auto sc4 = [&](const uint4& h) {
        return q < 2 ? (h.y & 0x3f3f3f3fu) : ((h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u));
      };
      auto mn4 = [&](const uint4& h) {
        return q < 2 ? (h.z & 0x3f3f3f3fu) : (((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u));
      };
      const uint32_t s0 = sc4(h0), s1 = sc4(h1), m0 = mn4(h0), m1 = mn4(h1);
      const uint32_t sel_lo = 0x7440u | (uint32_t)((2 * q) & 3), sel_hi = 0x7440u | (uint32_t)((2 * q + 1) & 3);
      // small integers as floats: byte into the 2^23 magic, minus 2^23 (exact)
      const float2 kMag = make_float2(-8388608.f, -8388608.f);
      const float2 sl = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(s0, 0x4b000000u, sel_lo)),
                                               __uint_as_float(__byte_perm(s1, 0x4b000000u, sel_lo))), kMag);
      const float2 sh = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(s0, 0x4b000000u, sel_hi)),
                                               __uint_as_float(__byte_perm(s1, 0x4b000000u, sel_hi))), kMag);
      const float2 mlo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(m0, 0x4b000000u, sel_lo)),
                                                __uint_as_float(__byte_perm(m1, 0x4b000000u, sel_lo))), kMag);
      const float2 mhi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(m0, 0x4b000000u, sel_hi)),
                                                __uint_as_float(__byte_perm(m1, 0x4b000000u, sel_hi))), kMag);
      const float2 d = make_float2(f16_ref(h0.x & 0xffffu), f16_ref(h1.x & 0xffffu));
      const float2 dm = make_float2(f16_ref(h0.x >> 16), f16_ref(h1.x >> 16));
      // dl = d * sc and ml = dmin * m: the reference's fp32 values (exact products)
      const float2 dl[2] = {__fmul2_rn(d, sl), __fmul2_rn(d, sh)};
      const float2 ml[2] = {__fmul2_rn(dm, mlo), __fmul2_rn(dm, mhi)};
      float2 v[BATCH][2];
      bool grow = false;
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          v[b][h] = __fmul2_rn(xv[b], dl[h]);
          mins[b][h] = fmaf(xv[b].x, ml[h].x, fmaf(xv[b].y, ml[h].y, mins[b][h]));
          const float a = fmaxf(fabsf(v[b][h].x), fabsf(v[b][h].y));
          if (!(a < 0x1p100f)) nonfin |= 1u << (2 * b + h);  // inf, NaN or past 2^100
          grow |= fmaxf(mag(v[b][h].x), mag(v[b][h].y)) >= bound[b];
        }
      if (__any_sync(0xffffffffu, grow)) {
        // rare: move the sums to fp32, then scale each batch row to 4-8x its largest |v|
        flush();
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          float m = fmaxf(fmaxf(mag(v[b][0].x), mag(v[b][0].y)), fmaxf(mag(v[b][1].x), mag(v[b][1].y)));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127 + 2;
          e = e < kExpMin ? kExpMin : (e > kExpMax ? kExpMax : e);
          scale[b] = pow2f(21 - e);
          step[b] = pow2f(e - 21);
          bound[b] = pow2f(e + 1);
        }
      }
      // ---- B table: three signed digits of n per row pair, batch row b, sub-block ----
#pragma unroll
      for (int b = 0; b < BATCH; ++b)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t wx = __float_as_uint(fmaf(v[b][h].x, scale[b], kMagic)) ^ 0x8080u;
          const uint32_t wy = __float_as_uint(fmaf(v[b][h].y, scale[b], kMagic)) ^ 0x8080u;
          uint8_t* col = tbl + (b >> 1) * kTblBytes + (2 * gl + h) * kSbStride + 4 * (b & 1) * kColStride + kap0;
#pragma unroll
          for (int j = 0; j < 3; ++j)
            *reinterpret_cast<uint16_t*>(col + j * kColStride) = (uint16_t)__byte_perm(wx, wy, j | ((4 + j) << 4));
        }
      __syncwarp();
      // ---- 4 chunks of 16 byte columns x 32 rows: low- and high-nibble MMAs per set ----
      const uint32_t lm = smem_u32(st) + lm_lane;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r0, r1, r2, r3;  // rows 0-7, 8-15, 16-23, 24-31 (pairs 2t, 2t+1), bytes 2g, 2g+1
        ldmatrix_x4_trans(lm + 16 * c, r0, r1, r2, r3);
        // A rows m = g: byte column 2g, m = g + 8: byte column 2g + 1
        const uint32_t a0 = __byte_perm(r0, r1, 0x6420), a1 = __byte_perm(r0, r1, 0x7531);
        const uint32_t a2 = __byte_perm(r2, r3, 0x6420), a3 = __byte_perm(r2, r3, 0x7531);
#pragma unroll
        for (int z = 0; z < NSET; ++z) {
          const uint8_t* tz = tbl + z * kTblBytes + (2 * (c >> 1)) * kSbStride + g * kColStride + 4 * t;
          const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(tz);
          const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(tz + 16);
          const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(tz + kSbStride);
          const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(tz + kSbStride + 16);
          mma_u8s8(acc[z][c][0], a0 & 0x0f0f0f0fu, a1 & 0x0f0f0f0fu, a2 & 0x0f0f0f0fu, a3 & 0x0f0f0f0fu, bl0, bl1);
          mma_u8s8(acc[z][c][1], a0 & 0xf0f0f0f0u, a1 & 0xf0f0f0f0u, a2 & 0xf0f0f0f0u, a3 & 0xf0f0f0f0u, bh0, bh1);
        }
      }
      __syncwarp();  // table and stage reads done
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty[s]));
    }
    flush();
    // min-term sums and flags of the lane's group: add over its 16 lanes
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        mins[b][0] += __shfl_xor_sync(0xffffffffu, mins[b][0], o);
        mins[b][1] += __shfl_xor_sync(0xffffffffu, mins[b][1], o);
      }
      nonfin |= __shfl_xor_sync(0xffffffffu, nonfin, o);
    }
  }

  // ---- per-warp outputs -> shared memory (the stage ring, now idle) ----
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem + kRedOff);  // [warp][b][the warp's 128 columns]
  if (warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int gg = c >> 1;
          // min sums and flags of sub-block (gg, h) sit in lanes 16 gg .. 16 gg + 15
          const float mA = __shfl_sync(0xffffffffu, mins[(2 * z) % BATCH][h], 16 * gg);
          const float mB = __shfl_sync(0xffffffffu, mins[(2 * z + 1) % BATCH][h], 16 * gg);
          const unsigned nf = __shfl_sync(0xffffffffu, nonfin, 16 * gg);
          const int b = 2 * z + (t >> 1);
          if ((t & 1) == 0 && b < BATCH && b < batch) {
            const float mn = (t >> 1) ? mB : mA;
            const bool bad = (nf >> (2 * b + h)) & 1u;
            // rows m = g, g + 8 of the chunk: byte columns 2g, 2g + 1 (+ 32: high nibbles)
            float* dst = red + (warp * 4 + b) * 128 + 64 * gg + 16 * (c & 1) + 2 * g + 32 * h;
            dst[0] = bad ? __int_as_float(0x7fc00000) : fac[z][c][h][0] - mn;
            dst[1] = bad ? __int_as_float(0x7fc00000) : fac[z][c][h][1] - mn;
          }
        }
  }
  __syncthreads();

  // ---- sum the warps in order: this CTA's partial y ----
  const int E = batch * 256;
  float* outbuf = red + kConsumers * 4 * 128;  // after the per-warp slots, still in the ring
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, n = e & 255, half = n >> 7, cl = n & 127;
    float v = 0.f;
    for (int w2 = half; w2 < kConsumers; w2 += 2) v += red[(w2 * 4 + b) * 128 + cl];  // warps of this half
    outbuf[e] = v;
  }
  __syncthreads();

  if (S == 1) {
    for (int e = threadIdx.x; e < E; e += kThreads)
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = outbuf[e];
    return;
  }
  // ---- split-K: publish this CTA's partial; the last CTA of the tile adds them up ----
  for (int e = threadIdx.x; e < E; e += kThreads)
    partials[((int64_t)split * batch + (e >> 8)) * N + tile * 256 + (e & 255)] = outbuf[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&counters[tile], 1u) == (unsigned)(S - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, n = e & 255;
    float sum = 0.f;
    for (int sp = 0; sp < S; ++sp)
      sum += __ldcg(partials + ((int64_t)sp * batch + b) * N + tile * 256 + n);
    y[(int64_t)b * N + tile * 256 + n] = sum;
  }
  if (threadIdx.x == 0) counters[tile] = 0u;  // leave the scratch ready for the next call
}

}  // namespace gmma

// ---- host side -----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnG)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnG encode_fn_g() {
  static EncodeTiledFnG fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnG>(p);
  });
  return fn;
}

template <int BATCH>
static cudaError_t launch_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                            int64_t RB, int batch, const GemvPlan& plan, void* scratch,
                            cudaStream_t st) {
  using namespace gmma;
  auto enc = encode_fn_g();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw;
  cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)RB};
  cuuint32_t box[2] = {(cuuint32_t)(kPitch / 2), (cuuint32_t)kRows};
  cuuint32_t es[2] = {1, 1};
  if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  auto kern = gemv_mma_kernel<BATCH>;
  constexpr int kSmem = Lay<(BATCH <= 2 ? 1 : 2)>::kSmem;
  static unsigned configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 32 || !(configured & (1u << dev))) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (dev < 32) configured |= (1u << dev);
  }
  unsigned* counters = static_cast<unsigned*>(scratch);
  float* partials = plan.splits > 1
                        ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + plan.counter_bytes)
                        : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)plan.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mw, x, y, (int)K, (int)N, batch, partials, counters);
}

// Whether the tensor-core kernel takes this call (batch 1..4; any K below 2^31 - 2^8).
bool gemv_mma_fits(const float*, int64_t K, int64_t N, int batch, const GemvPlan&) {
  return batch >= 1 && batch <= 4 && K >= 1 && K <= 0x7fffff00LL && N % 256 == 0;
}

// Tensor-core Q4_K GEMV for batch 1..4.
cudaError_t launch_gemv_mma_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, const GemvPlan& plan,
                                void* scratch, cudaStream_t st) {
  if (!gemv_mma_fits(x, K, N, batch, plan) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  if (batch == 1) return launch_t<1>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
  if (batch == 2) return launch_t<2>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
  return launch_t<4>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
}

cudaError_t gemv_mma_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_mma_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_mma_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
