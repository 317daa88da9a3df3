// vbq_gemv_mma.cu -- Q4_K dequant-GEMV on the integer tensor cores (decode, batch 1..4), and
// its Q5_K form (176-byte rows, fifth bits merged into the A fragments; see Geo / Q5).
//
//   y[b, n] = sum_k x[b, k] * deq(W)[k, n],  deq(W)[k, n] = dl[k, s] * q[k, n] - ml[k, s]
//
// (cpp/src/dequant.cpp:268-301, :739-780; s = the 32-column sub-block of n).  Regrouped as
//   y[b, n] = sum_k q[k, n] * v[b, k, s]  -  sum_k x[b, k] * ml[k, s],   v = x * dl,
// the first term runs on mma.sync m16n8k32 (u8 x s8 -> s32), two instructions per 1024
// weights:
//   * A (16 columns x 32 rows): the 4-bit codes as exact u8.  One byte-granular
//     ldmatrix.trans (m16n16, two matrices) hands each lane four rows of one byte column
//     per register, the MMA's A fragment as it stands; one LOP keeps the low nibbles (q)
//     or the high nibbles in place (16 q).
//   * B (32 rows x 8): v as a 22-bit fixed-point integer n on a power-of-two scale per warp
//     and batch row, in three signed byte digits.  One FFMA with the 1.5 * 2^23 magic puts
//     n + 2^22 in the float mantissa, one XOR turns its two low bytes into signed digits
//     (the top byte is already 0..127), one PRMT per digit packs two rows.  The digits sum
//     to n + 4161408; column 3 (7) of B is all ones, so the MMA also yields sum q, and the
//     offset comes off in int32 (top digit centred) before fp32.
//   * The s32 accumulators run across the CTA's stages (exact integer sums).  A stage
//     whose |v| outgrows the scale, or whose sampled |v| for some batch row (one value per
//     lane) all sit 16x or more below the value the scale was set from (warp-uniform
//     decisions; both rare on ordinary activations), first moves the sums so far to fp32
//     and then sets the scales again from this stage's full maximum.  The min term is
//     summed in fp32 on the side.
// Accuracy: each v is rounded to 2^-20 of the warp's largest |v| for its batch row in the
// stage that set the scale (headroom 2-4x), products and sums are exact, fp32 at the end.
// Because the scale also comes back down, an outlier activation (a channel 100-1000x its
// neighbours) coarsens only the rows of its own stage, not the rest of the warp's stages.
// A v that is not finite (or beyond 2^100) marks its batch row in the warp, whose 128
// outputs for that row are then NaN.
//
// Decomposition: a CTA owns one 256-column tile (one Q4_K block per row) and every S-th
// 128-row stage of the matrix (stages split, split + S, ...), so each CTA samples the
// whole row range.  The S splits of a tile form one thread-block cluster (S <= 16): splits
// 1 .. S-1 store their partial sums into split 0's shared memory with st.async, which
// counts the bytes on split 0's mbarrier, and exit; split 0 adds them in split order
// (deterministic) and writes y.  No global scratch, fence or atomic.  Warp 8 TMA-loads the stages (144 B per row) into a 4-deep ring; warps 0-7 each
// take 32 rows x 128 columns of a stage: the B table for their rows, then 4 x 2 MMAs per
// column set.  Each lane reads its two rows of x from global memory a stage ahead.  Waits
// are bounded.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>
#include <type_traits>

#include "vbq_common.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up); each
// translation unit keeps its own word (no relocatable device code).
__device__ unsigned g_gemv_mma_status = 0;


namespace gmma {

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 16 * kConsumers;   // rows per stage
constexpr int kStages = 4;  // a power of two (slot = stage & (kStages - 1))
// Row geometry of a stage: one Q4_K block (144 B, codes at byte 16) or, with Q5, one Q5_K
// block (176 B: d, dmin and the 12 scale bytes as in Q4_K, the 32 fifth-bit bytes at 16,
// codes at 48) per row.
template <bool Q5> struct Geo {
  static constexpr int kPitch = Q5 ? 176 : 144;
  static constexpr int kQs = Q5 ? 48 : 16;
  static constexpr int kStageBytes = kRows * kPitch;  // 18432 / 22528
  static constexpr int kTblOff = kStages * kStageBytes;
};
// B table per warp and column set: [4 local sub-blocks][8 columns][32 rows] s8, each
// column's rows ordered so that lane (g, t)'s two fragment words (k = 4t.., 16 + 4t..) are
// adjacent (one 8-byte load at byte 8t of column g; conflict-free per half warp).  Sub-block
// stride 288 B: the row-pair stores of the two lane halves land 16 banks apart.
constexpr int kColStride = 32;
constexpr int kSbStride = 288;
constexpr int kTblBytes = 4 * kSbStride;  // 1152
constexpr int kRedBytes = kConsumers * 4 * 128 * 4 + 4 * 256 * 4;  // per-warp outputs + CTA sum

struct Bars {
  uint64_t full[kStages], empty[kStages];
  uint64_t red;  // the cluster leader's: the other splits' partial sums have landed
  int abort;
};
constexpr int kRedOff = 0;  // the per-warp outputs reuse the stage ring afterwards
static_assert(kRedBytes <= kStages * Geo<false>::kStageBytes, "reduction buffer inside the ring");
template <int NSET, bool Q5 = false> struct Lay {
  static constexpr int kBarOff = Geo<Q5>::kTblOff + kConsumers * NSET * kTblBytes;
  // the leader's receive slots: splits 1 .. S-1, batch x 256 fp32 each (sized at launch)
  static constexpr int kRecvOff = kBarOff + 128;
  static constexpr int kSmem = kRecvOff + 128;  // + alignment slack; plus the slots
};
constexpr int kMaxSplit = 16;  // cluster size limit (non-portable above 8)

template <int BATCH, bool SWIGLU, bool Q5 = false>
__global__ void __launch_bounds__(kThreads, BATCH <= 2 ? 2 : 1)
gemv_mma_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ x,
                float* y, int K, int N, int batch, Epi epi) {
  using G = Geo<Q5>;
  constexpr int NSET = BATCH <= 2 ? 1 : 2;  // B column sets: two batch rows per set
  constexpr int kDownEvery = BATCH <= 2 ? 1 : 2;  // stages between shrink tests (a power of two)
  extern __shared__ uint8_t smem_raw[];
  // 128-byte aligned: TMA destinations and ldmatrix rows
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  using L = Lay<NSET, Q5>;
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 128-row stages split, split + S, split + 2S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto stage = [&](int s) { return smem + s * G::kStageBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), kConsumers);
    }
    mbar_init(smem_u32(&bars.red), 1);
    bars.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (S > 1) cluster_arrive();  // barriers initialised; waited for before any remote store
  // Programmatic dependent launch: the next kernel may start filling SMs as this grid
  // drains; weights are streamed before waiting for the previous grid (they never depend
  // on it), x, y and the scratch only after.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_mma_status, kStatusTimeout);
  };

  // flushed fp32 sums [set][chunk][low / high nibbles] of MMA row g (lanes t even) or
  // g + 8 (t odd), min-term sums [batch][low / high sub-block], non-finite flags (bit b)
  float fac[NSET][4][2];
  float mins[BATCH][2];
  unsigned nonfin = 0u;
#pragma unroll
  for (int z = 0; z < NSET; ++z)
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) fac[z][c][h] = 0.f;
#pragma unroll
  for (int b = 0; b < BATCH; ++b) mins[b][0] = mins[b][1] = 0.f;

  if (warp == kConsumers) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int it = 0;
      for (; it < nst && !*abort_flag; ++it) {
        const int s = it % kStages;
        if (it == kStages) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (!mbar_wait_hinted(smem_u32(&bars.empty[s]), ((it / kStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full[s]);
        mbar_arrive_expect_tx(fb, G::kStageBytes);
        tma_load_2d(smem_u32(stage(s)), &tmap_w, tile * (G::kPitch / 2), (split + S * it) * kRows, fb);
      }
      // every issued stage lands before the CTA may exit
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait_bounded(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    // warp: columns 128 gp .. + 127 (gp = warp & 1, a template constant below) and rows
    // rw .. rw + 31 of each stage
    auto consumer = [&](auto gp_c) {
      constexpr int GP = decltype(gp_c)::value;
      const int rw = 32 * (warp >> 1);
      // table role: rows rw + 2 rp, + 1 and local group gl (sub-blocks 2 q, 2 q + 1 of the
      // tile, q = 2 GP + gl)
      const int rp = lane & 15, gl = lane >> 4;
      // the MMA's k index is the row (0..31); row r is stored at byte 8 ((r & 15) >> 2) +
      // 4 (r >> 4) + (r & 3) of a column, so lane t's fragment words (rows 4t.., 16 + 4t..)
      // are adjacent; rows 2 rp, 2 rp + 1 are one 16-bit slot
      const int kap0 = 8 * ((rp & 7) >> 1) + 4 * (rp >> 3) + 2 * (rp & 1);
      const int g = lane >> 2, t = lane & 3;  // MMA fragment role
      uint8_t* tbl = smem + G::kTblOff + warp * NSET * kTblBytes;
      for (int i = lane; i < NSET * kTblBytes / 4; i += 32) reinterpret_cast<uint32_t*>(tbl)[i] = 0u;
      __syncwarp();
      for (int i = lane; i < NSET * 4 * 2 * 8; i += 32) {  // all-ones columns 3 and 7
        const int w8 = i & 7, c2 = (i >> 3) & 1, sb = (i >> 4) & 3, z = i >> 6;
        reinterpret_cast<uint32_t*>(tbl + z * kTblBytes + sb * kSbStride + (3 + 4 * c2) * kColStride)[w8] =
            0x01010101u;
      }
      __syncwarp();
      // the lane's B-table bytes: (set, sub-block 2 gl + h, batch column 4 (b & 1), row pair)
      uint8_t* const tcol = tbl + (2 * gl) * kSbStride + kap0;
      // the lane's B fragments: column g, k = 4t .. 4t + 3 and 16 + 4t .. 16 + 4t + 3
      const uint8_t* const tfrag = tbl + g * kColStride + 8 * t;
      const uint32_t sel_lo = 0x7440u | (uint32_t)(2 * gl), sel_hi = sel_lo + 1u;  // sub-block byte
      const int row0 = rw + 2 * rp;  // stage row of this lane's first row
      // ldmatrix: lane L gives row rw + L (matrix L >> 3, row L & 7) of the warp's qs bytes
      const uint32_t lm_lane = smem_u32(smem) + (uint32_t)((rw + lane) * G::kPitch + G::kQs + 64 * GP);
      asm volatile("griddepcontrol.wait;" ::: "memory");

      int acc[NSET][4][2][4];  // [set][chunk][low / high nibbles][fragment]
#pragma unroll
      for (int z = 0; z < NSET; ++z)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int h = 0; h < 2; ++h) acc[z][c][h][0] = acc[z][c][h][1] = acc[z][c][h][2] = acc[z][c][h][3] = 0;
      float scale[BATCH];  // powers of two; the step of batch row b is 1 / scale[b]
      // bit b: batch row b may be rescaled down (a row below `batch` whose scale was not set
      // from an all-zero stage)
      uint32_t down_ok = 0u;
      float2 mn2[BATCH][2];  // min-term sums, rows 2 rp / 2 rp + 1
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        scale[b] = 1.f;  // the first stage sets the scale
        mn2[b][0] = mn2[b][1] = make_float2(0.f, 0.f);
      }
      // s32 sums -> fp32.  Lanes t even hold digits 0, 1 of batch row 2z + t/2, lanes t odd
      // digit 2 and the code sum of the same row.  With the top digit centred (d2 - 64 per
      // code) the pair's parts are (a0 + 256 a1) and (65536 (a2 - 64 S) + 32896 S), S = sum q:
      // the int32 difference is exact and the fp32 terms stay within 2^-20 of the result.
      auto flush = [&]() {
        const int odd = t & 1;
        const float c1 = odd ? 65536.f : 1.f, c2 = odd ? 32896.f : 256.f;
        const int cen = odd ? 64 : 0;
#pragma unroll
        for (int z = 0; z < NSET; ++z) {
          const float sb = (t >> 1) ? ((2 * z + 1 < BATCH) ? inv_pow2(scale[(2 * z + 1) % BATCH]) : 0.f)
                                  : inv_pow2(scale[(2 * z) % BATCH]);
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              int* a = acc[z][c][h];
              float p0 = fmaf(c2, (float)a[1], c1 * (float)(a[0] - cen * a[1]));
              float p1 = fmaf(c2, (float)a[3], c1 * (float)(a[2] - cen * a[3]));
              // the pair's halves: lane t even keeps row g, lane t odd row g + 8
              const float mine = odd ? p1 : p0, other = odd ? p0 : p1;
              const float sum = mine + __shfl_xor_sync(0xffffffffu, other, 1);
              // Q4_K high nibbles are entered as 16 q; Q5_K codes always as q
              const float f = (h && !Q5) ? sb * 0.0625f : sb;
              fac[z][c][h] = fmaf(sum, f, fac[z][c][h]);
              a[0] = a[1] = a[2] = a[3] = 0;
            }
        }
      };

      // x rows of the lane, two stages ahead (L2 latency under a saturated HBM exceeds one
      // stage): k = the lane's first row in the stage being loaded
      int kx = split * kRows + row0;
      const int kstep = S * kRows;
      float2 xn[BATCH], xnn[BATCH];
      auto load_x = [&](int k, float2 (&xv)[BATCH]) {
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          xv[b].x = (b < batch && k < K) ? gemv_x<SWIGLU>(x, b, K, k) : 0.f;
          xv[b].y = (b < batch && k + 1 < K) ? gemv_x<SWIGLU>(x, b, K, k + 1) : 0.f;
        }
      };
      load_x(kx, xn);
      kx += kstep;
      load_x(kx, xnn);
      // one stage per iteration, not unrolled: the loop body already fills the instruction
      // cache (unrolling it 2x / 4x measured 3-7 % slower)
#pragma unroll 1
      for (int it = 0; it < nst; ++it) {
        const int u = it & (kStages - 1);
        const uint32_t par = (uint32_t)(it / kStages) & 1u;
        {
          float2 xv[BATCH];
#pragma unroll
          for (int b = 0; b < BATCH; ++b) {
            xv[b] = xn[b];
            xn[b] = xnn[b];
          }
          kx += kstep;
          load_x(kx, xnn);  // rows of the stage after next (zero past K)
          if (!__all_sync(0xffffffffu, mbar_wait_hinted(smem_u32(&bars.full[u]), par, kWaitBudgetCycles))) {
            if (lane == 0) give_up();
            break;
          }
          const uint8_t* st = smem + u * G::kStageBytes;
          // ---- scales of the lane's two rows (get_scale_min_k4, cpp/src/dequant.cpp:258-266,
          // four sub-blocks per word) ----
          const uint4 h0 = *reinterpret_cast<const uint4*>(st + row0 * G::kPitch);
          const uint4 h1 = *reinterpret_cast<const uint4*>(st + (row0 + 1) * G::kPitch);
          uint32_t s0, s1, m0, m1;
          if constexpr (GP == 0) {  // sub-blocks 0-3: 6-bit fields of scale bytes 0-3 / 4-7
            s0 = h0.y & 0x3f3f3f3fu;
            s1 = h1.y & 0x3f3f3f3fu;
            m0 = h0.z & 0x3f3f3f3fu;
            m1 = h1.z & 0x3f3f3f3fu;
          } else {  // sub-blocks 4-7: low / high nibbles of bytes 8-11 + top bits of 0-7
            s0 = (h0.w & 0x0f0f0f0fu) | ((h0.y >> 2) & 0x30303030u);
            s1 = (h1.w & 0x0f0f0f0fu) | ((h1.y >> 2) & 0x30303030u);
            m0 = ((h0.w >> 4) & 0x0f0f0f0fu) | ((h0.z >> 2) & 0x30303030u);
            m1 = ((h1.w >> 4) & 0x0f0f0f0fu) | ((h1.z >> 2) & 0x30303030u);
          }
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
          const float2 dl0 = __fmul2_rn(d, sl), dl1 = __fmul2_rn(d, sh);
          const float2 ml0 = __fmul2_rn(dm, mlo), ml1 = __fmul2_rn(dm, mhi);
          // v on the current scale: 1.5 * 2^23 + n in the float, in range exactly when the
          // float keeps the exponent of 2^23 (|n| < 2^22); NaN, inf and overflow leave it
          float2 v[BATCH][2];
          uint32_t w[BATCH][2][2];
          uint32_t out = 0u;
#pragma unroll
          for (int b = 0; b < BATCH; ++b) {
            v[b][0] = __fmul2_rn(xv[b], dl0);
            v[b][1] = __fmul2_rn(xv[b], dl1);
            mn2[b][0] = __ffma2_rn(xv[b], ml0, mn2[b][0]);
            mn2[b][1] = __ffma2_rn(xv[b], ml1, mn2[b][1]);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              w[b][h][0] = __float_as_uint(fmaf(v[b][h].x, scale[b], kMagic));
              w[b][h][1] = __float_as_uint(fmaf(v[b][h].y, scale[b], kMagic));
              out |= (w[b][h][0] ^ 0x4b000000u) | (w[b][h][1] ^ 0x4b000000u);
            }
          }
          // the shrink test (every stage up to batch 2, every second one above, where it costs
          // more): one of the lane's four values per batch row is the sample (the test only
          // decides whether to rescale; the rescale itself takes the full maximum).  The word
          // holds 1.5 * 2^23 + n when in range, so |n| < 2^16 <=> w - (1.5 * 2^23 - 2^16) is below
          // 2^17; an out-of-range word fails it and rescales through `out` anyway.
          bool shrink = false;
          if ((it & (kDownEvery - 1)) == 0) {
            uint32_t small = 0u;
#pragma unroll
            for (int b = 0; b < BATCH; ++b) small |= (w[b][0][0] - 0x4b3f0000u < 0x20000u) ? (1u << b) : 0u;
            shrink = __reduce_and_sync(0xffffffffu, small & down_ok) != 0u;
          }
          if (__any_sync(0xffffffffu, out >= (1u << 23)) || shrink || it == 0) {
            // rare (and the first stage): flag non-finite values, move the sums to fp32, then
            // scale each batch row to 2-4x its largest finite |v| and encode again.  The
            // max ignores NaN and is capped so that huge values do not rescale every stage.
            if (it > 0) flush();  // nothing accumulated before the first stage
#pragma unroll
            for (int b = 0; b < BATCH; ++b) {
              const float sum = (fabsf(v[b][0].x) + fabsf(v[b][0].y)) + (fabsf(v[b][1].x) + fabsf(v[b][1].y));
              nonfin |= (sum < 0x1p100f) ? 0u : (1u << b);  // NaN / inf propagate
              float m = fminf(fmaxf(fmaxf(fabsf(v[b][0].x), fabsf(v[b][0].y)),
                                    fmaxf(fabsf(v[b][1].x), fabsf(v[b][1].y))), 0x1p99f);
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
              int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127 + 1;
              e = e < kExpMin ? kExpMin : (e > kExpMax ? kExpMax : e);
              scale[b] = pow2f(21 - e);
              down_ok = (b < batch && e > kExpMin) ? (down_ok | (1u << b)) : (down_ok & ~(1u << b));
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                w[b][h][0] = __float_as_uint(fmaf(v[b][h].x, scale[b], kMagic));
                w[b][h][1] = __float_as_uint(fmaf(v[b][h].y, scale[b], kMagic));
              }
            }
          }
          // ---- B table: three signed digits of n per row pair, batch row b, sub-block ----
#pragma unroll
          for (int b = 0; b < BATCH; ++b)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t wx = w[b][h][0] ^ 0x8080u, wy = w[b][h][1] ^ 0x8080u;
              uint8_t* col = tcol + (b >> 1) * kTblBytes + h * kSbStride + 4 * (b & 1) * kColStride;
#pragma unroll
              for (int j = 0; j < 3; ++j)
                *reinterpret_cast<uint16_t*>(col + j * kColStride) = (uint16_t)__byte_perm(wx, wy, j | ((4 + j) << 4));
            }
          __syncwarp();
          // ---- 4 chunks of 16 byte columns x 32 rows: low- and high-nibble MMAs per set ----
          const uint32_t lm = lm_lane + (uint32_t)(u * G::kStageBytes);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t a[4];  // A rows m = g / g + 8: byte columns g / g + 8
            ldmatrix_a8_trans(lm + 16 * c, a[0], a[1], a[2], a[3]);
            uint32_t lo[4], hi[4];
            if constexpr (Q5) {
              // Q5_K (cpp/src/dequant.cpp:317-354): the fifth bits of code byte l' sit in byte
              // 16 + l' of the block (the reference steps its qh pointer 32 bytes a chunk),
              // 32 bytes before the code byte: the same ldmatrix 32 bytes lower puts them in
              // the same fragment places; bit 7 belongs to the low nibble's value, bit 3 to
              // the high nibble's.  Both codes enter as q (0..31).
              uint32_t hb[4];
              ldmatrix_a8_trans(lm + 16 * c - 32, hb[0], hb[1], hb[2], hb[3]);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                lo[i] = (a[i] & 0x0f0f0f0fu) | ((hb[i] >> 3) & 0x10101010u);
                hi[i] = ((a[i] >> 4) & 0x0f0f0f0fu) | ((hb[i] << 1) & 0x10101010u);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                lo[i] = a[i] & 0x0f0f0f0fu;
                hi[i] = a[i] & 0xf0f0f0f0u;
              }
            }
#pragma unroll
            for (int z = 0; z < NSET; ++z) {
              const uint8_t* tz = tfrag + z * kTblBytes + (2 * (c >> 1)) * kSbStride;
              const uint2 bl = *reinterpret_cast<const uint2*>(tz);
              const uint2 bh = *reinterpret_cast<const uint2*>(tz + kSbStride);
              mma_u8s8(acc[z][c][0], lo[0], lo[1], lo[2], lo[3], bl.x, bl.y);
              mma_u8s8(acc[z][c][1], hi[0], hi[1], hi[2], hi[3], bh.x, bh.y);
            }
          }
          __syncwarp();  // table and stage reads done
          if (lane == 0) mbar_arrive(smem_u32(&bars.empty[u]));
        }
      }
      flush();
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        mins[b][0] = mn2[b][0].x + mn2[b][0].y;
        mins[b][1] = mn2[b][1].x + mn2[b][1].y;
      }
    };
    if (warp & 1) consumer(std::integral_constant<int, 1>{});
    else consumer(std::integral_constant<int, 0>{});
    // min-term sums of the lane's group: add over its 16 lanes; flags over the warp (the
    // warp's scale is shared by both groups)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      if (o < 16) {
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          mins[b][0] += __shfl_xor_sync(0xffffffffu, mins[b][0], o);
          mins[b][1] += __shfl_xor_sync(0xffffffffu, mins[b][1], o);
        }
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
          if (b < BATCH && b < batch) {
            const float mn = (t >> 1) ? mB : mA;
            const bool bad = (nf >> b) & 1u;
            // row m = g (t even) / g + 8 (t odd) of the chunk: byte column g / g + 8
            // (+ 32: high nibbles)
            red[(warp * 4 + b) * 128 + 64 * gg + 16 * (c & 1) + g + 8 * (t & 1) + 32 * h] =
                bad ? __int_as_float(0x7fc00000) : fac[z][c][h] - mn;
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
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = epi_apply(epi, outbuf[e], e >> 8, N, tile * 256 + (e & 255));
    return;
  }
  // ---- split-K inside the cluster: splits 1 .. S-1 push their partials into the leader's
  // slots (st.async, counted on its barrier) and exit; the leader adds them in split order
  cluster_wait();  // every CTA of the cluster has initialised its barriers
  const uint32_t rank = cluster_rank();
  float* recv = reinterpret_cast<float*>(smem + L::kRecvOff);
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
    y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = epi_apply(epi, sum, e >> 8, N, tile * 256 + (e & 255));
  }
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

// Splits per tile: at most one wave (two CTAs per SM up to batch 2) and 16 (one cluster),
// the leader's receive slots inside the per-CTA shared memory budget, and room for every
// tile's cluster at once with 25 % to spare (cudaOccupancyMaxActiveClusters, cached per
// shape).  Measured on B200 (us per launch, batch 1): 4096 x 14336 S = 4: 11.6, S = 5
// (56 clusters in 56-59 places): 16.3; 4096 x 6144 S = 8: 8.3, S = 12: 11.7.
template <int BATCH, bool SW, bool Q5>
static int choose_splits(int64_t K, int64_t N, int batch, int smem_base) {
  using namespace gmma;
  const int tiles = (int)(N / 256);
  const int64_t tot_st = (K + kRows - 1) / kRows;
  const int slots = (BATCH <= 2 ? 2 : 1) * sm_count();
  int S = tiles > 0 ? slots / tiles : 1;
  if (S > kMaxSplit) S = kMaxSplit;
  if (S > tot_st) S = (int)tot_st;
  if (S < 1) S = 1;
  const int cap = BATCH <= 2 ? 112 * 1024 : 220 * 1024;  // 2 / 1 CTAs per SM
  if (gemv_split_override()) {
    S = gemv_split_override() > kMaxSplit ? kMaxSplit : gemv_split_override();
    if (S > tot_st) S = (int)tot_st;
    while (S > 1 && smem_base + (S - 1) * batch * 1024 > cap) --S;
    return S;
  }
  while (S > 1 && smem_base + (S - 1) * batch * 1024 > cap) --S;
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
    cfg.dynamicSmemBytes = smem_base + (S - 1) * batch * 1024;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, gmma::gemv_mma_kernel<BATCH, SW, Q5>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      active = 0;
    }
    // a quarter of headroom: clusters need S free slots in one GPC at once, and a grid
    // that fills every GPC to the last cluster leaves some clusters to a second wave
    // when the previous launch still holds slots (programmatic dependent launch)
    if (active * 4 >= tiles * 5) break;
  }
  if (n_cache < 32) cache[n_cache++] = Entry{tiles, batch, s_in, S};
  return S;
}

template <int BATCH, bool SWIGLU, bool Q5 = false>
static cudaError_t launch_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                            int64_t RB, int batch, cudaStream_t st, Epi epi) {
  using namespace gmma;
  auto enc = encode_fn_g();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw;
  if (!weight_map(reinterpret_cast<EncodeTiledFn>(enc), w, K, RB, Geo<Q5>::kPitch, kRows, &mw))
    return cudaErrorInvalidValue;
  auto kern = gemv_mma_kernel<BATCH, SWIGLU, Q5>;
  constexpr int kBase = Lay<(BATCH <= 2 ? 1 : 2), Q5>::kSmem;
  static DeviceOnce configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  const int S = choose_splits<BATCH, SWIGLU, Q5>(K, N, batch, kBase);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kBase + (S - 1) * batch * 1024;
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
  return cudaLaunchKernelEx(&cfg, kern, mw, x, y, (int)K, (int)N, batch, epi);
}

// Whether the tensor-core kernel takes this call (batch 1..16).  The s32 sums run over up
// to K / 4 rows per accumulator with terms below 240 * 128 in magnitude, so K is capped
// at 3 * 2^16 (exact below 2^31 with room to spare); longer rows take the fp32 kernel.
constexpr int64_t kMmaMaxK = 3 * 65536;
bool gemv_mma_fits(int64_t K, int64_t N, int batch) {
  return batch >= 1 && batch <= 16 && K >= 1 && K <= kMmaMaxK && N % 256 == 0 && N > 0;
}

// Tensor-core Q4_K GEMV.  Batches 5..16 go to the fp16 kernel (vbq_gemv_half.cu: one pass
// over the weights, activations tabled once per row) when x's rows are 16-byte aligned;
// otherwise to the integer wide kernel (x aligned, no SwiGLU input), else as consecutive
// launches over groups of 4 batch rows (each streams the weights again).  Measured on
// B200, 4096 x 14336: batch 8 grouped 33.2 us / wide 31.3 us / fp16 28.7 us; batch 16
// grouped 64.5 us / wide 51.9 us / fp16 40.4 us.
template <bool SW, bool Q5 = false>
static cudaError_t launch_group(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int nb, cudaStream_t st, Epi epi) {
  return nb == 1   ? launch_t<1, SW, Q5>(x, w, y, K, N, row_bytes, nb, st, epi)
         : nb == 2 ? launch_t<2, SW, Q5>(x, w, y, K, N, row_bytes, nb, st, epi)
                   : launch_t<4, SW, Q5>(x, w, y, K, N, row_bytes, nb, st, epi);
}

cudaError_t launch_gemv_mma_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_mma_fits(K, N, batch) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  if (gemv_half_fits(x, K, N, batch)) return launch_gemv_half_q4k(x, w, y, K, N, row_bytes, batch, st, f);
  // the wide kernel reads x by TMA, so a SwiGLU input runs in groups of 4 here
  if (batch > 4 && !f.swiglu_x && gemv_wide_fits(x, K, N, batch))
    return launch_gemv_wide_q4k(x, w, y, K, N, row_bytes, batch, st, f);
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int b0 = 0; b0 < batch; b0 += 4) {
    const int nb = batch - b0 < 4 ? batch - b0 : 4;
    const float* xg = x + (int64_t)b0 * xrow;
    float* yg = y + (int64_t)b0 * N;
    const Epi epi{f.bias, f.res ? f.res + (int64_t)b0 * N : nullptr};
    cudaError_t e = f.swiglu_x ? launch_group<true>(xg, w, yg, K, N, row_bytes, nb, st, epi)
                               : launch_group<false>(xg, w, yg, K, N, row_bytes, nb, st, epi);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Q5_K on the same kernel (batch 1..16, as groups of up to 4 batch rows): the Q4_K
// kernel with 176-byte rows and the fifth bits merged into its A fragments.  Rows of 176
// bytes are always whole 16-byte granules, so every width of whole 256-column tiles fits.
cudaError_t launch_gemv_mma_q5k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_mma_fits(K, N, batch) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int b0 = 0; b0 < batch; b0 += 4) {
    const int nb = batch - b0 < 4 ? batch - b0 : 4;
    const float* xg = x + (int64_t)b0 * xrow;
    float* yg = y + (int64_t)b0 * N;
    const Epi epi{f.bias, f.res ? f.res + (int64_t)b0 * N : nullptr};
    cudaError_t e = f.swiglu_x ? launch_group<true, true>(xg, w, yg, K, N, row_bytes, nb, st, epi)
                               : launch_group<false, true>(xg, w, yg, K, N, row_bytes, nb, st, epi);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ---------------------------------------------------------------------------------
// Diagnostic of the bounded-wait path: one warp waits on an mbarrier with the GEMV
// kernel's own hinted, bounded wait and, when the wait gives up, raises kStatusTimeout in
// this file's status word, as the kernel's give_up() does.  With arrive = 0 nothing ever
// arrives, so the wait runs out after `budget` cycles and the kernel returns normally:
// the timeout report is tested without a fault or a hang.  With arrive = 1 lane 0
// completes the phase first and the wait succeeds.
// ---------------------------------------------------------------------------------
namespace gmma {
__global__ void __launch_bounds__(32) wait_probe_kernel(long long budget, int arrive) {
  __shared__ uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    mbar_fence_init();
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) mbar_arrive(b);
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, mbar_wait_hinted(b, 0u, budget));
  if (threadIdx.x == 0) {
    if (!ok) atomicOr(&g_gemv_mma_status, kStatusTimeout);
    mbar_inval(b);
  }
}
}  // namespace gmma

cudaError_t launch_wait_probe(long long budget_cycles, int arrive, cudaStream_t st) {
  gmma::wait_probe_kernel<<<1, 32, 0, st>>>(budget_cycles, arrive);
  return cudaGetLastError();
}

cudaError_t gemv_mma_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_mma_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_mma_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
