// vbq_gemv_wide.cu -- Q4_K dequant-GEMV for batch 5..16 on the integer tensor cores.
//
// The arithmetic is the batch 1..4 kernel's (vbq_gemv_mma.cu): y[b, n] = sum_k q[k, n] *
// v[b, k, s] - sum_k x[b, k] * ml[k, s] with v = x * dl (cpp/src/dequant.cpp:268-301,
// :739-780), the codes as exact u8 A fragments of mma.sync m16n8k32 and v as three signed
// byte digits of a 22-bit fixed-point integer per batch row in the B columns (two batch
// rows and an all-ones column per set of 8), exact s32 accumulation across stages.
//
// What changes with 8 or 16 batch rows is the shape of a warp's work: its accumulators
// grow with the batch (4 or 8 column sets), so a warp takes one 16-byte chunk of the
// tile's quant bytes (32 columns: 16 low + 16 high nibbles) instead of four, and the 8
// consumer warps cover the 256-column tile over 32-row stages.  Warps 2G and 2G + 1 read
// the same two sub-blocks (2G, 2G + 1) and share one B table: each builds the digits of
// half the batch rows (lanes 0-15 / 16-31 a quarter each), a 64-thread named barrier per
// pair separates the table's writes from the MMAs' reads, and the pair agrees on every
// per-stage decision (a rescale, a bounded wait that gave up) through shared flags before
// that barrier, so neither warp can wait for one the other skips.  The stage's x rows ([batch][32] fp32) come by TMA with the weights, so nothing
// is prefetched in registers.  Flushed fp32 sums and the per-batch-row scales live in
// shared memory (they change only when a scale does).
//
// Split-K: the S splits of a tile form a thread-block cluster.  Each CTA leaves its 256 x
// batch partial sums in its own shared memory; after a cluster barrier, CTA r adds the
// partials of its slice of the columns (256 r / S .. 256 (r + 1) / S - 1) in split order
// (deterministic) reading the others' shared memory, and a second barrier keeps every CTA
// alive until all reads are done.  No receive buffer, so S is not limited by memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "vbq_common.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up).
__device__ unsigned g_gemv_wide_status = 0;

namespace gwide {
using namespace gmma;

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 32;                 // rows per stage
constexpr int kPitch = 144;               // one Q4_K block per row
constexpr int kWBytes = kRows * kPitch;   // 4608, a multiple of 128
constexpr int kStages = 12;
constexpr int kColStride = 32;            // B table: 32 rows of s8 per column
constexpr int kSbStride = 288;            // 8 columns + pad: the two lane halves 16 banks apart

template <int BATCH> struct Cfg {
  static constexpr int kSets = BATCH / 2;
  static constexpr int kXBytes = BATCH * kRows * 4;        // [BATCH][32] fp32
  static constexpr int kSlot = kWBytes + kXBytes;          // stage slot (multiple of 128)
  // set stride: a batch row's lane-half partner (B/4 sets apart) writes 16 banks away
  static constexpr int kSetStride = BATCH == 16 ? 592 : 608;
  static constexpr int kTbl = kSets * kSetStride;          // per warp pair
  static constexpr int kFac = kSets * 2 * 32 * 4;          // per warp: [set][lo/hi][lane]
  static constexpr int kRingOff = 0;
  static constexpr int kTblOff = kStages * kSlot;
  static constexpr int kPairs = kConsumers / 2;
  static constexpr int kFacOff = kTblOff + kPairs * kTbl;
  static constexpr int kStepOff = kFacOff + kConsumers * kFac;          // [pair][BATCH] fp32
  static constexpr int kMinOff = kStepOff + kPairs * BATCH * 4;         // [pair][BATCH][2]
  static constexpr int kFlagOff = kMinOff + kPairs * BATCH * 2 * 4;     // [warp][2] u32
  static constexpr int kBarOff = kFlagOff + kConsumers * 2 * 4;
  static constexpr int kSmem = kBarOff + 128 + 128;                     // + alignment slack
  static constexpr int kOutBytes = BATCH * 256 * 4;                     // partial sums
  static_assert(kSlot % 128 == 0, "TMA destinations 128-byte aligned");
  static_assert(kOutBytes <= kStages * kSlot, "partial sums inside the ring");
  static_assert(kSmem <= 220 * 1024, "shared memory per CTA");
};

struct Bars {
  uint64_t full[kStages], empty[kStages];
  int abort;
};

template <int BATCH>
__global__ void __launch_bounds__(kThreads, BATCH <= 8 ? 2 : 1)
gemv_wide_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 float* y, int K, int N, int batch, Epi epi) {
  using C = Cfg<BATCH>;
  constexpr int NSET = C::kSets;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  Bars& bars = *reinterpret_cast<Bars*>(smem + C::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 32-row stages split, split + S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto slot = [&](int s) { return smem + C::kRingOff + s * C::kSlot; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), kConsumers);
    }
    bars.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_wide_status, kStatusTimeout);
  };

  if (warp == kConsumers) {
    // ---------------------------- TMA producer ----------------------------
    // Weights stream before the wait for the previous grid; x (its output, maybe) after.
    if (lane == 0) {
      int it = 0;
      bool waited = false;
      auto issue_x = [&](int j) {
        tma_load_2d(smem_u32(slot(j % kStages) + kWBytes), &tmap_x, (split + S * j) * kRows, 0,
                    smem_u32(&bars.full[j % kStages]));
      };
      for (; it < nst && !*abort_flag; ++it) {
        const int s = it % kStages;
        if (it == kStages) {  // the ring is full: wait for the previous grid, then x
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
          for (int j = 0; j < kStages; ++j) issue_x(j);
        }
        if (!mbar_wait_hinted(smem_u32(&bars.empty[s]), ((it / kStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full[s]);
        mbar_arrive_expect_tx(fb, C::kSlot);
        tma_load_2d(smem_u32(slot(s)), &tmap_w, tile * (kPitch / 2), (split + S * it) * kRows, fb);
        if (waited) issue_x(it);
      }
      if (!waited) {  // fewer stages than the ring holds
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int j = 0; j < it; ++j) issue_x(j);
      }
      // every issued stage lands before the CTA may exit
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait_hinted(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    constexpr int QB = BATCH / 4;  // batch rows per lane (a quarter of the batch)
    const int c = warp;            // the tile's quant bytes 16c .. 16c + 15
    const int G = c >> 1;          // 64-column group: sub-blocks 2G (low), 2G + 1 (high)
    const int pr = G, par = c & 1; // warp pair (shares the B table) and the warp in it
    // table role: rows 2 rp, 2 rp + 1 of the stage, batch rows qd * QB .. + QB - 1
    const int rp = lane & 15, qd = 2 * par + (lane >> 4);
    const int kap0 = 8 * ((rp & 7) >> 1) + 4 * (rp >> 3) + 2 * (rp & 1);  // as in vbq_gemv_mma.cu
    const int g = lane >> 2, t = lane & 3;  // MMA fragment role
    uint8_t* tbl = smem + C::kTblOff + pr * C::kTbl;
    float* fac = reinterpret_cast<float*>(smem + C::kFacOff + warp * C::kFac);  // [set][h][lane]
    float* stp = reinterpret_cast<float*>(smem + C::kStepOff) + pr * BATCH;     // step per row
    volatile uint32_t* flags = reinterpret_cast<volatile uint32_t*>(smem + C::kFlagOff);  // [warp][2]
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + pr) : "memory"); };
    // the pair's table: each warp zeroes half and writes the all-ones columns 3 and 7 of
    // its half of the sets, then the pair meets before any digit is written
    for (int i = par * 32 + lane; i < C::kTbl / 4; i += 64) reinterpret_cast<uint32_t*>(tbl)[i] = 0u;
    for (int i = lane; i < NSET * 2 * 32; i += 32) fac[i] = 0.f;
    if (par == 0 && lane < BATCH) stp[lane] = 1.f;
    pair_sync();
    for (int i = par * 32 + lane; i < NSET * 2 * 2 * 8; i += 64) {
      const int w8 = i & 7, c2 = (i >> 3) & 1, h = (i >> 4) & 1, z = i >> 5;
      reinterpret_cast<uint32_t*>(tbl + z * C::kSetStride + h * kSbStride + (3 + 4 * c2) * kColStride)[w8] =
          0x01010101u;
    }
    pair_sync();
    const uint32_t sel_lo = 0x7440u | (uint32_t)((2 * G) & 3), sel_hi = 0x7440u | (uint32_t)((2 * G + 1) & 3);
    const uint8_t* const tfrag = tbl + g * kColStride + 8 * t;
    const uint32_t lm_lane = smem_u32(smem) + (uint32_t)(C::kRingOff + lane * kPitch + 16 + 16 * c);

    int acc[NSET][2][4];
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int h = 0; h < 2; ++h) acc[z][h][0] = acc[z][h][1] = acc[z][h][2] = acc[z][h][3] = 0;
    float scale[QB], mins[QB][2];
    uint32_t down_ok = 0u;  // bit b: batch row b may be rescaled down (see vbq_gemv_mma.cu)
#pragma unroll
    for (int j = 0; j < QB; ++j) {
      scale[j] = 1.f;
      mins[j][0] = mins[j][1] = 0.f;
    }
    unsigned nonfin = 0u;  // bit b: batch row b saw a non-finite v

    // s32 sums -> fp32 sums in shared memory (see vbq_gemv_mma.cu): lanes t even hold
    // digits 0, 1 of batch row 2z + t/2, lanes t odd digit 2 and the code sum
    auto flush = [&]() {
      const int odd = t & 1;
      const float c1 = odd ? 65536.f : 1.f, c2 = odd ? 32896.f : 256.f;
      const int cen = odd ? 64 : 0;
#pragma unroll
      for (int z = 0; z < NSET; ++z) {
        const float sb = stp[2 * z + (t >> 1)];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int* a = acc[z][h];
          const float p0 = fmaf(c2, (float)a[1], c1 * (float)(a[0] - cen * a[1]));
          const float p1 = fmaf(c2, (float)a[3], c1 * (float)(a[2] - cen * a[3]));
          const float mine = odd ? p1 : p0, other = odd ? p0 : p1;
          const float sum = mine + __shfl_xor_sync(0xffffffffu, other, 1);
          float& f = fac[(z * 2 + h) * 32 + lane];
          f = fmaf(sum, h ? sb * 0.0625f : sb, f);
          a[0] = a[1] = a[2] = a[3] = 0;
        }
      }
    };

    for (int it = 0; it < nst; ++it) {
      const int s = it % kStages;
      // a wait that gives up is acted on only after the pair's flag exchange below (the
      // stage's bytes are then stale but in bounds)
      const bool ok = __all_sync(0xffffffffu, mbar_wait_hinted(smem_u32(&bars.full[s]), (it / kStages) & 1,
                                                                kWaitBudgetCycles));
      const uint8_t* st = slot(s);
      // ---- scales of the lane's two rows, sub-blocks 2G and 2G + 1
      // (get_scale_min_k4, cpp/src/dequant.cpp:258-266) ----
      const uint4 h0 = *reinterpret_cast<const uint4*>(st + (2 * rp) * kPitch);
      const uint4 h1 = *reinterpret_cast<const uint4*>(st + (2 * rp + 1) * kPitch);
      uint32_t s0, s1, m0, m1;
      if (G < 2) {
        s0 = h0.y & 0x3f3f3f3fu;
        s1 = h1.y & 0x3f3f3f3fu;
        m0 = h0.z & 0x3f3f3f3fu;
        m1 = h1.z & 0x3f3f3f3fu;
      } else {
        s0 = (h0.w & 0x0f0f0f0fu) | ((h0.y >> 2) & 0x30303030u);
        s1 = (h1.w & 0x0f0f0f0fu) | ((h1.y >> 2) & 0x30303030u);
        m0 = ((h0.w >> 4) & 0x0f0f0f0fu) | ((h0.z >> 2) & 0x30303030u);
        m1 = ((h1.w >> 4) & 0x0f0f0f0fu) | ((h1.z >> 2) & 0x30303030u);
      }
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
      const float2 dl0 = __fmul2_rn(d, sl), dl1 = __fmul2_rn(d, sh);
      const float2 ml0 = __fmul2_rn(dm, mlo), ml1 = __fmul2_rn(dm, mhi);
      // ---- v = x * dl on the current scales (x rows from the stage slot) ----
      const float* xs = reinterpret_cast<const float*>(st + kWBytes);  // [BATCH][32]
      float2 v[QB][2];
      uint32_t w[QB][2][2];
      uint32_t out = 0u;
#pragma unroll
      for (int j = 0; j < QB; ++j) {
        const int b = qd * QB + j;
        const float2 xv = *reinterpret_cast<const float2*>(xs + b * kRows + 2 * rp);
        v[j][0] = __fmul2_rn(xv, dl0);
        v[j][1] = __fmul2_rn(xv, dl1);
        mins[j][0] = fmaf(xv.x, ml0.x, fmaf(xv.y, ml0.y, mins[j][0]));
        mins[j][1] = fmaf(xv.x, ml1.x, fmaf(xv.y, ml1.y, mins[j][1]));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          w[j][h][0] = __float_as_uint(fmaf(v[j][h].x, scale[j], kMagic));
          w[j][h][1] = __float_as_uint(fmaf(v[j][h].y, scale[j], kMagic));
          out |= (w[j][h][0] ^ 0x4b000000u) | (w[j][h][1] ^ 0x4b000000u);
        }
      }
      // the sampled shrink test (see vbq_gemv_mma.cu), every second 32-row stage: bit b of
      // `small` = batch row b's sample (one value per lane) is 16x or more below its scale,
      // |n| < 2^16.  Each lane half owns one quarter of the rows; the bits of the other
      // half's quarter are set, so the warp-wide AND below is each row's AND over the lanes
      // that own it.
      uint32_t small = 0u;
      if ((it & 1) == 0) {
#pragma unroll
        for (int j = 0; j < QB; ++j)
          small |= (fabsf(v[j][0].x) * scale[j] < 65536.f) ? (1u << (qd * QB + j)) : 0u;
        small = (small & down_ok) | (((1u << QB) - 1u) << ((qd ^ 1) * QB));
      }
      // the pair's decisions: either warp's wait gave up -> both leave; either warp's
      // digits left their range, or some batch row of the warp sits 16x or more below its
      // scale in every lane (or the first stage) -> both flush, then rescale
      const bool need = __any_sync(0xffffffffu, out >= (1u << 23)) ||
                        __reduce_and_sync(0xffffffffu, small) != 0u || it == 0;
      if (lane == 0) flags[2 * warp] = (need ? 1u : 0u) | (ok ? 0u : 2u);
      pair_sync();
      const uint32_t fl = flags[2 * warp] | flags[2 * (warp ^ 1)];
      if (fl & 2u) {
        if (!ok && lane == 0) give_up();
        break;
      }
      if (fl & 1u) {
        // rare (and the first stage): flag non-finite values, move the sums to fp32 with
        // the old steps (both warps, before either changes them), then scale each batch row
        // of this warp's half to 2-4x its largest finite |v| over the lane half, encode again
        if (it > 0) flush();
        pair_sync();
#pragma unroll
        for (int j = 0; j < QB; ++j) {
          const float sum = (fabsf(v[j][0].x) + fabsf(v[j][0].y)) + (fabsf(v[j][1].x) + fabsf(v[j][1].y));
          nonfin |= (sum < 0x1p100f) ? 0u : (1u << (qd * QB + j));
          float m = fminf(fmaxf(fmaxf(fabsf(v[j][0].x), fabsf(v[j][0].y)),
                                fmaxf(fabsf(v[j][1].x), fabsf(v[j][1].y))), 0x1p99f);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127 + 1;
          e = e < kExpMin ? kExpMin : (e > kExpMax ? kExpMax : e);
          scale[j] = pow2f(21 - e);
          {
            const uint32_t bit = 1u << (qd * QB + j);
            down_ok = (qd * QB + j < batch && e > kExpMin) ? (down_ok | bit) : (down_ok & ~bit);
          }
          if (rp == 0) stp[qd * QB + j] = pow2f(e - 21);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            w[j][h][0] = __float_as_uint(fmaf(v[j][h].x, scale[j], kMagic));
            w[j][h][1] = __float_as_uint(fmaf(v[j][h].y, scale[j], kMagic));
          }
        }
      }
      // ---- B table: three signed digits of n per row pair (this warp's batch rows) ----
#pragma unroll
      for (int j = 0; j < QB; ++j) {
        const int b = qd * QB + j;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t wx = w[j][h][0] ^ 0x8080u, wy = w[j][h][1] ^ 0x8080u;
          uint8_t* col = tbl + (b >> 1) * C::kSetStride + h * kSbStride + 4 * (b & 1) * kColStride + kap0;
#pragma unroll
          for (int dg = 0; dg < 3; ++dg)
            *reinterpret_cast<uint16_t*>(col + dg * kColStride) = (uint16_t)__byte_perm(wx, wy, dg | ((4 + dg) << 4));
        }
      }
      pair_sync();  // the pair's table is complete (and the steps, after a rescale)
      // ---- the chunk: 16 byte columns x 32 rows, low- and high-nibble MMAs per set ----
      {
        uint32_t a0, a1, a2, a3;  // A rows m = g / g + 8: byte columns g / g + 8
        ldmatrix_a8_trans(lm_lane + (uint32_t)(s * C::kSlot), a0, a1, a2, a3);
        const uint32_t l0 = a0 & 0x0f0f0f0fu, l1 = a1 & 0x0f0f0f0fu, l2 = a2 & 0x0f0f0f0fu, l3 = a3 & 0x0f0f0f0fu;
        const uint32_t u0 = a0 & 0xf0f0f0f0u, u1 = a1 & 0xf0f0f0f0u, u2 = a2 & 0xf0f0f0f0u, u3 = a3 & 0xf0f0f0f0u;
#pragma unroll
        for (int z = 0; z < NSET; ++z) {
          const uint8_t* tz = tfrag + z * C::kSetStride;
          const uint2 bl = *reinterpret_cast<const uint2*>(tz);
          const uint2 bhf = *reinterpret_cast<const uint2*>(tz + kSbStride);
          mma_u8s8(acc[z][0], l0, l1, l2, l3, bl.x, bl.y);
          mma_u8s8(acc[z][1], u0, u1, u2, u3, bhf.x, bhf.y);
        }
      }
      __syncwarp();  // table and stage reads done
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty[s]));
    }
    __syncwarp();
    flush();
    // min-term sums: add over the 16 lanes of a half; non-finite flags over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      if (o < 16) {
#pragma unroll
        for (int j = 0; j < QB; ++j) {
          mins[j][0] += __shfl_xor_sync(0xffffffffu, mins[j][0], o);
          mins[j][1] += __shfl_xor_sync(0xffffffffu, mins[j][1], o);
        }
      }
      nonfin |= __shfl_xor_sync(0xffffffffu, nonfin, o);
    }
    float* mns = reinterpret_cast<float*>(smem + C::kMinOff) + pr * BATCH * 2;  // [b][h]
    if (rp == 0) {
#pragma unroll
      for (int j = 0; j < QB; ++j) {
        mns[(qd * QB + j) * 2 + 0] = mins[j][0];
        mns[(qd * QB + j) * 2 + 1] = mins[j][1];
      }
    }
    if (lane == 0) flags[2 * warp + 1] = nonfin;  // this warp's batch rows' flags
  }

  // ---- this CTA's partial sums [BATCH][256] into the ring (idle now) ----
  __syncthreads();
  float* outp = reinterpret_cast<float*>(smem + C::kRingOff);
  if (warp < kConsumers) {
    const int c = warp, G = c >> 1, g = lane >> 2, t = lane & 3;
    const float* fac = reinterpret_cast<const float*>(smem + C::kFacOff + warp * C::kFac);
    const float* mns = reinterpret_cast<const float*>(smem + C::kMinOff) + G * BATCH * 2;
    const volatile uint32_t* flg = reinterpret_cast<const volatile uint32_t*>(smem + C::kFlagOff);
    const unsigned nf = flg[2 * warp + 1] | flg[2 * (warp ^ 1) + 1];  // the pair's rows
    // MMA row g (t even) / g + 8 (t odd) = byte column g / g + 8 of the chunk
    const int colb = 64 * G + 16 * (c & 1) + g + 8 * (t & 1);
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int b = 2 * z + (t >> 1);
        const float val = fac[(z * 2 + h) * 32 + lane] - mns[b * 2 + h];
        outp[b * 256 + colb + 32 * h] = ((nf >> b) & 1u) ? __int_as_float(0x7fc00000) : val;
      }
  }
  __syncthreads();

  if (S == 1) {
    for (int e = threadIdx.x; e < batch * 256; e += kThreads)
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = epi_apply(epi, outp[e], e >> 8, N, tile * 256 + (e & 255));
    return;
  }
  // ---- split-K across the cluster: CTA r adds columns n0 .. n1 - 1 of every split's
  // partial sums in split order; the second barrier keeps each CTA's shared memory alive
  // until every CTA has read it ----
  cluster_sync_all();
  const uint32_t rank = cluster_rank();
  const int n0 = (256 * (int)rank) / S, n1 = (256 * ((int)rank + 1)) / S, wdt = n1 - n0;
  const uint32_t base = smem_u32(outp);
  for (int idx = threadIdx.x; idx < batch * wdt; idx += kThreads) {
    const int b = idx / wdt, n = n0 + idx % wdt;
    const uint32_t off = (uint32_t)((b * 256 + n) * 4);
    float sum = 0.f;
    for (int sp = 0; sp < S; ++sp) sum += ld_cluster_f32(mapa_u32(base + off, (uint32_t)sp));
    y[(int64_t)b * N + tile * 256 + n] = epi_apply(epi, sum, b, N, tile * 256 + n);
  }
  cluster_sync_all();
}

}  // namespace gwide

// ---- host side -----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnW)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnW encode_fn_w() {
  static EncodeTiledFnW fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnW>(p);
  });
  return fn;
}

// Splits per tile: at most one wave (two CTAs per SM for batch 8, one for 16) and 16 (one
// cluster), and room for every tile's cluster with 25 % to spare (as the batch 1..4 kernel).
template <int BATCH>
static int choose_splits_wide(int64_t K, int64_t N) {
  using C = gwide::Cfg<BATCH>;
  const int tiles = (int)(N / 256);
  const int64_t tot_st = (K + gwide::kRows - 1) / gwide::kRows;
  const int slots = (BATCH <= 8 ? 2 : 1) * sm_count();
  int S = tiles > 0 ? slots / tiles : 1;
  if (S > 16) S = 16;
  if (S > tot_st) S = (int)tot_st;
  if (S < 1) S = 1;
  if (gemv_split_override()) {
    S = gemv_split_override() > 16 ? 16 : gemv_split_override();
    return S > tot_st ? (int)tot_st : S;
  }
  struct Entry { int64_t tiles; int s_in, s_out; };
  static Entry cache[16];
  static int n_cache = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_cache; ++i)
    if (cache[i].tiles == tiles && cache[i].s_in == S) return cache[i].s_out;
  const int s_in = S;
  for (; S > 1; --S) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)S, 1);
    cfg.blockDim = dim3(gwide::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, gwide::gemv_wide_kernel<BATCH>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      active = 0;
    }
    if (active * 4 >= tiles * 5) break;
  }
  if (n_cache < 16) cache[n_cache++] = Entry{tiles, s_in, S};
  return S;
}

template <int BATCH>
static cudaError_t launch_wide_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, cudaStream_t st, Epi epi) {
  using namespace gwide;
  using C = Cfg<BATCH>;
  auto enc = encode_fn_w();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw, mx;
  {
    cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)RB};
    cuuint32_t box[2] = {(cuuint32_t)(kPitch / 2), (cuuint32_t)kRows};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {  // x [batch][K] fp32; rows past K and batch rows past `batch` read as zeros
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)batch};
    cuuint64_t strides[1] = {(cuuint64_t)K * 4};
    cuuint32_t box[2] = {(cuuint32_t)kRows, (cuuint32_t)BATCH};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  auto kern = gemv_wide_kernel<BATCH>;
  static DeviceOnce configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  const int S = choose_splits_wide<BATCH>(K, N);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
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
  return cudaLaunchKernelEx(&cfg, kern, mw, mx, y, (int)K, (int)N, batch, epi);
}

// The wide kernel reads x through a TMA tensor map: rows of x 16-byte aligned.
// A warp's s32 sums run over up to K rows with terms below 240 * 128 in magnitude: K is
// capped at 2^16 (longer rows run as groups of 4 on the batch 1..4 kernel).
bool gemv_wide_fits(const float* x, int64_t K, int64_t N, int batch) {
  return batch >= 5 && batch <= 16 && K >= 1 && K <= 65536 && K % 4 == 0 && N % 256 == 0 &&
         N > 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
}

cudaError_t launch_gemv_wide_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  // x arrives by TMA as it is stored: no SwiGLU input here (the caller routes that away)
  if (!gemv_wide_fits(x, K, N, batch) || row_bytes % 16 != 0 || f.swiglu_x) return cudaErrorNotSupported;
  const Epi epi{f.bias, f.res};
  if (batch <= 8) return launch_wide_t<8>(x, w, y, K, N, row_bytes, batch, st, epi);
  return launch_wide_t<16>(x, w, y, K, N, row_bytes, batch, st, epi);
}

cudaError_t gemv_wide_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_wide_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_wide_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
