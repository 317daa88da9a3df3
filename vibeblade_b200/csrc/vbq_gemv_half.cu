// vbq_gemv_half.cu -- Q4_K dequant-GEMV for batch 5..16 on the fp16 tensor cores.
//
//   y[b, n] = sum_k x[b, k] * (dl[k, s] * q[k, n] - ml[k, s]),  dl = d * sc, ml = dmin * m
//
// (cpp/src/dequant.cpp:268-301, :739-780; s = the 32-column sub-block of n), regrouped as
//
//   y[b, n] = sum_k (sc * q)[k, n] * (x * d)[b, k]  -  sum_k m[k, s] * (x * dmin)[b, k]
//
// so that the matrix operand carries everything that changes along n and the activation
// operand only what changes along k:
//   * A (16 columns x 16 rows per mma.sync m16n8k16): sc * q, an integer in 0..945 and so
//     exact in fp16.  A byte-granular ldmatrix.trans gives each lane four rows of one code
//     byte per register; one LOP3 puts a nibble under the fp16 exponent of 1024 (1024 + q,
//     or 1024 + 16 q for the high nibble) and one HFMA2 with (sc, -1024 sc) or
//     (sc / 16, -64 sc) leaves sc * q exactly (the fused product is exact and representable).
//   * B (16 rows x 8 columns): v = x * d on a power-of-two scale per CTA and batch row,
//     split into fp16 hi + lo (22 significant bits); each batch row takes two B columns, so
//     the two partial sums add up in fp32 at the end.  The table is built once per CTA and
//     128-column group for all of the tile's 256 columns, not per sub-block.
//   * the min term: A = m (0..63, exact) for the tile's 8 sub-blocks, B = x * dmin on the
//     same scale, split the same way; one MMA per 16 rows and 8 B columns.
// fp32 accumulators.  A scale is set from the first stage's largest |v| (2^11 .. 2^12) and
// set again, with the sums so far multiplied by the exact power-of-two ratio, only when a
// later |v| reaches 2^15 (or when the first values were all zero); below the scale, hi + lo
// keep full precision down to 2^-14 of it and absolute precision 2^-25 under that.  A
// non-finite v marks its batch row, whose outputs are then NaN (as in vbq_gemv_mma.cu).
//
// Decomposition: a CTA owns one 256-column tile and every S-th 64-row stage of the matrix;
// the S splits of a tile form a thread-block cluster and add their partial sums in split
// order (deterministic) through distributed shared memory, as vbq_gemv_wide.cu does.  Warp
// 8 TMA-loads the stages (weights before the previous grid is waited for, x after) into a
// ring; consumer warp w owns code bytes 16w .. 16w + 15 of the block (columns 64c + 16h +
// 0..15 and 64c + 32 + 16h + 0..15, c = w / 2, h = w % 2) over every row, so no two warps
// share an output column.  Per stage the eight warps first build the next stage's tables
// together (a 256-thread named barrier publishes them and carries the rescale vote), then
// run this stage's MMAs.  Waits are bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "vbq_common.cuh"
#include "vbq_gemv_half.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up).
__device__ unsigned g_gemv_half_status = 0;

namespace ghalf {
using namespace gmma;

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 64;                  // rows per stage = 4 slices of 16
constexpr int kPitch = 144;                // one Q4_K block per row
constexpr int kWBytes = kRows * kPitch;    // 9216, a multiple of 128
constexpr float kOvf = 32768.f;            // |v| on the scale at which the scale is set again
constexpr int kTarget = 11;                // the scale puts the largest |v| in [2^11, 2^12)

template <int BATCH, bool SW> struct Cfg {
  static constexpr int kNC = 2 * BATCH;                        // B columns: (batch row, hi / lo)
  static constexpr int kNT = kNC / 8;                          // n8 tiles
  static constexpr int kXBytes = (SW ? 2 : 1) * BATCH * kRows * 4;  // [BATCH][64] fp32 (gate, up)
  static constexpr int kSlot = kWBytes + kXBytes;
  static constexpr int kStages = SW && BATCH == 16 ? 4 : 6;
  // tables of one stage: B and B-min [slice][column][16 fp16 in fragment order], the A
  // multipliers [slice][t][c][8 half2] (t stride padded to 144 B: the four t of a load
  // land in different banks), the min-term A [slice][t][sub-block][2 half2]
  static constexpr int kBT = 4 * kNC * 32;
  static constexpr int kST = 4 * 4 * 144;
  static constexpr int kMT = 4 * 4 * 8 * 8;
  static constexpr int kTbl = 2 * kBT + kST + kMT;
  static constexpr int kRingOff = 0;
  static constexpr int kTblOff = kStages * kSlot;              // two table buffers
  static constexpr int kMiscOff = kTblOff + 2 * kTbl;
  // misc: scale [16] f32, max [16] u32, non-finite bits u32, abort flag
  static constexpr int kBarOff = kMiscOff + 256;
  static constexpr int kSmem = kBarOff + 128 + 128;            // + alignment slack
  static constexpr int kOutBytes = BATCH * 256 * 4 + 4 * BATCH * 8 * 4;  // partial sums + mins
  static_assert(kSlot % 128 == 0, "TMA destinations 128-byte aligned");
  static_assert(kOutBytes <= kStages * kSlot, "partial sums inside the ring");
  static_assert(kSmem <= 113 * 1024, "two CTAs per SM");
};

struct Bars {
  uint64_t full[8], empty[8];
};

template <int BATCH, bool SW>
__global__ void __launch_bounds__(kThreads, 2)
gemv_half_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 float* y, int K, int N, int batch, Epi epi) {
  using C = Cfg<BATCH, SW>;
  constexpr int NC = C::kNC, NT = C::kNT, STG = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  Bars& bars = *reinterpret_cast<Bars*>(smem + C::kBarOff);
  float* sc_e = reinterpret_cast<float*>(smem + C::kMiscOff);             // [16] scale per batch row
  unsigned* maxv = reinterpret_cast<unsigned*>(smem + C::kMiscOff + 64);  // [16] |v| bits
  unsigned* nonfin = reinterpret_cast<unsigned*>(smem + C::kMiscOff + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 132);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto slot = [&](int s) { return smem + C::kRingOff + s * C::kSlot; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), kConsumers);
    }
    *nonfin = 0u;
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (threadIdx.x < 16) {
    sc_e[threadIdx.x] = 0.f;  // 0: not set yet
    maxv[threadIdx.x] = 0u;
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_half_status, kStatusTimeout);
  };

  // per-lane accumulators: [low / high nibble m-tile][n-tile][fragment], min term [n-tile]
  float acc[2][NT][4], accm[NT][4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[h][nt][0] = acc[h][nt][1] = acc[h][nt][2] = acc[h][nt][3] = 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) accm[nt][0] = accm[nt][1] = accm[nt][2] = accm[nt][3] = 0.f;

  if (warp == kConsumers) {
    // ---------------------------- TMA producer ----------------------------
    if (lane == 0) {
      int it = 0;
      bool waited = false;
      auto issue_x = [&](int j) {
        const uint32_t dst = smem_u32(slot(j % STG) + kWBytes);
        const uint32_t fb = smem_u32(&bars.full[j % STG]);
        const int k0 = (split + S * j) * kRows;
        tma_load_2d(dst, &tmap_x, k0, 0, fb);
        if constexpr (SW) tma_load_2d(dst + BATCH * kRows * 4, &tmap_x, K + k0, 0, fb);
      };
      for (; it < nst && !*abort_flag; ++it) {
        const int s = it % STG;
        if (it == STG) {  // the ring is full: wait for the previous grid, then x
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
          for (int j = 0; j < STG; ++j) issue_x(j);
        }
        if (!mbar_wait_hinted(smem_u32(&bars.empty[s]), ((it / STG) & 1) ^ 1, kWaitBudgetCycles)) {
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
      for (int j = (it > STG ? it - STG : 0); j < it; ++j)
        mbar_wait_hinted(smem_u32(&bars.full[j % STG]), (j / STG) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    const int c = warp >> 1, hh = warp & 1;  // code bytes 32c + 16hh .. + 15 of each row
    const int g = lane >> 2, t = lane & 3;   // MMA fragment role
    // table role: row pair p of the stage (slice pj, rows 4pt + pw and 4pt + pw + 2 of it)
    const int p = lane, pj = p >> 3, pt = (p >> 1) & 3, pw = p & 1;
    const int pr0 = 16 * pj + 4 * pt + pw, pr1 = pr0 + 2;
    auto tbl = [&](int q) { return smem + C::kTblOff + q * C::kTbl; };
    const uint32_t lm_lane = smem_u32(smem) + (uint32_t)(C::kRingOff + lane * kPitch + 16 + 32 * c + 16 * hh);

    // x * d and x * dmin of the lane's row pair for batch row b (0 past K)
    auto load_pair = [&](const uint8_t* st, int it, int b, float2& vd, float2& vm) {
      const float* xs = reinterpret_cast<const float*>(st + kWBytes);
      float x0, x1;
      if constexpr (SW) {
        x0 = swiglu1(xs[b * kRows + pr0], xs[BATCH * kRows + b * kRows + pr0]);
        x1 = swiglu1(xs[b * kRows + pr1], xs[BATCH * kRows + b * kRows + pr1]);
      } else {
        x0 = xs[b * kRows + pr0];
        x1 = xs[b * kRows + pr1];
      }
      const int k0 = (split + S * it) * kRows;
      if (k0 + pr0 >= K) x0 = 0.f;  // rows past K: zero weights, and x there may be anything
      if (k0 + pr1 >= K) x1 = 0.f;
      const uint32_t w0 = *reinterpret_cast<const uint32_t*>(st + pr0 * kPitch);
      const uint32_t w1 = *reinterpret_cast<const uint32_t*>(st + pr1 * kPitch);
      vd = make_float2(x0 * f16_ref(w0 & 0xffffu), x1 * f16_ref(w1 & 0xffffu));
      vm = make_float2(x0 * f16_ref(w0 >> 16), x1 * f16_ref(w1 >> 16));
    };

    // Tables of stage `it` into buffer q; returns whether some v needs a new scale.
    auto build = [&](int it, int q) -> bool {
      const uint8_t* st = slot(it % STG);
      uint8_t* T = tbl(q);
      bool ovf = false;
      // A multipliers and min-term A of sub-block s = warp for the lane's row pair
      {
        const int s = warp;
        const uint4 h0 = *reinterpret_cast<const uint4*>(st + pr0 * kPitch);
        const uint4 h1 = *reinterpret_cast<const uint4*>(st + pr1 * kPitch);
        int sc0, m0, sc1, m1;
        q4k_scale_min(s, h0.y, h0.z, h0.w, sc0, m0);
        q4k_scale_min(s, h1.y, h1.z, h1.w, sc1, m1);
        const float f0 = (float)sc0, f1 = (float)sc1;
        uint32_t mul, add;
        if (s & 1) {  // high nibbles: (1024 + 16 q) * sc / 16 - 64 sc
          mul = h2_bits(__floats2half2_rn(f0 * 0.0625f, f1 * 0.0625f));
          add = h2_bits(__floats2half2_rn(-64.f * f0, -64.f * f1));
        } else {      // low nibbles: (1024 + q) * sc - 1024 sc
          mul = h2_bits(__floats2half2_rn(f0, f1));
          add = h2_bits(__floats2half2_rn(-1024.f * f0, -1024.f * f1));
        }
        *reinterpret_cast<uint2*>(T + 2 * C::kBT + (pj * 4 + pt) * 144 + (s >> 1) * 32 + (s & 1) * 16 + pw * 8) =
            make_uint2(mul, add);
        *reinterpret_cast<uint32_t*>(T + 2 * C::kBT + C::kST + ((pj * 4 + pt) * 8 + s) * 8 + pw * 4) =
            h2_bits(__floats2half2_rn((float)m0, (float)m1));
      }
      // B and B-min columns of batch rows warp (+ 8) for the lane's row pair
#pragma unroll
      for (int i = 0; i < (BATCH + 7) / 8; ++i) {
        const int b = warp + 8 * i;
        if (b >= BATCH) break;
        float2 vd, vm;
        load_pair(st, it, b, vd, vm);
        const float se = sc_e[b];
        const float2 sd = make_float2(vd.x * se, vd.y * se), sm = make_float2(vm.x * se, vm.y * se);
        ovf |= !(fabsf(sd.x) < kOvf) | !(fabsf(sd.y) < kOvf) | !(fabsf(sm.x) < kOvf) | !(fabsf(sm.y) < kOvf);
        ovf |= se == 0.f && (vd.x != 0.f || vd.y != 0.f || vm.x != 0.f || vm.y != 0.f);
        const __half2 dh = __floats2half2_rn(sd.x, sd.y), mh = __floats2half2_rn(sm.x, sm.y);
        const float2 dhf = __half22float2(dh), mhf = __half22float2(mh);
        const __half2 dl = __floats2half2_rn(sd.x - dhf.x, sd.y - dhf.y);
        const __half2 ml = __floats2half2_rn(sm.x - mhf.x, sm.y - mhf.y);
        const int col = 8 * (b >> 2) + 2 * (b & 3);
        uint8_t* bd = T + (pj * NC + col) * 32 + 8 * pt + 4 * pw;
        *reinterpret_cast<uint32_t*>(bd) = h2_bits(dh);
        *reinterpret_cast<uint32_t*>(bd + 32) = h2_bits(dl);
        *reinterpret_cast<uint32_t*>(bd + C::kBT) = h2_bits(mh);
        *reinterpret_cast<uint32_t*>(bd + C::kBT + 32) = h2_bits(ml);
      }
      return ovf;
    };

    // Sets the scales again from stage `it`'s values (rows whose scale is unset or too
    // small for this stage), multiplies the sums so far by the exact ratio, and rebuilds
    // the stage's tables.  Entered by all 256 consumer threads together.
    auto rescale = [&](int it, int q) {
      if (threadIdx.x < BATCH) maxv[threadIdx.x] = 0u;
      bar_sync_c();
      const uint8_t* st = slot(it % STG);
#pragma unroll
      for (int i = 0; i < (BATCH + 7) / 8; ++i) {
        const int b = warp + 8 * i;
        if (b >= BATCH) break;
        float2 vd, vm;
        load_pair(st, it, b, vd, vm);
        float mx = 0.f;
        bool bad = false;
        const float a[4] = {fabsf(vd.x), fabsf(vd.y), fabsf(vm.x), fabsf(vm.y)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (a[j] <= 3.0e38f) mx = fmaxf(mx, a[j]);
          else bad = true;  // NaN or inf
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
          atomicMax(&maxv[b], __float_as_uint(mx));
          if (bad) atomicOr(nonfin, 1u << b);
        }
      }
      bar_sync_c();
      // new scale of batch row b (every thread computes the same from the same values)
      auto new_scale = [&](int b) -> float {
        const float old = sc_e[b];
        const float m = __uint_as_float(maxv[b]);
        if (old > 0.f && m * old < kOvf) return old;  // this row fits its scale
        if (m == 0.f) return old;                     // nothing to set it from
        int e = kTarget - ((int)((__float_as_uint(m) >> 23) & 0xffu) - 127);
        e = e < -126 ? -126 : (e > 126 ? 126 : e);
        return pow2f(e);
      };
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int b = 4 * nt + t;
        const float old = sc_e[b], nw = new_scale(b);
        const float r = (old > 0.f && nw != old) ? nw * inv_pow2(old) : 1.f;  // exact
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[0][nt][j] *= r;
          acc[1][nt][j] *= r;
          accm[nt][j] *= r;
        }
      }
      float nsc = 0.f;
      if (threadIdx.x < BATCH) nsc = new_scale(threadIdx.x);
      bar_sync_c();  // every thread has read the old scales
      if (threadIdx.x < BATCH) sc_e[threadIdx.x] = nsc;
      bar_sync_c();
      build(it, q);
      bar_sync_c();  // tables published
    };

    // MMAs of stage `it` from table buffer q
    auto mma_stage = [&](int it, int q) {
      const uint8_t* T = tbl(q);
      const uint32_t lm = lm_lane + (uint32_t)((it % STG) * C::kSlot);
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        uint32_t r0, r1, r2, r3;  // rows 32 grp + 4t .. (+ 16): byte column g / g + 8
        ldmatrix_a8_trans(lm + (uint32_t)(grp * 32 * kPitch), r0, r1, r2, r3);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const int j = 2 * grp + ks;
          const uint32_t ra = ks ? r2 : r0, rb = ks ? r3 : r1;
          const uint8_t* sp = T + 2 * C::kBT + (j * 4 + t) * 144 + c * 32;
          const uint4 sl = *reinterpret_cast<const uint4*>(sp);       // low-nibble sub-block
          const uint4 sh = *reinterpret_cast<const uint4*>(sp + 16);  // high-nibble sub-block
          // rows (4t, 4t + 2) as k = 2t, 2t + 1 and (4t + 1, 4t + 3) as k = 2t + 8, 2t + 9
          const uint32_t ra1 = ra >> 8, rb1 = rb >> 8;
          const uint32_t l0 = hfma2_u(lop_nib(ra, 0x000f000fu), sl.x, sl.y);
          const uint32_t l1 = hfma2_u(lop_nib(rb, 0x000f000fu), sl.x, sl.y);
          const uint32_t l2 = hfma2_u(lop_nib(ra1, 0x000f000fu), sl.z, sl.w);
          const uint32_t l3 = hfma2_u(lop_nib(rb1, 0x000f000fu), sl.z, sl.w);
          const uint32_t h0 = hfma2_u(lop_nib(ra, 0x00f000f0u), sh.x, sh.y);
          const uint32_t h1 = hfma2_u(lop_nib(rb, 0x00f000f0u), sh.x, sh.y);
          const uint32_t h2 = hfma2_u(lop_nib(ra1, 0x00f000f0u), sh.z, sh.w);
          const uint32_t h3 = hfma2_u(lop_nib(rb1, 0x00f000f0u), sh.z, sh.w);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint2 bb = *reinterpret_cast<const uint2*>(T + (j * NC + nt * 8 + g) * 32 + 8 * t);
            mma_f16(acc[0][nt], l0, l1, l2, l3, bb.x, bb.y);
            mma_f16(acc[1][nt], h0, h1, h2, h3, bb.x, bb.y);
          }
        }
      }
      if (warp < 4) {  // the min term of slice j = warp
        const uint2 am = *reinterpret_cast<const uint2*>(T + 2 * C::kBT + C::kST + ((warp * 4 + t) * 8 + g) * 8);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint2 bb = *reinterpret_cast<const uint2*>(T + C::kBT + (warp * NC + nt * 8 + g) * 32 + 8 * t);
          mma_f16(accm[nt], am.x, 0u, am.y, 0u, bb.x, bb.y);
        }
      }
    };

    // a full-barrier wait; once the kernel is aborting, waits are skipped (the values are
    // then garbage, and the status word reports the failure)
    auto wait_full = [&](int it) {
      if (*abort_flag) return;
      const bool ok = __all_sync(0xffffffffu, mbar_wait_hinted(smem_u32(&bars.full[it % STG]), (it / STG) & 1,
                                                               kWaitBudgetCycles));
      if (!ok && lane == 0) give_up();
    };

    if (nst > 0) {
      wait_full(0);
      rescale(0, 0);  // the first stage sets the scales
    }
#pragma unroll 1
    for (int it = 0; it < nst; ++it) {
      const int q = it & 1;
      bool ovf = false;
      if (it + 1 < nst) {
        wait_full(it + 1);
        ovf = build(it + 1, q ^ 1);
      }
      mma_stage(it, q);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty[it % STG]));
      if (bar_or_c(ovf)) rescale(it + 1, q ^ 1);  // ovf implies it + 1 < nst
    }
  }

  // ---- this CTA's partial sums [BATCH][256] and min sums [4][BATCH][8] into the ring ----
  __syncthreads();
  float* outp = reinterpret_cast<float*>(smem + C::kRingOff);
  float* minp = outp + BATCH * 256;
  if (warp < kConsumers) {
    const int c = warp >> 1, hh = warp & 1, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int b = 4 * nt + t;
      const float se = sc_e[b];
      const float inv = se > 0.f ? inv_pow2(se) : 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n0 = 64 * c + 32 * h + 16 * hh + g;
        outp[b * 256 + n0] = (acc[h][nt][0] + acc[h][nt][1]) * inv;
        outp[b * 256 + n0 + 8] = (acc[h][nt][2] + acc[h][nt][3]) * inv;
      }
      if (warp < 4) minp[(warp * BATCH + b) * 8 + g] = (accm[nt][0] + accm[nt][1]) * inv;
    }
  }
  __syncthreads();
  const unsigned nf = *nonfin;
  for (int e = threadIdx.x; e < BATCH * 256; e += kThreads) {
    const int b = e >> 8, s = (e & 255) >> 5;
    const float mn = ((minp[b * 8 + s] + minp[(BATCH + b) * 8 + s]) + minp[(2 * BATCH + b) * 8 + s]) +
                     minp[(3 * BATCH + b) * 8 + s];
    outp[e] = ((nf >> b) & 1u) ? __int_as_float(0x7fc00000) : outp[e] - mn;
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

}  // namespace ghalf

// ---- host side -----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnH)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnH encode_fn_h() {
  static EncodeTiledFnH fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnH>(p);
  });
  return fn;
}

// Splits per tile: at most one wave (two CTAs per SM) and 16 (one cluster), and room for
// every tile's cluster with 25 % to spare (as the other tensor-core GEMV kernels).
template <int BATCH, bool SW>
static int choose_splits_half(int64_t K, int64_t N) {
  using C = ghalf::Cfg<BATCH, SW>;
  const int tiles = (int)(N / 256);
  const int64_t tot_st = (K + ghalf::kRows - 1) / ghalf::kRows;
  int S = tiles > 0 ? 2 * sm_count() / tiles : 1;
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
    cfg.blockDim = dim3(ghalf::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int active = 0;
    if (cudaOccupancyMaxActiveClusters(&active, ghalf::gemv_half_kernel<BATCH, SW>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      active = 0;
    }
    if (active * 4 >= tiles * 5) break;
  }
  if (n_cache < 16) cache[n_cache++] = Entry{tiles, s_in, S};
  return S;
}

template <int BATCH, bool SW>
static cudaError_t launch_half_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, cudaStream_t st, Epi epi) {
  using namespace ghalf;
  using C = Cfg<BATCH, SW>;
  auto enc = encode_fn_h();
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
  {  // x [batch][K] (or [batch][2K]: gate | up) fp32; batch rows past `batch` read as zeros
    const int64_t width = SW ? 2 * K : K;
    cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)batch};
    cuuint64_t strides[1] = {(cuuint64_t)width * 4};
    cuuint32_t box[2] = {(cuuint32_t)kRows, (cuuint32_t)BATCH};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  auto kern = gemv_half_kernel<BATCH, SW>;
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
  const int S = choose_splits_half<BATCH, SW>(K, N);
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

// VBQ_GEMV_INT8=1 keeps batch 5..16 on the integer kernels (comparison runs).
static bool int8_override() {
  static const bool v = [] {
    const char* env = getenv("VBQ_GEMV_INT8");
    return env && atoi(env) == 1;
  }();
  return v;
}

// x arrives by TMA: rows of x (and the gate | up halves of a SwiGLU input) 16-byte aligned.
// Batches 2..4 stay on the integer kernel, which is faster there (Llama-8B decode layer on
// B200: batch 4 67.7 us integer / 96.8 us here; batch 8 125.9 / 114.3; batch 16 206.6 /
// 164.7).
bool gemv_half_fits(const float* x, int64_t K, int64_t N, int batch) {
  return !int8_override() && batch >= 5 && batch <= 16 && K >= 1 && K <= (1 << 24) && K % 4 == 0 &&
         N % 256 == 0 && N > 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
}

cudaError_t launch_gemv_half_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_half_fits(x, K, N, batch) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  const Epi epi{f.bias, f.res};
  if (f.swiglu_x) {
    if (batch <= 8) return launch_half_t<8, true>(x, w, y, K, N, row_bytes, batch, st, epi);
    return launch_half_t<16, true>(x, w, y, K, N, row_bytes, batch, st, epi);
  }
  if (batch <= 8) return launch_half_t<8, false>(x, w, y, K, N, row_bytes, batch, st, epi);
  return launch_half_t<16, false>(x, w, y, K, N, row_bytes, batch, st, epi);
}

cudaError_t gemv_half_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_half_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_half_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
