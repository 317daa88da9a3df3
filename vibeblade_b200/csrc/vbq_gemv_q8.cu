// vbq_gemv_q8.cu -- Q8_0 dequant-GEMV on the integer tensor cores (decode, batch 1..4), and
// the same kernel for the reference dispatcher's 32-value 4- and 5-bit blocks (Q4_0, Q4_1,
// Q5_0, Q5_1; template F, see QF below).
//
//   y[b, n] = sum_k x[b, k] * d[k, j] * q[k, n]      (GGUF Q8_0: 34-byte blocks of 32 columns,
//   fp16 scale d then 32 int8 codes; cpp/src/cuda_kernels.cu:718-735, vibeblade/loader.py:129)
//
// The codes are the s8 A operand of mma.sync m16n8k32 as they are; v = x * d per (row,
// block) goes into the B columns as three signed byte digits of a 22-bit fixed-point
// integer on a power-of-two scale per warp and batch row, with an all-ones column for the
// digits' offset, as in the Q4_K kernel (vbq_gemv_mma.cu).  Accumulation is exact s32.
// As there, the scale is set again (after a flush to fp32) when a stage's |v| outgrows it
// or sits 16x or more below the value it was set from, so an outlier activation coarsens
// only its own stage's rows.
//
// Layout: a CTA owns one 256-column tile (8 blocks, 272 bytes of each row) and every S-th
// 64-row stage.  A block's codes start 2 bytes into it, so rows are only 2-byte aligned
// and ldmatrix cannot read them: each lane gathers its A fragment with 16-bit shared loads
// (two rows x two codes per load pair) and byte permutes.  8 consumer warps = 2 row slices
// (32 rows) x 4 column quarters (2 blocks = 64 columns); warp 8 TMA-loads the stages.
// Split-K: the S splits of a tile form a cluster; splits 1..S-1 push their partial sums
// into split 0's shared memory with st.async and exit, split 0 adds them in split order.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "vbq_common.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {

__device__ unsigned g_gemv_q8_status = 0;

namespace gq8 {
using namespace gmma;

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 64;                 // rows per stage
constexpr int kStages = 4;
constexpr int kColStride = 32;
constexpr int kSbStride = 288;            // per block: 8 columns + pad (lane halves 8 banks apart)
constexpr int kTblBytes = 2 * kSbStride;  // the warp's 2 blocks, one column set
constexpr int kRedBytes = kConsumers * 4 * 64 * 4 + 4 * 256 * 4;  // [warp][b][64] + [b][256]

struct Bars {
  uint64_t full[kStages], empty[kStages];
  uint64_t red;
  int abort;
};
// Block formats the kernel reads: Q8_0 (s8 codes), and the 32-value 4- and 5-bit blocks
// of the reference's dispatcher (cpp/src/dequant.cpp:23-93: value i = nibble i & 1 of code
// byte i >> 1, fifth bit = bit i of the 32-bit qh), whose codes enter the MMA as u8 with
// their offset (-8 q, -16 q) or min term (+ m) summed apart in fp32.
template <int F> struct QF;
template <> struct QF<kQ8_0> {
  static constexpr int kBB = 34, kCO = 2, kQH = -1, kM = -1;
  static constexpr bool kNib = false;
  static constexpr float kOff = 0.f;
};
template <> struct QF<kQ4_0> {
  static constexpr int kBB = 18, kCO = 2, kQH = -1, kM = -1;
  static constexpr bool kNib = true;
  static constexpr float kOff = -8.f;   // (q - 8) * d
};
template <> struct QF<kQ4_1> {
  static constexpr int kBB = 20, kCO = 4, kQH = -1, kM = 2;
  static constexpr bool kNib = true;
  static constexpr float kOff = 0.f;    // d * q + m
};
template <> struct QF<kQ5_0> {
  static constexpr int kBB = 22, kCO = 6, kQH = 2, kM = -1;
  static constexpr bool kNib = true;
  static constexpr float kOff = -16.f;  // (q - 16) * d
};
template <> struct QF<kQ5_1> {
  static constexpr int kBB = 24, kCO = 8, kQH = 4, kM = 2;
  static constexpr bool kNib = true;
  static constexpr float kOff = 0.f;    // d * q + m
};
// a row of a stage: the tile's 8 blocks (kTile = 272 / 144 / 160 / 176 / 192 bytes), loaded
// by a TMA box kPitch bytes wide.  Q4_1 and Q5_1 take 16 bytes more (the next tile's first
// bytes, or zeros past the row): at 160 / 192 bytes the rows a lane group gathers (2t apart)
// fall into 2 / 1 bank groups; at 176 / 208 into 4.
template <int F> struct Geo {
  static constexpr int kTile = 8 * QF<F>::kBB;
  static constexpr int kPitch = kTile + ((F == kQ4_1 || F == kQ5_1) ? 16 : 0);
  static constexpr int kStageBytes = kRows * kPitch;  // a multiple of 128
  static constexpr int kTblOff = kStages * kStageBytes;
  static_assert(kStageBytes % 128 == 0, "stages stay 128-byte aligned");
  static_assert(kRedBytes <= kStages * kStageBytes, "reduction buffer inside the ring");
};
template <int NSET, int F = kQ8_0> struct Lay {
  static constexpr int kBarOff = Geo<F>::kTblOff + kConsumers * NSET * kTblBytes;
  static constexpr int kRecvOff = kBarOff + 128;
  static constexpr int kSmem = kRecvOff + 128;  // + alignment slack; plus the receive slots
};

__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t saddr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(saddr));
  return (uint32_t)v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}

template <int BATCH, bool SWIGLU, int F = kQ8_0>
__global__ void __launch_bounds__(kThreads, 2)
gemv_q8_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ x,
               float* y, int K, int N, int batch, Epi epi) {
  using Q = QF<F>;
  constexpr int kPitch = Geo<F>::kPitch, kStageBytes = Geo<F>::kStageBytes;
  constexpr int NSET = BATCH <= 2 ? 1 : 2;  // B column sets: two batch rows per set
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  using L = Lay<NSET, F>;
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 64-row stages split, split + S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto stage = [&](int s) { return smem + s * kStageBytes; };

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
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_q8_status, kStatusTimeout);
  };

  float fac[NSET][4];  // flushed fp32 sums [set][chunk]: MMA row g (lanes t even) / g + 8 (t odd)
  unsigned nonfin = 0u;
  // 4- and 5-bit formats: the offset / min term of the lane's table block and rows, per
  // batch row (summed over the block's 16 lanes at the end)
  float mo[BATCH];
#pragma unroll
  for (int b = 0; b < BATCH; ++b) mo[b] = 0.f;
#pragma unroll
  for (int z = 0; z < NSET; ++z)
#pragma unroll
    for (int k = 0; k < 4; ++k) fac[z][k] = 0.f;

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
        mbar_arrive_expect_tx(fb, kStageBytes);
        tma_load_2d(smem_u32(stage(s)), &tmap_w, tile * (Geo<F>::kTile / 2), (split + S * it) * kRows, fb);
      }
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait_hinted(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    const int rw = 32 * (warp >> 2);  // row slice: rows rw .. rw + 31 of each stage
    const int cq = warp & 3;          // column quarter: blocks 2cq, 2cq + 1
    // table role: rows rw + 2 rp, + 1 and block 2cq + gl
    const int rp = lane & 15, gl = lane >> 4;
    const int kap0 = 8 * (rp & 3) + 4 * (rp >> 3) + 2 * ((rp >> 2) & 1);
    const int g = lane >> 2, t = lane & 3;  // MMA fragment role
    uint8_t* tbl = smem + Geo<F>::kTblOff + warp * NSET * kTblBytes;
    for (int i = lane; i < NSET * kTblBytes / 4; i += 32) reinterpret_cast<uint32_t*>(tbl)[i] = 0u;
    __syncwarp();
    for (int i = lane; i < NSET * 2 * 2 * 8; i += 32) {  // all-ones columns 3 and 7
      const int w8 = i & 7, c2 = (i >> 3) & 1, jb = (i >> 4) & 1, z = i >> 5;
      reinterpret_cast<uint32_t*>(tbl + z * kTblBytes + jb * kSbStride + (3 + 4 * c2) * kColStride)[w8] =
          0x01010101u;
    }
    __syncwarp();
    uint8_t* const tcol = tbl + gl * kSbStride + kap0;
    const uint8_t* const tfrag = tbl + g * kColStride + 8 * t;
    const int row0 = rw + 2 * rp;
    const int blk = 2 * cq + gl;  // this lane's table block
    // A gather: lane (g, t) reads codes 2g, 2g + 1 of rows rw + 8i + 2t (+1) of a chunk
    const uint32_t a_lane = smem_u32(smem) + (uint32_t)((rw + 2 * t) * kPitch + Q::kCO + 2 * g);

    asm volatile("griddepcontrol.wait;" ::: "memory");

    int acc[NSET][4][4];  // [set][chunk][fragment]
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[z][k][0] = acc[z][k][1] = acc[z][k][2] = acc[z][k][3] = 0;
    float scale[BATCH];  // powers of two; the step of batch row b is 1 / scale[b]
    uint32_t down_ok = 0u;  // rows that may be rescaled down (see vbq_gemv_mma.cu)
#pragma unroll
    for (int b = 0; b < BATCH; ++b) scale[b] = 1.f;
    // s32 sums -> fp32 (see vbq_gemv_mma.cu): lanes t even hold digits 0, 1 of batch row
    // 2z + t/2, lanes t odd digit 2 and the code sum; the pair adds its halves
    auto flush = [&]() {
      const int odd = t & 1;
      const float c1 = odd ? 65536.f : 1.f, c2 = odd ? 32896.f : 256.f;
      const int cen = odd ? 64 : 0;
#pragma unroll
      for (int z = 0; z < NSET; ++z) {
        const float sb = (t >> 1) ? ((2 * z + 1 < BATCH) ? inv_pow2(scale[(2 * z + 1) % BATCH]) : 0.f)
                                  : inv_pow2(scale[(2 * z) % BATCH]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          int* a = acc[z][k];
          const float p0 = fmaf(c2, (float)a[1], c1 * (float)(a[0] - cen * a[1]));
          const float p1 = fmaf(c2, (float)a[3], c1 * (float)(a[2] - cen * a[3]));
          const float mine = odd ? p1 : p0, other = odd ? p0 : p1;
          const float sum = mine + __shfl_xor_sync(0xffffffffu, other, 1);
          fac[z][k] = fmaf(sum, sb, fac[z][k]);
          a[0] = a[1] = a[2] = a[3] = 0;
        }
      }
    };

    int kx = split * kRows + row0;
    const int kstep = S * kRows;
    auto load_x = [&](int k, float2 (&xv)[BATCH]) {
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        xv[b].x = (b < batch && k < K) ? gemv_x<SWIGLU>(x, b, K, k) : 0.f;
        xv[b].y = (b < batch && k + 1 < K) ? gemv_x<SWIGLU>(x, b, K, k + 1) : 0.f;
      }
    };
    float2 xn[BATCH], xnn[BATCH];
    load_x(kx, xn);
    kx += kstep;
    load_x(kx, xnn);
#pragma unroll 1
    for (int it = 0; it < nst; ++it) {
      const int s = it & (kStages - 1);
      float2 xv[BATCH];
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        xv[b] = xn[b];
        xn[b] = xnn[b];
      }
      kx += kstep;
      load_x(kx, xnn);
      if (!__all_sync(0xffffffffu, mbar_wait_hinted(smem_u32(&bars.full[s]), (uint32_t)(it / kStages) & 1u,
                                                      kWaitBudgetCycles))) {
        if (lane == 0) give_up();
        break;
      }
      const uint8_t* st = stage(s);
      // ---- v = x * d for the lane's two rows of its block (fp16 scale, IEEE) ----
      // (the reference converts the 4- and 5-bit blocks' fp16 fields with its f16_to_f32)
      const uint16_t hd0 = *reinterpret_cast<const uint16_t*>(st + row0 * kPitch + Q::kBB * blk);
      const uint16_t hd1 = *reinterpret_cast<const uint16_t*>(st + (row0 + 1) * kPitch + Q::kBB * blk);
      const float2 d = Q::kNib ? make_float2(f16_ref(hd0), f16_ref(hd1)) : make_float2(f16_ieee(hd0), f16_ieee(hd1));
      float2 v[BATCH];
      uint32_t w[BATCH][2];
      uint32_t out = 0u;
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        v[b] = __fmul2_rn(xv[b], d);
        if constexpr (Q::kM >= 0) {  // + x * m
          const float m0 = f16_ref(*reinterpret_cast<const uint16_t*>(st + row0 * kPitch + Q::kBB * blk + Q::kM));
          const float m1 = f16_ref(*reinterpret_cast<const uint16_t*>(st + (row0 + 1) * kPitch + Q::kBB * blk + Q::kM));
          mo[b] = fmaf(xv[b].x, m0, fmaf(xv[b].y, m1, mo[b]));
        } else if constexpr (Q::kNib) {  // - 8 v / - 16 v
          mo[b] = fmaf(Q::kOff, v[b].x + v[b].y, mo[b]);
        }
        w[b][0] = __float_as_uint(fmaf(v[b].x, scale[b], kMagic));
        w[b][1] = __float_as_uint(fmaf(v[b].y, scale[b], kMagic));
        out |= (w[b][0] ^ 0x4b000000u) | (w[b][1] ^ 0x4b000000u);
      }
      // the sampled shrink test, as in vbq_gemv_mma.cu (every second stage at batch 4)
      bool shrink = false;
      if ((it & ((BATCH <= 2 ? 1 : 2) - 1)) == 0) {
        uint32_t small = 0u;
#pragma unroll
        for (int b = 0; b < BATCH; ++b) small |= (fabsf(v[b].x) * scale[b] < 65536.f) ? (1u << b) : 0u;
        shrink = __reduce_and_sync(0xffffffffu, small & down_ok) != 0u;
      }
      if (__any_sync(0xffffffffu, out >= (1u << 23)) || shrink || it == 0) {
        // rare (and the first stage): see vbq_gemv_mma.cu
        if (it > 0) flush();
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const float sum = fabsf(v[b].x) + fabsf(v[b].y);
          nonfin |= (sum < 0x1p100f) ? 0u : (1u << b);
          float m = fminf(fmaxf(fabsf(v[b].x), fabsf(v[b].y)), 0x1p99f);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          int e = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127 + 1;
          e = e < kExpMin ? kExpMin : (e > kExpMax ? kExpMax : e);
          scale[b] = pow2f(21 - e);
          down_ok = (b < batch && e > kExpMin) ? (down_ok | (1u << b)) : (down_ok & ~(1u << b));
          w[b][0] = __float_as_uint(fmaf(v[b].x, scale[b], kMagic));
          w[b][1] = __float_as_uint(fmaf(v[b].y, scale[b], kMagic));
        }
      }
      // ---- B table: three signed digits of n per row pair ----
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const uint32_t wx = w[b][0] ^ 0x8080u, wy = w[b][1] ^ 0x8080u;
        uint8_t* col = tcol + (b >> 1) * kTblBytes + 4 * (b & 1) * kColStride;
#pragma unroll
        for (int dg = 0; dg < 3; ++dg)
          *reinterpret_cast<uint16_t*>(col + dg * kColStride) = (uint16_t)__byte_perm(wx, wy, dg | ((4 + dg) << 4));
      }
      __syncwarp();
      // ---- 4 chunks of 16 codes x 32 rows: one MMA per set ----
      const uint32_t sbase = a_lane + (uint32_t)(s * kStageBytes);
      if constexpr (!Q::kNib) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t cb = sbase + (uint32_t)(34 * (2 * cq + (k >> 1)) + 16 * (k & 1));
          uint32_t r[4];  // rows 8i + 2t (low half) and 8i + 2t + 1 (high half), codes 2g, 2g + 1
#pragma unroll
          for (int i = 0; i < 4; ++i)
            r[i] = __byte_perm(lds_u16(cb + (uint32_t)(8 * i * kPitch)), lds_u16(cb + (uint32_t)((8 * i + 1) * kPitch)),
                               0x5410);
          // A rows m = g: code column 2g, m = g + 8: code column 2g + 1
          const uint32_t a0 = __byte_perm(r[0], r[1], 0x6420), a1 = __byte_perm(r[0], r[1], 0x7531);
          const uint32_t a2 = __byte_perm(r[2], r[3], 0x6420), a3 = __byte_perm(r[2], r[3], 0x7531);
#pragma unroll
          for (int z = 0; z < NSET; ++z) {
            const uint2 bf = *reinterpret_cast<const uint2*>(tfrag + z * kTblBytes + (k >> 1) * kSbStride);
            mma_s8s8(acc[z][k], a0, a1, a2, a3, bf.x, bf.y);
          }
        }
      } else {
        // a block's 16 code bytes hold its 32 values: the same gather as Q8_0's half block,
        // then low nibbles (values 4g, 4g + 2 for A rows g, g + 8) and high nibbles (4g + 1,
        // 4g + 3) as two u8 MMAs: chunk k = 2 * (local block) + nibble
#pragma unroll
        for (int jb = 0; jb < 2; ++jb) {
          const uint32_t cb = sbase + (uint32_t)(Q::kBB * (2 * cq + jb));
          uint32_t r[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            r[i] = __byte_perm(lds_u16(cb + (uint32_t)(8 * i * kPitch)), lds_u16(cb + (uint32_t)((8 * i + 1) * kPitch)),
                               0x5410);
          const uint32_t a[4] = {__byte_perm(r[0], r[1], 0x6420), __byte_perm(r[0], r[1], 0x7531),
                                 __byte_perm(r[2], r[3], 0x6420), __byte_perm(r[2], r[3], 0x7531)};
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            lo[q] = a[q] & 0x0f0f0f0fu;
            hi[q] = (a[q] >> 4) & 0x0f0f0f0fu;
          }
          if constexpr (Q::kQH >= 0) {
            // fifth bits: bits 4g .. 4g + 3 of each row's qh (values 4g .. 4g + 3), one byte
            // per row in the same row order as the fragment words (rows 8i + 2t, + 1)
            const uint32_t hbase = cb - (uint32_t)(Q::kCO + 2 * g) + (uint32_t)(Q::kQH + (g >> 1));
            const uint32_t nsh = 4u * (uint32_t)(g & 1);
            uint32_t hw[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t acc4 = 0u;
#pragma unroll
              for (int i2 = 0; i2 < 2; ++i2)
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                  const int i = 2 * hh + i2;
                  const uint32_t byte = lds_u8(hbase + (uint32_t)((8 * i + rr) * kPitch));
                  acc4 |= ((byte >> nsh) & 0xfu) << (8 * (2 * i2 + rr));
                }
              hw[hh] = acc4;  // bytes: rows (i, A), (i, B), (i + 1, A), (i + 1, B)
            }
            // A words 0 / 2 (code byte 2g: values 4g lo, 4g + 1 hi), 1 / 3 (byte 2g + 1:
            // values 4g + 2 lo, 4g + 3 hi); the fifth bit goes to bit 4 of each code byte
            lo[0] |= (hw[0] & 0x01010101u) << 4;
            lo[1] |= ((hw[0] >> 2) & 0x01010101u) << 4;
            lo[2] |= (hw[1] & 0x01010101u) << 4;
            lo[3] |= ((hw[1] >> 2) & 0x01010101u) << 4;
            hi[0] |= ((hw[0] >> 1) & 0x01010101u) << 4;
            hi[1] |= ((hw[0] >> 3) & 0x01010101u) << 4;
            hi[2] |= ((hw[1] >> 1) & 0x01010101u) << 4;
            hi[3] |= ((hw[1] >> 3) & 0x01010101u) << 4;
          }
#pragma unroll
          for (int z = 0; z < NSET; ++z) {
            const uint2 bf = *reinterpret_cast<const uint2*>(tfrag + z * kTblBytes + jb * kSbStride);
            mma_u8s8(acc[z][2 * jb], lo[0], lo[1], lo[2], lo[3], bf.x, bf.y);
            mma_u8s8(acc[z][2 * jb + 1], hi[0], hi[1], hi[2], hi[3], bf.x, bf.y);
          }
        }
      }
      __syncwarp();  // table and stage reads done
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty[s]));
    }
    flush();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      if (o < 16) {  // offset terms: the 16 lanes of a table block hold its 32 rows
#pragma unroll
        for (int b = 0; b < BATCH; ++b) mo[b] += __shfl_xor_sync(0xffffffffu, mo[b], o);
      }
      nonfin |= __shfl_xor_sync(0xffffffffu, nonfin, o);
    }
  }

  // ---- per-warp outputs -> shared memory (the stage ring, now idle) ----
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [warp][b][64 columns of the warp]
  if (warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int z = 0; z < NSET; ++z)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int b = 2 * z + (t >> 1);
        // the offset term of local block k >> 1 sits in lanes 16 (k >> 1) .. + 15 (every
        // lane shuffles: the store below is conditional)
        const float oA = __shfl_sync(0xffffffffu, mo[(2 * z) % BATCH], 16 * (k >> 1));
        const float oB = __shfl_sync(0xffffffffu, mo[(2 * z + 1) % BATCH], 16 * (k >> 1));
        if (b < BATCH && b < batch) {
          // Q8_0: chunk k is half k & 1 of block k >> 1, A rows g / g + 8 its codes 2g / 2g + 1;
          // 4- and 5-bit: nibble k & 1 of block k >> 1, A rows g / g + 8 values 4g / 4g + 2
          const int col = Q::kNib ? 32 * (k >> 1) + 4 * g + 2 * (t & 1) + (k & 1)
                                  : 32 * (k >> 1) + 16 * (k & 1) + 2 * g + (t & 1);
          const float o = Q::kNib ? ((t >> 1) ? oB : oA) : 0.f;
          red[(warp * 4 + b) * 64 + col] = ((nonfin >> b) & 1u) ? __int_as_float(0x7fc00000) : fac[z][k] + o;
        }
      }
  }
  __syncthreads();
  // ---- sum the two row slices in order: this CTA's partial y ----
  const int E = batch * 256;
  float* outbuf = red + kConsumers * 4 * 64;
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, n = e & 255, cq = n >> 6, cl = n & 63;
    outbuf[e] = red[(cq * 4 + b) * 64 + cl] + red[((cq + 4) * 4 + b) * 64 + cl];
  }
  __syncthreads();
  if (S == 1) {
    for (int e = threadIdx.x; e < E; e += kThreads)
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = epi_apply(epi, outbuf[e], e >> 8, N, tile * 256 + (e & 255));
    return;
  }
  // ---- split-K inside the cluster (as vbq_gemv_mma.cu) ----
  cluster_wait();
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

}  // namespace gq8

// ---- host side -----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnQ)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnQ encode_fn_q() {
  static EncodeTiledFnQ fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnQ>(p);
  });
  return fn;
}

// Splits per tile as for the Q4_K kernel: one wave of two CTAs per SM, at most 16, the
// leader's receive slots inside the shared memory budget, 25 % spare cluster places.
template <int BATCH, bool SW, int F>
static int choose_splits_q8(int64_t K, int64_t N, int batch, int smem_base) {
  using namespace gq8;
  const int tiles = (int)(N / 256);
  const int64_t tot_st = (K + kRows - 1) / kRows;
  // resident CTAs per SM: two for Q8_0 (272-byte rows); the 4- and 5-bit forms' smaller
  // stages fit three where their registers allow (queried once per device)
  int per_sm = 2;
  if constexpr (F != kQ8_0) {
    static DeviceOnce queried;
    static DeviceSlots slots_per_sm;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
      if (!queried.done(dev)) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_q8_kernel<BATCH, SW, F>, kThreads,
                                                          smem_base + 8 * 1024) != cudaSuccess) {
          cudaGetLastError();
          n = 2;
        }
        slots_per_sm.set(dev, n < 2 ? 2 : (n > 3 ? 3 : n));
        queried.mark(dev);
      }
      per_sm = slots_per_sm.get(dev);
    }
  }
  int S = tiles > 0 ? per_sm * sm_count() / tiles : 1;
  if (S > 16) S = 16;
  if (S > tot_st) S = (int)tot_st;
  if (S < 1) S = 1;
  const int cap = per_sm >= 3 ? 72 * 1024 : 112 * 1024;  // per_sm CTAs per SM
  if (gemv_split_override()) {
    S = gemv_split_override() > 16 ? 16 : gemv_split_override();
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
    if (cudaOccupancyMaxActiveClusters(&active, gemv_q8_kernel<BATCH, SW, F>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      active = 0;
    }
    if (active * 4 >= tiles * 5) break;
  }
  if (n_cache < 32) cache[n_cache++] = Entry{tiles, batch, s_in, S};
  return S;
}

template <int BATCH, bool SWIGLU, int F = kQ8_0>
static cudaError_t launch_q8_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t RB, int batch, cudaStream_t st, Epi epi) {
  using namespace gq8;
  auto enc = encode_fn_q();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw;
  if (!weight_map(reinterpret_cast<EncodeTiledFn>(enc), w, K, RB, Geo<F>::kPitch, kRows, &mw))
    return cudaErrorInvalidValue;
  auto kern = gemv_q8_kernel<BATCH, SWIGLU, F>;
  constexpr int kBase = Lay<(BATCH <= 2 ? 1 : 2), F>::kSmem;
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
  const int S = choose_splits_q8<BATCH, SWIGLU, F>(K, N, batch, kBase);
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

// The s32 sums run over up to K / 2 rows per accumulator with terms of at most 128 * 128
// in magnitude: K is capped at 3 * 2^16 (longer rows take the fp32 kernel).
bool gemv_q8_fits(int64_t K, int64_t N, int batch) {
  return batch >= 1 && batch <= 16 && K >= 1 && K <= 3 * 65536 && N % 256 == 0 && N > 0;
}

// Tensor-core Q8_0 GEMV; batches above 4 run as launches over groups of 4 batch rows.
template <bool SW, int F = kQ8_0>
static cudaError_t launch_q8_group(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                   int64_t row_bytes, int nb, cudaStream_t st, Epi epi) {
  return nb == 1   ? launch_q8_t<1, SW, F>(x, w, y, K, N, row_bytes, nb, st, epi)
         : nb == 2 ? launch_q8_t<2, SW, F>(x, w, y, K, N, row_bytes, nb, st, epi)
                   : launch_q8_t<4, SW, F>(x, w, y, K, N, row_bytes, nb, st, epi);
}

cudaError_t launch_gemv_q8_mma(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_q8_fits(K, N, batch) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int b0 = 0; b0 < batch; b0 += 4) {
    const int nb = batch - b0 < 4 ? batch - b0 : 4;
    const float* xg = x + (int64_t)b0 * xrow;
    float* yg = y + (int64_t)b0 * N;
    const Epi epi{f.bias, f.res ? f.res + (int64_t)b0 * N : nullptr};
    cudaError_t e = f.swiglu_x ? launch_q8_group<true>(xg, w, yg, K, N, row_bytes, nb, st, epi)
                               : launch_q8_group<false>(xg, w, yg, K, N, row_bytes, nb, st, epi);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Q4_0 / Q4_1 / Q5_0 / Q5_1 on the same kernel (batch 1..16 as groups of 4): rows of 8
// blocks are 144 / 160 / 176 / 192 bytes, whole 16-byte granules at any width of whole
// 256-column tiles.
template <int F>
static cudaError_t launch_q4x(const float* x, const void* w, float* y, int64_t K, int64_t N,
                              int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int b0 = 0; b0 < batch; b0 += 4) {
    const int nb = batch - b0 < 4 ? batch - b0 : 4;
    const float* xg = x + (int64_t)b0 * xrow;
    float* yg = y + (int64_t)b0 * N;
    const Epi epi{f.bias, f.res ? f.res + (int64_t)b0 * N : nullptr};
    cudaError_t e = f.swiglu_x ? launch_q8_group<true, F>(xg, w, yg, K, N, row_bytes, nb, st, epi)
                               : launch_q8_group<false, F>(xg, w, yg, K, N, row_bytes, nb, st, epi);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_gemv_q4x_mma(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f) {
  if (!gemv_q8_fits(K, N, batch) || row_bytes % 16 != 0) return cudaErrorNotSupported;
  switch (qtype) {
    case kQ4_0: return launch_q4x<kQ4_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ4_1: return launch_q4x<kQ4_1>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_0: return launch_q4x<kQ5_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_1: return launch_q4x<kQ5_1>(x, w, y, K, N, row_bytes, batch, st, f);
    default: return cudaErrorNotSupported;
  }
}

cudaError_t gemv_q8_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_q8_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_q8_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
