// vbq_gemm.cu -- quantized-weight GEMM on the sm_100a tensor cores (prefill).
//
//   C[m, n] = sum_k A[m, k] * deq(W)[k, n]
//
// A is bf16 [M, K] row-major, W the reference's K x N block layout (quant blocks along N,
// cpp/src/dequant.cpp:739-771), C fp32 or bf16 [M, N].  The reference has no batched GEMM:
// its engine runs one gemv_dequant per token (cpp/src/fast_model.cpp:645-660).
//
// One CTA computes a 256 x 256 tile of C with tcgen05 MMAs accumulating in tensor memory
// (two 128 x 256 fp32 accumulators = all 512 TMEM columns).  Per 64-deep K step:
//   * warp 0 (one lane) TMA-loads the two 128 x 64 A boxes (128-byte swizzle) and the raw
//     quant bytes of the 64 W rows of the tile's 256 columns into a 3-deep ring;
//   * warps 2-9 dequantize the raw bytes to bf16 straight into the K-major, 128-byte
//     swizzled B tile the MMA reads (2-deep ring), warp w handling K rows 8(w-2)..+7;
//   * warp 1 (one lane) issues 2 x 4 tcgen05.mma (M=128, N=256, K=16) and commits them to
//     the barriers that free the A and B stages.
// After the last K step the dequant warps read the accumulators out of tensor memory
// (tcgen05.ld) and store C.  Every mbarrier wait is bounded; a wait that gives up records
// kStatusTimeout in the device status word and the CTA drains and exits.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {

__device__ unsigned g_gemm_status = 0;

namespace gemm {

constexpr int BM = 256, BN = 256, BK = 64;
constexpr int kThreads = 320;            // 10 warps
constexpr int kLoadStages = 3, kBStages = 2;
constexpr int kABoxBytes = 128 * BK * 2;  // one 128 x 64 bf16 box
constexpr int kBBytes = BN * BK * 2;      // 256 x 64 bf16 B tile
constexpr int kTmemCols = 512;

template <int QT> struct Raw {
  static constexpr int kTileBytes = Tile<QT>::kBytes;                       // 144 / 210 / 272
  static constexpr int kPitch = (QT == kQ6_K) ? 224 : kTileBytes;           // TMA box row
  static constexpr int kBytes = kPitch * BK;                                // per stage
  static constexpr int kSlot = (kBytes + 1023) / 1024 * 1024;
};

template <int QT> struct Smem {
  static constexpr int kStageBytes = 2 * kABoxBytes + Raw<QT>::kSlot;
  static constexpr int kLoadOff = 0;
  static constexpr int kBOff = kLoadStages * kStageBytes;
  static constexpr int kTblOff = kBOff + kBStages * kBBytes;  // per-warp scale tables
  static constexpr int kBarOff = kTblOff + 8 * 768;
  // barriers: full_load[3], empty_load[3], full_b[2], empty_b[2], acc_full, + tmem ptr, abort
  static constexpr int kTotal = kBarOff + 128;
  static constexpr int kAlloc = kTotal + 1024;  // slack for 1024-byte alignment
};

// ---- tcgen05 / TMA primitives (inline PTX, sm_100a) ----------------------------------
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: rows of 128 B, 8-row atoms 1024 B apart (SBO),
  // LBO unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B).
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one lane per thread)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// ---- dequantization: one thread = 8 K rows x 8 consecutive columns ---------------------
// Warp w (w = 2..9) owns K rows 8(w-2)..8(w-2)+7 of every stage, lane l the columns
// 8l..8l+7 of the tile.  Every weight value is produced as the reference's fp32 value
// (one rounding per product and per difference, cpp/src/dequant.cpp:268-301, :359-402 and
// the Q8_0 block of cpp/src/cuda_kernels.cu:718-735), then rounded once to bf16.
//
// A small integer q becomes the float (magic + q) with one byte permute: the magic's
// exponent makes its mantissa LSB worth exactly 1, so a packed fp32x2 add or fma removes
// it without rounding.  Q4_K folds that into the product: fma(2^23 + q, dl, -2^23 dl) is
// dl*q rounded once (2^23 dl is exact).  The result equals the reference's value up to
// the sign of an exact zero, for every finite block scale.
//
// Two K rows of one column form one packed bf16x2 word; the four words of a column make
// the 16-byte chunk the MMA reads.
constexpr float kTwo23 = 8388608.0f;     // 2^23
constexpr float kOneHalf23 = 12582912.0f; // 1.5 * 2^23: magic 0x4b4000xx = 1.5*2^23 + xx
constexpr uint32_t kMagic23 = 0x4b000000u, kMagic15 = 0x4b400000u;

// byte i of w as the low byte of magic k (k's bytes 0 and 1 are zero)
// result bytes: [byte I of w, k.byte0, k.byte2, k.byte3]; k.byte0 is zero for both magics
template <int I>
__device__ __forceinline__ float magic_byte(uint32_t w, uint32_t k) {
  return __uint_as_float(__byte_perm(w, k, 0x7640u | (uint32_t)I));
}
template <int QT> struct Producer;

// Q4_K: all 256 columns of the tile are one block; lane l's columns lie in sub-block
// l >> 2 (low nibbles for even sub-blocks, high for odd).  The (dl, ml) pair of each of
// the warp's 8 rows x 8 sub-blocks is computed once per stage into a per-warp table.
template <> struct Producer<kQ4_K> {
  static constexpr int kPitch = 144;
  static constexpr int kTableBytes = 768;  // float4 [4 row pairs][8 sub-blocks] + float2 [4][8]
  __device__ __forceinline__ static void table(const uint8_t* rows, int lane, uint8_t* tbl) {
    const int sb = lane & 7, p = lane >> 3;
    const Q4kScaleRecipe rec(sb);
    float dl[2], ml[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 hd = *reinterpret_cast<const uint4*>(rows + (2 * p + h) * kPitch);
      int sc, mn;
      rec.apply(hd.y, hd.z, hd.w, sc, mn);
      dl[h] = __fmul_rn(f16_ref(hd.x & 0xffffu), (float)sc);
      ml[h] = __fmul_rn(f16_ref(hd.x >> 16), (float)mn);
    }
    reinterpret_cast<float4*>(tbl)[p * 8 + sb] =
        make_float4(dl[0], dl[1], __fmul_rn(-kTwo23, dl[0]), __fmul_rn(-kTwo23, dl[1]));
    reinterpret_cast<float2*>(tbl + 512)[p * 8 + sb] = make_float2(-ml[0], -ml[1]);
  }
  float2 dl[4], c[4], nm[4];
  uint32_t w[8][2];
  template <bool>
  __device__ __forceinline__ void load(const uint8_t* rows, int lane, const uint8_t* tbl) {
    const int sb = lane >> 2;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float4 a = reinterpret_cast<const float4*>(tbl)[p * 8 + sb];
      dl[p] = make_float2(a.x, a.y);
      c[p] = make_float2(a.z, a.w);
      nm[p] = reinterpret_cast<const float2*>(tbl + 512)[p * 8 + sb];
    }
    const int off = 16 + 32 * (lane >> 3) + 8 * (lane & 3);
    const uint32_t hs = (uint32_t)((lane >> 2) & 1) * 4u;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint2 q = *reinterpret_cast<const uint2*>(rows + r * kPitch + off);
      w[r][0] = (q.x >> hs) & 0x0f0f0f0fu;
      w[r][1] = (q.y >> hs) & 0x0f0f0f0fu;
    }
  }
  template <int I>
  __device__ __forceinline__ uint32_t pair(int p) const {
    const float2 m = make_float2(magic_byte<I & 3>(w[2 * p][I >> 2], kMagic23),
                                 magic_byte<I & 3>(w[2 * p + 1][I >> 2], kMagic23));
    const float2 v = __fadd2_rn(__ffma2_rn(m, dl[p], c[p]), nm[p]);
    return pack_bf16x2(v.x, v.y);
  }
};

// Q6_K (reference layout): lane l's 8 values take ql bytes 4l..4l+3 and qh bytes 2l, 2l+1
// and share scale l >> 1.  The 6-bit codes are assembled byte-wise: even columns in one
// word, odd columns in another.
template <> struct Producer<kQ6_K> {
  static constexpr int kPitch = 224;
  static constexpr int kTableBytes = 512;  // float2 [4 row pairs][16 scales]
  __device__ __forceinline__ static void table(const uint8_t* rows, int lane, uint8_t* tbl) {
    const int s = lane & 15;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int p = (lane >> 4) + 2 * j;
      float ds[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint8_t* row = rows + (2 * p + h) * kPitch;
        ds[h] = __fmul_rn(f16_ref(ld_u16(row + 208)), (float)(int8_t)row[192 + s]);
      }
      reinterpret_cast<float2*>(tbl)[p * 16 + s] = make_float2(ds[0], ds[1]);
    }
  }
  float2 ds[4];
  uint32_t ue[8], uo[8];
  template <bool kMisaligned>  // the block starts 2 mod 4 within the staged row
  __device__ __forceinline__ void load(const uint8_t* rows, int lane, const uint8_t* tbl) {
#pragma unroll
    for (int p = 0; p < 4; ++p) ds[p] = reinterpret_cast<const float2*>(tbl)[p * 16 + (lane >> 1)];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint8_t* row = rows + r * kPitch;
      uint32_t q;
      if constexpr (kMisaligned) {
        const uint32_t* a = reinterpret_cast<const uint32_t*>(row + 4 * lane - 2);
        q = __byte_perm(a[0], a[1], 0x5432u);
      } else {
        q = *reinterpret_cast<const uint32_t*>(row + 4 * lane);
      }
      // qh bytes h0 (fields of columns 0-3), h1 (4-7) as [h0, h0, h1, h1]
      const uint32_t hh = __byte_perm(ld_u16(row + 128 + 2 * lane), 0u, 0x1100u);
      // high bits of column 2j: field 2j -> bits 4-5 of byte j; column 2j+1: field 2j+1
      ue[r] = (q & 0x0f0f0f0fu) | ((hh << 4) & 0x00300030u) | (hh & 0x30003000u);
      uo[r] = ((q >> 4) & 0x0f0f0f0fu) | ((hh << 2) & 0x00300030u) | ((hh >> 2) & 0x30003000u);
    }
  }
  template <int I>
  __device__ __forceinline__ uint32_t pair(int p) const {
    const uint32_t* u = (I & 1) ? uo : ue;
    const float2 m = make_float2(magic_byte<(I >> 1)>(u[2 * p], kMagic15),
                                 magic_byte<(I >> 1)>(u[2 * p + 1], kMagic15));
    const float2 q = __fadd2_rn(m, make_float2(-(kOneHalf23 + 32.0f), -(kOneHalf23 + 32.0f)));
    const float2 v = __fmul2_rn(ds[p], q);
    return pack_bf16x2(v.x, v.y);
  }
};

// Q8_0 (GGUF 34-byte block, fp16 scale): the tile's 256 columns are 8 blocks; lane l's
// 8 values are bytes 8(l & 3)..+7 of block l >> 2, 2 bytes off a 4-byte boundary for
// even blocks.
template <> struct Producer<kQ8_0> {
  static constexpr int kPitch = 272;
  static constexpr int kTableBytes = 0;
  __device__ __forceinline__ static void table(const uint8_t*, int, uint8_t*) {}
  float2 d[4];
  uint32_t w[8][2];
  template <bool>
  __device__ __forceinline__ void load(const uint8_t* rows, int lane, const uint8_t*) {
    const int boff = 34 * (lane >> 2);
    const int a = boff + 2 + 8 * (lane & 3);
    const int base = a & ~3;
    const uint32_t sel = (a & 2) ? 0x5432u : 0x3210u;
    float dr[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint8_t* row = rows + r * kPitch;
      const uint32_t* x = reinterpret_cast<const uint32_t*>(row + base);
      const uint32_t x0 = x[0], x1 = x[1], x2 = x[2];
      w[r][0] = __byte_perm(x0, x1, sel) ^ 0x80808080u;  // q + 128 as unsigned bytes
      w[r][1] = __byte_perm(x1, x2, sel) ^ 0x80808080u;
      dr[r] = f16_ieee(ld_u16(row + boff));
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) d[p] = make_float2(dr[2 * p], dr[2 * p + 1]);
  }
  template <int I>
  __device__ __forceinline__ uint32_t pair(int p) const {
    const float2 m = make_float2(magic_byte<I & 3>(w[2 * p][I >> 2], kMagic15),
                                 magic_byte<I & 3>(w[2 * p + 1][I >> 2], kMagic15));
    const float2 q = __fadd2_rn(m, make_float2(-(kOneHalf23 + 128.0f), -(kOneHalf23 + 128.0f)));
    const float2 v = __fmul2_rn(q, d[p]);
    return pack_bf16x2(v.x, v.y);
  }
};

// Value I of lane l (column 8l + I of the tile) goes to B row 8l + ((I + l) & 7): the 8
// lanes of each 16-byte store phase then hit 8 different swizzle chunks.  The epilogue
// undoes this rotation inside each group of 8 accumulator columns.
template <int QT, int I>
__device__ __forceinline__ void store_column(const Producer<QT>& pr, uint8_t* bt, const uint32_t (&off)[8]) {
  const uint4 chunk = make_uint4(pr.template pair<I>(0), pr.template pair<I>(1),
                                 pr.template pair<I>(2), pr.template pair<I>(3));
  *reinterpret_cast<uint4*>(bt + off[I]) = chunk;
}
template <int QT>
__device__ __forceinline__ void store_all(const Producer<QT>& pr, uint8_t* bt, const uint32_t (&off)[8]) {
  store_column<QT, 0>(pr, bt, off);
  store_column<QT, 1>(pr, bt, off);
  store_column<QT, 2>(pr, bt, off);
  store_column<QT, 3>(pr, bt, off);
  store_column<QT, 4>(pr, bt, off);
  store_column<QT, 5>(pr, bt, off);
  store_column<QT, 6>(pr, bt, off);
  store_column<QT, 7>(pr, bt, off);
}

struct Bars {
  uint64_t full_load[kLoadStages], empty_load[kLoadStages];
  uint64_t full_b[kBStages], empty_b[kBStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
};

template <int QT, bool BF16_OUT>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
            const uint8_t* __restrict__ w, void* __restrict__ c, int M, int K, int N, int64_t RB) {
  using L = Smem<QT>;
  using R = Raw<QT>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (128-byte swizzle atoms); derived from the array so that the
  // compiler keeps shared-memory addressing
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int m0 = m_tile * BM;
  const int nk = (K + BK - 1) / BK;

  auto a_box = [&](int s, int h) { return smem + L::kLoadOff + s * L::kStageBytes + h * kABoxBytes; };
  auto raw_stage = [&](int s) { return smem + L::kLoadOff + s * L::kStageBytes + 2 * kABoxBytes; };
  auto b_stage = [&](int t) { return smem + L::kBOff + t * kBBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLoadStages; ++s) {
      mbar_init(smem_u32(&bars.full_load[s]), 1);
      mbar_init(smem_u32(&bars.empty_load[s]), 1 + 8);  // MMA commit + 8 dequant warps
    }
    for (int t = 0; t < kBStages; ++t) {
      mbar_init(smem_u32(&bars.full_b[t]), 8);
      mbar_init(smem_u32(&bars.empty_b[t]), 1);
    }
    mbar_init(smem_u32(&bars.acc_full), 1);
    bars.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {  // whole warp: allocate the 512 accumulator columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&bars.tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  volatile int* abort_flag = &bars.abort;

  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemm_status, kStatusTimeout);
  };

  // Q6_K tiles start inside a 16-byte chunk; the TMA box starts at the chunk
  int tile_x = n_tile * R::kTileBytes;
  const int raw_off = (QT == kQ6_K) ? (tile_x & 15) : 0;
  tile_x &= ~15;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      const uint32_t bytes = 2 * kABoxBytes + R::kBytes;
      int it = 0;
      for (; it < nk && !*abort_flag; ++it) {
        const int s = it % kLoadStages;
        const uint32_t parity = ((it / kLoadStages) & 1) ^ 1;
        if (!mbar_wait_bounded(smem_u32(&bars.empty_load[s]), parity, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full_load[s]);
        mbar_arrive_expect_tx(fb, bytes);
        tma_load_2d(smem_u32(a_box(s, 0)), &tmap_a, it * BK, m0, fb);
        tma_load_2d(smem_u32(a_box(s, 1)), &tmap_a, it * BK, m0 + 128, fb);
        tma_load_2d(smem_u32(raw_stage(s)), &tmap_w, tile_x / 2, it * BK, fb);
      }
      // drain: every issued stage must land before the CTA may exit
      for (int j = (it > kLoadStages ? it - kLoadStages : 0); j < it; ++j)
        mbar_wait_bounded(smem_u32(&bars.full_load[j % kLoadStages]), (j / kLoadStages) & 1,
                          kWaitBudgetCycles);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      int it = 0;
      for (; it < nk && !*abort_flag; ++it) {
        const int s = it % kLoadStages, t = it % kBStages;
        if (!mbar_wait_bounded(smem_u32(&bars.full_load[s]), (it / kLoadStages) & 1, kWaitBudgetCycles) ||
            !mbar_wait_bounded(smem_u32(&bars.full_b[t]), (it / kBStages) & 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        tc_fence_after();
        const uint64_t a0 = smem_desc_sw128(smem_u32(a_box(s, 0)));
        const uint64_t a1 = smem_desc_sw128(smem_u32(a_box(s, 1)));
        const uint64_t b = smem_desc_sw128(smem_u32(b_stage(t)));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          // +32 bytes per 16-element K step inside the 128-byte swizzle atom (+2 encoded)
          umma_bf16(tmem, a0 + 2 * kk, b + 2 * kk, acc);
          umma_bf16(tmem + 256, a1 + 2 * kk, b + 2 * kk, acc);
        }
        umma_commit(smem_u32(&bars.empty_load[s]));
        umma_commit(smem_u32(&bars.empty_b[t]));
      }
      umma_commit(smem_u32(&bars.acc_full));  // arrives once every MMA issued so far is done
      // tensor memory is freed below only after the MMAs writing it have finished
      if (!mbar_wait_bounded(smem_u32(&bars.acc_full), 0, kWaitBudgetCycles)) give_up();
    }
  } else {
    // ------------------------------ dequant warps ------------------------------
    using P = Producer<QT>;
    const int kc = warp - 2;  // this warp's 8 K rows of each stage
    uint8_t* tbl = smem + L::kTblOff + kc * 768;
    uint32_t off[8];          // B-tile byte offset of value i's 16-byte chunk
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rot = (i + lane) & 7;
      off[i] = (uint32_t)((8 * lane + rot) * 128 + ((kc ^ rot) << 4));
    }
    const bool mis = (raw_off & 2) != 0;
    for (int it = 0; it < nk; ++it) {
      if (*abort_flag) break;
      const int s = it % kLoadStages, t = it % kBStages;
      if (!mbar_wait_bounded(smem_u32(&bars.full_load[s]), (it / kLoadStages) & 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      const uint8_t* rows = raw_stage(s) + 8 * kc * P::kPitch + raw_off;
      if constexpr (P::kTableBytes > 0) {
        P::table(rows, lane, tbl);
        __syncwarp();
      }
      P pr;
      if (mis) pr.template load<true>(rows, lane, tbl);
      else pr.template load<false>(rows, lane, tbl);
      __syncwarp();  // every lane holds its raw bytes and scales in registers
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty_load[s]));
      if (!mbar_wait_bounded(smem_u32(&bars.empty_b[t]), ((it / kBStages) & 1) ^ 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      store_all<QT>(pr, b_stage(t), off);
      fence_proxy_async_smem();  // make the generic stores visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars.full_b[t]));
    }

    // ------------------------------ epilogue ------------------------------
    const bool ok = !*abort_flag &&
                    mbar_wait_bounded(smem_u32(&bars.acc_full), 0, kWaitBudgetCycles);
    if (!ok) {
      if (lane == 0) give_up();
    } else {
      tc_fence_after();
      const int quarter = warp & 3;             // TMEM lanes 32*quarter .. +31
      const int half = (warp - 2) >> 2;         // accumulator 0 (warps 2-5) or 1 (warps 6-9)
      const int row = m0 + half * 128 + quarter * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 256);
      // accumulator column 8L + p holds tile column 8L + ((p - L) & 7) (the producer's
      // rotation); with 64 columns per step, L & 7 is 4h + g for group g of half h
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 64) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t r[32], o[32];
          tmem_ld32(tbase + cb + 32 * h, r);
#pragma unroll
          for (int g = 0; g < 4; ++g)
#pragma unroll
            for (int q = 0; q < 8; ++q) o[8 * g + q] = r[8 * g + ((q + 4 * h + g) & 7)];
          if (row < M) {
            const int64_t off = (int64_t)row * N + (int64_t)n_tile * BN + cb + 32 * h;
            if constexpr (BF16_OUT) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(c) + off);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q]), __uint_as_float(o[8 * q + 1])),
                                    pack_bf16x2(__uint_as_float(o[8 * q + 2]), __uint_as_float(o[8 * q + 3])),
                                    pack_bf16x2(__uint_as_float(o[8 * q + 4]), __uint_as_float(o[8 * q + 5])),
                                    pack_bf16x2(__uint_as_float(o[8 * q + 6]), __uint_as_float(o[8 * q + 7])));
            } else {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(c) + off);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                dst[q] = make_float4(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]),
                                     __uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3]));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace gemm

// ---- host side -----------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link needed)
static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

template <int QT, bool BF16_OUT>
static cudaError_t launch_gemm_t(const void* a, const void* w, void* c, int64_t M, int64_t K,
                                 int64_t N, int64_t RB, cudaStream_t st) {
  using namespace gemm;
  using L = Smem<QT>;
  using R = Raw<QT>;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap ma, mw;
  {  // A: [M][K] bf16, boxes of 128 rows x 64 K, 128-byte swizzle
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {BK, 128};
    cuuint32_t es[2] = {1, 1};
    if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {  // W: [K][RB] bytes as uint16, boxes of 64 rows x one tile's (aligned) bytes
    cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)K};
    cuuint64_t strides[1] = {(cuuint64_t)RB};
    cuuint32_t box[2] = {(cuuint32_t)(R::kPitch / 2), BK};
    cuuint32_t es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  auto kern = gemm_kernel<QT, BF16_OUT>;
  static unsigned configured = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 32 || !(configured & (1u << dev))) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    if (dev < 32) configured |= (1u << dev);
  }
  const dim3 grid((unsigned)(N / BN), (unsigned)((M + BM - 1) / BM), 1);
  kern<<<grid, kThreads, L::kAlloc, st>>>(ma, mw, static_cast<const uint8_t*>(w), c, (int)M, (int)K,
                                          (int)N, RB);
  return cudaGetLastError();
}

cudaError_t launch_gemm(int qtype, const void* a, const void* w, void* c, int64_t M, int64_t K,
                        int64_t N, int64_t row_bytes, int c_dtype, cudaStream_t st) {
  const bool bf = c_dtype == 1;
  switch (qtype) {
    case kQ4_K: return bf ? launch_gemm_t<kQ4_K, true>(a, w, c, M, K, N, row_bytes, st)
                          : launch_gemm_t<kQ4_K, false>(a, w, c, M, K, N, row_bytes, st);
    case kQ6_K: return bf ? launch_gemm_t<kQ6_K, true>(a, w, c, M, K, N, row_bytes, st)
                          : launch_gemm_t<kQ6_K, false>(a, w, c, M, K, N, row_bytes, st);
    case kQ8_0: return bf ? launch_gemm_t<kQ8_0, true>(a, w, c, M, K, N, row_bytes, st)
                          : launch_gemm_t<kQ8_0, false>(a, w, c, M, K, N, row_bytes, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemm_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemm_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
