// vbq_gemm.cu -- quantized-weight GEMM on the sm_100a tensor cores (prefill).
//
//   C[m, n] = sum_k A[m, k] * deq(W)[k, n]
//
// A is bf16 [M, K] row-major, W the reference's K x N block layout (quant blocks along N,
// cpp/src/dequant.cpp:739-771), C fp32 or bf16 [M, N].  The reference has no batched GEMM:
// its engine runs one gemv_dequant per token (cpp/src/fast_model.cpp:645-660).
//
// A CTA pair (a 2-CTA cluster; rank 0 is the leader) computes a 512 x 256 tile of C with
// cta_group::2 tcgen05 MMAs: M = 256 spread over the pair (128 rows per CTA), N = 256,
// K = 16, fp32 accumulators in tensor memory.  Each CTA holds two 128 x 256 accumulators
// (pair rows 128r.. and 256 + 128r.., all 512 TMEM columns).  Each CTA dequantizes only
// its 128-column half of the weight tile and holds 128 of the pair's A rows; the pair MMA
// reads both CTAs' halves.  Per 64-deep K step:
//   * warp 0 (one lane) TMA-loads the CTA's two 128 x 64 A boxes (128-byte swizzle); the
//     bytes are reported to the leader's barrier (3-deep ring, freed by the MMAs);
//   * warp 18 (one lane) TMA-loads the raw quant bytes of the 64 W rows into a 3-deep
//     ring that the dequant warps free as soon as the bytes are in registers.  With an odd
//     depth a slot alternates between the two dequant groups, so each slot has one "full"
//     barrier per group.  A parity wait for phase k also passes while the barrier is still
//     in phase k - 1 (same test, other parity); on a barrier shared with the other group,
//     a group could reach its next visit of a slot (phase k) before the other group's
//     load (phase k - 1) had landed, read stale bytes, release the slot early and let the
//     producer arrive again on a phase whose arrival was spent;
//   * warps 2-17 dequantize the raw bytes to bf16 into the K-major, 128-byte swizzled B
//     half-tile (4-deep ring): warps 2-9 take the even K steps, warps 10-17 the odd ones,
//     each warp 8 K rows x 128 columns; they arrive on the leader's B barrier;
//   * the leader's warp 1 (one lane) issues 2 x 4 MMAs and commits them to barriers in
//     both CTAs.
// After the last K step warps 2-17 of each CTA read its accumulators out of tensor memory
// (tcgen05.ld) and store C.  Every mbarrier wait is bounded; a wait that gives up records
// kStatusTimeout in the device status word, raises the abort flag of both CTAs, and the
// pair drains and exits.  No TMA load here uses cluster multicast.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {

__device__ unsigned g_gemm_status = 0;

namespace gemm {

constexpr int BMP = 512, BN = 256, BK = 64;  // pair tile rows, tile columns, K step
constexpr int kHalfN = BN / 2;               // columns dequantized per CTA
constexpr int kDeqWarps = 16;                // two groups of 8, alternating K steps
constexpr int kThreads = 32 * (3 + kDeqWarps);  // + A TMA, MMA, raw TMA warps
constexpr int kRawWarp = 2 + kDeqWarps;
constexpr int kAStages = 3, kRStages = 3, kBStages = 4;
// raw steps it and it + kRCycle use the same slot and the same dequant group (it & 1)
constexpr int kRCycle = (kRStages % 2) ? 2 * kRStages : kRStages;
static_assert(kBStages % 2 == 0, "each B slot belongs to one dequant group");
constexpr int kABoxBytes = 128 * BK * 2;      // one 128 x 64 bf16 box
constexpr int kBBytes = kHalfN * BK * 2;      // 128 x 64 bf16 B half-tile
constexpr int kTableBytes = 384;              // per dequant warp
constexpr int kTmemCols = 512;

template <int QT> struct Raw {
  static constexpr int kTileBytes = Tile<QT>::kBytes;                       // 144 / 210 / 272
  static constexpr int kPitch = (QT == kQ6_K) ? 240 : kTileBytes;           // TMA box row
  static constexpr int kBytes = kPitch * BK;                                // per stage
  static constexpr int kSlot = (kBytes + 1023) / 1024 * 1024;
};

struct Bars {
  uint64_t full_a[kAStages], empty_a[kAStages];
  uint64_t full_raw[kRStages][2], empty_raw[kRStages];  // full: per slot and dequant group
  uint64_t full_b[kBStages], empty_b[kBStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort;
};

template <int QT> struct Smem {
  static constexpr int kAOff = 0;
  static constexpr int kRawOff = kAOff + kAStages * 2 * kABoxBytes;
  static constexpr int kBOff = kRawOff + kRStages * Raw<QT>::kSlot;
  static constexpr int kTblOff = kBOff + kBStages * kBBytes;
  static constexpr int kBarOff = kTblOff + kDeqWarps * kTableBytes;
  static constexpr int kTotal = kBarOff + (int)((sizeof(Bars) + 127) / 128 * 128);
  static constexpr int kAlloc = kTotal + 1024;  // slack for 1024-byte alignment
  static_assert(kAlloc <= 232448, "shared memory per CTA");
};

// ---- tcgen05 / TMA / cluster primitives (inline PTX, sm_100a) ------------------------
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
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, N = 256, M = 256
// (the pair's M; each CTA's tensor core produces 128 of the rows).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// Whole-cluster barrier (every thread of both CTAs).  Only reached after bounded waits.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// try_wait with cluster-scope acquire, for barriers that threads of the peer CTA arrive on
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint32_t bar, uint32_t parity,
                                                          long long budget) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > budget) return false;
  }
  return true;
}

// TMA tile load into this CTA's shared memory, bytes reported to `bar` in this CTA
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
// TMA tile load into this CTA's shared memory, bytes reported to a barrier of the CTA
// pair (`bar` is a shared::cluster address); no multicast
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at `bar`'s offset in both CTAs once the issued MMAs are done
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(bar), "h"((uint16_t)3)
      : "memory");
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
// In CTA r, dequant warp q (0..7 within its group) owns K rows 8q..8q+7 of a stage and
// the CTA's 128 tile columns; each lane 4 rows x 8 columns.  Every weight value is produced as the reference's fp32 value (one rounding per
// product and per difference, cpp/src/dequant.cpp:268-301, :359-402 and the Q8_0 block of
// cpp/src/cuda_kernels.cu:718-735), then rounded once to bf16.
//
// A small integer q becomes the float (magic + q) with one byte permute: the magic's
// exponent makes its mantissa LSB worth exactly 1, so a packed fp32x2 add or fma removes
// it without rounding.  Q4_K folds that into the product: fma(2^23 + q, dl, -2^23 dl) is
// dl*q rounded once (2^23 dl is exact).  The result equals the reference's value up to
// the sign of an exact zero, for every finite block scale.
//
// Two K rows of one column form one packed bf16x2 word; a lane's two words for a column
// are half of the 16-byte chunk (8 K rows) the MMA reads.
constexpr float kTwo23 = 8388608.0f;      // 2^23
constexpr float kOneHalf23 = 12582912.0f; // 1.5 * 2^23: magic 0x4b4000xx = 1.5*2^23 + xx
constexpr uint32_t kMagic23 = 0x4b000000u, kMagic15 = 0x4b400000u;

// result bytes: [byte I of w, k.byte0, k.byte2, k.byte3]; k.byte0 is zero for both magics
template <int I>
__device__ __forceinline__ float magic_byte(uint32_t w, uint32_t k) {
  return __uint_as_float(__byte_perm(w, k, 0x7640u | (uint32_t)I));
}

// Where a thread's rows and columns are: lane l takes column group lc = l >> 1 (tile
// columns 128*rank + 8*lc .. +7) and row quad rq = l & 1 (rows 4rq .. 4rq+3 of its warp's
// 8 rows).  Adjacent lanes differ in rq, so each half-warp's 8-byte stores cover 8
// column groups x both row quads: 16 distinct 8-byte slots, no bank conflict.  Scale
// tables are indexed by the warp's row pair p = 2*rq + pp, stored at slot 2*pp + rq so
// that one load instruction reads adjacent entries.
struct Lane {
  int lc;    // column group
  int rq;    // row quad
  int rank;  // CTA rank in the pair: which half of the tile's columns
};
__device__ __forceinline__ int pair_slot(int p) { return 2 * (p & 1) + (p >> 1); }

template <int QT> struct Producer;

// Q4_K: the tile's 256 columns are one block; this CTA's half covers sub-blocks
// 4r .. 4r+3, lane l's columns lie in sub-block 4r + (lc >> 2).  The (dl, ml) pair of each
// of the warp's 8 rows x 4 sub-blocks is computed once per stage into a per-warp table.
template <> struct Producer<kQ4_K> {
  static constexpr int kPitch = 144;
  // table: float4 (dl_r, dl_r+1, -2^23 dl_r, -2^23 dl_r+1) [4 row pairs][4 sub-blocks],
  // then float2 (-ml_r, -ml_r+1) [4][4] at byte 256
  __device__ __forceinline__ static void table(const uint8_t* wrows, int lane, int rank,
                                               uint8_t* tbl) {
    if (lane >= 16) return;
    const int sbl = lane & 3, p = lane >> 2;
    const Q4kScaleRecipe rec(4 * rank + sbl);
    float dl[2], ml[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 hd = *reinterpret_cast<const uint4*>(wrows + (2 * p + h) * kPitch);
      int sc, mn;
      rec.apply(hd.y, hd.z, hd.w, sc, mn);
      dl[h] = __fmul_rn(f16_ref(hd.x & 0xffffu), (float)sc);
      ml[h] = __fmul_rn(f16_ref(hd.x >> 16), (float)mn);
    }
    const int e = pair_slot(p) * 4 + sbl;
    reinterpret_cast<float4*>(tbl)[e] =
        make_float4(dl[0], dl[1], __fmul_rn(-kTwo23, dl[0]), __fmul_rn(-kTwo23, dl[1]));
    reinterpret_cast<float2*>(tbl + 256)[e] = make_float2(-ml[0], -ml[1]);
  }
  float2 dl[2], c[2], nm[2];
  uint32_t w[4][2];
  template <bool>
  __device__ __forceinline__ void load(const uint8_t* rows, const Lane& ln, const uint8_t* tbl) {
    const int sbl = ln.lc >> 2;
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      const int e = (2 * pp + ln.rq) * 4 + sbl;
      const float4 a = reinterpret_cast<const float4*>(tbl)[e];
      dl[pp] = make_float2(a.x, a.y);
      c[pp] = make_float2(a.z, a.w);
      nm[pp] = reinterpret_cast<const float2*>(tbl + 256)[e];
    }
    // column 128r + 8lc + i: 64-value group g = 2r + (lc >> 3), low nibbles when the
    // column's offset in the group is below 32
    const int off = 16 + 32 * (2 * ln.rank + (ln.lc >> 3)) + 8 * (ln.lc & 3);
    const uint32_t hs = (uint32_t)((ln.lc >> 2) & 1) * 4u;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
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

// Q6_K (reference layout): column 128r + 8lc + i takes ql bytes 64r + 4lc .. +3, qh bytes
// 32r + 2lc, +1 and scale 8r + (lc >> 1).  The 6-bit codes are assembled byte-wise: even
// columns in one word, odd columns in another.
template <> struct Producer<kQ6_K> {
  static constexpr int kPitch = 240;
  // table: float2 (d*sc_r, d*sc_r+1) [4 row pairs][8 scales]
  __device__ __forceinline__ static void table(const uint8_t* wrows, int lane, int rank,
                                               uint8_t* tbl) {
    const int sl = lane & 7, p = lane >> 3;
    float ds[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint8_t* row = wrows + (2 * p + h) * kPitch;
      ds[h] = __fmul_rn(f16_ref(ld_u16(row + 208)), (float)(int8_t)row[192 + 8 * rank + sl]);
    }
    reinterpret_cast<float2*>(tbl)[pair_slot(p) * 8 + sl] = make_float2(ds[0], ds[1]);
  }
  float2 ds[2];
  uint32_t ue[4], uo[4];
  template <bool kMisaligned>  // the block starts 2 mod 4 within the staged row
  __device__ __forceinline__ void load(const uint8_t* rows, const Lane& ln, const uint8_t* tbl) {
#pragma unroll
    for (int pp = 0; pp < 2; ++pp)
      ds[pp] = reinterpret_cast<const float2*>(tbl)[(2 * pp + ln.rq) * 8 + (ln.lc >> 1)];
    const int qlo = 64 * ln.rank + 4 * ln.lc, qho = 128 + 32 * ln.rank + 2 * ln.lc;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint8_t* row = rows + r * kPitch;
      uint32_t q;
      if constexpr (kMisaligned) {
        const uint32_t* a = reinterpret_cast<const uint32_t*>(row + qlo - 2);
        q = __byte_perm(a[0], a[1], 0x5432u);
      } else {
        q = *reinterpret_cast<const uint32_t*>(row + qlo);
      }
      // qh bytes h0 (fields of columns 0-3), h1 (4-7) as [h0, h0, h1, h1]
      const uint32_t hh = __byte_perm(ld_u16(row + qho), 0u, 0x1100u);
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

// Q8_0 (GGUF 34-byte block, fp16 scale): the tile's 256 columns are 8 blocks; column
// 128r + 8lc + i is byte 8(lc & 3) + i of block 4r + (lc >> 2), 2 bytes off a 4-byte
// boundary for even blocks.
template <> struct Producer<kQ8_0> {
  static constexpr int kPitch = 272;
  __device__ __forceinline__ static void table(const uint8_t*, int, int, uint8_t*) {}
  float2 d[2];
  uint32_t w[4][2];
  template <bool>
  __device__ __forceinline__ void load(const uint8_t* rows, const Lane& ln, const uint8_t*) {
    const int boff = 34 * (4 * ln.rank + (ln.lc >> 2));
    const int a = boff + 2 + 8 * (ln.lc & 3);
    const int base = a & ~3;
    const uint32_t sel = (a & 2) ? 0x5432u : 0x3210u;
    float dr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint8_t* row = rows + r * kPitch;
      const uint32_t* x = reinterpret_cast<const uint32_t*>(row + base);
      const uint32_t x0 = x[0], x1 = x[1], x2 = x[2];
      w[r][0] = __byte_perm(x0, x1, sel) ^ 0x80808080u;  // q + 128 as unsigned bytes
      w[r][1] = __byte_perm(x1, x2, sel) ^ 0x80808080u;
      dr[r] = f16_ieee(ld_u16(row + boff));
    }
#pragma unroll
    for (int p = 0; p < 2; ++p) d[p] = make_float2(dr[2 * p], dr[2 * p + 1]);
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

// Value I of column group lc goes to B row 8lc + ((I + lc) & 7), in the 8-byte half of
// its 16-byte chunk that holds the lane's row quad.  The epilogue undoes the rotation
// inside each group of 8 accumulator columns.
template <int QT, int I>
__device__ __forceinline__ void store_column(const Producer<QT>& pr, uint8_t* bt, const uint32_t (&off)[8]) {
  *reinterpret_cast<uint2*>(bt + off[I]) = make_uint2(pr.template pair<I>(0), pr.template pair<I>(1));
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

// GROUPED: the rows of A and C are split into n_seg consecutive segments (seg[s] ..
// seg[s+1], device memory), segment s multiplied by weight slab s (the third coordinate of
// tmap_w).  Work item blockIdx.y walks the segments' 512-row tiles; items past the last
// tile exit at once (both CTAs of a pair share blockIdx.y).
// SWI (SwiGLU fused, bf16 out): pair tile j makes h[rows, 128 j .. 128 j + 127] =
// silu(x W_gate) * (x W_up) for those columns.  CTA 0 dequantizes gate columns 128 j ..
// (half j % 2 of gate tile j / 2, tmap_w), CTA 1 the same columns of up (tmap_w2), so the
// pair MMA's N = 256 are the gate and up values of one column range and each CTA's
// accumulator holds both for its rows; the dequantization work per tile is unchanged.  The
// gate and up values are rounded to bf16 before the SwiGLU, as when the GEMM writes them
// and `vbq_swiglu_rows` reads them back, so the fused output has the same bits.
template <int QT, bool BF16_OUT, bool GROUPED, bool SWI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
            const __grid_constant__ CUtensorMap tmap_w2, void* c, int M, int K, int N,
            const int* __restrict__ seg, int n_seg, GemmEpi ep) {
  static_assert(!SWI || BF16_OUT, "the fused SwiGLU writes bf16");
  using L = Smem<QT>;
  using R = Raw<QT>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (128-byte swizzle atoms); derived from the array so that the
  // compiler keeps shared-memory addressing.  Both CTAs get the same offsets, which the
  // pair MMA relies on.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int n_tile = blockIdx.x >> 1;  // SWI: the 128-column chunk of h
  // the weight tile this CTA reads and which 128 of its 256 columns it dequantizes
  const int w_tile = SWI ? (n_tile >> 1) : n_tile;
  const int w_half = SWI ? (n_tile & 1) : (int)cluster_rank();
  const CUtensorMap* tw = (SWI && cluster_rank() == 1) ? &tmap_w2 : &tmap_w;
  int m0 = blockIdx.y * BMP, row_end = M, slab = 0;
  if constexpr (GROUPED) {
    int w = (int)blockIdx.y;
    bool found = false;
    for (int sidx = 0; sidx < n_seg && !found; ++sidx) {
      const int a = seg[sidx], b = seg[sidx + 1];
      const int tiles = b > a ? (b - a + BMP - 1) / BMP : 0;
      if (w < tiles) {
        m0 = a + w * BMP;
        row_end = b;
        slab = sidx;
        found = true;
      } else {
        w -= tiles;
      }
    }
    if (!found) return;  // before any barrier: the whole pair leaves together
  }
  const int nk = (K + BK - 1) / BK;
  const bool two_acc = m0 + 256 < row_end;  // pair rows 256..511 hold data

  auto a_box = [&](int s, int h) { return smem + L::kAOff + (2 * s + h) * kABoxBytes; };
  auto raw_stage = [&](int q) { return smem + L::kRawOff + q * R::kSlot; };
  auto b_stage = [&](int t) { return smem + L::kBOff + t * kBBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(smem_u32(&bars.full_a[s]), 1);   // leader: its expect_tx arrival
      mbar_init(smem_u32(&bars.empty_a[s]), 1);  // MMA commit
    }
    for (int q = 0; q < kRStages; ++q) {
      mbar_init(smem_u32(&bars.full_raw[q][0]), 1);
      mbar_init(smem_u32(&bars.full_raw[q][1]), 1);
      mbar_init(smem_u32(&bars.empty_raw[q]), kDeqWarps / 2);  // the warps of one group
    }
    for (int t = 0; t < kBStages; ++t) {
      mbar_init(smem_u32(&bars.full_b[t]), kDeqWarps);  // leader: one group x 2 CTAs
      mbar_init(smem_u32(&bars.empty_b[t]), 1);  // MMA commit
    }
    mbar_init(smem_u32(&bars.acc_full), 1);
    bars.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {  // whole warp, both CTAs: the 512 accumulator columns of the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&bars.tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = bars.tmem_base;
  volatile int* abort_flag = &bars.abort;
  const uint32_t peer_abort = mapa(smem_u32(&bars.abort), rank ^ 1u);

  auto give_up = [&]() {
    *abort_flag = 1;
    st_cluster_u32(peer_abort, 1u);
    atomicOr(&g_gemm_status, kStatusTimeout);
  };

  // Q6_K tiles start inside a 16-byte chunk; the TMA box starts at the chunk
  int tile_x = w_tile * R::kTileBytes;
  const int raw_off = (QT == kQ6_K) ? (tile_x & 15) : 0;
  tile_x &= ~15;

  if (warp == 0) {
    // --------------------------- A producer (both CTAs) ---------------------------
    if (lane == 0) {
      for (int it = 0; it < nk && !*abort_flag; ++it) {
        const int s = it % kAStages;
        if (!mbar_wait_bounded(smem_u32(&bars.empty_a[s]), ((it / kAStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(smem_u32(&bars.full_a[s]), 4 * kABoxBytes);
        const uint32_t fa = mapa(smem_u32(&bars.full_a[s]), 0u);
        tma_load_2d_pair(smem_u32(a_box(s, 0)), &tmap_a, it * BK, m0 + 128 * (int)rank, fa);
        tma_load_2d_pair(smem_u32(a_box(s, 1)), &tmap_a, it * BK, m0 + 256 + 128 * (int)rank, fa);
      }
    }
  } else if (warp == kRawWarp) {
    // --------------------------- raw weight producer ---------------------------
    if (lane == 0) {
      int it = 0;
      for (; it < nk && !*abort_flag; ++it) {
        const int q = it % kRStages;
        if (!mbar_wait_bounded(smem_u32(&bars.empty_raw[q]), ((it / kRStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full_raw[q][it & 1]);  // the consuming group's
        mbar_arrive_expect_tx(fb, R::kBytes);
        if constexpr (GROUPED) tma_load_3d(smem_u32(raw_stage(q)), tw, tile_x / 2, it * BK, slab, fb);
        else tma_load_2d(smem_u32(raw_stage(q)), tw, tile_x / 2, it * BK, fb);
      }
      // drain: every issued raw stage must land before the CTA may exit
      for (int j = (it > kRStages ? it - kRStages : 0); j < it; ++j)
        mbar_wait_bounded(smem_u32(&bars.full_raw[j % kRStages][j & 1]), (j / kRCycle) & 1, kWaitBudgetCycles);
    }
  } else if (warp == 1) {
    // --------------------------- MMA issuer (leader) ---------------------------
    if (rank == 0 && lane == 0) {
      for (int it = 0; it < nk && !*abort_flag; ++it) {
        const int s = it % kAStages, t = it % kBStages;
        if (!mbar_wait_bounded(smem_u32(&bars.full_a[s]), (it / kAStages) & 1, kWaitBudgetCycles) ||
            !mbar_wait_bounded_cluster(smem_u32(&bars.full_b[t]), (it / kBStages) & 1, kWaitBudgetCycles)) {
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
          umma_bf16_pair(tmem, a0 + 2 * kk, b + 2 * kk, acc);
          if (two_acc) umma_bf16_pair(tmem + 256, a1 + 2 * kk, b + 2 * kk, acc);
        }
        umma_commit_pair(smem_u32(&bars.empty_a[s]));
        umma_commit_pair(smem_u32(&bars.empty_b[t]));
      }
      umma_commit_pair(smem_u32(&bars.acc_full));  // arrives once every MMA issued is done
      // tensor memory is freed only after the MMAs writing it have finished
      if (!mbar_wait_bounded(smem_u32(&bars.acc_full), 0, kWaitBudgetCycles)) give_up();
    }
    // Tail, both CTAs: the last commits of every A / B slot arrive on this CTA's empty
    // barriers through the pair's multicast, and nothing else waits for them.  The CTA may
    // not exit (and a CTA of the next wave take its shared memory) while one of those
    // arrivals is in flight, so wait for each slot's final phase.  After an abort some of
    // those MMAs were never issued: skip.
    if (lane == 0 && !*abort_flag) {
      bool ok = true;
      for (int j = (nk > kAStages ? nk - kAStages : 0); ok && j < nk; ++j)
        ok = mbar_wait_bounded_cluster(smem_u32(&bars.empty_a[j % kAStages]), (j / kAStages) & 1,
                                       kWaitBudgetCycles);
      for (int j = (nk > kBStages ? nk - kBStages : 0); ok && j < nk; ++j)
        ok = mbar_wait_bounded_cluster(smem_u32(&bars.empty_b[j % kBStages]), (j / kBStages) & 1,
                                       kWaitBudgetCycles);
      if (!ok && !*abort_flag) give_up();
    }
  } else {
    // ------------------------------ dequant warps ------------------------------
    using P = Producer<QT>;
    const int dw = warp - 2;
    const int grp = dw >> 3;  // group g dequantizes the K steps it = g, g + 2, ...
    const int wq = dw & 7;    // this warp's 8 K rows of each step: 8 wq .. +7
    const Lane ln{lane >> 1, lane & 1, w_half};
    uint8_t* tbl = smem + L::kTblOff + dw * kTableBytes;
    uint32_t off[8];  // B half-tile byte offset of value i's 8-byte half-chunk
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rot = (i + ln.lc) & 7;  // wq is the 8-row K chunk within the step
      off[i] = (uint32_t)((8 * ln.lc + rot) * 128 + ((wq ^ rot) << 4) + 8 * ln.rq);
    }
    const bool mis = (raw_off & 2) != 0;
    const uint32_t full_b0 = mapa(smem_u32(&bars.full_b[0]), 0u);
    for (int it = grp; it < nk; it += 2) {
      if (*abort_flag) break;
      const int q = it % kRStages, t = it % kBStages;
      // this group's own barrier of the slot: its phases are exactly this group's visits
      if (!mbar_wait_bounded(smem_u32(&bars.full_raw[q][grp]), (it / kRCycle) & 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      const uint8_t* wrows = raw_stage(q) + 8 * wq * P::kPitch + raw_off;
      if constexpr (QT != kQ8_0) {
        P::table(wrows, lane, w_half, tbl);
        __syncwarp();
      }
      P pr;
      const uint8_t* rows = wrows + 4 * ln.rq * P::kPitch;
      if (mis) pr.template load<true>(rows, ln, tbl);
      else pr.template load<false>(rows, ln, tbl);
      __syncwarp();  // every lane holds its raw bytes and scales in registers
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty_raw[q]));
      if (!mbar_wait_bounded(smem_u32(&bars.empty_b[t]), ((it / kBStages) & 1) ^ 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      store_all<QT>(pr, b_stage(t), off);
      fence_proxy_async_smem();  // make the generic stores visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(smem_u32(&bars.full_b[t]));
        else mbar_arrive_cluster(full_b0 + 8u * (uint32_t)t);
      }
    }

    // ------------------------------ epilogue ------------------------------
    const bool ok = !*abort_flag &&
                    mbar_wait_bounded(smem_u32(&bars.acc_full), 0, kWaitBudgetCycles);
    if (!ok) {
      if (lane == 0 && !*abort_flag) give_up();
    } else {
      tc_fence_after();
      // 16 warps = 4 TMEM lane quarters x 2 accumulators x 2 column halves; a warp may
      // only read the lane quarter warp % 4
      const int quarter = warp & 3;
      const int half = (dw >> 2) & 1;  // accumulator 0 (pair rows 128r..) or 1 (256 + 128r..)
      const int col0 = (dw >> 3) * (BN / 2);
      const int row = m0 + half * 256 + (int)rank * 128 + quarter * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 256);
      if constexpr (SWI) {
        // accumulator columns 0..127: gate, 128..255: up, of h columns 128 n_tile + 0..127;
        // this warp takes h columns c0 .. c0 + 63 (the producer's rotation as below)
        const int c0 = (dw >> 3) * 64;
        if (half == 0 || two_acc) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {  // unrolled: the rotation indexes registers
            uint32_t rg[32], ru[32];
            tmem_ld32(tbase + c0 + 32 * hh, rg);
            tmem_ld32(tbase + 128 + c0 + 32 * hh, ru);
            if (row < row_end) {
              uint32_t o[16];
#pragma unroll
              for (int g = 0; g < 4; ++g)
#pragma unroll
                for (int qq = 0; qq < 8; qq += 2) {
                  const uint32_t gp = pack_bf16x2(__uint_as_float(rg[8 * g + ((qq + 4 * hh + g) & 7)]),
                                                  __uint_as_float(rg[8 * g + ((qq + 1 + 4 * hh + g) & 7)]));
                  const uint32_t up = pack_bf16x2(__uint_as_float(ru[8 * g + ((qq + 4 * hh + g) & 7)]),
                                                  __uint_as_float(ru[8 * g + ((qq + 1 + 4 * hh + g) & 7)]));
                  const float2 gf = make_float2(__uint_as_float(gp << 16), __uint_as_float(gp & 0xffff0000u));
                  const float2 uf = make_float2(__uint_as_float(up << 16), __uint_as_float(up & 0xffff0000u));
                  o[4 * g + qq / 2] = pack_bf16x2(silu_ref(sanitize(gf.x)) * sanitize(uf.x),
                                                  silu_ref(sanitize(gf.y)) * sanitize(uf.y));
                }
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(c) + (int64_t)row * N +
                                                    (int64_t)n_tile * 128 + c0 + 32 * hh);
#pragma unroll
              for (int x = 0; x < 4; ++x) dst[x] = make_uint4(o[4 * x], o[4 * x + 1], o[4 * x + 2], o[4 * x + 3]);
            }
          }
        }
      } else if (half == 0 || two_acc) {
        // accumulator column 8L + p holds tile column 8L + ((p - L) & 7) (the producer's
        // rotation, L & 7 = lc & 7); with 64 columns per step L & 7 is 4h + g for group g
        // of half-step h
#pragma unroll 1
        for (int cb = col0; cb < col0 + BN / 2; cb += 64) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32], o[32];
            tmem_ld32(tbase + cb + 32 * h, r);
#pragma unroll
            for (int g = 0; g < 4; ++g)
#pragma unroll
              for (int qq = 0; qq < 8; ++qq) o[8 * g + qq] = r[8 * g + ((qq + 4 * h + g) & 7)];
            if (row < row_end) {
              const int64_t off64 = (int64_t)row * N + (int64_t)n_tile * BN + cb + 32 * h;
              if (ep.bias) {  // bias of these 32 columns (the same for every row)
                const float4* bp = reinterpret_cast<const float4*>(ep.bias + (int64_t)n_tile * BN + cb + 32 * h);
#pragma unroll
                for (int x = 0; x < 8; ++x) {
                  const float4 t = __ldg(bp + x);
                  o[4 * x] = __float_as_uint(__uint_as_float(o[4 * x]) + t.x);
                  o[4 * x + 1] = __float_as_uint(__uint_as_float(o[4 * x + 1]) + t.y);
                  o[4 * x + 2] = __float_as_uint(__uint_as_float(o[4 * x + 2]) + t.z);
                  o[4 * x + 3] = __float_as_uint(__uint_as_float(o[4 * x + 3]) + t.w);
                }
              }
              if (ep.res) {  // residual of the row's 32 columns, read before the store below
                if constexpr (BF16_OUT) {
                  const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(ep.res) + off64);
#pragma unroll
                  for (int x = 0; x < 4; ++x) {
                    const uint4 t = rp[x];
                    const uint32_t wv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                      o[8 * x + 2 * q] = __float_as_uint(__uint_as_float(o[8 * x + 2 * q]) + __uint_as_float(wv[q] << 16));
                      o[8 * x + 2 * q + 1] =
                          __float_as_uint(__uint_as_float(o[8 * x + 2 * q + 1]) + __uint_as_float(wv[q] & 0xffff0000u));
                    }
                  }
                } else {
                  const float4* rp = reinterpret_cast<const float4*>(static_cast<const float*>(ep.res) + off64);
#pragma unroll
                  for (int x = 0; x < 8; ++x) {
                    const float4 t = rp[x];
                    o[4 * x] = __float_as_uint(__uint_as_float(o[4 * x]) + t.x);
                    o[4 * x + 1] = __float_as_uint(__uint_as_float(o[4 * x + 1]) + t.y);
                    o[4 * x + 2] = __float_as_uint(__uint_as_float(o[4 * x + 2]) + t.z);
                    o[4 * x + 3] = __float_as_uint(__uint_as_float(o[4 * x + 3]) + t.w);
                  }
                }
              }
              if constexpr (BF16_OUT) {
                uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(c) + off64);
#pragma unroll
                for (int x = 0; x < 4; ++x)
                  dst[x] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * x]), __uint_as_float(o[8 * x + 1])),
                                      pack_bf16x2(__uint_as_float(o[8 * x + 2]), __uint_as_float(o[8 * x + 3])),
                                      pack_bf16x2(__uint_as_float(o[8 * x + 4]), __uint_as_float(o[8 * x + 5])),
                                      pack_bf16x2(__uint_as_float(o[8 * x + 6]), __uint_as_float(o[8 * x + 7])));
              } else {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(c) + off64);
#pragma unroll
                for (int x = 0; x < 8; ++x)
                  dst[x] = make_float4(__uint_as_float(o[4 * x]), __uint_as_float(o[4 * x + 1]),
                                       __uint_as_float(o[4 * x + 2]), __uint_as_float(o[4 * x + 3]));
              }
            }
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  // warp-uniform decision: the cluster barrier below must be reached convergently
  if (__shfl_sync(0xffffffffu, *abort_flag, 0)) {
    // A load this CTA issued reports to the leader's barrier, which may never complete
    // after an abort; give such loads time to land before the shared memory is released.
    for (int i = 0; i < 64; ++i) __nanosleep(1000);
  }
  __syncwarp();
  cluster_sync_all();  // neither CTA frees TMEM or exits while the pair's MMAs may run
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
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

// Plain GEMM: slab_bytes == 0, seg == nullptr, rows = M.  Grouped: `n_seg` slabs of
// `slab_bytes` each starting at w, rows of A / C split by seg[0..n_seg] (device), `rows`
// the total row count (seg[n_seg] at most).
template <int QT, bool BF16_OUT, bool GROUPED, bool SWI>
static cudaError_t launch_gemm_t(const void* a, const void* w, const void* w2, void* c, int64_t rows,
                                 int64_t K, int64_t N, int64_t RB, int64_t slab_bytes, const int* seg,
                                 int n_seg, cudaStream_t st, GemmEpi ep) {
  using namespace gemm;
  using L = Smem<QT>;
  using R = Raw<QT>;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap ma, mw, mw2;
  {  // A: [rows][K] bf16, boxes of 128 rows x 64 K, 128-byte swizzle
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {BK, 128};
    cuuint32_t es[2] = {1, 1};
    if (enc(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // W (and, fused with SwiGLU, the up matrix W2): [slab][K][RB] bytes as uint16, boxes of
  // 64 rows x one tile's (aligned) bytes.  A fused call covers I = N columns of each.
  // The map's rows end at the matrix's own N columns (a packed gate | up row is longer than
  // either part): a box reaching past them (the last Q6_K tile's 240 bytes) reads zeros,
  // never the next part or memory past the buffer.
  const int64_t row_n = (N / Fmt<QT>::kValues) * Fmt<QT>::kBytes;
  for (int m = 0; m < (SWI ? 2 : 1); ++m) {
    cuuint64_t dims[3] = {(cuuint64_t)(row_n / 2), (cuuint64_t)K, (cuuint64_t)(GROUPED ? n_seg : 1)};
    cuuint64_t strides[2] = {(cuuint64_t)RB, (cuuint64_t)(GROUPED ? slab_bytes : RB * K)};
    cuuint32_t box[3] = {(cuuint32_t)(R::kPitch / 2), BK, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(m ? &mw2 : &mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, GROUPED ? 3 : 2, const_cast<void*>(m ? w2 : w), dims,
            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (!SWI) mw2 = mw;
  auto kern = gemm_kernel<QT, BF16_OUT, GROUPED, SWI>;
  static DeviceOnce configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured.done(dev)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return e;
    configured.mark(dev);
  }
  // two CTAs (one cluster) per 512 x 256 tile of C; grouped: an upper bound on the
  // segments' tile count (each segment adds at most one partial tile)
  const int64_t items = GROUPED ? (rows + BMP - 1) / BMP + n_seg : (rows + BMP - 1) / BMP;
  // SWI: one pair per 128 columns of h (= per 256 columns of gate | up)
  const dim3 grid((unsigned)(2 * (SWI ? N / 128 : N / BN)), (unsigned)items, 1);
  kern<<<grid, kThreads, L::kAlloc, st>>>(ma, mw, mw2, c, (int)rows, (int)K, (int)N, seg, n_seg, ep);
  return cudaGetLastError();
}

template <bool GROUPED>
static cudaError_t dispatch_gemm(int qtype, const void* a, const void* w, void* c, int64_t rows,
                                 int64_t K, int64_t N, int64_t row_bytes, int c_dtype,
                                 int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st,
                                 const GemmEpi& ep) {
  const bool bf = c_dtype == 1;
#define VBQ_GEMM_CASE(QT)                                                                       \
  case QT:                                                                                      \
    return bf ? launch_gemm_t<QT, true, GROUPED, false>(a, w, w, c, rows, K, N, row_bytes, slab_bytes, \
                                                        seg, n_seg, st, ep)                      \
              : launch_gemm_t<QT, false, GROUPED, false>(a, w, w, c, rows, K, N, row_bytes,        \
                                                         slab_bytes, seg, n_seg, st, ep);
  switch (qtype) {
    VBQ_GEMM_CASE(kQ4_K)
    VBQ_GEMM_CASE(kQ6_K)
    VBQ_GEMM_CASE(kQ8_0)
    default: return cudaErrorInvalidValue;
  }
#undef VBQ_GEMM_CASE
}

cudaError_t launch_gemm(int qtype, const void* a, const void* w, void* c, int64_t M, int64_t K,
                        int64_t N, int64_t row_bytes, int c_dtype, cudaStream_t st, const GemmEpi& ep) {
  return dispatch_gemm<false>(qtype, a, w, c, M, K, N, row_bytes, c_dtype, 0, nullptr, 0, st, ep);
}

cudaError_t launch_gemm_grouped(int qtype, const void* a, const void* w, void* c, int64_t rows,
                                int64_t K, int64_t N, int64_t row_bytes, int c_dtype,
                                int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st) {
  return dispatch_gemm<true>(qtype, a, w, c, rows, K, N, row_bytes, c_dtype, slab_bytes, seg,
                             n_seg, st, GemmEpi{});
}

// Fused SwiGLU: h bf16 [rows, I] = silu(a W_gate) * (a W_up), W_gate / W_up K x I with row
// stride row_bytes (plain) or slabs as the grouped GEMM (slab_bytes > 0, seg, n_seg).
template <bool GROUPED>
static cudaError_t dispatch_gemm_swiglu(int qtype, const void* a, const void* wg, const void* wu, void* h,
                                        int64_t rows, int64_t K, int64_t I, int64_t row_bytes,
                                        int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st) {
  switch (qtype) {
    case kQ4_K:
      return launch_gemm_t<kQ4_K, true, GROUPED, true>(a, wg, wu, h, rows, K, I, row_bytes, slab_bytes, seg,
                                                       n_seg, st, GemmEpi{});
    case kQ6_K:
      return launch_gemm_t<kQ6_K, true, GROUPED, true>(a, wg, wu, h, rows, K, I, row_bytes, slab_bytes, seg,
                                                       n_seg, st, GemmEpi{});
    case kQ8_0:
      return launch_gemm_t<kQ8_0, true, GROUPED, true>(a, wg, wu, h, rows, K, I, row_bytes, slab_bytes, seg,
                                                       n_seg, st, GemmEpi{});
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm_swiglu(int qtype, const void* a, const void* w_gate, const void* w_up, void* h,
                               int64_t M, int64_t K, int64_t I, int64_t row_bytes, cudaStream_t st) {
  return dispatch_gemm_swiglu<false>(qtype, a, w_gate, w_up, h, M, K, I, row_bytes, 0, nullptr, 0, st);
}

cudaError_t launch_gemm_grouped_swiglu(int qtype, const void* a, const void* w_gate, const void* w_up,
                                       void* h, int64_t rows, int64_t K, int64_t I, int64_t row_bytes,
                                       int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st) {
  return dispatch_gemm_swiglu<true>(qtype, a, w_gate, w_up, h, rows, K, I, row_bytes, slab_bytes, seg,
                                    n_seg, st);
}

cudaError_t gemm_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemm_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
