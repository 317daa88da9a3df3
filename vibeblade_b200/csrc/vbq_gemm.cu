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
  static constexpr int kBarOff = kBOff + kBStages * kBBytes;
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

// ---- dequantization: one thread = one K row-octet x one 8-column group ---------------
// prep() reads a row's bytes for the thread's 8 columns (shared memory, broadcast-friendly:
// all lanes of a warp read the same row); value(i) gives column i of that row in fp32,
// bit-identical to the reference's dequantizers (one rounding per product/difference).
// Small integers become floats exactly via the 2^23 + v bit pattern.
__device__ __forceinline__ float small_to_f(uint32_t v) {
  return __uint_as_float(0x4b000000u | v) - 8388608.0f;
}

template <int QT> struct Deq;

template <> struct Deq<kQ4_K> {
  float dl, ml;
  uint32_t q0, q1, hs;
  __device__ __forceinline__ void prep(const uint8_t* __restrict__ rp, int ng,
                                       const Q4kScaleRecipe& rec) {
    const uint4 h = *reinterpret_cast<const uint4*>(rp);
    int sc, mn;
    rec.apply(h.y, h.z, h.w, sc, mn);
    const float d = f16_ref(h.x & 0xffffu), dmin = f16_ref(h.x >> 16);
    dl = __fmul_rn(d, (float)sc);
    ml = __fmul_rn(dmin, (float)mn);
    const int g = ng >> 3;
    const uint2 q = *reinterpret_cast<const uint2*>(rp + 16 + 32 * g + 8 * (ng & 3));
    q0 = q.x;
    q1 = q.y;
    hs = ((ng >> 2) & 1) * 4;  // high nibbles for odd sub-blocks
  }
  __device__ __forceinline__ float value(int i) const {
    const uint32_t w = i < 4 ? q0 : q1;
    const uint32_t nib = (w >> (8 * (i & 3) + hs)) & 0xfu;
    return __fsub_rn(__fmul_rn(dl, small_to_f(nib)), ml);
  }
};

template <> struct Deq<kQ6_K> {
  float ds;
  uint32_t ql, qh;
  __device__ __forceinline__ void prep(const uint8_t* __restrict__ bp, int ng,
                                       const Q4kScaleRecipe&) {
    const float d = f16_ref(ld_u16(bp + 208));
    const int sc = (int)(int8_t)bp[192 + (ng >> 1)];
    ds = __fmul_rn(d, (float)sc);
    ql = ld_u32_a2(bp + 4 * ng);
    qh = ld_u16(bp + 128 + 2 * ng);
  }
  __device__ __forceinline__ float value(int i) const {
    const uint32_t u = ((ql >> (4 * i)) & 0xfu) | (((qh >> (2 * i)) & 0x3u) << 4);
    return __fmul_rn(ds, small_to_f(u) - 32.0f);
  }
};

template <> struct Deq<kQ8_0> {
  float d;
  uint32_t w0, w1;
  __device__ __forceinline__ void prep(const uint8_t* __restrict__ rp, int ng,
                                       const Q4kScaleRecipe&) {
    const uint8_t* bp = rp + 34 * (ng >> 2);
    d = f16_ieee(ld_u16(bp));
    const uint8_t* q = bp + 2 + 8 * (ng & 3);
    w0 = ld_u32_a2(q);
    w1 = ld_u32_a2(q + 4);
  }
  __device__ __forceinline__ float value(int i) const {
    const uint32_t w = i < 4 ? w0 : w1;
    const uint32_t b = ((w >> (8 * (i & 3))) & 0xffu) ^ 0x80u;  // q + 128
    return __fmul_rn(small_to_f(b) - 128.0f, d);
  }
};

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
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
    const int kc = warp - 2;  // this warp's 8 K rows of each stage
    const int ng = lane;      // 8-column group: columns 8*ng .. 8*ng+7
    const Q4kScaleRecipe rec(2 * (ng >> 3) + ((ng >> 2) & 1));  // Q4_K sub-block of the group
    for (int it = 0; it < nk; ++it) {
      if (*abort_flag) break;
      const int s = it % kLoadStages, t = it % kBStages;
      if (!mbar_wait_bounded(smem_u32(&bars.full_load[s]), (it / kLoadStages) & 1, kWaitBudgetCycles) ||
          !mbar_wait_bounded(smem_u32(&bars.empty_b[t]), ((it / kBStages) & 1) ^ 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      const uint8_t* raw = raw_stage(s);
      Deq<QT> rows[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) rows[r].prep(raw + (8 * kc + r) * R::kPitch + raw_off, ng, rec);
      // K-major, 128-byte swizzled B tile: column n's values of rows 8kc..8kc+7 form the
      // 16-byte chunk (kc ^ (n & 7)) of smem row n.  Lane l writes its columns in the order
      // i = (jj + l) & 7, so the 8 lanes of each store phase hit 8 different chunks.
      uint8_t* bt = b_stage(t);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int i = (jj + lane) & 7;
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = rows[r].value(i);
        const uint4 chunk = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                       pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        const int n = 8 * ng + i;
        *reinterpret_cast<uint4*>(bt + n * 128 + ((kc ^ (n & 7)) << 4)) = chunk;
      }
      fence_proxy_async_smem();  // make the generic stores visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&bars.full_b[t]));
        mbar_arrive(smem_u32(&bars.empty_load[s]));
      }
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
#pragma unroll 1
      for (int cb = 0; cb < BN; cb += 32) {
        uint32_t r[32];
        tmem_ld32(tbase + cb, r);
        if (row < M) {
          const int64_t off = (int64_t)row * N + (int64_t)n_tile * BN + cb;
          if constexpr (BF16_OUT) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(c) + off);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dst[q] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1])),
                                  pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                                  pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                                  pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(c) + off);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                   __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
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
