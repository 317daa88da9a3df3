// vbq_gemv.cu -- fused dequant-GEMV for decode (batch 1..16) on sm_100a.
//
// Computes y[b, n] = sum_k x[b, k] * deq(W)[k, n] for W laid out like the reference's
// gemv_dequant (cpp/src/dequant.cpp:739-780): K rows, quant blocks along N.  The
// reference dequantizes each row into scratch and runs an axpy on one core; here the
// whole matrix streams through HBM once.
//
// Decomposition
//   * A CTA owns one 256-value column tile (one Q4_K / Q6_K block, eight Q8_0 blocks per
//     row) and a K-slice.  The S CTAs that split K for the same tile form one
//     thread-block cluster (S <= 16) and reduce their partial sums through distributed
//     shared memory, in rank order, so results are deterministic and no workspace or
//     second launch is needed.
//   * Rows stream global -> shared through a 4-stage cp.async pipeline (64 rows per
//     stage).  Copies are the 16-byte-aligned superset of each row's tile bytes, so
//     Q6_K's 210-byte blocks at 2-byte offsets need no special casing on the load side.
//   * Each thread owns VPT consecutive outputs of the tile for B batch rows and walks
//     the rows of its row-lane.  A quant q becomes the float 1 + q/2^m with one funnel
//     shift and one LOP3 (q placed in the top mantissa bits), and the accumulation is
//     acc += (2^m * x * scale) * (1 + q/2^m); the constant part is subtracted once at
//     the end per sub-block.  Products are summed with packed fp32x2 FMAs.
//   Accuracy: fp32 throughout; the offset trick costs < 5 bits of the 24-bit
//   significand on the running sum (max-norm relative error ~1e-6 at K = 14336).
#include <cooperative_groups.h>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace cg = cooperative_groups;

namespace vbq {

template <int QT, int B, int VPT>
struct GemvCfg {
  static constexpr int kThreads = 256;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kTPR = 256 / VPT;             // threads sharing one row's tile
  static constexpr int kRowLanes = kThreads / kTPR;  // rows processed side by side
  static constexpr int kRows = 64;                   // rows per pipeline stage
  static constexpr int kRowsPerThread = kRows / kRowLanes;
  static constexpr int kTileBytes = Tile<QT>::kBytes;  // 144 / 210 / 272
  // shared-memory row pitch: Q6_K rows start at any even offset inside a 16-byte chunk,
  // and ceil16(14 + 210) = 224 bytes always covers the block.
  static constexpr int kPitch = (QT == kQ6_K) ? 224 : kTileBytes;
  static constexpr int kChunks = kPitch / 16;
  static constexpr int kStages = 4;
  static constexpr int kWBytes = kRows * kPitch;
  static constexpr int kXBytes = B * kRows * 4;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kPipeBytes = kStages * kStageBytes + 16;  // +16: tail pad for ld_u32_a2
  static constexpr int kBC = B < 4 ? B : 4;  // batch rows per cross-warp reduction round
  static constexpr int kRedBytes = kWarps * kBC * 256 * 4;
  static constexpr int kOutBytes = B * 256 * 4;
  static constexpr int kSmem = (kPipeBytes > kRedBytes ? kPipeBytes : kRedBytes) + kOutBytes;
  static_assert(kPitch % 16 == 0, "pitch");
  static_assert(kRows % kRowLanes == 0, "rows");
};

__device__ __forceinline__ uint32_t rotl(uint32_t w, int s) { return __funnelshift_l(w, w, s); }
__device__ __forceinline__ float fbits(uint32_t u) { return __uint_as_float(u); }

// Per-row contribution of one thread: values [v0, v0+VPT) of the 256-value tile.
// acc[b][p] holds outputs v0+2p, v0+2p+1; corr[b][g] the per-group constant.
template <int QT, int B, int VPT>
struct RowMath;

// Q4_K: one 32-value sub-block per thread (VPT <= 32), f = 1 + q/16.
template <int B, int VPT>
struct RowMath<kQ4_K, B, VPT> {
  static constexpr int kGroups = 1;
  __device__ __forceinline__ static void run(const uint8_t* __restrict__ rp, const float* xv,
                                             int v0, float2 (&acc)[B][VPT / 2],
                                             float (&corr)[B][kGroups]) {
    const uint4 h = *reinterpret_cast<const uint4*>(rp);
    const float d = f16_ref(h.x & 0xffffu);
    const float dmin = f16_ref(h.x >> 16);
    const int s = v0 >> 5;
    int sc, mn;
    q4k_scale_min(s, h.y, h.z, h.w, sc, mn);
    const float ds16 = d * (float)(16 * sc);
    const float dm = dmin * (float)mn;
    const uint8_t* qp = rp + 16 + 32 * (s >> 1) + (v0 & 31);
    uint32_t wq[VPT / 4];
    if constexpr (VPT >= 16) {
#pragma unroll
      for (int i = 0; i < VPT / 16; ++i) {
        const uint4 t = reinterpret_cast<const uint4*>(qp)[i];
        wq[4 * i + 0] = t.x; wq[4 * i + 1] = t.y; wq[4 * i + 2] = t.z; wq[4 * i + 3] = t.w;
      }
    } else {
      const uint2 t = *reinterpret_cast<const uint2*>(qp);
      wq[0] = t.x; wq[1] = t.y;
    }
    const int hs = (s & 1) * 4;  // high nibbles for odd sub-blocks
    int amt[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) amt[i] = (19 - 8 * i - hs) & 31;
    float a[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      a[b] = xv[b] * ds16;
      corr[b][0] += fmaf(xv[b], dm, a[b]);
    }
#pragma unroll
    for (int p = 0; p < VPT / 2; ++p) {
      const int t0 = 2 * p, t1 = 2 * p + 1;
      const float f0 = fbits((rotl(wq[t0 >> 2], amt[t0 & 3]) & 0x00780000u) | 0x3f800000u);
      const float f1 = fbits((rotl(wq[t1 >> 2], amt[t1 & 3]) & 0x00780000u) | 0x3f800000u);
      const float2 f = make_float2(f0, f1);
#pragma unroll
      for (int b = 0; b < B; ++b) acc[b][p] = ffma2(f, make_float2(a[b], a[b]), acc[b][p]);
    }
  }
  __device__ __forceinline__ static int group_of(int t) { return 0; }
};

// Q6_K (reference layout): u = lo | hi<<4 in 0..63, f = 1 + u/64; int8 scale per 16.
template <int B, int VPT>
struct RowMath<kQ6_K, B, VPT> {
  static constexpr int kGroups = VPT >= 16 ? VPT / 16 : 1;
  __device__ __forceinline__ static void run(const uint8_t* __restrict__ bp, const float* xv,
                                             int v0, float2 (&acc)[B][VPT / 2],
                                             float (&corr)[B][kGroups]) {
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
        uint32_t u = (rotl(ql[t >> 3], (17 - 4 * (t & 7)) & 31) & 0x001e0000u) | 0x3f800000u;
        u |= rotl(qh[t >> 4], (21 - 2 * (t & 15)) & 31) & 0x00600000u;
        fv[e] = fbits(u);
      }
      const float2 f = make_float2(fv[0], fv[1]);
      const int g = (2 * p) >> 4;
#pragma unroll
      for (int b = 0; b < B; ++b)
        acc[b][p] = ffma2(f, make_float2(a[g][b], a[g][b]), acc[b][p]);
    }
  }
  __device__ __forceinline__ static int group_of(int t) { return t >> 4; }
};

// Q8_0 (GGUF block): u = q + 128 in 0..255, f = 1 + u/256.
template <int B, int VPT>
struct RowMath<kQ8_0, B, VPT> {
  static constexpr int kGroups = 1;
  __device__ __forceinline__ static void run(const uint8_t* __restrict__ rp, const float* xv,
                                             int v0, float2 (&acc)[B][VPT / 2],
                                             float (&corr)[B][kGroups]) {
    const uint8_t* bp = rp + 34 * (v0 >> 5);
    const float d = f16_ieee(ld_u16(bp));
    uint32_t wq[VPT / 4];
#pragma unroll
    for (int i = 0; i < VPT / 4; ++i) wq[i] = ld_u32_a2(bp + 2 + (v0 & 31) + 4 * i) ^ 0x80808080u;
    const float d256 = d * 256.0f;
    float a[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      a[b] = xv[b] * d256;
      corr[b][0] = fmaf(1.5f, a[b], corr[b][0]);
    }
#pragma unroll
    for (int p = 0; p < VPT / 2; ++p) {
      const int t0 = 2 * p, t1 = 2 * p + 1;
      const float f0 = fbits((rotl(wq[t0 >> 2], (15 - 8 * (t0 & 3)) & 31) & 0x007f8000u) | 0x3f800000u);
      const float f1 = fbits((rotl(wq[t1 >> 2], (15 - 8 * (t1 & 3)) & 31) & 0x007f8000u) | 0x3f800000u);
      const float2 f = make_float2(f0, f1);
#pragma unroll
      for (int b = 0; b < B; ++b) acc[b][p] = ffma2(f, make_float2(a[b], a[b]), acc[b][p]);
    }
  }
  __device__ __forceinline__ static int group_of(int t) { return 0; }
};

template <int QT, int B, int VPT>
__device__ __forceinline__ void gemv_issue_stage(uint8_t* sW, float* sX, const uint8_t* __restrict__ w,
                                                 const float* __restrict__ x, int64_t RB, int64_t K,
                                                 int64_t tile, int64_t kbeg, int64_t kend,
                                                 int batch) {
  using C = GemvCfg<QT, B, VPT>;
  for (int slot = threadIdx.x; slot < C::kRows * C::kChunks; slot += C::kThreads) {
    const int r = slot / C::kChunks;
    const int ch = slot - r * C::kChunks;
    const int64_t k = kbeg + r;
    if (k >= kend) continue;
    const uintptr_t a = reinterpret_cast<uintptr_t>(w + k * RB + tile * C::kTileBytes);
    const uintptr_t a0 = a & ~uintptr_t(15);
    const int nbytes = (int)(((a + C::kTileBytes + 15) & ~uintptr_t(15)) - a0);
    if (ch * 16 >= nbytes) continue;
    cp_async16(sW + r * C::kPitch + ch * 16, reinterpret_cast<const void*>(a0 + ch * 16));
  }
  for (int slot = threadIdx.x; slot < B * C::kRows; slot += C::kThreads) {
    const int b = slot / C::kRows;
    const int r = slot - b * C::kRows;
    const int64_t k = kbeg + r;
    if (b < batch && k < kend) cp_async4(sX + slot, x + (int64_t)b * K + k);
    else sX[slot] = 0.0f;
  }
}

template <int QT, int B, int VPT>
__global__ void __launch_bounds__(256) gemv_kernel(const float* __restrict__ x,
                                                   const uint8_t* __restrict__ w,
                                                   float* __restrict__ y, int64_t K, int64_t N,
                                                   int64_t RB, int64_t kslice, int batch) {
  using C = GemvCfg<QT, B, VPT>;
  using M = RowMath<QT, B, VPT>;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();

  const int64_t tile = blockIdx.x;
  const int64_t k0 = (int64_t)blockIdx.y * kslice;
  const int64_t k1 = (k0 + kslice < K) ? k0 + kslice : K;
  const int nst = k1 > k0 ? (int)((k1 - k0 + C::kRows - 1) / C::kRows) : 0;

  const int tid = threadIdx.x;
  const int c = tid % C::kTPR;   // chunk of the tile
  const int rl = tid / C::kTPR;  // row lane
  const int v0 = c * VPT;

  float2 acc[B][VPT / 2];
  float corr[B][M::kGroups];
#pragma unroll
  for (int b = 0; b < B; ++b) {
#pragma unroll
    for (int p = 0; p < VPT / 2; ++p) acc[b][p] = make_float2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < M::kGroups; ++g) corr[b][g] = 0.f;
  }

  auto stage_w = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_x = [&](int s) { return reinterpret_cast<float*>(smem + s * C::kStageBytes + C::kWBytes); };

#pragma unroll
  for (int s = 0; s < C::kStages - 1; ++s) {
    if (s < nst)
      gemv_issue_stage<QT, B, VPT>(stage_w(s), stage_x(s), w, x, RB, K, tile,
                                   k0 + (int64_t)s * C::kRows, k1, batch);
    cp_async_commit();
  }

  for (int it = 0; it < nst; ++it) {
    const int nxt = it + C::kStages - 1;
    if (nxt < nst)
      gemv_issue_stage<QT, B, VPT>(stage_w(nxt % C::kStages), stage_x(nxt % C::kStages), w, x,
                                   RB, K, tile, k0 + (int64_t)nxt * C::kRows, k1, batch);
    cp_async_commit();
    cp_async_wait<C::kStages - 1>();
    __syncthreads();

    const int st = it % C::kStages;
    const uint8_t* sW = stage_w(st);
    const float* sX = stage_x(st);
    const int64_t kb = k0 + (int64_t)it * C::kRows;
#pragma unroll
    for (int i = 0; i < C::kRowsPerThread; ++i) {
      const int r = rl + i * C::kRowLanes;
      const int64_t k = kb + r;
      if (k < k1) {
        float xv[B];
#pragma unroll
        for (int b = 0; b < B; ++b) xv[b] = sX[b * C::kRows + r];
        int off = 0;
        if constexpr (QT == kQ6_K)
          off = (int)(reinterpret_cast<uintptr_t>(w + k * RB + tile * C::kTileBytes) & 15u);
        M::run(sW + r * C::kPitch + off, xv, v0, acc, corr);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- fold the per-group constants, then reduce row lanes inside the warp ----
#pragma unroll
  for (int b = 0; b < B; ++b) {
#pragma unroll
    for (int p = 0; p < VPT / 2; ++p) {
      acc[b][p].x -= corr[b][M::group_of(2 * p)];
      acc[b][p].y -= corr[b][M::group_of(2 * p + 1)];
    }
  }
#pragma unroll
  for (int off = C::kTPR; off < 32; off <<= 1) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
      for (int p = 0; p < VPT / 2; ++p) {
        acc[b][p].x += __shfl_xor_sync(0xffffffffu, acc[b][p].x, off);
        acc[b][p].y += __shfl_xor_sync(0xffffffffu, acc[b][p].y, off);
      }
    }
  }

  // ---- across warps, in kBC-row rounds, into outbuf[B][256] ----
  float* red = reinterpret_cast<float*>(smem);
  constexpr int kRedRegion = (C::kPipeBytes > C::kRedBytes ? C::kPipeBytes : C::kRedBytes);
  float* outbuf = reinterpret_cast<float*>(smem + kRedRegion);
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int bc0 = 0; bc0 < B; bc0 += C::kBC) {
    if (lane < C::kTPR) {
#pragma unroll
      for (int bb = 0; bb < C::kBC; ++bb) {
        float4* dst = reinterpret_cast<float4*>(red + (warp * C::kBC + bb) * 256 + v0);
#pragma unroll
        for (int p = 0; p < VPT / 4; ++p)
          dst[p] = make_float4(acc[bc0 + bb][2 * p].x, acc[bc0 + bb][2 * p].y,
                               acc[bc0 + bb][2 * p + 1].x, acc[bc0 + bb][2 * p + 1].y);
      }
    }
    __syncthreads();
    for (int e = tid; e < C::kBC * 256; e += C::kThreads) {
      float s = 0.f;
#pragma unroll
      for (int wv = 0; wv < C::kWarps; ++wv) s += red[wv * C::kBC * 256 + e];
      outbuf[bc0 * 256 + e] = s;
    }
    __syncthreads();
  }

  // ---- across the cluster (split-K), rank order, through distributed shared memory ----
  cluster.sync();
  const int S = (int)cluster.num_blocks();
  const int q = (int)cluster.block_rank();
  const int E = batch * 256;
  const int per = (E + S - 1) / S;
  const int e_end = (q + 1) * per < E ? (q + 1) * per : E;
  for (int e = q * per + tid; e < e_end; e += C::kThreads) {
    float s = 0.f;
    for (int rnk = 0; rnk < S; ++rnk) s += cluster.map_shared_rank(outbuf, rnk)[e];
    const int b = e >> 8, n = e & 255;
    y[(int64_t)b * N + tile * 256 + n] = s;
  }
  cluster.sync();
}

template <int QT, int B, int VPT>
static cudaError_t launch_gemv_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, cudaStream_t st) {
  using C = GemvCfg<QT, B, VPT>;
  auto kern = gemv_kernel<QT, B, VPT>;
  static unsigned configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 32 || !(configured & (1u << dev))) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    if (dev < 32) configured |= (1u << dev);
  }
  const int64_t tiles = N / 256;
  // Split K so that the grid has about two CTAs per SM; S is a power of two <= 16.
  int S = 1;
  while (S < 16 && tiles * S < 2 * 148) S <<= 1;
  const int64_t max_s = (K + C::kRows - 1) / C::kRows;
  while (S > 1 && S > max_s) S >>= 1;
  int64_t kslice = (K + S - 1) / S;
  kslice = (kslice + C::kRows - 1) / C::kRows * C::kRows;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)tiles, (unsigned)S, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)S;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, x, static_cast<const uint8_t*>(w), y, K, N, RB, kslice,
                            batch);
}

template <int QT>
static cudaError_t launch_gemv_q(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t RB, int batch, cudaStream_t st) {
  if (batch <= 1) return launch_gemv_t<QT, 1, 32>(x, w, y, K, N, RB, batch, st);
  if (batch <= 2) return launch_gemv_t<QT, 2, 32>(x, w, y, K, N, RB, batch, st);
  if (batch <= 4) return launch_gemv_t<QT, 4, 16>(x, w, y, K, N, RB, batch, st);
  if (batch <= 8) return launch_gemv_t<QT, 8, 8>(x, w, y, K, N, RB, batch, st);
  return launch_gemv_t<QT, 16, 8>(x, w, y, K, N, RB, batch, st);
}

cudaError_t launch_gemv(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                        int64_t row_bytes, int batch, cudaStream_t st) {
  if (N % 256 != 0 || batch < 1 || batch > 16) return cudaErrorNotSupported;
  switch (qtype) {
    case kQ4_K: return launch_gemv_q<kQ4_K>(x, w, y, K, N, row_bytes, batch, st);
    case kQ6_K: return launch_gemv_q<kQ6_K>(x, w, y, K, N, row_bytes, batch, st);
    case kQ8_0: return launch_gemv_q<kQ8_0>(x, w, y, K, N, row_bytes, batch, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vbq
