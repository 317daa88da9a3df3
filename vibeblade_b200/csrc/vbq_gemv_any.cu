// vbq_gemv_any.cu -- the generic fused dequant-GEMV: any weight type the reference's
// gemv_dequant takes (F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K,
// Q6_K, Q8_K), any N that is a multiple of the type's block (1 / 32 / 256 values) and any
// batch (groups of 4 rows on the grid's z dimension).
//
//   y[b, n] = sum_k x[b, k] * deq(W)[k, n]  (+ bias[n]) (+ res[b, n])
//
// (with the fused-input option, x[b, k] = silu(gate) * up of a packed [batch, 2K] buffer)
//
// (cpp/src/dequant.cpp:739-780, every type its switch at :748-763 lists that this library
// reads).  The tiled kernels cover N % 256 == 0 in the quantized types; this one takes what
// they do not: the MoE router (cpp/src/fast_model.cpp:861: N = n_experts, usually an F32 or
// F16 tensor in GGUF files), Q8_0 rows whose width is a multiple of 32 but not of 256,
// unquantized weights of any width, and the block types outside the path's three (Q4_0 /
// Q4_1 / Q5_0 / Q5_1 / Q2_K / Q3_K / Q5_K / Q8_K files).
//
// Decomposition: a CTA owns one 256-column segment of the output, a K-slice and a group of
// up to 4 batch rows; its 8 warps take the slice's rows in turn (row k to warp k % 8), lane l
// dequantizes values 8 l .. 8 l + 7 of the row's segment (vbq_decode.cuh, the reference's
// values bit for bit) and accumulates x[b, k] * value in fp32 (the reference accumulates in
// fp32 too, in row order).  The warps' sums meet in shared memory in warp order; the S
// K-slices of a segment form one thread-block cluster and the leader adds the other CTAs'
// sums, read from their shared memory, in split order.  Deterministic, no scratch, no
// atomics.  HBM-bound for large N, latency-bound for the tiny router GEMV.
#include <cuda_runtime.h>

#include "vbq_common.cuh"
#include "vbq_decode.cuh"
#include "vbq_gemv_mma.cuh"
#include "vbq_internal.h"

namespace vbq {
namespace gany {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxBatch = 4;   // batch rows per CTA
constexpr int kMaxSplit = 8;   // portable cluster size
constexpr int kRowUnroll = 4;  // rows in flight per warp

template <int QT, int B, bool SWIGLU>
__global__ void __launch_bounds__(kThreads)
gemv_any_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w, float* y, Epi epi,
                int K, int N, int64_t RB, int batch, int kslice) {
  // [warp][b][256] partial sums, then [b][256] CTA sums (read by the cluster leader)
  __shared__ __align__(16) float red[kWarps * B * 256];
  __shared__ __align__(16) float cta_sum[B * 256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seg = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // this CTA's group of batch rows
  x += (int64_t)blockIdx.z * B * (SWIGLU ? 2 * (int64_t)K : (int64_t)K);
  y += (int64_t)blockIdx.z * B * N;
  if (epi.res) epi.res += (int64_t)blockIdx.z * B * N;
  batch = batch - (int)blockIdx.z * B < B ? batch - (int)blockIdx.z * B : B;
  const int64_t v0 = (int64_t)seg * 256 + 8 * lane;  // first column of this lane
  const bool active = v0 < N;
  const bool ragged = Fmt<QT>::kValues == 1 && v0 + 8 > N;  // unquantized rows only
  const uint8_t* const wseg = w + (int64_t)seg * Tile<QT>::kBytes;
  const int k0 = split * kslice;
  const int k1 = (k0 + kslice < K) ? k0 + kslice : K;

  asm volatile("griddepcontrol.wait;" ::: "memory");  // x / res come from the previous grid
  float acc[B][8];
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[b][i] = 0.f;

  if (active) {
    // rows k0 + warp, + 8, ...; kRowUnroll of them decoded before their FMAs
    for (int k = k0 + warp; k < k1; k += kWarps * kRowUnroll) {
      float v[kRowUnroll][8];
      float xv[kRowUnroll][B];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u) {
        const int kk = k + u * kWarps;
        if (kk < k1) {
          const uint8_t* unit = wseg + (int64_t)kk * RB;
          if constexpr (Fmt<QT>::kValues == 1) {
            if (ragged) decode_tail<QT>(unit, lane, (int)(N - v0), v[u]);
            else decode8<QT>(unit, lane, v[u]);
          } else {
            decode8<QT>(unit, lane, v[u]);
          }
#pragma unroll
          for (int b = 0; b < B; ++b) xv[u][b] = (b < batch) ? gemv_x<SWIGLU>(x, b, K, kk) : 0.f;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
#pragma unroll
          for (int b = 0; b < B; ++b) xv[u][b] = 0.f;
        }
      }
      // rows in increasing order within the warp's share (fp32 FMAs)
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
#pragma unroll
        for (int b = 0; b < B; ++b)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[b][i] = fmaf(xv[u][b], v[u][i], acc[b][i]);
    }
  }
  // ---- warps -> CTA sum (warp order) ----
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float4* dst = reinterpret_cast<float4*>(red + (warp * B + b) * 256 + 8 * lane);
    dst[0] = make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
    dst[1] = make_float4(acc[b][4], acc[b][5], acc[b][6], acc[b][7]);
  }
  __syncthreads();
  const int c = threadIdx.x;  // column of the segment this thread sums
#pragma unroll
  for (int b = 0; b < B; ++b) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += red[(q * B + b) * 256 + c];
    cta_sum[b * 256 + c] = s;
  }
  // ---- K-slices -> the cluster leader (split order), then the output ----
  if (S > 1) gmma::cluster_sync_all();  // every CTA's sums are in its shared memory
  if (split == 0) {
    const int64_t n = (int64_t)seg * 256 + c;
    if (n < N) {
      const uint32_t local = smem_u32(cta_sum);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b >= batch) break;
        float s = cta_sum[b * 256 + c];
        for (int r = 1; r < S; ++r) {
          float o;
          const uint32_t ra = gmma::mapa_u32(local + (uint32_t)((b * 256 + c) * 4), (uint32_t)r);
          asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(o) : "r"(ra) : "memory");
          s += o;
        }
        y[(int64_t)b * N + n] = epi_apply(epi, s, b, N, n);
      }
    }
  }
  if (S > 1) gmma::cluster_sync_all();  // the leader's remote reads are done before exit
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int QT, int B, bool SW>
static cudaError_t launch_any_t(const float* x, const void* w, float* y, Epi epi, int64_t K,
                                int64_t N, int64_t RB, int batch, cudaStream_t st) {
  const int segs = (int)((N + 255) / 256);
  // splits: enough CTAs for ~4 per SM, each slice at least 64 rows
  int S = (4 * sm_count() + segs - 1) / segs;
  const int64_t max_by_rows = (K + 63) / 64;
  if (S > max_by_rows) S = (int)max_by_rows;
  if (S > kMaxSplit) S = kMaxSplit;
  if (S < 1) S = 1;
  int64_t kslice = (K + S - 1) / S;
  kslice = (kslice + kWarps - 1) / kWarps * kWarps;
  S = (int)((K + kslice - 1) / kslice);
  if (S < 1) S = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)segs, (unsigned)S, (unsigned)((batch + B - 1) / B));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
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
  return cudaLaunchKernelEx(&cfg, gemv_any_kernel<QT, B, SW>, x, static_cast<const uint8_t*>(w), y,
                            epi, (int)K, (int)N, RB, batch, (int)kslice);
}

template <int QT, bool SW>
static cudaError_t launch_any_b(const float* x, const void* w, float* y, Epi epi, int64_t K,
                                int64_t N, int64_t RB, int batch, cudaStream_t st) {
  if (batch <= 1) return launch_any_t<QT, 1, SW>(x, w, y, epi, K, N, RB, batch, st);
  if (batch <= 2) return launch_any_t<QT, 2, SW>(x, w, y, epi, K, N, RB, batch, st);
  return launch_any_t<QT, 4, SW>(x, w, y, epi, K, N, RB, batch, st);
}

template <int QT>
static cudaError_t launch_any_q(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t RB, int batch, cudaStream_t st, const GemvFuse& f) {
  const Epi epi{f.bias, f.res};
  return f.swiglu_x ? launch_any_b<QT, true>(x, w, y, epi, K, N, RB, batch, st)
                    : launch_any_b<QT, false>(x, w, y, epi, K, N, RB, batch, st);
}

}  // namespace gany

cudaError_t launch_gemv_any(int qtype, const float* x, const void* w, float* y, int64_t K,
                            int64_t N, int64_t row_bytes, int batch, cudaStream_t st,
                            const GemvFuse& f) {
  if (batch < 1 || K < 1 || N < 1 || K > INT32_MAX || N > INT32_MAX) return cudaErrorInvalidValue;
  if ((batch + gany::kMaxBatch - 1) / gany::kMaxBatch > 65535) return cudaErrorInvalidValue;
  // Q4_0 / Q4_1 / Q5_0 / Q5_1 decode batches on the integer tensor cores (the Q8_0 kernel's
  // 4- and 5-bit forms)
  if ((qtype == kQ4_0 || qtype == kQ4_1 || qtype == kQ5_0 || qtype == kQ5_1) && batch <= 16 &&
      gemv_q8_fits(K, N, batch) && row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0) {
    const cudaError_t e = launch_gemv_q4x_mma(qtype, x, w, y, K, N, row_bytes, batch, st, f);
    if (e != cudaErrorNotSupported) return e;
  }
  // Q5_K decode batches on the integer tensor cores (the Q4_K kernel's Q5_K form)
  if (qtype == kQ5_K && batch <= 16 && gemv_mma_fits(K, N, batch) && row_bytes % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(w) & 15u) == 0) {
    const cudaError_t e = launch_gemv_mma_q5k(x, w, y, K, N, row_bytes, batch, st, f);
    if (e != cudaErrorNotSupported) return e;
  }
  if (gemv_stage_takes(qtype, K, N, row_bytes, w)) {
    const cudaError_t e = launch_gemv_stage(qtype, x, w, y, K, N, row_bytes, batch, st, f);
    if (e != cudaErrorNotSupported) return e;  // else: a K-slice too long for its shared memory
  }
  switch (qtype) {
    case kF32: return gany::launch_any_q<kF32>(x, w, y, K, N, row_bytes, batch, st, f);
    case kF16: return gany::launch_any_q<kF16>(x, w, y, K, N, row_bytes, batch, st, f);
    case kBF16: return gany::launch_any_q<kBF16>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ8_0: return gany::launch_any_q<kQ8_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ4_K: return gany::launch_any_q<kQ4_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ6_K: return gany::launch_any_q<kQ6_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ4_0: return gany::launch_any_q<kQ4_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ4_1: return gany::launch_any_q<kQ4_1>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_0: return gany::launch_any_q<kQ5_0>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_1: return gany::launch_any_q<kQ5_1>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ2_K: return gany::launch_any_q<kQ2_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ3_K: return gany::launch_any_q<kQ3_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ5_K: return gany::launch_any_q<kQ5_K>(x, w, y, K, N, row_bytes, batch, st, f);
    case kQ8_K: return gany::launch_any_q<kQ8_K>(x, w, y, K, N, row_bytes, batch, st, f);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vbq
