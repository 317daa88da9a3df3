// vbq_moe.cu -- the mixture-of-experts FFN around the grouped dequant-GEMM.
//
// Reference semantics: vibeblade/moe.py:170-206 (ExpertRouter.route: softmax over the
// clipped logits, top-k, renormalised weights) and :407-505 (moe_ffn_silu: per selected
// expert down(silu(gate x) * (up x)) with the projections clipped to +-65504, weighted sum
// over the k slots, output sanitised).  The C++ engine's per-token loop
// (cpp/src/fast_model.cpp:534-571, :844-903) computes the same thing one token and one
// expert at a time; its slab stride (ggml_type_size per element, :852-854) is not used
// here: slab e starts at e * K * row_bytes(type, N).
//
// Device pipeline (all on the caller's stream): route -> stable sort of the (token, slot)
// entries by expert into row segments -> gather the rows of x as bf16 -> grouped GEMMs
// gate and up (bf16 out) -> SwiGLU -> grouped GEMM down (fp32) -> weighted combine.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {
namespace {

constexpr int kMaxTopK = 8;

// One thread per token.  Probabilities are recomputed on each selection pass with the same
// arithmetic, so the comparisons are consistent; ties go to the lower expert index.
__global__ void route_kernel(const float* __restrict__ logits, int T, int E, int topk,
                             int32_t* __restrict__ idx, float* __restrict__ weight) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const float* l = logits + (int64_t)t * E;
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) mx = fmaxf(mx, fminf(fmaxf(l[e], -50.0f), 50.0f));
  float sum = 0.0f;
  for (int e = 0; e < E; ++e) sum += expf(fminf(fmaxf(l[e], -50.0f), 50.0f) - mx);
  int chosen[kMaxTopK];
  float w[kMaxTopK];
  float wsum = 0.0f;
  for (int k = 0; k < topk; ++k) {
    int best = -1;
    float bp = -1.0f;
    for (int e = 0; e < E; ++e) {
      bool taken = false;
      for (int j = 0; j < k; ++j) taken |= (chosen[j] == e);
      if (taken) continue;
      const float p = expf(fminf(fmaxf(l[e], -50.0f), 50.0f) - mx) / sum;
      if (p > bp) {
        bp = p;
        best = e;
      }
    }
    chosen[k] = best;
    w[k] = bp;
    wsum += bp;
  }
  const float div = wsum < 1e-12f ? 1.0f : wsum;
  for (int k = 0; k < topk; ++k) {
    idx[(int64_t)t * topk + k] = chosen[k];
    weight[(int64_t)t * topk + k] = w[k] / div;
  }
}

// Single CTA.  Counts per expert, exclusive scan into seg, then one warp assigns rows to
// the entries in entry order (stable), 32 entries at a time.
__global__ void sort_kernel(const int32_t* __restrict__ idx, int n, int E, int32_t* __restrict__ seg,
                            int32_t* __restrict__ pos, int32_t* __restrict__ tok, int topk) {
  extern __shared__ int32_t sh[];  // cnt[E], next[E]
  int32_t* cnt = sh;
  int32_t* next = sh + E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int e = idx[j];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      seg[e] = run;
      next[e] = run;
      run += cnt[e];
    }
    seg[E] = run;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const unsigned lane = threadIdx.x;
    for (int base = 0; base < n; base += 32) {
      const int j = base + (int)lane;
      const int e = (j < n) ? idx[j] : -1;
      const bool valid = e >= 0 && e < E;
      const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
      const int rank = __popc(same & ((1u << lane) - 1u));
      const int row = valid ? next[e] + rank : -1;
      __syncwarp();
      if (valid && rank == 0) next[e] += __popc(same);
      __syncwarp();
      if (j < n) {
        pos[j] = row;
        if (valid) tok[row] = j / topk;
      }
    }
  }
}

// Single CTA, every warp busy: warp w takes the contiguous entries [w c, (w + 1) c) and
// counts them per expert; a scan over (expert, warp) in warp order gives each warp its
// first row per expert; each warp then assigns rows to its entries in entry order, 32 at
// a time.  The same stable order as sort_kernel (entry order within an expert).
constexpr int kSortWarps = 32;
__global__ void sort_parallel_kernel(const int32_t* __restrict__ idx, int n, int E,
                                     int32_t* __restrict__ seg, int32_t* __restrict__ pos,
                                     int32_t* __restrict__ tok, int topk) {
  extern __shared__ int32_t sh[];  // cnt[kSortWarps][E]: counts, then each warp's next row
  const int warp = threadIdx.x >> 5;
  const unsigned lane = threadIdx.x & 31u;
  for (int i = threadIdx.x; i < kSortWarps * E; i += blockDim.x) sh[i] = 0;
  __syncthreads();
  const int chunk = (n + kSortWarps - 1) / kSortWarps;
  const int j0 = warp * chunk, j1 = min(n, j0 + chunk);
  int32_t* mine = sh + warp * E;
  for (int base = j0; base < j1; base += 32) {
    const int j = base + (int)lane;
    const int e = (j < j1) ? idx[j] : -1;
    const bool valid = e >= 0 && e < E;
    const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
    if (valid && __popc(same & ((1u << lane) - 1u)) == 0) mine[e] += __popc(same);
    __syncwarp();
  }
  __syncthreads();
  // expert e: the warps' first rows in warp order, then the segment offsets
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kSortWarps; ++w) {
      const int c = sh[w * E + e];
      sh[w * E + e] = run;
      run += c;
    }
    seg[e + 1] = run;  // the expert's total, scanned below
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    seg[0] = 0;
    for (int e = 0; e < E; ++e) {
      const int c = seg[e + 1];
      seg[e] = run;
      run += c;
    }
    seg[E] = run;
  }
  __syncthreads();
  for (int e = (int)lane; e < E; e += 32) mine[e] += seg[e];  // + the segment start
  __syncwarp();
  for (int base = j0; base < j1; base += 32) {
    const int j = base + (int)lane;
    const int e = (j < j1) ? idx[j] : -1;
    const bool valid = e >= 0 && e < E;
    const unsigned same = __match_any_sync(0xffffffffu, valid ? e : -1);
    const int rank = __popc(same & ((1u << lane) - 1u));
    const int row = valid ? mine[e] + rank : -1;
    __syncwarp();
    if (valid && rank == 0) mine[e] += __popc(same);
    __syncwarp();
    if (j < j1) {
      pos[j] = row;
      if (valid) tok[row] = j / topk;
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// a_perm[row, :] = bf16(x[tok[row], :]); one CTA per row, 8 values per thread step
__global__ void gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ tok, int H,
                              uint4* __restrict__ a_perm) {
  const int row = blockIdx.x;
  const float4* src = reinterpret_cast<const float4*>(x + (int64_t)tok[row] * H);
  uint4* dst = a_perm + (int64_t)row * (H / 8);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    const float4 a = src[2 * i], b = src[2 * i + 1];
    dst[i] = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y),
                        pack_bf16(b.z, b.w));
  }
}

// sanitize() and silu_ref() are in vbq_common.cuh (shared with the fused GEMV input).

// silu(g) * u on 8 bf16 / 4 fp32 values (one 16-byte vector of each), inputs sanitised
__device__ __forceinline__ uint4 swiglu_vec(uint4 gv, uint4 uv, std::true_type /*bf16*/) {
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 g2 = *reinterpret_cast<const __nv_bfloat162*>(&gw[q]);
    const __nv_bfloat162 u2 = *reinterpret_cast<const __nv_bfloat162*>(&uw[q]);
    const float2 gf = __bfloat1622float2(g2), uf = __bfloat1622float2(u2);
    o[q] = pack_bf16(silu_ref(sanitize(gf.x)) * sanitize(uf.x), silu_ref(sanitize(gf.y)) * sanitize(uf.y));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ uint4 swiglu_vec(uint4 gq, uint4 uq, std::false_type /*fp32*/) {
  const float4 gv = *reinterpret_cast<const float4*>(&gq), uv = *reinterpret_cast<const float4*>(&uq);
  const float4 r = make_float4(silu_ref(sanitize(gv.x)) * sanitize(uv.x), silu_ref(sanitize(gv.y)) * sanitize(uv.y),
                               silu_ref(sanitize(gv.z)) * sanitize(uv.z), silu_ref(sanitize(gv.w)) * sanitize(uv.w));
  return *reinterpret_cast<const uint4*>(&r);
}

template <bool BF16>
__global__ void swiglu_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u,
                              uint4* __restrict__ h, int64_t nv) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * blockDim.x)
    h[i] = swiglu_vec(g[i], u[i], std::integral_constant<bool, BF16>{});
}

// rows of [g | u] (each row: the gate half then the up half, w vectors each) -> rows of
// h = silu(g) * u (w vectors each): the output of one GEMM / GEMV over gate and up packed
// side by side
template <bool BF16>
__global__ void swiglu_rows_kernel(const uint4* __restrict__ gu, uint4* __restrict__ h,
                                   int64_t rows, int64_t w) {
  const int64_t total = rows * w;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / w, c = i - r * w;
    const uint4* row = gu + r * 2 * w;
    h[i] = swiglu_vec(row[c], row[w + c], std::integral_constant<bool, BF16>{});
  }
}

// out[t, d] = sanitize(((0 + w0 y0) + w1 y1) + ...), each product and sum rounded once,
// in slot order as the reference's accumulation loop (vibeblade/moe.py:466-475)
__global__ void combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ pos,
                               const float* __restrict__ weight, int topk, int H,
                               float* __restrict__ out) {
  const int t = blockIdx.x;
  for (int d = threadIdx.x; d < H; d += blockDim.x) {
    float acc = 0.0f;
    for (int k = 0; k < topk; ++k) {
      const int r = pos[(int64_t)t * topk + k];
      const float v = r >= 0 ? y[(int64_t)r * H + d] : 0.0f;
      acc = __fadd_rn(acc, __fmul_rn(weight[(int64_t)t * topk + k], v));
    }
    out[(int64_t)t * H + d] = sanitize(acc);
  }
}

// combine_kernel on 16-byte vectors (H % 4 == 0, aligned rows): the same products and sums
// per value, in the same order
__global__ void combine4_kernel(const float4* __restrict__ y, const int32_t* __restrict__ pos,
                                const float* __restrict__ weight, int topk, int H4,
                                float4* __restrict__ out) {
  const int t = blockIdx.x;
  for (int d = threadIdx.x; d < H4; d += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < topk; ++k) {
      const int r = pos[(int64_t)t * topk + k];
      const float4 v = r >= 0 ? y[(int64_t)r * H4 + d] : make_float4(0.f, 0.f, 0.f, 0.f);
      const float w = weight[(int64_t)t * topk + k];
      acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
      acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
      acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
      acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
    }
    out[(int64_t)t * H4 + d] = make_float4(sanitize(acc.x), sanitize(acc.y), sanitize(acc.z), sanitize(acc.w));
  }
}

}  // namespace

cudaError_t launch_moe_route(const float* logits, int T, int E, int topk, int32_t* idx,
                             float* weight, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (topk < 1 || topk > kMaxTopK || topk > E) return cudaErrorInvalidValue;
  route_kernel<<<(T + 127) / 128, 128, 0, st>>>(logits, T, E, topk, idx, weight);
  return cudaGetLastError();
}

cudaError_t launch_moe_sort(const int32_t* idx, int T, int E, int topk, int32_t* seg,
                            int32_t* pos, int32_t* tok, cudaStream_t st) {
  const size_t shm_par = (size_t)kSortWarps * E * sizeof(int32_t);
  if (shm_par <= 48 * 1024) {
    sort_parallel_kernel<<<1, 32 * kSortWarps, shm_par, st>>>(idx, T * topk, E, seg, pos, tok, topk);
    return cudaGetLastError();
  }
  const size_t shm = (size_t)2 * E * sizeof(int32_t);
  if (shm > 48 * 1024) return cudaErrorInvalidValue;
  sort_kernel<<<1, 1024, shm, st>>>(idx, T * topk, E, seg, pos, tok, topk);
  return cudaGetLastError();
}

cudaError_t launch_moe_gather(const float* x, const int32_t* tok, int rows, int H, void* a_perm,
                              cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  gather_kernel<<<rows, 128, 0, st>>>(x, tok, H, static_cast<uint4*>(a_perm));
  return cudaGetLastError();
}

static int grid_for(int64_t items) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (items + 255) / 256;
  return (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
}

cudaError_t launch_swiglu(const void* g, const void* u, void* h, int64_t n, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 <= 0) return cudaSuccess;
  swiglu_kernel<true><<<grid_for(n8), 256, 0, st>>>(static_cast<const uint4*>(g),
                                                    static_cast<const uint4*>(u), static_cast<uint4*>(h), n8);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_f32(const float* g, const float* u, float* h, int64_t n, cudaStream_t st) {
  const int64_t n4 = n / 4;
  if (n4 <= 0) return cudaSuccess;
  swiglu_kernel<false><<<grid_for(n4), 256, 0, st>>>(reinterpret_cast<const uint4*>(g),
                                                     reinterpret_cast<const uint4*>(u),
                                                     reinterpret_cast<uint4*>(h), n4);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_rows(const void* gu, void* h, int64_t rows, int64_t n, bool bf16,
                               cudaStream_t st) {
  const int64_t w = bf16 ? n / 8 : n / 4;  // 16-byte vectors per half row
  if (rows <= 0 || w <= 0) return cudaSuccess;
  if (bf16)
    swiglu_rows_kernel<true><<<grid_for(rows * w), 256, 0, st>>>(static_cast<const uint4*>(gu),
                                                                 static_cast<uint4*>(h), rows, w);
  else
    swiglu_rows_kernel<false><<<grid_for(rows * w), 256, 0, st>>>(static_cast<const uint4*>(gu),
                                                                  static_cast<uint4*>(h), rows, w);
  return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float* y, const int32_t* pos, const float* weight, int T,
                               int topk, int H, float* out, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  if (H % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0)
    combine4_kernel<<<T, 256, 0, st>>>(reinterpret_cast<const float4*>(y), pos, weight, topk, H / 4,
                                       reinterpret_cast<float4*>(out));
  else
    combine_kernel<<<T, 256, 0, st>>>(y, pos, weight, topk, H, out);
  return cudaGetLastError();
}

}  // namespace vbq
