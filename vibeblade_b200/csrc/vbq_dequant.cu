// vbq_dequant.cu -- k-quant block dequantization to fp32 / bf16 (sm_100a).
//
// Device form of the reference's dequantize_row for every type its dispatcher takes
// (cpp/src/dequant.cpp:407-425: the k-quants Q2_K..Q8_K, Q4_0 / Q4_1 / Q5_0 / Q5_1, F32 /
// F16 / BF16) and of the GGUF Q8_0 block (cpp/src/cuda_kernels.cu:718-735).  Values are
// bit-identical to the reference: every product and difference the reference rounds
// separately is rounded separately here (__fmul_rn / __fsub_rn stop the compiler from
// contracting them into an FMA).
//
// Work unit: 256 consecutive values of one row (one block of a 256-value type, eight
// blocks of a 32-value type), one warp per unit, 8 values per lane, so each warp writes
// 1 KB (fp32) or 512 B (bf16) of contiguous output.  The kernel is HBM-bound on its writes.
#include "vbq_common.cuh"
#include "vbq_decode.cuh"
#include "vbq_internal.h"

namespace vbq {

template <int QT, typename OutT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w,
                                                      OutT* __restrict__ out, int64_t rows,
                                                      int64_t n, int64_t row_bytes,
                                                      bool vec_ok) {
  const int lane = threadIdx.x & 31;
  const int64_t units_per_row = (n + 255) / 256;
  const int64_t total = rows * units_per_row;
  const int64_t warp0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  constexpr int kUnitBytes = Tile<QT>::kBytes;
  for (int64_t u = warp0; u < total; u += nwarps) {
    const int64_t r = u / units_per_row;
    const int64_t j = u - r * units_per_row;
    const int64_t v0 = j * 256 + 8 * lane;  // first value of this lane within the row
    if (v0 >= n) continue;                  // ragged tail of a single row
    const uint8_t* unit = w + r * row_bytes + j * kUnitBytes;
    float v[8];
    if constexpr (Fmt<QT>::kValues == 1) {
      if (v0 + 8 > n) decode_tail<QT>(unit, lane, (int)(n - v0), v);
      else decode8<QT>(unit, lane, v);
    } else {
      decode8<QT>(unit, lane, v);
    }
    OutT* o = out + r * n + v0;
    if (vec_ok && v0 + 8 <= n) {
      if constexpr (sizeof(OutT) == 4) {
        float4* o4 = reinterpret_cast<float4*>(o);
        o4[0] = make_float4(v[0], v[1], v[2], v[3]);
        o4[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        __nv_bfloat162 p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4*>(o) = *reinterpret_cast<uint4*>(p);
      }
    } else {
      const int lim = (int)((n - v0) < 8 ? (n - v0) : 8);
      for (int i = 0; i < lim; ++i) {
        if constexpr (sizeof(OutT) == 4) o[i] = v[i];
        else o[i] = __float2bfloat16_rn(v[i]);
      }
    }
  }
}

template <int QT, typename OutT>
static cudaError_t launch_dequant_t(const void* w, void* out, int64_t rows, int64_t n,
                                    int64_t row_bytes, cudaStream_t st) {
  const int64_t units = rows * ((n + 255) / 256);
  const int warps_per_cta = 8;
  int64_t ctas = (units + warps_per_cta - 1) / warps_per_cta;
  const int64_t cap = 148LL * 16;  // grid-stride beyond 16 CTAs per SM
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) &&
                      (n % (sizeof(OutT) == 4 ? 4 : 8) == 0);
  dequant_kernel<QT, OutT><<<(unsigned)ctas, 256, 0, st>>>(
      static_cast<const uint8_t*>(w), static_cast<OutT*>(out), rows, n, row_bytes, vec_ok);
  return cudaGetLastError();
}

cudaError_t launch_dequant(int qtype, const void* w, void* out, int64_t rows, int64_t n,
                           int64_t row_bytes, int out_dtype, cudaStream_t st) {
  const bool bf = out_dtype == 1;
  switch (qtype) {
#define VBQ_DEQ_CASE(QT)                                                                  \
  case QT:                                                                                \
    return bf ? launch_dequant_t<QT, __nv_bfloat16>(w, out, rows, n, row_bytes, st)       \
              : launch_dequant_t<QT, float>(w, out, rows, n, row_bytes, st);
    VBQ_DEQ_CASE(kQ4_K)
    VBQ_DEQ_CASE(kQ6_K)
    VBQ_DEQ_CASE(kQ8_0)
    VBQ_DEQ_CASE(kF32)
    VBQ_DEQ_CASE(kF16)
    VBQ_DEQ_CASE(kBF16)
    VBQ_DEQ_CASE(kQ4_0)
    VBQ_DEQ_CASE(kQ4_1)
    VBQ_DEQ_CASE(kQ5_0)
    VBQ_DEQ_CASE(kQ5_1)
    VBQ_DEQ_CASE(kQ2_K)
    VBQ_DEQ_CASE(kQ3_K)
    VBQ_DEQ_CASE(kQ5_K)
    VBQ_DEQ_CASE(kQ8_K)
#undef VBQ_DEQ_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace vbq
