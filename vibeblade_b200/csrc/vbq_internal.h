// vbq_internal.h -- launchers shared between the kernel files and the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vbq {

cudaError_t launch_dequant(int qtype, const void* w, void* out, int64_t rows, int64_t n,
                           int64_t row_bytes, int out_dtype, cudaStream_t st);

// Split-K plan of the fused dequant-GEMV for the current device.
struct GemvPlan {
  int splits;            // CTAs per 256-column tile along K
  int64_t kslice;        // rows per CTA
  int64_t counter_bytes; // scratch prefix holding one counter per tile (0 when splits == 1)
  size_t scratch_bytes;  // counters + splits * batch * N fp32 partial sums
};
GemvPlan plan_gemv(int64_t K, int64_t N, int batch);

// Fused dequant-GEMV; batch in 1..16.  `scratch` must hold plan.scratch_bytes with its
// counter prefix zero (the kernel leaves it zero).  Returns cudaErrorNotSupported for
// shapes the kernels do not cover (the C-ABI layer checks shapes first).
cudaError_t launch_gemv(int qtype, const float* x, const void* w, float* y, int64_t K,
                        int64_t N, int64_t row_bytes, int batch, const GemvPlan& plan,
                        void* scratch, cudaStream_t st);

// tcgen05 dequant-GEMM: a bf16 [M,K], W K x N blocks, c fp32 (c_dtype 0) / bf16 (1) [M,N].
cudaError_t launch_gemm(int qtype, const void* a, const void* w, void* c, int64_t M, int64_t K,
                        int64_t N, int64_t row_bytes, int c_dtype, cudaStream_t st);
cudaError_t gemm_status(unsigned* out, bool clear);

// Sticky device status bits of the GEMV kernels (kStatusTimeout = 1); synchronous.
cudaError_t gemv_status(unsigned* out, bool clear);

}  // namespace vbq
