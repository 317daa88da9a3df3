// vbq_internal.h -- launchers shared between the kernel files and the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vbq {

cudaError_t launch_dequant(int qtype, const void* w, void* out, int64_t rows, int64_t n,
                           int64_t row_bytes, int out_dtype, cudaStream_t st);

// Fused dequant-GEMV; batch in 1..16.  Returns cudaErrorNotSupported for shapes the
// kernels do not cover (the C-ABI layer checks shapes first).
cudaError_t launch_gemv(int qtype, const float* x, const void* w, float* y, int64_t K,
                        int64_t N, int64_t row_bytes, int batch, cudaStream_t st);

}  // namespace vbq
