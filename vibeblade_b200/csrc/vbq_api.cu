// vbq_api.cu -- the extern "C" boundary declared in include/vbq.h.
//
// Argument checks mirror the reference's failure modes and messages:
//   * unsupported type -> "Unsupported dequant type: <id>" (cpp/src/dequant.cpp:423)
//     and "gemv_dequant: unsupported type <id>" (cpp/src/dequant.cpp:764);
//   * CUDA failures -> the runtime's error string, like CUDA_CHECK
//     (cpp/src/cuda_kernels.cu:24-40), but returned as a status instead of thrown.
#include <cstdio>
#include <cstring>
#include <string>

#include "vbq.h"
#include "vbq_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int ok() {
  g_last_error.clear();
  return VBQ_OK;
}

bool supported(int32_t t) { return t == VBQ_TYPE_Q4_K || t == VBQ_TYPE_Q6_K || t == VBQ_TYPE_Q8_0; }

int64_t block_values(int32_t t) { return t == VBQ_TYPE_Q8_0 ? 32 : 256; }
int64_t block_bytes(int32_t t) {
  return t == VBQ_TYPE_Q8_0 ? 34 : (t == VBQ_TYPE_Q4_K ? 144 : 210);
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int cuda_fail(cudaError_t e, const char* what) {
  return fail(VBQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

const char* vbq_last_error(void) { return g_last_error.c_str(); }

int vbq_version(void) { return 100; }

int vbq_row_bytes(int32_t type, int64_t n, int64_t* out_bytes) {
  if (!supported(type)) return fail(VBQ_ERR_TYPE, "Unsupported dequant type: " + std::to_string(type));
  if (!out_bytes) return fail(VBQ_ERR_NULL, "vbq_row_bytes: out_bytes is NULL");
  if (n < 0) return fail(VBQ_ERR_SHAPE, "vbq_row_bytes: n < 0");
  *out_bytes = (n / block_values(type)) * block_bytes(type);
  return ok();
}

int vbq_dequantize(const void* w, void* out, int64_t rows, int64_t n, int32_t type,
                   int32_t out_dtype, void* stream) {
  if (!supported(type)) return fail(VBQ_ERR_TYPE, "Unsupported dequant type: " + std::to_string(type));
  if (out_dtype != VBQ_DTYPE_F32 && out_dtype != VBQ_DTYPE_BF16)
    return fail(VBQ_ERR_SHAPE, "vbq_dequantize: out_dtype must be VBQ_DTYPE_F32 or VBQ_DTYPE_BF16");
  if (rows < 0 || n < 0) return fail(VBQ_ERR_SHAPE, "vbq_dequantize: negative size");
  if (rows == 0 || n == 0) return ok();
  const int64_t bv = block_values(type);
  if (rows > 1 && n % bv != 0)
    return fail(VBQ_ERR_SHAPE, "vbq_dequantize: n = " + std::to_string(n) +
                                   " is not a multiple of the block size " + std::to_string(bv) +
                                   " (only a single row may be ragged)");
  if (!w || !out) return fail(VBQ_ERR_NULL, "vbq_dequantize: NULL pointer");
  if (!aligned(w, 2) || !aligned(out, out_dtype == VBQ_DTYPE_F32 ? 4 : 2))
    return fail(VBQ_ERR_ALIGN, "vbq_dequantize: w must be 2-byte aligned and out element-aligned");
  const int64_t rb = (n / bv) * block_bytes(type);
  cudaError_t e = vbq::launch_dequant(type, w, out, rows, n, rb, out_dtype,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_dequantize launch");
  return ok();
}

int vbq_gemv(const float* x, const void* w, float* y, int64_t K, int64_t N, int32_t type,
             int32_t batch, void* stream) {
  if (!supported(type)) return fail(VBQ_ERR_TYPE, "gemv_dequant: unsupported type " + std::to_string(type));
  if (K < 0 || N < 0) return fail(VBQ_ERR_SHAPE, "vbq_gemv: negative size");
  if (batch < 1 || batch > 16)
    return fail(VBQ_ERR_SHAPE, "vbq_gemv: batch must be in 1..16, got " + std::to_string(batch));
  const int64_t bv = block_values(type);
  if (N % bv != 0)
    return fail(VBQ_ERR_SHAPE, "vbq_gemv: N = " + std::to_string(N) +
                                   " is not a multiple of the block size " + std::to_string(bv));
  if (N == 0) return ok();
  if (!x || !w || !y) return fail(VBQ_ERR_NULL, "vbq_gemv: NULL pointer");
  if (!aligned(x, 4) || !aligned(y, 16) || !aligned(w, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_gemv: w and y must be 16-byte aligned, x 4-byte aligned");
  if (N % 256 != 0)
    return fail(VBQ_ERR_UNSUPPORTED,
                "vbq_gemv: N must be a multiple of 256 (Q8_0 rows of a partial 256-value tile are not implemented)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)batch * (size_t)N * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv memset");
    return ok();
  }
  const int64_t rb = (N / bv) * block_bytes(type);
  cudaError_t e = vbq::launch_gemv(type, x, w, y, K, N, rb, batch, st);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv launch");
  return ok();
}

}  // extern "C"
