// vbq_api.cu -- the extern "C" boundary declared in include/vbq.h.
//
// Argument checks mirror the reference's failure modes and messages:
//   * unsupported type -> "Unsupported dequant type: <id>" (cpp/src/dequant.cpp:423)
//     and "gemv_dequant: unsupported type <id>" (cpp/src/dequant.cpp:764);
//   * CUDA failures -> the runtime's error string, like CUDA_CHECK
//     (cpp/src/cuda_kernels.cu:24-40), but returned as a status instead of thrown.
#include <cuda.h>

#include <cstdio>
#include <cstring>
#include <mutex>
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

// the quantized weight types of the path (tiled GEMV kernels, tensor-core GEMM, MoE)
bool quantized(int32_t t) { return t == VBQ_TYPE_Q4_K || t == VBQ_TYPE_Q6_K || t == VBQ_TYPE_Q8_0; }
// the reference dispatcher's other block types (cpp/src/dequant.cpp:412-422): dequantize
// and the generic GEMV read them
bool other_block_type(int32_t t) {
  switch (t) {
    case VBQ_TYPE_Q4_0: case VBQ_TYPE_Q4_1: case VBQ_TYPE_Q5_0: case VBQ_TYPE_Q5_1:
    case VBQ_TYPE_Q2_K: case VBQ_TYPE_Q3_K: case VBQ_TYPE_Q5_K: case VBQ_TYPE_Q8_K:
      return true;
    default:
      return false;
  }
}
// every weight type the library reads (dequantize, GEMV): the reference's dequantize_row and
// gemv_dequant take the same set (cpp/src/dequant.cpp:407-425, :748-765)
bool supported(int32_t t) {
  return quantized(t) || other_block_type(t) || t == VBQ_TYPE_F32 || t == VBQ_TYPE_F16 ||
         t == VBQ_TYPE_BF16;
}

// values and bytes per block (cpp/include/ggml_types.h:31-71; Q8_0 the 34-byte GGUF block)
int64_t block_values(int32_t t) {
  switch (t) {
    case VBQ_TYPE_F32: case VBQ_TYPE_F16: case VBQ_TYPE_BF16: return 1;
    case VBQ_TYPE_Q4_0: case VBQ_TYPE_Q4_1: case VBQ_TYPE_Q5_0: case VBQ_TYPE_Q5_1:
    case VBQ_TYPE_Q8_0: return 32;
    default: return 256;  // Q2_K .. Q8_K
  }
}
int64_t block_bytes(int32_t t) {
  switch (t) {
    case VBQ_TYPE_Q4_0: return 18;
    case VBQ_TYPE_Q4_1: return 20;
    case VBQ_TYPE_Q5_0: return 22;
    case VBQ_TYPE_Q5_1: return 24;
    case VBQ_TYPE_Q8_0: return 34;
    case VBQ_TYPE_Q2_K: return 84;
    case VBQ_TYPE_Q3_K: return 110;
    case VBQ_TYPE_Q4_K: return 144;
    case VBQ_TYPE_Q5_K: return 176;
    case VBQ_TYPE_Q6_K: return 210;
    case VBQ_TYPE_Q8_K: return 292;
    case VBQ_TYPE_F32: return 4;
    default: return 2;  // F16, BF16
  }
}

// The generic GEMV kernel takes unquantized weights and widths that are not whole
// 256-column tiles; the tiled kernels the rest.
bool gemv_generic(int32_t t, int64_t N) { return !quantized(t) || N % 256 != 0; }

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

// Batches above 16 run as launches over groups of up to 16 rows (the kernels' limit), in
// order on the stream, sharing the scratch (each launch leaves it zero-filled).
constexpr int32_t kMaxBatch = 32, kLaunchBatch = 16;

// batch limit of the generic kernel (groups of 4 rows on a grid dimension of 65535)
constexpr int32_t kMaxBatchGeneric = 4 * 65535;

static int gemv_checks(int32_t type, int64_t K, int64_t N, int32_t batch) {
  if (!supported(type)) return fail(VBQ_ERR_TYPE, "gemv_dequant: unsupported type " + std::to_string(type));
  if (K < 0 || N < 0) return fail(VBQ_ERR_SHAPE, "vbq_gemv: negative size");
  const int32_t max_batch = gemv_generic(type, N) ? kMaxBatchGeneric : kMaxBatch;
  if (batch < 1 || batch > max_batch)
    return fail(VBQ_ERR_SHAPE, "vbq_gemv: batch must be in 1.." + std::to_string(max_batch) + ", got " +
                                   std::to_string(batch));
  const int64_t bv = block_values(type);
  if (N % bv != 0)
    return fail(VBQ_ERR_SHAPE, "vbq_gemv: N = " + std::to_string(N) +
                                   " is not a multiple of the block size " + std::to_string(bv));
  return VBQ_OK;
}

// the largest plan among the launches of a call (a full group of 16 and the remainder):
// the most scratch, and the longest counter prefix any of the launches uses
static vbq::GemvPlan gemv_call_plan(int64_t K, int64_t N, int32_t batch, int32_t type) {
  vbq::GemvPlan p = vbq::plan_gemv(K, N, batch < kLaunchBatch ? batch : kLaunchBatch, type);
  const int32_t rem = batch % kLaunchBatch;
  if (batch > kLaunchBatch && rem != 0) {
    const vbq::GemvPlan q = vbq::plan_gemv(K, N, rem, type);
    const int64_t counters = q.counter_bytes > p.counter_bytes ? q.counter_bytes : p.counter_bytes;
    if (q.scratch_bytes > p.scratch_bytes) p = q;
    p.counter_bytes = counters;
  }
  return p;
}

static cudaError_t launch_gemv_groups(int32_t type, const float* x, const void* w, float* y,
                                      int64_t K, int64_t N, int64_t rb, int32_t batch,
                                      void* scratch, cudaStream_t st,
                                      const vbq::GemvFuse& f = vbq::GemvFuse{}) {
  const int64_t xrow = f.swiglu_x ? 2 * K : K;
  for (int32_t b0 = 0; b0 < batch; b0 += kLaunchBatch) {
    const int32_t nb = batch - b0 < kLaunchBatch ? batch - b0 : kLaunchBatch;
    const vbq::GemvPlan plan = vbq::plan_gemv(K, N, nb, type);
    vbq::GemvFuse fg = f;
    if (f.res) fg.res = f.res + (int64_t)b0 * N;
    cudaError_t e = vbq::launch_gemv(type, x + (int64_t)b0 * xrow, w, y + (int64_t)b0 * N, K, N, rb, nb,
                                     plan, scratch, st, fg);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int vbq_gemv_scratch_bytes(int64_t K, int64_t N, int32_t type, int32_t batch, size_t* bytes) {
  if (int rc = gemv_checks(type, K, N, batch)) return rc;
  if (!bytes) return fail(VBQ_ERR_NULL, "vbq_gemv_scratch_bytes: bytes is NULL");
  *bytes = (K == 0 || N == 0 || gemv_generic(type, N)) ? 0 : gemv_call_plan(K, N, batch, type).scratch_bytes;
  return ok();
}

// vbq_gemv and vbq_gemv_ex: `who` names the entry in messages, `f` the optional fusions
static int gemv_impl(const char* who, const float* x, const void* w, float* y, int64_t K, int64_t N,
                     int32_t type, int32_t batch, void* scratch, size_t scratch_bytes, void* stream,
                     const vbq::GemvFuse& f) {
  const std::string nm(who);
  if (int rc = gemv_checks(type, K, N, batch)) return rc;
  if (N == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool epi = f.bias || f.res;
  if (K == 0) {  // empty sum: the reference zeroes out and adds nothing (dequant.cpp:767)
    if (!y) return fail(VBQ_ERR_NULL, nm + ": NULL pointer");
    if (epi) return fail(VBQ_ERR_SHAPE, nm + ": K must be positive when a bias or residual is added");
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)batch * (size_t)N * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, (nm + " memset").c_str());
    return ok();
  }
  if (!x || !w || !y) return fail(VBQ_ERR_NULL, nm + ": NULL pointer");
  if (!aligned(x, 4) || !aligned(y, 16) || !aligned(w, 16))
    return fail(VBQ_ERR_ALIGN, nm + ": w and y must be 16-byte aligned, x 4-byte aligned");
  if ((f.bias && !aligned(f.bias, 4)) || (f.res && !aligned(f.res, 4)))
    return fail(VBQ_ERR_ALIGN, nm + ": bias and residual must be 4-byte aligned");
  if (K > (int64_t)INT32_MAX || N > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, nm + ": sizes above 2^31 are not supported");
  if (gemv_generic(type, N)) {
    const int64_t rbg = (N / block_values(type)) * block_bytes(type);
    cudaError_t e = vbq::launch_gemv_any(type, x, w, y, K, N, rbg, batch, st, f);
    if (e != cudaSuccess) return cuda_fail(e, (nm + " launch").c_str());
    return ok();
  }
  const vbq::GemvPlan plan = gemv_call_plan(K, N, batch, type);
  if (plan.scratch_bytes > 0) {
    if (!scratch || scratch_bytes < plan.scratch_bytes)
      return fail(VBQ_ERR_WORKSPACE, nm + ": scratch needs " + std::to_string(plan.scratch_bytes) +
                                         " bytes (vbq_gemv_scratch_bytes), got " + std::to_string(scratch_bytes));
    if (!aligned(scratch, 16)) return fail(VBQ_ERR_ALIGN, nm + ": scratch must be 16-byte aligned");
  }
  const int64_t rb = (N / block_values(type)) * block_bytes(type);
  cudaError_t e = launch_gemv_groups(type, x, w, y, K, N, rb, batch, scratch, st, f);
  if (e != cudaSuccess) return cuda_fail(e, (nm + " launch").c_str());
  return ok();
}

int vbq_gemv(const float* x, const void* w, float* y, int64_t K, int64_t N, int32_t type,
             int32_t batch, void* scratch, size_t scratch_bytes, void* stream) {
  return gemv_impl("vbq_gemv", x, w, y, K, N, type, batch, scratch, scratch_bytes, stream, vbq::GemvFuse{});
}

int vbq_gemv_ex(const float* x, const void* w, float* y, int64_t K, int64_t N, int32_t type,
                int32_t batch, int32_t flags, const float* bias, const float* residual, void* scratch,
                size_t scratch_bytes, void* stream) {
  if (flags & ~VBQ_GEMV_X_SWIGLU) return fail(VBQ_ERR_SHAPE, "vbq_gemv_ex: unknown flags " + std::to_string(flags));
  vbq::GemvFuse f;
  f.swiglu_x = (flags & VBQ_GEMV_X_SWIGLU) != 0;
  f.bias = bias;
  f.res = residual;
  return gemv_impl("vbq_gemv_ex", x, w, y, K, N, type, batch, scratch, scratch_bytes, stream, f);
}

static int gemm_impl(const void* a, const void* w, void* c, int64_t M, int64_t K, int64_t N, int32_t type,
                     int32_t c_dtype, void* stream, const vbq::GemmEpi& ep) {
  if (!quantized(type)) return fail(VBQ_ERR_TYPE, "gemm_dequant: unsupported type " + std::to_string(type));
  if (c_dtype != VBQ_DTYPE_F32 && c_dtype != VBQ_DTYPE_BF16)
    return fail(VBQ_ERR_SHAPE, "vbq_gemm: c_dtype must be VBQ_DTYPE_F32 or VBQ_DTYPE_BF16");
  if (M < 0 || K < 0 || N < 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm: negative size");
  if (N % 256 != 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm: N must be a multiple of 256");
  if (M == 0 || N == 0) return ok();
  if (K == 0) {
    if (!c) return fail(VBQ_ERR_NULL, "vbq_gemm: NULL pointer");
    if (ep.bias || ep.res) return fail(VBQ_ERR_SHAPE, "vbq_gemm_ex: K must be positive when a bias or residual is added");
    cudaError_t e = cudaMemsetAsync(c, 0, (size_t)M * N * (c_dtype == VBQ_DTYPE_F32 ? 4 : 2),
                                    static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemm memset");
    return ok();
  }
  if (!a || !w || !c) return fail(VBQ_ERR_NULL, "vbq_gemm: NULL pointer");
  if (K % 8 != 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm: K must be a multiple of 8 (16-byte rows of A)");
  if (M > (int64_t)INT32_MAX || K > (int64_t)INT32_MAX || N > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_gemm: sizes above 2^31 are not supported");
  const int64_t rb = (N / block_values(type)) * block_bytes(type);
  if (rb % 16 != 0)
    return fail(VBQ_ERR_UNSUPPORTED, "vbq_gemm: weight rows must be a multiple of 16 bytes (Q6_K: N % 2048 == 0)");
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(c, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_gemm: a, w and c must be 16-byte aligned");
  if ((ep.bias && !aligned(ep.bias, 16)) || (ep.res && !aligned(ep.res, 16)))
    return fail(VBQ_ERR_ALIGN, "vbq_gemm_ex: bias and residual must be 16-byte aligned");
  cudaError_t e = vbq::launch_gemm(type, a, w, c, M, K, N, rb, c_dtype, static_cast<cudaStream_t>(stream), ep);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemm launch");
  return ok();
}

int vbq_gemm(const void* a, const void* w, void* c, int64_t M, int64_t K, int64_t N, int32_t type,
             int32_t c_dtype, void* stream) {
  return gemm_impl(a, w, c, M, K, N, type, c_dtype, stream, vbq::GemmEpi{});
}

int vbq_gemm_swiglu(const void* a, const void* w_gate, const void* w_up, void* h, int64_t M, int64_t K,
                    int64_t I, int32_t type, int64_t row_bytes, void* stream) {
  if (!quantized(type)) return fail(VBQ_ERR_TYPE, "gemm_dequant: unsupported type " + std::to_string(type));
  if (M < 0 || K < 0 || I < 0 || row_bytes < 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm_swiglu: negative size");
  if (I % 256 != 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm_swiglu: I must be a multiple of 256");
  if (M == 0 || I == 0) return ok();
  if (!h) return fail(VBQ_ERR_NULL, "vbq_gemm_swiglu: NULL pointer");
  if (K == 0) {  // gate = up = 0: silu(0) * 0
    cudaError_t e = cudaMemsetAsync(h, 0, (size_t)M * I * 2, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemm_swiglu memset");
    return ok();
  }
  if (!a || !w_gate || !w_up) return fail(VBQ_ERR_NULL, "vbq_gemm_swiglu: NULL pointer");
  if (K % 8 != 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm_swiglu: K must be a multiple of 8 (16-byte rows of A)");
  if (M > (int64_t)INT32_MAX || K > (int64_t)INT32_MAX || I > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_gemm_swiglu: sizes above 2^31 are not supported");
  const int64_t rb = (I / block_values(type)) * block_bytes(type);
  const int64_t stride = row_bytes ? row_bytes : rb;
  if (stride < rb) return fail(VBQ_ERR_SHAPE, "vbq_gemm_swiglu: row_bytes below the rows' " + std::to_string(rb) + " bytes");
  if (stride % 16 != 0)
    return fail(VBQ_ERR_UNSUPPORTED, "vbq_gemm_swiglu: weight rows must be a multiple of 16 bytes apart");
  if (!aligned(a, 16) || !aligned(w_gate, 16) || !aligned(w_up, 16) || !aligned(h, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_gemm_swiglu: a, w_gate, w_up and h must be 16-byte aligned");
  cudaError_t e = vbq::launch_gemm_swiglu(type, a, w_gate, w_up, h, M, K, I, stride,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemm_swiglu launch");
  return ok();
}

int vbq_gemm_ex(const void* a, const void* w, void* c, int64_t M, int64_t K, int64_t N, int32_t type,
                int32_t c_dtype, const float* bias, const void* residual, void* stream) {
  vbq::GemmEpi ep;
  ep.bias = bias;
  ep.res = residual;
  return gemm_impl(a, w, c, M, K, N, type, c_dtype, stream, ep);
}

int vbq_device_status(int32_t* status, int32_t clear) {
  if (!status) return fail(VBQ_ERR_NULL, "vbq_device_status: status is NULL");
  unsigned g = 0, g2 = 0, g3 = 0, g4 = 0, g5 = 0, g6 = 0, g7 = 0, g8 = 0;
  cudaError_t e = vbq::gemv_status(&g, clear != 0);
  if (e == cudaSuccess) e = vbq::gemm_status(&g2, clear != 0);
  if (e == cudaSuccess) e = vbq::gemv_mma_status(&g3, clear != 0);
  if (e == cudaSuccess) e = vbq::gemv_wide_status(&g4, clear != 0);
  if (e == cudaSuccess) e = vbq::gemv_q8_status(&g5, clear != 0);
  if (e == cudaSuccess) e = vbq::gemv_half_status(&g6, clear != 0);
  if (e == cudaSuccess) e = vbq::gemv_q6_status(&g7, clear != 0);
  if (e == cudaSuccess) e = vbq::peer_status(&g8, clear != 0);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_device_status");
  g |= g2 | g3 | g4 | g5 | g6 | g7 | g8;
  *status = (int32_t)g;
  if (g & 1u) return fail(VBQ_ERR_TIMEOUT, "a bounded device-side wait gave up (a copy never completed)");
  return ok();
}

int vbq_debug_wait_probe(int64_t budget_cycles, int32_t arrive, void* stream) {
  if (budget_cycles < 1 || budget_cycles > (int64_t)1 << 31)
    return fail(VBQ_ERR_SHAPE, "vbq_debug_wait_probe: budget_cycles must be in 1..2^31");
  if (arrive != 0 && arrive != 1) return fail(VBQ_ERR_SHAPE, "vbq_debug_wait_probe: arrive must be 0 or 1");
  cudaError_t e = vbq::launch_wait_probe((long long)budget_cycles, arrive, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_debug_wait_probe launch");
  return ok();
}

int vbq_peer_allreduce(const float* const* data, int32_t* const* flags, int32_t world, int32_t rank,
                       int32_t epoch, int64_t n, float* out, int64_t timeout_cycles, void* stream) {
  if (world < 1 || world > 8) return fail(VBQ_ERR_SHAPE, "vbq_peer_allreduce: world must be in 1..8");
  if (rank < 0 || rank >= world) return fail(VBQ_ERR_SHAPE, "vbq_peer_allreduce: rank out of range");
  if (epoch < 1) return fail(VBQ_ERR_SHAPE, "vbq_peer_allreduce: epoch must be positive");
  if (n < 0) return fail(VBQ_ERR_SHAPE, "vbq_peer_allreduce: negative n");
  if (!data || !flags || (n > 0 && !out)) return fail(VBQ_ERR_NULL, "vbq_peer_allreduce: NULL pointer");
  for (int32_t p = 0; p < world; ++p) {
    if (!data[p] || !flags[p]) return fail(VBQ_ERR_NULL, "vbq_peer_allreduce: NULL peer pointer");
    if (!aligned(data[p], 16) || !aligned(flags[p], 4))
      return fail(VBQ_ERR_ALIGN, "vbq_peer_allreduce: peer data must be 16-byte aligned, flags 4-byte");
  }
  if (out && !aligned(out, 16)) return fail(VBQ_ERR_ALIGN, "vbq_peer_allreduce: out must be 16-byte aligned");
  const long long budget = timeout_cycles > 0 ? (long long)timeout_cycles : 2000000000LL;
  cudaError_t e = vbq::launch_peer_allreduce(data, reinterpret_cast<int* const*>(flags), world, rank, epoch, n,
                                             out, budget, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_peer_allreduce launch");
  return ok();
}

int vbq_ipc_export(const void* ptr, void* handle64, int64_t* offset) {
  if (!ptr || !handle64 || !offset) return fail(VBQ_ERR_NULL, "vbq_ipc_export: NULL pointer");
  cudaError_t e = vbq::ipc_export(ptr, handle64, offset);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_ipc_export");
  return ok();
}

int vbq_ipc_import(const void* handle64, int64_t offset, void** ptr) {
  if (!handle64 || !ptr) return fail(VBQ_ERR_NULL, "vbq_ipc_import: NULL pointer");
  if (offset < 0) return fail(VBQ_ERR_SHAPE, "vbq_ipc_import: negative offset");
  cudaError_t e = vbq::ipc_import(handle64, offset, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_ipc_import");
  return ok();
}

int vbq_ipc_close(void* ptr, int64_t offset) {
  if (!ptr) return fail(VBQ_ERR_NULL, "vbq_ipc_close: NULL pointer");
  cudaError_t e = vbq::ipc_close(ptr, offset);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_ipc_close");
  return ok();
}

}  // extern "C"

// ---------------------------------------------------------------------------------
// GEMV with library-owned scratch, for callers that cannot allocate device memory.
//
// Some hosts of this library own every byte of device memory: a serving engine that
// reserves the whole HBM at start-up for its weight and KV-cache pools and forbids later
// cudaMalloc calls (which can also synchronise the device and stall its other streams),
// or a plugin that only ever receives the host application's buffers.  Such callers have
// nowhere to put vbq_gemv's split-K scratch.  This entry point uses a fixed array in the
// library's own device memory instead; it exists on every GPU that loads the library,
// from load until process exit.
// ---------------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_gemv_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
// device address of the array per device ordinal, and the id of the context it was looked
// up in (a context created anew, e.g. after cudaDeviceReset, gets a new id and a new
// lookup: the old address would point into freed memory)
void* g_static_ptr[64] = {nullptr};
unsigned long long g_static_ctx[64] = {0};

// id of the context current on this thread (0 when none is current yet).  The two driver
// calls come through the runtime's driver entry point, so the library needs no libcuda
// link (it loads on machines without a driver; its calls then fail with a status).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
unsigned long long current_context_id() {
  static const CtxGetCurrentFn get_current = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetCurrentFn>(p) : nullptr;
  }();
  static const CtxGetIdFn get_id = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    return (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetIdFn>(p) : nullptr;
  }();
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id) return 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the array on the current device.  Host code must not pass
// g_gemv_static_scratch itself to a kernel: on the host it names a stand-in, not device
// memory.  The address is looked up once per device and context, with that device current.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv_static_scratch: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(VBQ_ERR_UNSUPPORTED, "vbq_gemv_static_scratch: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_static_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_static_ptr[dev] || ctx == 0 || ctx != g_static_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gemv_static_scratch);  // makes the primary context current
    if (e != cudaSuccess || !p)
      return cuda_fail(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                       "vbq_gemv_static_scratch: cudaGetSymbolAddress");
    g_static_ptr[dev] = p;
    g_static_ctx[dev] = current_context_id();
  }
  *out = g_static_ptr[dev];
  return VBQ_OK;
}

}  // namespace

extern "C" int vbq_gemv_static_scratch(const float* x, const void* w, float* y, int64_t K,
                                       int64_t N, int32_t type, int32_t batch, void* stream) {
  if (int rc = gemv_checks(type, K, N, batch)) return rc;
  if (N == 0) return ok();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    if (!y) return fail(VBQ_ERR_NULL, "vbq_gemv_static_scratch: NULL pointer");
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)batch * (size_t)N * sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv_static_scratch memset");
    return ok();
  }
  if (!x || !w || !y) return fail(VBQ_ERR_NULL, "vbq_gemv_static_scratch: NULL pointer");
  if (!aligned(x, 4) || !aligned(y, 16) || !aligned(w, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_gemv_static_scratch: w and y must be 16-byte aligned, x 4-byte aligned");
  if (K > (int64_t)INT32_MAX || N > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_gemv_static_scratch: sizes above 2^31 are not supported");
  if (gemv_generic(type, N)) {  // the generic kernel needs no scratch
    const int64_t rbg = (N / block_values(type)) * block_bytes(type);
    cudaError_t e = vbq::launch_gemv_any(type, x, w, y, K, N, rbg, batch, st);
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv_static_scratch launch");
    return ok();
  }
  const vbq::GemvPlan plan = gemv_call_plan(K, N, batch, type);
  if (plan.scratch_bytes > kStaticScratchBytes)
    return fail(VBQ_ERR_WORKSPACE,
                "vbq_gemv_static_scratch: this shape needs " + std::to_string(plan.scratch_bytes) +
                    " bytes of scratch, above the library's fixed " +
                    std::to_string(kStaticScratchBytes) +
                    "; use vbq_gemv with caller scratch (or a smaller batch / N)");
  void* scratch = nullptr;
  if (plan.scratch_bytes > 0) {
    if (int rc = static_scratch(&scratch)) return rc;
    // the array keeps the previous call's contents; the tile counters must start at zero
    cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)plan.counter_bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv_static_scratch counter reset");
  }
  const int64_t rb = (N / block_values(type)) * block_bytes(type);
  cudaError_t e = launch_gemv_groups(type, x, w, y, K, N, rb, batch, scratch, st);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemv_static_scratch launch");
  return ok();
}

// ---------------------------------------------------------------------------------
// Grouped GEMM over weight slabs, and the MoE FFN built on it.
// ---------------------------------------------------------------------------------
namespace {

// Shape rules of the tcgen05 GEMM for one K x N weight slab; *rb gets the row bytes.
int gemm_shape_checks(const char* who, int32_t type, int64_t K, int64_t N, int64_t* rb) {
  const std::string w(who);
  if (!quantized(type)) return fail(VBQ_ERR_TYPE, w + ": unsupported type " + std::to_string(type));
  if (K <= 0 || N <= 0) return fail(VBQ_ERR_SHAPE, w + ": K and N must be positive");
  if (N % 256 != 0) return fail(VBQ_ERR_SHAPE, w + ": N must be a multiple of 256");
  if (K % 8 != 0) return fail(VBQ_ERR_SHAPE, w + ": K must be a multiple of 8 (16-byte rows of A)");
  if (K > (int64_t)INT32_MAX || N > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, w + ": sizes above 2^31 are not supported");
  *rb = (N / block_values(type)) * block_bytes(type);
  if (*rb % 16 != 0)
    return fail(VBQ_ERR_UNSUPPORTED, w + ": weight rows must be a multiple of 16 bytes (Q6_K: N % 2048 == 0)");
  return VBQ_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace of vbq_moe_ffn, in order: routing (idx, weight), segments, entry rows, row
// tokens, gathered activations (bf16), gate and up projections (bf16; SwiGLU overwrites
// gate), down projection (fp32).
struct MoeLayout {
  size_t idx, weight, seg, pos, tok, a, g, u, y, total;
};
MoeLayout moe_layout(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  MoeLayout l{};
  const size_t R = (size_t)T * (size_t)k;
  size_t o = 0;
  l.idx = o;    o += align256(R * 4);
  l.weight = o; o += align256(R * 4);
  l.seg = o;    o += align256((size_t)(E + 1) * 4);
  l.pos = o;    o += align256(R * 4);
  l.tok = o;    o += align256(R * 4);
  l.a = o;      o += align256(R * (size_t)H * 2);
  l.g = o;      o += align256(R * (size_t)I * 2);
  l.u = o;      o += align256(R * (size_t)I * 2);
  l.y = o;      o += align256(R * (size_t)H * 4);
  l.total = o;
  return l;
}

}  // namespace

extern "C" {

int vbq_gemm_grouped(const void* a, const void* w, int64_t slab_bytes, void* c, int64_t rows,
                     int64_t K, int64_t N, int32_t type, int32_t c_dtype, const int32_t* seg,
                     int32_t n_seg, void* stream) {
  int64_t rb = 0;
  const int rc = gemm_shape_checks("vbq_gemm_grouped", type, K, N, &rb);
  if (rc != VBQ_OK) return rc;
  if (c_dtype != VBQ_DTYPE_F32 && c_dtype != VBQ_DTYPE_BF16)
    return fail(VBQ_ERR_SHAPE, "vbq_gemm_grouped: c_dtype must be VBQ_DTYPE_F32 or VBQ_DTYPE_BF16");
  if (rows < 0 || n_seg < 0) return fail(VBQ_ERR_SHAPE, "vbq_gemm_grouped: negative size");
  if (rows > (int64_t)INT32_MAX) return fail(VBQ_ERR_SHAPE, "vbq_gemm_grouped: rows above 2^31");
  if (rows == 0 || n_seg == 0) return ok();
  if (!a || !w || !c || !seg) return fail(VBQ_ERR_NULL, "vbq_gemm_grouped: NULL pointer");
  if (slab_bytes < K * rb || slab_bytes % 16 != 0)
    return fail(VBQ_ERR_SHAPE, "vbq_gemm_grouped: slab_bytes must be >= K * row_bytes and a multiple of 16");
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(c, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_gemm_grouped: a, w and c must be 16-byte aligned");
  cudaError_t e = vbq::launch_gemm_grouped(type, a, w, c, rows, K, N, rb, c_dtype, slab_bytes, seg,
                                           n_seg, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_gemm_grouped launch");
  return ok();
}

int vbq_moe_route(const float* logits, int64_t T, int32_t E, int32_t topk, int32_t* idx,
                  float* weight, void* stream) {
  if (T < 0 || E <= 0 || topk < 1 || topk > 8 || topk > E || T > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_moe_route: need T >= 0, 1 <= topk <= min(8, E)");
  if (T == 0) return ok();
  if (!logits || !idx || !weight) return fail(VBQ_ERR_NULL, "vbq_moe_route: NULL pointer");
  cudaError_t e = vbq::launch_moe_route(logits, (int)T, E, topk, idx, weight,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_moe_route launch");
  return ok();
}

int vbq_moe_sort(const int32_t* idx, int64_t T, int32_t E, int32_t topk, int32_t* seg,
                 int32_t* pos, int32_t* tok, void* stream) {
  if (T < 0 || E <= 0 || E > 4096 || topk < 1 || topk > 8 || T * topk > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_moe_sort: need T >= 0, 1 <= E <= 4096, 1 <= topk <= 8");
  if (!idx || !seg || !pos || !tok) return fail(VBQ_ERR_NULL, "vbq_moe_sort: NULL pointer");
  cudaError_t e = vbq::launch_moe_sort(idx, (int)T, E, topk, seg, pos, tok,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_moe_sort launch");
  return ok();
}

int vbq_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int32_t E, int32_t topk,
                            size_t* bytes) {
  if (!bytes) return fail(VBQ_ERR_NULL, "vbq_moe_workspace_bytes: bytes is NULL");
  if (T < 0 || H <= 0 || I <= 0 || E <= 0 || topk < 1 || topk > 8 || topk > E)
    return fail(VBQ_ERR_SHAPE, "vbq_moe_workspace_bytes: bad sizes");
  *bytes = moe_layout(T, H, I, E, topk).total;
  return ok();
}

int vbq_moe_ffn(const float* x, const float* logits, const void* w_gate, const void* w_up,
                const void* w_down, float* out, int64_t T, int64_t H, int64_t I, int32_t E,
                int32_t topk, int32_t type_gate, int32_t type_up, int32_t type_down,
                void* workspace, size_t workspace_bytes, void* stream) {
  int64_t rb_g = 0, rb_u = 0, rb_d = 0;
  int rc = gemm_shape_checks("vbq_moe_ffn (gate)", type_gate, H, I, &rb_g);
  if (rc == VBQ_OK) rc = gemm_shape_checks("vbq_moe_ffn (up)", type_up, H, I, &rb_u);
  if (rc == VBQ_OK) rc = gemm_shape_checks("vbq_moe_ffn (down)", type_down, I, H, &rb_d);
  if (rc != VBQ_OK) return rc;
  if (T < 0 || E <= 0 || E > 4096 || topk < 1 || topk > 8 || topk > E ||
      T * topk > (int64_t)INT32_MAX)
    return fail(VBQ_ERR_SHAPE, "vbq_moe_ffn: need T >= 0, 1 <= E <= 4096, 1 <= topk <= min(8, E)");
  if (T == 0) return ok();
  if (!x || !logits || !w_gate || !w_up || !w_down || !out || !workspace)
    return fail(VBQ_ERR_NULL, "vbq_moe_ffn: NULL pointer");
  const MoeLayout l = moe_layout(T, H, I, E, topk);
  if (workspace_bytes < l.total)
    return fail(VBQ_ERR_WORKSPACE, "vbq_moe_ffn: workspace needs " + std::to_string(l.total) + " bytes");
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(w_gate, 16) || !aligned(w_up, 16) ||
      !aligned(w_down, 16) || !aligned(workspace, 256))
    return fail(VBQ_ERR_ALIGN, "vbq_moe_ffn: x, out, weights 16-byte and workspace 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* idx = reinterpret_cast<int32_t*>(ws + l.idx);
  float* wt = reinterpret_cast<float*>(ws + l.weight);
  int32_t* seg = reinterpret_cast<int32_t*>(ws + l.seg);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + l.pos);
  int32_t* tok = reinterpret_cast<int32_t*>(ws + l.tok);
  const int64_t R = T * topk;
  cudaError_t e = vbq::launch_moe_route(logits, (int)T, E, topk, idx, wt, st);
  if (e == cudaSuccess) e = vbq::launch_moe_sort(idx, (int)T, E, topk, seg, pos, tok, st);
  if (e == cudaSuccess) e = vbq::launch_moe_gather(x, tok, (int)R, (int)H, ws + l.a, st);
  if (type_gate == type_up) {  // gate | up and SwiGLU in one grouped GEMM (the same bits)
    if (e == cudaSuccess)
      e = vbq::launch_gemm_grouped_swiglu(type_gate, ws + l.a, w_gate, w_up, ws + l.g, R, H, I, rb_g,
                                          H * rb_g, seg, E, st);
  } else {
    if (e == cudaSuccess)
      e = vbq::launch_gemm_grouped(type_gate, ws + l.a, w_gate, ws + l.g, R, H, I, rb_g, VBQ_DTYPE_BF16,
                                   H * rb_g, seg, E, st);
    if (e == cudaSuccess)
      e = vbq::launch_gemm_grouped(type_up, ws + l.a, w_up, ws + l.u, R, H, I, rb_u, VBQ_DTYPE_BF16,
                                   H * rb_u, seg, E, st);
    if (e == cudaSuccess) e = vbq::launch_swiglu(ws + l.g, ws + l.u, ws + l.g, R * I, st);
  }
  if (e == cudaSuccess)
    e = vbq::launch_gemm_grouped(type_down, ws + l.g, w_down, ws + l.y, R, I, H, rb_d, VBQ_DTYPE_F32,
                                 I * rb_d, seg, E, st);
  if (e == cudaSuccess)
    e = vbq::launch_moe_combine(reinterpret_cast<const float*>(ws + l.y), pos, wt, (int)T, topk,
                                (int)H, out, st);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_moe_ffn launch");
  return ok();
}

}  // extern "C"

extern "C" int vbq_swiglu(const void* g, const void* u, void* h, int64_t n, int32_t dtype,
                          void* stream) {
  if (dtype != VBQ_DTYPE_F32 && dtype != VBQ_DTYPE_BF16)
    return fail(VBQ_ERR_SHAPE, "vbq_swiglu: dtype must be VBQ_DTYPE_F32 or VBQ_DTYPE_BF16");
  if (n < 0) return fail(VBQ_ERR_SHAPE, "vbq_swiglu: negative size");
  if (n == 0) return ok();
  if (!g || !u || !h) return fail(VBQ_ERR_NULL, "vbq_swiglu: NULL pointer");
  if (n % 8 != 0) return fail(VBQ_ERR_SHAPE, "vbq_swiglu: n must be a multiple of 8");
  if (!aligned(g, 16) || !aligned(u, 16) || !aligned(h, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_swiglu: g, u and h must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = dtype == VBQ_DTYPE_BF16
                      ? vbq::launch_swiglu(g, u, h, n, st)
                      : vbq::launch_swiglu_f32(static_cast<const float*>(g), static_cast<const float*>(u),
                                               static_cast<float*>(h), n, st);
  if (e != cudaSuccess) return cuda_fail(e, "vbq_swiglu launch");
  return ok();
}

extern "C" int vbq_swiglu_rows(const void* gu, void* h, int64_t rows, int64_t n, int32_t dtype,
                               void* stream) {
  if (dtype != VBQ_DTYPE_F32 && dtype != VBQ_DTYPE_BF16)
    return fail(VBQ_ERR_SHAPE, "vbq_swiglu_rows: dtype must be VBQ_DTYPE_F32 or VBQ_DTYPE_BF16");
  if (rows < 0 || n < 0) return fail(VBQ_ERR_SHAPE, "vbq_swiglu_rows: negative size");
  if (rows == 0 || n == 0) return ok();
  if (!gu || !h) return fail(VBQ_ERR_NULL, "vbq_swiglu_rows: NULL pointer");
  if (n % 8 != 0) return fail(VBQ_ERR_SHAPE, "vbq_swiglu_rows: n must be a multiple of 8");
  if (!aligned(gu, 16) || !aligned(h, 16))
    return fail(VBQ_ERR_ALIGN, "vbq_swiglu_rows: gu and h must be 16-byte aligned");
  cudaError_t e = vbq::launch_swiglu_rows(gu, h, rows, n, dtype == VBQ_DTYPE_BF16,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "vbq_swiglu_rows launch");
  return ok();
}
