// vbq_internal.h -- launchers shared between the kernel files and the C-ABI layer.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace vbq {

// One-time per-device set-up of a kernel's launch attributes.  Each launcher keeps one
// of these (a function-local static): `done(dev)` tells whether device `dev` is set up,
// `mark(dev)` records it.  The flag word is atomic, so first calls from several host
// threads never race on it; at worst two of them both run the set-up, which only sets
// the same attributes twice.  Devices past 63 are set up on every call.
struct DeviceOnce {
  std::atomic<uint64_t> bits{0};
  bool done(int dev) const {
    return dev < 64 && (bits.load(std::memory_order_acquire) >> dev & 1u);
  }
  void mark(int dev) {
    if (dev < 64) bits.fetch_or(uint64_t(1) << dev, std::memory_order_acq_rel);
  }
};

// A per-device int a launcher computes once (resident CTAs per SM, say): set before the
// launcher's DeviceOnce mark, read after its done() check, so a reader that sees the mark
// sees the value.  Devices past 63 read 1.
struct DeviceSlots {
  std::atomic<int> v[64] = {};
  void set(int dev, int x) {
    if (dev < 64) v[dev].store(x, std::memory_order_release);
  }
  int get(int dev) const {
    const int x = dev < 64 ? v[dev].load(std::memory_order_acquire) : 1;
    return x > 0 ? x : 1;
  }
};

cudaError_t launch_dequant(int qtype, const void* w, void* out, int64_t rows, int64_t n,
                           int64_t row_bytes, int out_dtype, cudaStream_t st);

// Optional fusions of a GEMV call (vbq_gemv_ex): the input as SwiGLU of a packed gate | up
// buffer [batch, 2K] (x then points there), and a bias [N] and a residual [batch, N] added
// to the output (the residual may be y itself).
struct GemvFuse {
  bool swiglu_x = false;
  const float* bias = nullptr;
  const float* res = nullptr;
};

// Split-K plan of the fused dequant-GEMV for the current device.
struct GemvPlan {
  int splits;            // CTAs per 256-column tile along K
  int64_t kslice;        // rows per CTA
  int64_t counter_bytes; // scratch prefix holding one counter per tile (0 when splits == 1)
  size_t scratch_bytes;  // counters + splits * batch * N fp32 partial sums
};
// `qtype` selects the kernel: the tensor-core Q4_K kernel (batch 1..4) reduces its K-splits
// inside a thread-block cluster and needs no scratch.
GemvPlan plan_gemv(int64_t K, int64_t N, int batch, int qtype);
int sm_count();
int gemv_split_override();  // VBQ_GEMV_SPLIT (tuning), 0 when unset

// Fused dequant-GEMV; batch in 1..16.  `scratch` must hold plan.scratch_bytes with its
// counter prefix zero (the kernel leaves it zero).  Returns cudaErrorNotSupported for
// shapes the kernels do not cover (the C-ABI layer checks shapes first).
cudaError_t launch_gemv(int qtype, const float* x, const void* w, float* y, int64_t K,
                        int64_t N, int64_t row_bytes, int batch, const GemvPlan& plan,
                        void* scratch, cudaStream_t st, const GemvFuse& f = GemvFuse{});

// Generic GEMV (vbq_gemv_any.cu): any type the library reads, any N that is a multiple of
// the block, any batch (groups of 4 rows on the grid), optional bias [N] and residual
// [batch, N] added to the output; no scratch.  The reference dispatcher's other block types
// (Q4_0 .. Q8_K) go to the staged kernel (vbq_gemv_stage.cu) when it takes the shape.
cudaError_t launch_gemv_any(int qtype, const float* x, const void* w, float* y, int64_t K,
                            int64_t N, int64_t row_bytes, int batch, cudaStream_t st,
                            const GemvFuse& f = GemvFuse{});

// Q4_0 / Q4_1 / Q5_0 / Q5_1 on the Q8_0 integer tensor-core kernel (vbq_gemv_q8.cu), batch
// 1..16 as groups of 4, when gemv_q8_fits() and the rows are whole 16-byte granules.
cudaError_t launch_gemv_q4x_mma(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f);

// Q5_K on the Q4_K integer tensor-core kernel (vbq_gemv_mma.cu), batch 1..16 as groups of 4,
// when gemv_mma_fits() and the rows are whole 16-byte granules.
cudaError_t launch_gemv_mma_q5k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f);

// Staged GEMV for Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, Q8_K (vbq_gemv_stage.cu): takes
// N a multiple of its column unit (256, or 512 for Q3_K), 4-byte-aligned rows, a 16-byte
// aligned w and K * row_bytes a multiple of 16.
bool gemv_stage_takes(int qtype, int64_t K, int64_t N, int64_t row_bytes, const void* w);
cudaError_t launch_gemv_stage(int qtype, const float* x, const void* w, float* y, int64_t K, int64_t N,
                              int64_t row_bytes, int batch, cudaStream_t st, const GemvFuse& f);

// Tensor-core (integer mma.sync) Q4_K GEMV, batch 1..16, when gemv_mma_fits(); the K-splits
// of a tile form one thread-block cluster and add up in the leader's shared memory.
bool gemv_mma_fits(int64_t K, int64_t N, int batch);
// Tensor-core Q8_0 GEMV (vbq_gemv_q8.cu), batch 1..16 (groups of 4 above 4), no scratch.
bool gemv_q8_fits(int64_t K, int64_t N, int batch);
cudaError_t launch_gemv_q8_mma(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t row_bytes, int batch, cudaStream_t st,
                               const GemvFuse& f = GemvFuse{});
cudaError_t gemv_q8_status(unsigned* out, bool clear);
// Tensor-core Q6_K GEMV (vbq_gemv_q6.cu), batch 1, no scratch; w 16-byte aligned and
// row_bytes the natural N / 256 * 210.
bool gemv_q6_fits(int64_t K, int64_t N, int batch);
cudaError_t launch_gemv_q6_mma(const float* x, const void* w, float* y, int64_t K, int64_t N,
                               int64_t row_bytes, int batch, cudaStream_t st,
                               const GemvFuse& f = GemvFuse{});
cudaError_t gemv_q6_status(unsigned* out, bool clear);
// Batch 5..16 kernel (vbq_gemv_wide.cu): x read by TMA, so rows of x 16-byte aligned.
bool gemv_wide_fits(const float* x, int64_t K, int64_t N, int batch);
cudaError_t launch_gemv_wide_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t row_bytes, int batch, cudaStream_t st,
                                 const GemvFuse& f = GemvFuse{});
cudaError_t gemv_wide_status(unsigned* out, bool clear);
// Batch 5..16 Q4_K kernel on the fp16 tensor cores (vbq_gemv_half.cu): x read by TMA (rows
// of x 16-byte aligned, K % 4 == 0); a SwiGLU input is read as its gate | up halves.
bool gemv_half_fits(const float* x, int64_t K, int64_t N, int batch);
cudaError_t launch_gemv_half_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                 int64_t row_bytes, int batch, cudaStream_t st,
                                 const GemvFuse& f = GemvFuse{});
cudaError_t gemv_half_status(unsigned* out, bool clear);
cudaError_t launch_gemv_mma_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, cudaStream_t st,
                                const GemvFuse& f = GemvFuse{});

// Optional epilogue of the GEMM: bias fp32 [N] and a residual [M, N] of c's element type
// (it may be c itself) added to the fp32 accumulator before the store.
struct GemmEpi {
  const float* bias = nullptr;
  const void* res = nullptr;
};

// tcgen05 dequant-GEMM: a bf16 [M,K], W K x N blocks, c fp32 (c_dtype 0) / bf16 (1) [M,N].
cudaError_t launch_gemm(int qtype, const void* a, const void* w, void* c, int64_t M, int64_t K,
                        int64_t N, int64_t row_bytes, int c_dtype, cudaStream_t st,
                        const GemmEpi& ep = GemmEpi{});
// Grouped form: rows of A / C split by the device array seg[0..n_seg] into segments,
// segment s multiplied by the K x N slab at w + s * slab_bytes.
cudaError_t launch_gemm_grouped(int qtype, const void* a, const void* w, void* c, int64_t rows,
                                int64_t K, int64_t N, int64_t row_bytes, int c_dtype,
                                int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st);
// The gate | up GEMM fused with SwiGLU: h bf16 [M, I] = silu(a W_gate) * (a W_up), both
// weights K x I with row stride row_bytes (same type); the grouped form takes slabs as
// launch_gemm_grouped.  The result has the bits of the two GEMMs (bf16 out) followed by
// launch_swiglu.
cudaError_t launch_gemm_swiglu(int qtype, const void* a, const void* w_gate, const void* w_up, void* h,
                               int64_t M, int64_t K, int64_t I, int64_t row_bytes, cudaStream_t st);
cudaError_t launch_gemm_grouped_swiglu(int qtype, const void* a, const void* w_gate, const void* w_up,
                                       void* h, int64_t rows, int64_t K, int64_t I, int64_t row_bytes,
                                       int64_t slab_bytes, const int* seg, int n_seg, cudaStream_t st);
cudaError_t gemm_status(unsigned* out, bool clear);

// MoE pieces (vbq_moe.cu).  Routing of T tokens over E experts from fp32 logits [T, E]:
// softmax (logits clipped to +-50), top-k (ties to the lower index), renormalised.
cudaError_t launch_moe_route(const float* logits, int T, int E, int topk, int32_t* idx,
                             float* weight, cudaStream_t st);
// Stable counting sort of the T*topk (token, slot) entries by expert: seg[E + 1] segment
// offsets, pos[T*topk] the sorted row of each entry, tok[T*topk] the token of each row.
cudaError_t launch_moe_sort(const int32_t* idx, int T, int E, int topk, int32_t* seg,
                            int32_t* pos, int32_t* tok, cudaStream_t st);
// a_perm[row] = bf16(x[tok[row]]), x fp32 [T, H]
cudaError_t launch_moe_gather(const float* x, const int32_t* tok, int rows, int H, void* a_perm,
                              cudaStream_t st);
// h = bf16(silu(g) * u) over n bf16 values, with the reference's clipping (in place in g ok)
cudaError_t launch_swiglu(const void* g, const void* u, void* h, int64_t n, cudaStream_t st);
cudaError_t launch_swiglu_f32(const float* g, const float* u, float* h, int64_t n, cudaStream_t st);
cudaError_t launch_swiglu_rows(const void* gu, void* h, int64_t rows, int64_t n, bool bf16,
                               cudaStream_t st);
// out[t] = sum_slot weight[t, slot] * y[pos[t * topk + slot]], fp32 [T, H], sanitised
cudaError_t launch_moe_combine(const float* y, const int32_t* pos, const float* weight, int T,
                               int topk, int H, float* out, cudaStream_t st);

cudaError_t gemv_mma_status(unsigned* out, bool clear);
// One warp waiting on an mbarrier with the GEMV's bounded wait (vbq_debug_wait_probe).
cudaError_t launch_wait_probe(long long budget_cycles, int arrive, cudaStream_t st);

// One-shot all-reduce over peer memory (vbq_peer.cu): out = sum over p of data[p][0 .. n),
// after publishing `epoch` to every peer's flags[rank] and waiting (bounded) for theirs.
cudaError_t launch_peer_allreduce(const float* const* data, int* const* flags, int world, int rank,
                                  int epoch, int64_t n, float* out, long long budget_cycles,
                                  cudaStream_t st);
cudaError_t peer_status(unsigned* out, bool clear);
// CUDA IPC of a buffer that may sit inside a larger allocation (64-byte handle + offset).
cudaError_t ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
cudaError_t ipc_import(const void* handle, int64_t offset, void** ptr_out);
cudaError_t ipc_close(void* ptr, int64_t offset);

// Sticky device status bits of the GEMV kernels (kStatusTimeout = 1); synchronous.
cudaError_t gemv_status(unsigned* out, bool clear);

}  // namespace vbq
