/*
 * vbq.h -- C ABI of the B200 (sm_100a) GGUF k-quant dequantize-and-multiply library.
 *
 * The library is the device-side replacement for VibeBlade's quantized matmul path
 * (kevin046/VibeBlade, cpp/src/dequant.cpp and cpp/include/dequant.h).  Every entry
 * point takes plain device pointers, sizes and a CUDA stream (as `void*`, NULL = the
 * legacy default stream), enqueues its work on that stream and returns without
 * synchronising.  No entry point allocates device memory.
 *
 * Matrix convention (the reference's, cpp/include/dequant.h:24-35): a weight matrix
 * is K rows of N values; each row is a run of quant blocks along N, rows are
 * vbq_row_bytes(type, N) bytes apart, and gemv computes y[n] = sum_k x[k] * W[k][n].
 *
 * Type ids are the reference's ggml_type values (cpp/include/ggml_types.h:11-27).
 *
 * Dequantized values are bit-identical to the reference CPU functions
 * (dequantize_row_q4_K / _q6_K, cpp/src/dequant.cpp:268-301, :359-402), including
 * their fp16 conversion (cpp/src/fp16_compat.cpp:13-35).  Q8_0 uses the GGUF block
 * with an fp16 scale, like the reference's CUDA kernel (cpp/src/cuda_kernels.cu:718-735).
 *
 * Return value: VBQ_OK (0) or one of the VBQ_ERR_* codes; vbq_last_error() returns
 * the message of the last failure on the calling thread.
 */
#ifndef VBQ_H
#define VBQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (cpp/include/ggml_types.h:11-27).  Q4_K, Q6_K and Q8_0 are the path's
 * quantized types (every entry point); the unquantized ones are read by vbq_dequantize and
 * vbq_gemv (GGUF files keep small tensors such as the MoE router, ffn_gate_inp,
 * unquantized), and so are the reference dispatcher's other block types (Q4_0, Q4_1, Q5_0,
 * Q5_1, Q2_K, Q3_K, Q5_K, Q8_K: cpp/src/dequant.cpp:412-422), each in the reference's own
 * reading of its block.  Q8_1 (9) is not read, as in the reference. */
#define VBQ_TYPE_F32 0
#define VBQ_TYPE_F16 1
#define VBQ_TYPE_Q4_0 2
#define VBQ_TYPE_Q4_1 3
#define VBQ_TYPE_Q5_0 6
#define VBQ_TYPE_Q5_1 7
#define VBQ_TYPE_Q8_0 8
#define VBQ_TYPE_Q2_K 10
#define VBQ_TYPE_Q3_K 11
#define VBQ_TYPE_Q4_K 12
#define VBQ_TYPE_Q5_K 13
#define VBQ_TYPE_Q6_K 14
#define VBQ_TYPE_Q8_K 15
#define VBQ_TYPE_BF16 30

/* element types of outputs / activations */
#define VBQ_DTYPE_F32 0
#define VBQ_DTYPE_BF16 1

/* status codes */
#define VBQ_OK 0
#define VBQ_ERR_TYPE 1        /* unsupported ggml type (reference: "Unsupported dequant type") */
#define VBQ_ERR_SHAPE 2       /* bad sizes: N not a block multiple, batch out of range, ... */
#define VBQ_ERR_ALIGN 3       /* a pointer or stride breaks an alignment rule */
#define VBQ_ERR_NULL 4        /* a required pointer is NULL */
#define VBQ_ERR_CUDA 5        /* a CUDA runtime call or kernel launch failed */
#define VBQ_ERR_TIMEOUT 6     /* a bounded device-side wait gave up (see vbq_gemm) */
#define VBQ_ERR_UNSUPPORTED 7 /* a valid request this build does not implement */
#define VBQ_ERR_WORKSPACE 8   /* workspace missing or too small */
#define VBQ_ERR_FORMAT 9      /* a GGUF file is malformed (vbq_gguf.h; the reference's messages) */
#define VBQ_ERR_IO 10         /* a file cannot be opened, read or mapped */
#define VBQ_ERR_NOT_FOUND 11  /* no GGUF metadata key of the asked kind */

/* Message of the last failing call on this thread ("" after success). */
const char* vbq_last_error(void);

/* Library version, as major*10000 + minor*100 + patch. */
int vbq_version(void);

/* Row stride in bytes of a K x N matrix of `type`: (N / block_values) * block_bytes,
 * truncating like gemv_dequant (cpp/src/dequant.cpp:749-763).  Host-only helper. */
int vbq_row_bytes(int32_t type, int64_t n, int64_t* out_bytes);

/*
 * Dequantize a K x N matrix (K rows of vbq_row_bytes(type, N) bytes) into fp32 or
 * bf16 [K, N], row-major.  With rows == 1 it is the device form of
 * `void dequantize_row(const void* row, float* out, int64_t n, ggml_type)`
 * (cpp/include/dequant.h:11); then n may be ragged (not a block multiple) and only n
 * values are written.  For rows > 1, n must be a multiple of the block size.
 * bf16 output rounds the fp32 dequantized value to nearest-even.  Every type the
 * reference's dispatcher takes is read, with its reading of each block (among them its
 * Q2_K adding dmin without a sub-block min, Q3_K high bits from hmask[0..15] only, Q5_K
 * fifth bits from 32 bytes further on per 64-value chunk, Q8_K's interleaved 33-byte
 * sub-blocks: cpp/src/dequant.cpp:128-245, :317-354).
 */
int vbq_dequantize(const void* w, void* out, int64_t rows, int64_t n, int32_t type,
                   int32_t out_dtype, void* stream);

/*
 * Scratch bytes vbq_gemv needs for this shape on the current device (0 when the call
 * needs none).  The reference's gemv_dequant also takes caller-owned scratch
 * (cpp/include/dequant.h:34); here it holds the split-K partial sums.
 */
int vbq_gemv_scratch_bytes(int64_t K, int64_t N, int32_t type, int32_t batch, size_t* bytes);

/*
 * Batched fused dequant-GEMV, the device form of
 * `void gemv_dequant(const float* x, const void* W, float* out, int64_t K, int64_t N,
 *                    ggml_type, float* scratch)` (cpp/include/dequant.h:27-35) and of
 * `cuda::gemv_dequant(d_x, d_weights, d_y, K, M, ggml_type, d_scratch, stream)`
 * (cpp/include/cuda_kernels.h:191-199):
 *     y[b, n] = sum_k x[b, k] * deq(W)[k, n],  b < batch (1..32 on the tiled kernels, above
 *     16 as consecutive launches over groups of up to 16 batch rows; any batch up to
 *     262140 on the generic kernel below, e.g. a prefill's tokens through the MoE router).
 * x is fp32 [batch, K], y fp32 [batch, N], both row-major.  N must be a multiple of
 * the block size (256 for the K-quants, 32 for Q4_0/Q4_1/Q5_0/Q5_1/Q8_0, 1 for
 * F32/F16/BF16); widths that are whole 256-column tiles of Q4_K, Q6_K or Q8_0 run on the
 * tiled kernels, as do batches up to 16 of Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q5_K (no scratch);
 * the rest (the MoE router's N = n_experts, unquantized weights, the other block types) on
 * generic and staged kernels without scratch.
 * W and y must be 16-byte aligned, x 4-byte aligned.  F16 weights are read through the
 * reference's f16_to_f32 (fp16 subnormals doubled), BF16 as the top half of an fp32.
 * scratch: caller-owned device memory of at least vbq_gemv_scratch_bytes(); it must be
 * zero-filled before its first use, every call leaves it zero-filled again, and two
 * calls that may run at the same time must not share it.  NULL is allowed when the
 * size is 0.  Results are deterministic (the split-K partials are added in a fixed
 * order).
 */
int vbq_gemv(const float* x, const void* w, float* y, int64_t K, int64_t N, int32_t type,
             int32_t batch, void* scratch, size_t scratch_bytes, void* stream);

/*
 * vbq_gemv with the FFN's element-wise steps fused in (no counterpart call in the
 * reference, which runs them as separate loops around its gemv_dequant calls):
 *   * flags & VBQ_GEMV_X_SWIGLU: x points at a [batch, 2K] buffer holding the output of a
 *     gate | up matmul (gate values in columns 0..K-1, up in K..2K-1), and the GEMV's input
 *     is x'[b, k] = silu(gate[b, k]) * up[b, k], computed where the kernel reads it, with
 *     vbq_swiglu's sanitising and arithmetic (cpp/src/fast_model.cpp:946-953) -- the down
 *     projection without a SwiGLU pass of its own;
 *   * bias (fp32 [N], may be NULL) is added to every output row (the Q/K/V biases,
 *     cpp/src/fast_model.cpp:659-668);
 *   * residual (fp32 [batch, N], may be NULL) is added as well (the residual adds after o
 *     and down, :813-824, :990-998); it may be y itself, but must not overlap y otherwise.
 * Same shapes, scratch and results as vbq_gemv otherwise (K >= 1 when an addend is given).
 * Q4_K batches above 4 with the SwiGLU input run as groups of 4 rows.
 */
#define VBQ_GEMV_X_SWIGLU 1
int vbq_gemv_ex(const float* x, const void* w, float* y, int64_t K, int64_t N, int32_t type,
                int32_t batch, int32_t flags, const float* bias, const float* residual,
                void* scratch, size_t scratch_bytes, void* stream);

/*
 * Quantized-weight GEMM on the tcgen05 tensor cores (prefill):
 *     C[m, n] = sum_k A[m, k] * deq(W)[k, n]
 * A is bf16 [M, K] row-major, C fp32 (VBQ_DTYPE_F32) or bf16 (VBQ_DTYPE_BF16) [M, N]
 * row-major, W the K x N block layout above.  Weight tiles are dequantized to bf16 in
 * shared memory (values rounded to nearest-even from the reference's fp32 values) and
 * multiplied with fp32 accumulation in tensor memory.  The reference has no batched GEMM;
 * its engine makes one gemv_dequant call per token (cpp/src/fast_model.cpp:645-660),
 * which this replaces.  Requirements: N % 256 == 0, K % 8 == 0, weight rows a multiple of
 * 16 bytes (Q6_K: N % 2048 == 0), A, W, C 16-byte aligned.  No workspace.  A device-side
 * wait that gives up is reported by vbq_device_status (outputs then undefined).
 */
int vbq_gemm(const void* a, const void* w, void* c, int64_t M, int64_t K, int64_t N,
             int32_t type, int32_t c_dtype, void* stream);

/*
 * vbq_gemm with the adds that follow the reference's matmuls fused into the epilogue (no
 * counterpart call in the reference): bias (fp32 [N], 16-byte aligned, may be NULL) is
 * added to every row, the Q/K/V biases (cpp/src/fast_model.cpp:659-668); residual ([M, N]
 * of c's element type, 16-byte aligned, may be NULL, may be c itself but must not overlap
 * it otherwise) is added too, the residual adds after o and down (:813-824, :990-998).
 * The sums are formed in fp32 on the accumulator and rounded once to c's type.
 */
int vbq_gemm_ex(const void* a, const void* w, void* c, int64_t M, int64_t K, int64_t N,
                int32_t type, int32_t c_dtype, const float* bias, const void* residual,
                void* stream);

/*
 * The gate | up GEMM fused with SwiGLU (prefill):
 *     h[m, j] = silu(sum_k A[m, k] deq(W_gate)[k, j]) * (sum_k A[m, k] deq(W_up)[k, j])
 * (cpp/src/fast_model.cpp:906-953: gate and up projections, then silu(gate) * up).  A bf16
 * [M, K]; W_gate and W_up K x I matrices of one type (Q4_K, Q6_K, Q8_0) whose rows are
 * row_bytes apart (0: (I / block_values) * block_bytes; a gate | up matrix packed side by
 * side passes its own row stride and w_up = w_gate + the gate part's bytes); h bf16 [M, I].
 * The result has the bits of two vbq_gemm calls with bf16 output followed by
 * vbq_swiglu, without the [M, 2I] intermediate.  I % 256 == 0, K % 8 == 0, pointers
 * 16-byte aligned, row_bytes a multiple of 16.
 */
int vbq_gemm_swiglu(const void* a, const void* w_gate, const void* w_up, void* h, int64_t M, int64_t K,
                    int64_t I, int32_t type, int64_t row_bytes, void* stream);

/*
 * vbq_gemv with library-owned scratch, for callers that cannot allocate device memory --
 * for example an engine that reserves all of HBM for its own pools at start-up and allows
 * no later cudaMalloc (which may also synchronise the device), or a plugin that only gets
 * the host application's buffers.  This entry point has no counterpart in the reference.
 *
 * Same arguments and results as vbq_gemv, without the scratch pair.  The split-K scratch
 * is a fixed 8 MiB array in the library's device memory (present on every GPU that loads
 * the library until the process exits); shapes whose scratch would exceed it return
 * VBQ_ERR_WORKSPACE.  The call allocates nothing.  Its first call on a device looks up
 * the array's device address once (cudaGetSymbolAddress, with that device current); make
 * that first call before any stream capture.  The address belongs to the device's current
 * context: after cudaDeviceReset (or any new primary context) the next call looks it up
 * again, so make that call before a capture as well.  Every call on a device shares the array
 * and the array keeps the previous call's contents (the call zeroes the part that must
 * start at zero), so calls that may overlap on the GPU -- different streams, or graphs
 * replayed concurrently -- race and must be serialised by the caller.
 */
int vbq_gemv_static_scratch(const float* x, const void* w, float* y, int64_t K, int64_t N,
                            int32_t type, int32_t batch, void* stream);

/*
 * Grouped quantized-weight GEMM over weight slabs (the MoE expert GEMM; the reference's
 * slab loop is cpp/src/fast_model.cpp:844-903, vibeblade/moe.py:458-470).  The rows of A
 * (bf16 [rows, K]) and C ([rows, N], c_dtype as vbq_gemm) are split into n_seg
 * consecutive segments by seg (DEVICE int32 [n_seg + 1], nondecreasing, seg[n_seg] <=
 * rows); segment s is multiplied by the K x N slab at w + s * slab_bytes.  slab_bytes is
 * the per-expert stride, normally tensor_nbytes(type, K, N) = K * row_bytes, a multiple
 * of 16 (the reference's own stride, ggml_type_size per element at :852-854, is not
 * used).  Rows outside every segment are left untouched.  Same shape rules as vbq_gemm.
 * The segments are read on the device, so the call never synchronises.
 */
int vbq_gemm_grouped(const void* a, const void* w, int64_t slab_bytes, void* c, int64_t rows,
                     int64_t K, int64_t N, int32_t type, int32_t c_dtype, const int32_t* seg,
                     int32_t n_seg, void* stream);

/*
 * MoE routing (vibeblade/moe.py:170-206, ExpertRouter.route after its matmul; C++:
 * softmax + top_k_select, cpp/src/fast_model.cpp:534-549, :861-872): for each of T tokens,
 * softmax over the E logits (fp32 [T, E], clipped to +-50), the topk largest
 * probabilities in descending order (ties to the lower expert index; the reference leaves
 * the order of equal values unspecified), renormalised to sum 1.  idx int32 [T, topk],
 * weight fp32 [T, topk], all device memory.  topk <= 8.
 */
int vbq_moe_route(const float* logits, int64_t T, int32_t E, int32_t topk, int32_t* idx,
                  float* weight, void* stream);

/*
 * The MoE dispatch's grouping of (token, slot) entries by expert (the reference sends each
 * slot's tokens to their experts one slot at a time, vibeblade/moe.py:462-475; here one
 * stable counting sort on the device): idx int32 [T, topk] is the expert of each entry
 * (entries outside 0..E-1 are skipped); seg int32 [E + 1] receives the row ranges (expert
 * e owns rows seg[e] .. seg[e + 1] - 1), pos int32 [T * topk] the row of entry j (-1 when
 * skipped) and tok int32 [T * topk] the token of each row (j / topk).  Within an expert,
 * rows follow entry order.  All device memory; E <= 4096.
 */
int vbq_moe_sort(const int32_t* idx, int64_t T, int32_t E, int32_t topk, int32_t* seg,
                 int32_t* pos, int32_t* tok, void* stream);

/* Workspace bytes vbq_moe_ffn needs for these sizes. */
int vbq_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int32_t E, int32_t topk,
                            size_t* bytes);

/*
 * MoE SwiGLU FFN (vibeblade/moe.py:407-505 moe_ffn_silu without a shared expert):
 *     out[t] = sum over the token's topk experts e of
 *              weight[t, e] * down_e( silu(gate_e x[t]) * up_e x[t] )
 * x fp32 [T, H], logits fp32 [T, E] (router output), out fp32 [T, H].  w_gate / w_up hold
 * E slabs of H x I weights, w_down E slabs of I x H, each in the block layout above and
 * packed back to back (slab stride = tensor_nbytes).  The gate and up projections are
 * clipped to +-65504 (NaN to 0) before SwiGLU and the output is sanitised the same way,
 * as the reference does.  Activations enter the tensor cores as bf16 (x, and the SwiGLU
 * product), accumulation is fp32.  workspace: device memory of vbq_moe_workspace_bytes(),
 * 256-byte aligned; it needs no initialisation.  Shape rules: I and H multiples of 256
 * (and of 2048 for Q6_K), E <= 4096, topk <= 8.
 */
int vbq_moe_ffn(const float* x, const float* logits, const void* w_gate, const void* w_up,
                const void* w_down, float* out, int64_t T, int64_t H, int64_t I, int32_t E,
                int32_t topk, int32_t type_gate, int32_t type_up, int32_t type_down,
                void* workspace, size_t workspace_bytes, void* stream);

/*
 * SwiGLU of the FFN (cpp/src/fast_model.cpp:946-953, vibeblade/moe.py:36-50, :472-474):
 *     h[i] = silu(g[i]) * u[i],  silu(x) = x * sigmoid(x),
 * with g and u first sanitised as the reference's MoE path does (NaN -> 0, clip to
 * +-65504).  n values of dtype VBQ_DTYPE_F32 or VBQ_DTYPE_BF16 (computed in fp32, bf16
 * output rounded to nearest-even); n % 8 == 0; h may alias g.
 */
int vbq_swiglu(const void* g, const void* u, void* h, int64_t n, int32_t dtype, void* stream);

/*
 * SwiGLU over the output of one matmul whose weight columns hold the gate and up
 * projections side by side (a tensor-parallel rank's gate and up shards packed into one
 * K x 2n block matrix, so that one GEMM / GEMV computes both): gu is [rows, 2n] (gate
 * values in columns 0..n-1, up values in n..2n-1), h is [rows, n], h[r, i] =
 * silu(gu[r, i]) * gu[r, n + i] with the same sanitising and rounding as vbq_swiglu.
 * n % 8 == 0; gu and h 16-byte aligned; h must not overlap gu.
 */
int vbq_swiglu_rows(const void* gu, void* h, int64_t rows, int64_t n, int32_t dtype,
                    void* stream);

/*
 * Device-side status of the library's kernels on the current device: bit 0 set means a
 * bounded wait inside a kernel gave up (VBQ_ERR_TIMEOUT is returned then), which leaves
 * that call's outputs undefined and its scratch in need of re-zeroing.  Reads
 * synchronously; `clear` resets the bits.  The reference has no counterpart (its CUDA
 * path throws on the host, cpp/src/cuda_kernels.cu:24-40).
 */
int vbq_device_status(int32_t* status, int32_t clear);

/*
 * Diagnostic of the failure report above (no counterpart in the reference): launches one
 * warp that waits on a shared-memory mbarrier with the same bounded wait the GEMV kernels
 * use.  arrive = 1: the warp completes the barrier's phase itself and the wait succeeds.
 * arrive = 0: nothing arrives, the wait gives up after budget_cycles SM clock cycles
 * (1 .. 2^31, about 1 s at most) and records the timeout bit that vbq_device_status then
 * reports as VBQ_ERR_TIMEOUT.  The kernel always returns; the context stays usable.
 */
int vbq_debug_wait_probe(int64_t budget_cycles, int32_t arrive, void* stream);

/*
 * One-shot all-reduce of fp32 partial outputs over peer memory, for the row-split layers
 * of tensor parallelism at decode (replaces the collective after the o and down GEMVs of a
 * split layer; the reference runs those layers whole on one device,
 * cpp/src/fast_model.cpp:813-824, :990-998).  One process per GPU; every rank calls it
 * with the same epoch and n.
 *   data[p]  (host array of `world` device pointers): rank p's partial of this call, n
 *            floats, 16-byte aligned, readable from this device (CUDA IPC); data[rank] is
 *            this rank's own, written by the work queued before on `stream`.
 *   flags[p] (host array): rank p's flag array of 8 int32 (zero-filled once at set-up),
 *            writable from this device; slot q holds the last epoch rank q published.
 *   epoch:   1, 2, 3, ... per call; a rank's partials alternate between two buffers by
 *            the epoch's parity (a buffer is rewritten only two calls later).
 *   out:     n floats (16-byte aligned), the sum over p = 0 .. world - 1 in that order,
 *            the same bits on every rank.
 * The wait for the peers is bounded by timeout_cycles SM clock cycles (<= 0: about 1 s);
 * a wait that gives up is reported by vbq_device_status as VBQ_ERR_TIMEOUT and `out` is
 * then not the sum.  No multicast; world <= 8.
 */
int vbq_peer_allreduce(const float* const* data, int32_t* const* flags, int32_t world, int32_t rank,
                       int32_t epoch, int64_t n, float* out, int64_t timeout_cycles, void* stream);

/*
 * CUDA IPC of a device buffer for vbq_peer_allreduce's set-up (no counterpart in the
 * reference).  vbq_ipc_export writes the 64-byte handle of the allocation holding ptr and
 * ptr's offset in it (the buffer may sit inside a caching allocator's block);
 * vbq_ipc_import, in another process, maps that allocation for the current device (peer
 * access enabled on first use) and returns the buffer's address there; vbq_ipc_close
 * unmaps it (same ptr and offset).  None of them allocates device memory.
 */
int vbq_ipc_export(const void* ptr, void* handle64, int64_t* offset);
int vbq_ipc_import(const void* handle64, int64_t offset, void** ptr);
int vbq_ipc_close(void* ptr, int64_t offset);

#ifdef __cplusplus
}
#endif
#endif /* VBQ_H */
