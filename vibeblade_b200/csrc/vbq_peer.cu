// vbq_peer.cu -- one-shot all-reduce of fp32 partial outputs over NVLink peer memory.
//
// The decode step of a row-split layer (tensor parallelism: o and down split by rows,
// cpp/src/fast_model.cpp:813-824 and :990-998 run them whole on one device) leaves each
// rank with a partial y of a few KB to a few hundred KB, to be summed over the ranks.  A
// general collective library pays several microseconds of latency for that; here each
// rank's GEMV writes its partial straight into a buffer every peer can read (CUDA IPC,
// one process per GPU), and one small kernel per rank
//   1. publishes "my partial of call `epoch` is ready" by a system-scope release store of
//      `epoch` into slot `rank` of every peer's flag array,
//   2. waits (bounded) until every peer has published the same epoch in its own flags
//      (acquire loads),
//   3. sums the W partials in rank order (0, 1, ..., W - 1), reading the peers' buffers
//      over NVLink, so every rank computes the same bits.
// The data buffers are double-buffered by the epoch's parity: a rank writes call e + 1's
// partial into the slot its peers read for call e - 1, which they finished before they
// published call e (stream order on every rank), so no slot is overwritten while it is
// read.  Flags only grow (>= test).  The kernel issues no multicast and no TMA; every
// wait is bounded, and a wait that gives up raises kStatusTimeout in this file's status
// word and returns (the output is then not the sum).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {

__device__ unsigned g_peer_status = 0;

namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 512;

struct PeerArgs {
  const float* data[kMaxRanks];  // rank p's partial of this call (its slot for the epoch)
  int* flags[kMaxRanks];         // rank p's flag array: [kMaxRanks] ints, slot q written by rank q
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid: CTAs over slices of n; every CTA waits for the flags itself (no inter-CTA sync)
__global__ void __launch_bounds__(kThreads)
peer_allreduce_kernel(const __grid_constant__ PeerArgs a, int world, int rank, int epoch, int64_t n,
                      float* __restrict__ out, long long budget) {
  // the previous kernel on this stream (the GEMV writing this rank's partial) has finished
  // and its writes are visible once the dependency resolves
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (blockIdx.x == 0 && threadIdx.x < world) {
    // publish: every prior write of this device is ordered before the release (cumulative)
    __threadfence_system();
    st_release_sys(a.flags[threadIdx.x] + rank, epoch);
  }
  __shared__ int ok_all;
  if (threadIdx.x == 0) ok_all = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    const int* f = a.flags[rank] + threadIdx.x;
    bool ok = ld_acquire_sys(f) >= epoch;
    if (!ok) {
      const long long t0 = clock64();
      while (!(ok = ld_acquire_sys(f) >= epoch)) {
        if (clock64() - t0 > budget) break;
        __nanosleep(64);
      }
    }
    if (!ok) {
      ok_all = 0;
      atomicOr(&g_peer_status, kStatusTimeout);
    }
  }
  __syncthreads();
  if (!ok_all) return;
  // sum in rank order, 4 floats at a time where n allows (buffers are 16-byte aligned)
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n4; i += stride) {
    float4 s = __ldcv(reinterpret_cast<const float4*>(a.data[0]) + i);
    for (int p = 1; p < world; ++p) {
      const float4 v = __ldcv(reinterpret_cast<const float4*>(a.data[p]) + i);
      s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
  }
  for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride) {
    float s = __ldcv(a.data[0] + i);
    for (int p = 1; p < world; ++p) s += __ldcv(a.data[p] + i);
    out[i] = s;
  }
}

}  // namespace peer

cudaError_t launch_peer_allreduce(const float* const* data, int* const* flags, int world, int rank,
                                  int epoch, int64_t n, float* out, long long budget_cycles,
                                  cudaStream_t st) {
  if (world < 1 || world > peer::kMaxRanks || rank < 0 || rank >= world || n < 0)
    return cudaErrorInvalidValue;
  peer::PeerArgs a = {};
  for (int p = 0; p < world; ++p) {
    a.data[p] = data[p];
    a.flags[p] = flags[p];
  }
  // a few CTAs: the step is latency-bound (W x n x 4 bytes over NVLink)
  int64_t ctas = (n / 4 + peer::kThreads - 1) / peer::kThreads;
  if (ctas < 1) ctas = 1;
  if (ctas > 32) ctas = 32;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, 1, 1);
  cfg.blockDim = dim3(peer::kThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer::peer_allreduce_kernel, a, world, rank, epoch, n, out,
                            budget_cycles);
}

// ---- CUDA IPC of a buffer inside a caching allocator's block -------------------------
// The handle names the whole allocation that holds `ptr`; the offset of `ptr` from the
// allocation's base travels with it, and the importer adds it back.
// The driver's address-range query, resolved at run time like the tensor-map encoder (the
// library has no link-time dependency on the driver).
typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
static AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  });
  return fn;
}

cudaError_t ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  const AddrRangeFn range = addr_range_fn();
  if (!range) return cudaErrorNotSupported;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return e;
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return cudaSuccess;
}
// maps the peer's allocation into this process for the current device (peer access enabled
// on first use); *ptr_out = base + offset
cudaError_t ipc_import(const void* handle, int64_t offset, void** ptr_out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return e;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return cudaSuccess;
}
cudaError_t ipc_close(void* ptr, int64_t offset) {
  return cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
}

cudaError_t peer_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_peer_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
