// vbq_gemv_mma.cu -- Q4_K dequant-GEMV on the tensor cores (decode, batch 1..4).
//
//   y[b, n] = sum_k x[b, k] * deq(W)[k, n],  deq(W)[k, n] = dl[k, s] * q[k, n] - ml[k, s]
//
// (cpp/src/dequant.cpp:268-301, :739-780; s = the 32-column sub-block of n).  The scalar
// GEMV spends ~5.5 instructions per weight and is issue-bound; here a weight costs about
// one.  The sum is regrouped as
//   y[b, n] = sum_k q[k, n] * x'[b, k, s]  -  sum_k x[b, k] * ml[k, s],   x' = x * dl,
// and the first term runs on mma.sync (bf16 x bf16 -> fp32):
//   * A (16 columns x 16 rows): the quant codes as exact bf16 integers.  ldmatrix.trans
//     hands each lane the bytes of two consecutive rows for the same columns, so one LOP3
//     (plus a shift for odd bytes / high nibbles) makes the bf16 pair (128 + q, 128 + q')
//     the MMA fragment wants.  High nibbles are placed 3 bits up (128 + 8 q).
//   * B (16 rows x 8): x' split into two bf16 (hi + lo, ~16 significant bits, fp32
//     range) for each batch row: columns 2b and 2b + 1; high-nibble sub-blocks use x' / 8.
//   * The constant parts -- 128 * sum x' (16 * sum x' for high nibbles) and the min term --
//     are summed per sub-block on the side and subtracted once at the end.
// Accuracy: ~2^-17 relative per term from the bf16 split, fp32 accumulation.
//
// Decomposition: a CTA owns one 256-column tile (one Q4_K block per row) and every S-th
// 128-row stage of the matrix (stages split, split + S, ...), so each CTA samples the
// whole row range; its partial sums go to the caller's scratch and the CTA finishing a
// tile last adds the S partials in split order (deterministic) and resets the tile's
// counter.  Warp 8 TMA-loads the stages (144 B per row) into a 4-deep ring; warps 0-7 each
// take 32 rows x 128 columns of a stage: the B table for their rows, then 2 groups x
// 4 kinds of MMAs plus two constant ones.  The CTA's x rows sit in shared memory.  Waits
// are bounded.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>

#include "vbq_common.cuh"
#include "vbq_internal.h"

namespace vbq {

// Sticky error bits of this file's kernel (kStatusTimeout: a bounded wait gave up); each
// translation unit keeps its own word (no relocatable device code).
__device__ unsigned g_gemv_mma_status = 0;


namespace gmma {

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kRows = 16 * kConsumers;   // rows per stage
constexpr int kPitch = 144;              // one Q4_K block per row
constexpr int kStageBytes = kRows * kPitch;  // 18432
constexpr int kStages = 4;
// x' table per warp and column set: [4 local sub-blocks][8 columns of B][32 rows] bf16,
// column stride 80 B so that the 32 lanes' 4-byte fragment loads hit 32 different banks
constexpr int kColStride = 80;
constexpr int kTblBytes = 4 * 8 * kColStride;  // 2560
constexpr int kRedBytes = kConsumers * 4 * 256 * 4 + 4 * 256 * 4;  // per-warp partials + sum

struct Bars {
  uint64_t full[kStages], empty[kStages];
  int abort;
};
constexpr int kTblOff = kStages * kStageBytes;
constexpr int kRedOff = 0;  // the per-warp partial outputs reuse the stage ring afterwards
static_assert(kRedBytes <= kStages * kStageBytes, "reduction buffer inside the ring");
template <int NSET> struct Lay {
  static constexpr int kBarOff = kTblOff + kConsumers * NSET * kTblBytes;
  static constexpr int kXOff = kBarOff + 128;      // the CTA's slice of x, [batch][kslice] fp32
  static constexpr int kFixed = kXOff + 128;       // + alignment slack; plus the x slice
};

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t saddr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(saddr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// bf16 code pairs from one ldmatrix.trans register R = [row k: bytes 2g, 2g+1 | row k+1:
// bytes 2g, 2g+1] (16-bit halves): low half = row k, high half = row k+1
__device__ __forceinline__ uint32_t even_lo(uint32_t r) { return (r & 0x000f000fu) | 0x43004300u; }
__device__ __forceinline__ uint32_t even_hi(uint32_t r) { return ((r >> 1) & 0x00780078u) | 0x43004300u; }
__device__ __forceinline__ uint32_t odd_lo(uint32_t r) { return ((r >> 8) & 0x000f000fu) | 0x43004300u; }
__device__ __forceinline__ uint32_t odd_hi(uint32_t r) { return ((r >> 9) & 0x00780078u) | 0x43004300u; }

__device__ __forceinline__ uint16_t bf16_bits(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&h);
}

template <int BATCH>
__global__ void __launch_bounds__(kThreads, BATCH <= 2 ? 2 : 1)
gemv_mma_kernel(const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ x,
                float* __restrict__ y, int K, int N, int kslice, int batch,
                float* __restrict__ partials, unsigned* __restrict__ counters) {
  constexpr int NSET = BATCH <= 2 ? 1 : 2;  // B column sets: two batch rows per set
  extern __shared__ uint8_t smem_raw[];
  // 128-byte aligned: TMA destinations and ldmatrix rows
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  using L = Lay<NSET>;
  Bars& bars = *reinterpret_cast<Bars*>(smem + L::kBarOff);
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y, S = gridDim.y;
  // CTA `split` takes the 128-row stages split, split + S, split + 2S, ... of the matrix
  const int tot_st = (K + kRows - 1) / kRows;
  const int nst = split < tot_st ? (tot_st - split + S - 1) / S : 0;
  auto stage = [&](int s) { return smem + s * kStageBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars.full[s]), 1);
      mbar_init(smem_u32(&bars.empty[s]), kConsumers);
    }
    bars.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  // Programmatic dependent launch: the next kernel may start filling SMs as this grid
  // drains; weights are streamed before waiting for the previous grid (they never depend
  // on it), x, y and the scratch only after.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  volatile int* abort_flag = &bars.abort;
  auto give_up = [&]() {
    *abort_flag = 1;
    atomicOr(&g_gemv_mma_status, kStatusTimeout);
  };

  // [set][local group][kind: even-lo, odd-lo, even-hi, odd-hi][fragment]; constant-A MMAs
  // [set][local group][low / high sub-block][fragment]
  float acc[NSET][2][4][4], cacc[NSET][2][2][4];
#pragma unroll
  for (int z = 0; z < NSET; ++z)
#pragma unroll
    for (int g = 0; g < 2; ++g) {
#pragma unroll
      for (int f = 0; f < 4; ++f) {
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[z][g][k][f] = 0.f;
        cacc[z][g][0][f] = 0.f;
        cacc[z][g][1][f] = 0.f;
      }
    }

  if (warp == kConsumers) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int it = 0;
      for (; it < nst && !*abort_flag; ++it) {
        const int s = it % kStages;
        if (it == kStages) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (!mbar_wait_bounded(smem_u32(&bars.empty[s]), ((it / kStages) & 1) ^ 1, kWaitBudgetCycles)) {
          give_up();
          break;
        }
        const uint32_t fb = smem_u32(&bars.full[s]);
        mbar_arrive_expect_tx(fb, kStageBytes);
        tma_load_2d(smem_u32(stage(s)), &tmap_w, tile * (kPitch / 2), (split + S * it) * kRows, fb);
      }
      // every issued stage lands before the CTA may exit
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        mbar_wait_bounded(smem_u32(&bars.full[j % kStages]), (j / kStages) & 1, kWaitBudgetCycles);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
  } else {
    // ------------------------------ consumers ------------------------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // this CTA's slice of x into shared memory once (the 8 consumer warps, coalesced)
    float* xs = reinterpret_cast<float*>(smem + L::kXOff);
    for (int i = threadIdx.x; i < BATCH * kslice; i += 32 * kConsumers) {
      const int b = i / kslice, li = i % kslice, lst = li / kRows;
      const int k = (split + S * lst) * kRows + li % kRows;
      xs[i] = (b < batch && lst < nst && k < K) ? __ldg(x + (int64_t)b * K + k) : 0.f;
    }
    uint8_t* tbl = smem + kTblOff + warp * NSET * kTblBytes;
    const int gp = warp & 1;          // this warp's groups 2gp, 2gp+1 (columns 128gp..+127)
    const int rw = 32 * (warp >> 1);  // and its 32 rows of each stage
    for (int i = lane; i < NSET * kTblBytes / 4; i += 32) reinterpret_cast<uint32_t*>(tbl)[i] = 0u;
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumers) : "memory");  // consumers only
    // table role: rows 2rp, 2rp+1 of the warp's 32 and local group gl = global group q
    // (sub-blocks 2q low nibbles, 2q + 1 high nibbles)
    const int rp = lane & 15, gl = lane >> 4, q = 2 * gp + gl;
    const uint32_t sel_lo = 0x7440u | (uint32_t)((2 * q) & 3), sel_hi = 0x7440u | (uint32_t)((2 * q + 1) & 3);
    const int g = lane >> 2, t = lane & 3;  // MMA fragment role
    // ldmatrix: lane gives the row address of matrix lane >> 3 (rows 0-7 / 8-15 x bytes
    // 0-15 / 16-31 of a group's 32 quant bytes)
    const int lm_row = rw + 8 * ((lane >> 3) & 1) + (lane & 7);
    const int lm_col = 16 + 64 * gp + 16 * (lane >> 4);
    for (int it = 0; it < nst; ++it) {
      if (*abort_flag) break;
      const int s = it % kStages;
      if (!mbar_wait_bounded(smem_u32(&bars.full[s]), (it / kStages) & 1, kWaitBudgetCycles)) {
        give_up();
        break;
      }
      const uint8_t* st = stage(s);
      // ---- B operand table for the warp's 32 rows: per local sub-block and batch row b,
      // columns 4(b&1) .. +3 of set b>>1 hold x' (hi, lo) and x * ml / 128 (hi, lo) ----
      {
        const int rl = rw + 2 * rp;  // stage row of this lane's first row
        const int kk = it * kRows + rl;     // offset in the CTA's K-slice
        const uint4 h0 = *reinterpret_cast<const uint4*>(st + rl * kPitch);
        const uint4 h1 = *reinterpret_cast<const uint4*>(st + (rl + 1) * kPitch);
        // get_scale_min_k4 (cpp/src/dequant.cpp:258-266), four sub-blocks per word
        auto sc4 = [&](const uint4& h) {
          return q < 2 ? (h.y & 0x3f3f3f3fu) : ((h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u));
        };
        auto mn4 = [&](const uint4& h) {
          return q < 2 ? (h.z & 0x3f3f3f3fu) : (((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u));
        };
        const uint32_t s0 = sc4(h0), s1 = sc4(h1), m0 = mn4(h0), m1 = mn4(h1);
        // small integers as floats: byte into the 2^23 magic, minus 2^23 (exact)
        const float2 kMag = make_float2(-8388608.f, -8388608.f);
        const float2 sl = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(s0, 0x4b000000u, sel_lo)),
                                                 __uint_as_float(__byte_perm(s1, 0x4b000000u, sel_lo))), kMag);
        const float2 sh = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(s0, 0x4b000000u, sel_hi)),
                                                 __uint_as_float(__byte_perm(s1, 0x4b000000u, sel_hi))), kMag);
        const float2 ml_ = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(m0, 0x4b000000u, sel_lo)),
                                                  __uint_as_float(__byte_perm(m1, 0x4b000000u, sel_lo))), kMag);
        const float2 mh_ = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(m0, 0x4b000000u, sel_hi)),
                                                  __uint_as_float(__byte_perm(m1, 0x4b000000u, sel_hi))), kMag);
        const float2 d = make_float2(f16_ref(h0.x & 0xffffu), f16_ref(h1.x & 0xffffu));
        const float2 dm = make_float2(f16_ref(h0.x >> 16), f16_ref(h1.x >> 16));
        // dl = d * sc (the reference's fp32 value, exact); high-nibble codes are 8 q, so
        // their x' is x * dl / 8; the min term enters as x * (dmin * m) / 128
        const float2 dl_lo = __fmul2_rn(d, sl);
        const float2 dl_hi = __fmul2_rn(__fmul2_rn(d, make_float2(0.125f, 0.125f)), sh);
        const float2 dm128 = __fmul2_rn(dm, make_float2(0.0078125f, 0.0078125f));
        const float2 ml_lo = __fmul2_rn(dm128, ml_), ml_hi = __fmul2_rn(dm128, mh_);
        uint32_t* tw = reinterpret_cast<uint32_t*>(tbl);
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const float2 xv = make_float2(xs[b * kslice + kk], xs[b * kslice + kk + 1]);
          // rows past the slice end read 0 (xs is zero-padded there: kk + 1 < kslice)
          const float2 v[4] = {__fmul2_rn(xv, dl_lo), __fmul2_rn(xv, ml_lo), __fmul2_rn(xv, dl_hi),
                               __fmul2_rn(xv, ml_hi)};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            // hi = bf16(v), lo = bf16(v - hi): two K rows per 32-bit word
            const __nv_bfloat162 hb = __floats2bfloat162_rn(v[u].x, v[u].y);
            const float2 hf = __bfloat1622float2(hb);
            const __nv_bfloat162 lb = __floats2bfloat162_rn(v[u].x - hf.x, v[u].y - hf.y);
            const int sbl = 2 * gl + (u >> 1);  // local sub-block 0..3
            const int n = 4 * (b & 1) + 2 * (u & 1);
            uint32_t* col = tw + ((b >> 1) * kTblBytes + sbl * 8 * kColStride + n * kColStride) / 4 + rp;
            col[0] = *reinterpret_cast<const uint32_t*>(&hb);
            col[kColStride / 4] = *reinterpret_cast<const uint32_t*>(&lb);
          }
        }
      }
      __syncwarp();
      // ---- 2 groups x 2 row halves x (4 kinds + 2 constant) m16n8k16 MMAs per set ----
      const uint32_t lm_base = smem_u32(st) + lm_row * kPitch + lm_col;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int gg = j & 1, hr = j >> 1;  // local group, 16-row half
        uint32_t r0, r1, r2, r3;  // matrices: rows 0-7 / 8-15 x bytes 0-15 / 16-31
        ldmatrix_x4_trans(lm_base + 16 * hr * kPitch + 32 * gg, r0, r1, r2, r3);
        const uint32_t el0 = even_lo(r0), el1 = even_lo(r2), el2 = even_lo(r1), el3 = even_lo(r3);
        const uint32_t ol0 = odd_lo(r0), ol1 = odd_lo(r2), ol2 = odd_lo(r1), ol3 = odd_lo(r3);
        const uint32_t eh0 = even_hi(r0), eh1 = even_hi(r2), eh2 = even_hi(r1), eh3 = even_hi(r3);
        const uint32_t oh0 = odd_hi(r0), oh1 = odd_hi(r2), oh2 = odd_hi(r1), oh3 = odd_hi(r3);
#pragma unroll
        for (int z = 0; z < NSET; ++z) {
          const uint8_t* tz = tbl + z * kTblBytes;
          const uint32_t* bl = reinterpret_cast<const uint32_t*>(tz + (2 * gg) * 8 * kColStride + g * kColStride) + 8 * hr;
          const uint32_t* bh = reinterpret_cast<const uint32_t*>(tz + (2 * gg + 1) * 8 * kColStride + g * kColStride) + 8 * hr;
          const uint32_t bl0 = bl[t], bl1 = bl[t + 4], bh0 = bh[t], bh1 = bh[t + 4];
          // A rows m = g (bytes 0-15) and g + 8 (bytes 16-31); k = 2t.. (rows 0-7), 2t+8..
          mma_bf16(acc[z][gg][0], el0, el1, el2, el3, bl0, bl1);
          mma_bf16(acc[z][gg][1], ol0, ol1, ol2, ol3, bl0, bl1);
          mma_bf16(acc[z][gg][2], eh0, eh1, eh2, eh3, bh0, bh1);
          mma_bf16(acc[z][gg][3], oh0, oh1, oh2, oh3, bh0, bh1);
          // A = 128 everywhere: 128 * sum x' (columns 4j, 4j+1) and sum x * ml (4j+2, +3)
          mma_bf16(cacc[z][gg][0], 0x43004300u, 0x43004300u, 0x43004300u, 0x43004300u, bl0, bl1);
          mma_bf16(cacc[z][gg][1], 0x43004300u, 0x43004300u, 0x43004300u, 0x43004300u, bh0, bh1);
        }
      }
      __syncwarp();  // table and stage reads done
      if (lane == 0) mbar_arrive(smem_u32(&bars.empty[s]));
    }
  }

  // ---- per-warp partial outputs -> shared memory (the stage ring, now idle) ----
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem + kRedOff);  // [warp][b][256]
  if (warp < kConsumers) {
    const int g = lane >> 2, t = lane & 3, gp = warp & 1;
#pragma unroll
    for (int z = 0; z < NSET; ++z) {
      const int b = 2 * z + (t >> 1);  // batch row of this lane's columns
#pragma unroll
      for (int gg = 0; gg < 2; ++gg) {
        // the constant MMAs' rows are all equal: lane t even holds 128 * sum x', t odd
        // (the next lane) the min term of the same batch row
        const float c_lo = cacc[z][gg][0][0] + cacc[z][gg][0][1];
        const float c_hi = cacc[z][gg][1][0] + cacc[z][gg][1][1];
        const float corr_lo = c_lo + __shfl_down_sync(0xffffffffu, c_lo, 1);
        const float corr_hi = c_hi + __shfl_down_sync(0xffffffffu, c_hi, 1);
        if ((t & 1) == 0 && b < BATCH) {
          float* dst = red + (warp * 4 + b) * 256;
#pragma unroll
          for (int kind = 0; kind < 4; ++kind) {
            // kind 0 / 1: even / odd byte, low nibble; 2 / 3: high nibble (+32 columns)
            const float corr = (kind >> 1) ? corr_hi : corr_lo;
            const int c0 = 128 * gp + 64 * gg + 2 * g + (kind & 1) + (kind >> 1) * 32;
            dst[c0] = acc[z][gg][kind][0] + acc[z][gg][kind][1] - corr;       // m = g
            dst[c0 + 16] = acc[z][gg][kind][2] + acc[z][gg][kind][3] - corr;  // m = g + 8
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- sum the warps in order: this CTA's partial y ----
  const int E = batch * 256;
  float* outbuf = red + kConsumers * 4 * 256;  // after the per-warp slots, still in the ring
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, n = e & 255;
    float v = 0.f;
#pragma unroll
    for (int w2 = (n >> 7); w2 < kConsumers; w2 += 2) v += red[(w2 * 4 + b) * 256 + n];  // warps of this half
    outbuf[e] = v;
  }
  __syncthreads();

  if (S == 1) {
    for (int e = threadIdx.x; e < E; e += kThreads)
      y[(int64_t)(e >> 8) * N + tile * 256 + (e & 255)] = outbuf[e];
    return;
  }
  // ---- split-K: publish this CTA's partial; the last CTA of the tile adds them up ----
  for (int e = threadIdx.x; e < E; e += kThreads)
    partials[((int64_t)split * batch + (e >> 8)) * N + tile * 256 + (e & 255)] = outbuf[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&counters[tile], 1u) == (unsigned)(S - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < E; e += kThreads) {
    const int b = e >> 8, n = e & 255;
    float sum = 0.f;
    for (int sp = 0; sp < S; ++sp)
      sum += __ldcg(partials + ((int64_t)sp * batch + b) * N + tile * 256 + n);
    y[(int64_t)b * N + tile * 256 + n] = sum;
  }
  if (threadIdx.x == 0) counters[tile] = 0u;  // leave the scratch ready for the next call
}

}  // namespace gmma

// ---- host side -----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFnG)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnG encode_fn_g() {
  static EncodeTiledFnG fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnG>(p);
  });
  return fn;
}

template <int BATCH>
static cudaError_t launch_t(const float* x, const void* w, float* y, int64_t K, int64_t N,
                            int64_t RB, int batch, const GemvPlan& plan, void* scratch,
                            cudaStream_t st) {
  using namespace gmma;
  auto enc = encode_fn_g();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap mw;
  cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)K};
  cuuint64_t strides[1] = {(cuuint64_t)RB};
  cuuint32_t box[2] = {(cuuint32_t)(kPitch / 2), (cuuint32_t)kRows};
  cuuint32_t es[2] = {1, 1};
  if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(w), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  auto kern = gemv_mma_kernel<BATCH>;
  static unsigned configured = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  constexpr int kMaxDyn = 220 * 1024;  // below the 227 KB limit: the kernel's static bytes
  const int smem = Lay<(BATCH <= 2 ? 1 : 2)>::kFixed + BATCH * (int)plan.kslice * 4;
  if (smem > kMaxDyn) return cudaErrorNotSupported;
  if (dev >= 32 || !(configured & (1u << dev))) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDyn);
    if (e != cudaSuccess) return e;
    if (dev < 32) configured |= (1u << dev);
  }
  unsigned* counters = static_cast<unsigned*>(scratch);
  float* partials = plan.splits > 1
                        ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + plan.counter_bytes)
                        : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 256), (unsigned)plan.splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mw, x, y, (int)K, (int)N, (int)plan.kslice, batch,
                            partials, counters);
}

// Whether the tensor-core kernel takes this call: its CTA keeps the x slice in shared
// memory (slices that would not fit go to the scalar kernel).
bool gemv_mma_fits(const float*, int64_t K, int64_t, int batch, const GemvPlan& plan) {
  const int B = batch <= 1 ? 1 : batch <= 2 ? 2 : 4;
  return batch >= 1 && batch <= 4 && K <= 0x7fffffff && plan.kslice % gmma::kRows == 0 &&
         gmma::Lay<2>::kFixed + (int64_t)B * plan.kslice * 4 <= 220 * 1024;
}

// Tensor-core Q4_K GEMV for batch 1..4 (the plan's K-slices are multiples of 128 rows).
cudaError_t launch_gemv_mma_q4k(const float* x, const void* w, float* y, int64_t K, int64_t N,
                                int64_t row_bytes, int batch, const GemvPlan& plan,
                                void* scratch, cudaStream_t st) {
  if (N % 256 != 0 || !gemv_mma_fits(x, K, N, batch, plan) || row_bytes % 16 != 0)
    return cudaErrorNotSupported;
  if (batch == 1) return launch_t<1>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
  if (batch == 2) return launch_t<2>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
  return launch_t<4>(x, w, y, K, N, row_bytes, batch, plan, scratch, st);
}

cudaError_t gemv_mma_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_gemv_mma_status, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0;
  return cudaMemcpyToSymbol(g_gemv_mma_status, &zero, sizeof(unsigned));
}

}  // namespace vbq
