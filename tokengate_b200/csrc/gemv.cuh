// Decode projections: y = x W^T for a few rows (the decode step's B <= 8
// tokens), HBM-bound on the weight read — the q/k/v, o, gate/up, down and
// lm_head projections of the reference's decode layers (transformers
// Qwen3DecoderLayer / lm_head under tokengate/e2e_gate/decode/gate_decode.py:199-219).
//
// x: (B, K) bf16 (row stride ld_x), W: (N, K) bf16 row-major (row stride
// ld_w), y: (B, N) bf16. The rows of x sit in shared memory; each warp
// streams its weight rows with 16-byte loads (lane l: elements 8l..8l+7 of
// every 256-element slice, several slices in flight), keeps B partial sums
// per row, and reduces them across the warp at the end. SwiGLU form: W is
// the fused [gate (I rows); up (I rows)] weight and the warp that owns
// output j reads gate row j and up row I + j, writing
// act[b, j] = bf16(bf16(silu(bf16(g))) * bf16(u)) — the rounding points of
// a bf16 GEMM output followed by the SwiGLU glue.
#pragma once

#include "ptx.cuh"
#include "e2e_gate.cuh"  // bf16_round

namespace tg {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

struct GemvParams {
  const __nv_bfloat16* x;
  int64_t ld_x;
  const __nv_bfloat16* w;
  int64_t ld_w;
  __nv_bfloat16* y;
  int64_t ld_y;
  int B, N, K;   // N: output columns (SwiGLU: the intermediate size I; W has 2I rows)
};

__device__ __forceinline__ float gemv_silu(float g) {
  // the eager op: g / (1 + exp(-g)) in fp32, IEEE division
  return g / (1.f + expf(-g));
}

// R weight rows per warp pass (SwiGLU: the gate row and its up row). A warp
// loads kGemvBatch 512-byte slices of its row(s) at a time into registers
// (a whole K = 2048 row in one batch) and issues the next batch (the rest of
// the row, or its next row) as soon as the current one is consumed; the
// first batch is issued before x is staged, so the two reads overlap.
// Launched with programmatic stream serialization: before waiting for the
// kernel that produces x, each warp prefetches the weight rows of its first
// two passes into L2 (a hint only: the rows are loaded after the wait).
constexpr int kGemvBatch = 8;

// A whole long row in one batch for the plain form with few rows (K up to
// 6144: 24 slices), where a row per warp in 8-slice batches leaves the
// launch bound by the latency of dependent loads.
constexpr int kGemvLongBatch = 24;

template <int R, int NB>
__device__ __forceinline__ void gemv_load_batch(uint4 (&wv)[R][NB], const __nv_bfloat16* w, const GemvParams& p,
                                                int64_t n, int s0, int n_slices, int lane) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const uint4* row = reinterpret_cast<const uint4*>(w + (n + r * p.N) * p.ld_w + 8 * lane) + 32 * s0;
#pragma unroll
    for (int u = 0; u < NB; ++u)
      if (s0 + u < n_slices) wv[r][u] = ld_nc_v4(row + 32 * u);
  }
}

// NB: 512-byte slices per batch (kGemvBatch, or kGemvLongBatch).
template <int BT, bool kSwiGlu, int NB = kGemvBatch>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) uint8_t gsm[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(gsm);  // [BT][K]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int K = p.K;
  constexpr int R = kSwiGlu ? 2 : 1;
  const int n_slices = K / 256;
  const int64_t warp_global = (int64_t)blockIdx.x * kGemvWarps + warp;
  const int64_t n_warps = (int64_t)gridDim.x * kGemvWarps;
  if (lane < 2 * R) {
    const int64_t n = warp_global + (lane / R) * n_warps;
    if (n < p.N) prefetch_l2_bulk(p.w + (n + (lane % R) * p.N) * p.ld_w, (uint32_t)K * 2u);
  }
  griddep_wait();
  const __nv_bfloat16* x = p.x;
  const __nv_bfloat16* w = p.w;
  uint4 wv[R][NB];
  if (warp_global < p.N) gemv_load_batch<R, NB>(wv, w, p, warp_global, 0, n_slices, lane);
  // x rows into shared memory (rows past B are zero)
  for (int i = t; i < BT * (K / 8); i += kGemvThreads) {
    const int b = i / (K / 8), c = i - b * (K / 8);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (b < p.B) v = *reinterpret_cast<const uint4*>(x + (int64_t)b * p.ld_x + 8 * c);
    reinterpret_cast<uint4*>(xs + (int64_t)b * K)[c] = v;
  }
  __syncthreads();
  griddep_launch_dependents();

  for (int64_t n = warp_global; n < p.N; n += n_warps) {
    float acc[R][BT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < BT; ++b) acc[r][b] = 0.f;
    for (int s0 = 0; s0 < n_slices; s0 += NB) {
#pragma unroll
      for (int u = 0; u < NB; ++u) {
        if (s0 + u < n_slices) {
#pragma unroll
          for (int b = 0; b < BT; ++b) {
            const uint4 xv = reinterpret_cast<const uint4*>(xs + (int64_t)b * K + 256 * (s0 + u))[lane];
            const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const uint32_t ww[4] = {wv[r][u].x, wv[r][u].y, wv[r][u].z, wv[r][u].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                acc[r][b] = fmaf(__uint_as_float(ww[e] << 16), __uint_as_float(xw[e] << 16), acc[r][b]);
                acc[r][b] = fmaf(__uint_as_float(ww[e] & 0xFFFF0000u), __uint_as_float(xw[e] & 0xFFFF0000u),
                                 acc[r][b]);
              }
            }
          }
        }
      }
      // the next batch: the rest of this row, else the first of the next
      if (s0 + NB < n_slices)
        gemv_load_batch<R, NB>(wv, w, p, n, s0 + NB, n_slices, lane);
      else if (n + n_warps < p.N)
        gemv_load_batch<R, NB>(wv, w, p, n + n_warps, 0, n_slices, lane);
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int b = 0; b < BT; ++b)
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], off);
    if (lane < BT && lane < p.B) {
      float val = 0.f;
#pragma unroll
      for (int b = 0; b < BT; ++b)
        if (b == lane) {
          if (kSwiGlu) {
            const float g = bf16_round(acc[0][b]), u = bf16_round(acc[R - 1][b]);
            val = bf16_round(gemv_silu(g)) * u;
          } else {
            val = acc[0][b];
          }
        }
      p.y[(int64_t)lane * p.ld_y + n] = __float2bfloat16_rn(val);
    }
  }
}

}  // namespace tg
