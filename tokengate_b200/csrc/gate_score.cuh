// Gate scorer: score = logsigmoid(w . h_row) over the state rows of each
// request — the synthetic linear gate of the gated prefill (a 1-wide fp32
// readout plus log-sigmoid; the reference scores with gate(h_art.to(fp32)),
// tokengate/e2e_gate/gate_module/gate_forward.py:1396-1407).
//
// HBM-bound. gate_score_bulk_kernel: one producer warp per CTA streams the
// CTA's contiguous range of state rows into a ring of shared-memory stages
// with bulk copies (the TMA engine, one copy per row, completion on an
// mbarrier per stage), 16 consumer warps (8 for rows over 4 KB) reduce one row each per stage
// from shared memory with their slice of w in registers. gate_score_kernel
// (one warp per row, 16-byte non-allocating loads with a one-row prefetch)
// is kept for rows that are not 16-byte aligned.
// Arithmetic contract (reproducible bit for bit on the host):
//   lane l accumulates, for i = 0..NV-1 and e = 0..7, the products of the
//   elements 8*(l + 32*i) + e in that order with fused multiply-adds into one
//   fp32 accumulator starting at 0; the 32 partials are combined by the xor
//   butterfly (offsets 16, 8, 4, 2, 1); logsigmoid uses IEEE +,-,*,/,fma only
//   (tg_logsigmoid below).
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kScoreMaxReq = 128;

struct ScoreParams {
  const __nv_bfloat16* h;
  int64_t h_sb, h_ss;
  const float* w;
  float* out;
  int64_t out_sb;
  int B;
  int64_t total_rows;
  int begin[kScoreMaxReq];
  int64_t row_off[kScoreMaxReq + 1];  // prefix sums of the row counts
  int64_t rows_per_cta;               // bulk kernel: contiguous rows per CTA
  unsigned int* err;
};

constexpr unsigned int ERR_SCORE = 1u << 13;
// rows per stage (one per consumer warp), stages, threads (consumers + one
// producer warp) and shared memory of the bulk kernel for NV 16-byte vectors
// per lane (rows of NV * 512 bytes)
template <int NV>
__host__ __device__ constexpr int score_rows() { return NV <= 8 ? 16 : 8; }
template <int NV>
__host__ __device__ constexpr int score_stages() { return NV <= 8 ? 3 : 2; }
template <int NV>
__host__ __device__ constexpr int score_threads() { return (score_rows<NV>() + 1) * 32; }
template <int NV>
__host__ __device__ constexpr int score_bulk_smem() {
  return score_stages<NV>() * score_rows<NV>() * NV * 512 + 16 * score_stages<NV>() + 128;
}

// exp(-a) for a >= 0 by Cody-Waite reduction a = k ln2 - r, |r| <= ln2/2, and a
// degree-7 Taylor polynomial for exp(r); IEEE operations only.
__device__ __forceinline__ float tg_exp_neg(float a) {
  if (a > 104.0f) return 0.0f;
  const float kInvLn2 = 1.44269504088896341f;
  const float kLn2Hi = 0.693145751953125f;         // 0x3F317200
  const float kLn2Lo = 1.42860682030941723212e-6f;  // ln2 - kLn2Hi
  const float k = rintf(__fmul_rn(a, kInvLn2));
  float r = __fmaf_rn(k, kLn2Hi, -a);
  r = __fmaf_rn(k, kLn2Lo, r);  // r = k ln2 - a, exp(-a) = 2^-k exp(r)
  float q = 1.98412698412698413e-4f;  // 1/7!
  q = __fmaf_rn(q, r, 1.38888888888888889e-3f);
  q = __fmaf_rn(q, r, 8.33333333333333333e-3f);
  q = __fmaf_rn(q, r, 4.16666666666666667e-2f);
  q = __fmaf_rn(q, r, 1.66666666666666667e-1f);
  q = __fmaf_rn(q, r, 0.5f);
  q = __fmaf_rn(q, r, 1.0f);
  q = __fmaf_rn(q, r, 1.0f);
  // scale by 2^-k, k in [0, 150]: two exact power-of-two steps
  int ki = (int)k;
  const int k1 = ki > 100 ? 100 : ki;
  const int k2 = ki - k1;
  q = __fmul_rn(q, __int_as_float((127 - k1) << 23));
  if (k2 > 0) q = __fmul_rn(q, __int_as_float((127 - k2) << 23));
  return q;
}

// log1p(x) for x in [0, 1]: log(u) + (x - (u - 1)) / u with u = 1 + x, and
// log(u) = j ln2 + 2 atanh((m - 1) / (m + 1)), m = u / 2^j in [sqrt(1/2), sqrt(2)].
__device__ __forceinline__ float tg_log1p_unit(float x) {
  if (x < 2.44140625e-4f) {  // 2^-12: three series terms are exact to fp32
    float s = __fmaf_rn(x, 0.333333333333333333f, -0.5f);
    s = __fmul_rn(s, x);
    return __fmaf_rn(s, x, x);
  }
  const float u = __fadd_rn(1.0f, x);
  const float corr = __fdiv_rn(__fsub_rn(x, __fsub_rn(u, 1.0f)), u);
  float m = u;
  float j = 0.0f;
  if (u > 1.41421356237309505f) {
    m = __fmul_rn(u, 0.5f);
    j = 1.0f;
  }
  const float f = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float f2 = __fmul_rn(f, f);
  float s = 7.69230769230769231e-2f;  // 1/13
  s = __fmaf_rn(s, f2, 9.09090909090909091e-2f);
  s = __fmaf_rn(s, f2, 1.11111111111111111e-1f);
  s = __fmaf_rn(s, f2, 1.42857142857142857e-1f);
  s = __fmaf_rn(s, f2, 2.0e-1f);
  s = __fmaf_rn(s, f2, 3.33333333333333333e-1f);
  s = __fmul_rn(s, f2);
  const float two_f = __fmul_rn(2.0f, f);
  const float logm = __fmaf_rn(two_f, s, two_f);
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.42860682030941723212e-6f;
  const float lo = __fmaf_rn(j, kLn2Lo, __fadd_rn(logm, corr));
  return __fmaf_rn(j, kLn2Hi, lo);
}

__device__ __forceinline__ float tg_logsigmoid(float z) {
  const float a = fabsf(z);
  const float e = tg_exp_neg(a);
  const float l = tg_log1p_unit(e);
  return __fsub_rn(fminf(z, 0.0f), l);
}

template <int NV>
__global__ void __launch_bounds__(256) gate_score_kernel(const ScoreParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;

  float wr[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4* wp = reinterpret_cast<const float4*>(p.w + 8 * (lane + 32 * i));
    const float4 a = __ldg(wp), c = __ldg(wp + 1);
    wr[i][0] = a.x; wr[i][1] = a.y; wr[i][2] = a.z; wr[i][3] = a.w;
    wr[i][4] = c.x; wr[i][5] = c.y; wr[i][6] = c.z; wr[i][7] = c.w;
  }

  // rows are visited in increasing order by each warp; `req` tracks the
  // request of the row, the next row's 16-byte vectors are loaded before the
  // current row is reduced
  int req = 0, nreq = 0;
  auto row_ptr = [&](int64_t g, int& rq) {
    while (g >= p.row_off[rq + 1]) ++rq;
    const int64_t r = g - p.row_off[rq];
    return p.h + (int64_t)rq * p.h_sb + (int64_t)(p.begin[rq] + r) * p.h_ss;
  };
  constexpr bool kPrefetch = NV <= 8;  // wider rows would spill the second buffer
  uint4 hv[NV], hn[kPrefetch ? NV : 1];
  int64_t g = warp_global;
  if (kPrefetch && g < p.total_rows) {
    const __nv_bfloat16* row = row_ptr(g, nreq);
#pragma unroll
    for (int i = 0; i < NV; ++i) hn[i] = ld_nc_v4(reinterpret_cast<const uint4*>(row + 8 * (lane + 32 * i)));
  }
  for (; g < p.total_rows; g += n_warps) {
    if constexpr (kPrefetch) {
      req = nreq;
#pragma unroll
      for (int i = 0; i < NV; ++i) hv[i] = hn[i];
      const int64_t gn = g + n_warps;
      if (gn < p.total_rows) {
        const __nv_bfloat16* row = row_ptr(gn, nreq);
#pragma unroll
        for (int i = 0; i < NV; ++i) hn[i] = ld_nc_v4(reinterpret_cast<const uint4*>(row + 8 * (lane + 32 * i)));
      }
    } else {
      const __nv_bfloat16* row = row_ptr(g, req);
#pragma unroll
      for (int i = 0; i < NV; ++i) hv[i] = ld_nc_v4(reinterpret_cast<const uint4*>(row + 8 * (lane + 32 * i)));
    }
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv[i]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = __uint_as_float(hw[e] << 16);
        const float hi = __uint_as_float(hw[e] & 0xFFFF0000u);
        acc = __fmaf_rn(lo, wr[i][2 * e], acc);
        acc = __fmaf_rn(hi, wr[i][2 * e + 1], acc);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    if (lane == 0) p.out[(int64_t)req * p.out_sb + (g - p.row_off[req])] = tg_logsigmoid(acc);
  }
}

template <int NV>
__global__ void __launch_bounds__(score_threads<NV>(), 1) gate_score_bulk_kernel(const ScoreParams p) {
  constexpr int kScoreRowsPerStage = score_rows<NV>();
  constexpr int ST = score_stages<NV>();
  constexpr int ROWB = NV * 512;  // bytes of one bf16 row
  extern __shared__ __align__(128) uint8_t s_smem[];
  const uint32_t sbase = smem_u32(s_smem);
  const uint32_t full = sbase + ST * kScoreRowsPerStage * ROWB;
  const uint32_t empty = full + 8 * ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int k = 0; k < ST; ++k) {
      mbar_init(full + 8u * k, 1);
      mbar_init(empty + 8u * k, kScoreRowsPerStage);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t g0 = (int64_t)blockIdx.x * p.rows_per_cta;
  const int64_t g1 = g0 + p.rows_per_cta < p.total_rows ? g0 + p.rows_per_cta : p.total_rows;
  const int n_it = (int)((g1 - g0 + kScoreRowsPerStage - 1) / kScoreRowsPerStage);

  if (warp == kScoreRowsPerStage) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int rq = 0;
      for (int it = 0; it < n_it; ++it) {
        const int k = it % ST;
        if (it >= ST && !mbar_wait(empty + 8u * k, (uint32_t)((it / ST) - 1) & 1u, p.err, ERR_SCORE)) break;
        const int64_t gb = g0 + (int64_t)it * kScoreRowsPerStage;
        const int nr = (int)(g1 - gb < kScoreRowsPerStage ? g1 - gb : kScoreRowsPerStage);
        mbar_arrive_expect_tx(full + 8u * k, (uint32_t)(nr * ROWB));
        for (int w = 0; w < nr; ++w) {
          const int64_t g = gb + w;
          while (g >= p.row_off[rq + 1]) ++rq;
          const __nv_bfloat16* row = p.h + (int64_t)rq * p.h_sb + (p.begin[rq] + (g - p.row_off[rq])) * p.h_ss;
          bulk_load(sbase + (uint32_t)((k * kScoreRowsPerStage + w) * ROWB), row, ROWB, full + 8u * k);
        }
      }
    }
    return;
  }
  // ------------------------------------------------------------------ consumers
  float wr[NV][8];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4* wp = reinterpret_cast<const float4*>(p.w + 8 * (lane + 32 * i));
    const float4 a = __ldg(wp), c = __ldg(wp + 1);
    wr[i][0] = a.x; wr[i][1] = a.y; wr[i][2] = a.z; wr[i][3] = a.w;
    wr[i][4] = c.x; wr[i][5] = c.y; wr[i][6] = c.z; wr[i][7] = c.w;
  }
  int rq = 0;
  for (int it = 0; it < n_it; ++it) {
    const int k = it % ST;
    if (!__all_sync(0xffffffffu, mbar_wait(full + 8u * k, (uint32_t)(it / ST) & 1u, p.err, ERR_SCORE))) break;
    const int64_t g = g0 + (int64_t)it * kScoreRowsPerStage + warp;
    if (g < g1) {
      const uint8_t* rowp = s_smem + (k * kScoreRowsPerStage + warp) * ROWB;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(rowp + 16 * (lane + 32 * i));
        const uint32_t hw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = __uint_as_float(hw[e] << 16);
          const float hi = __uint_as_float(hw[e] & 0xFFFF0000u);
          acc = __fmaf_rn(lo, wr[i][2 * e], acc);
          acc = __fmaf_rn(hi, wr[i][2 * e + 1], acc);
        }
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
        acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
      while (g >= p.row_off[rq + 1]) ++rq;
      if (lane == 0) p.out[(int64_t)rq * p.out_sb + (g - p.row_off[rq])] = tg_logsigmoid(acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + 8u * k);
  }
}

}  // namespace tg
