// Gate scorer: score = logsigmoid(w . h_row) over the state rows of each
// request — the synthetic linear gate of the gated prefill (a 1-wide fp32
// readout plus log-sigmoid; the reference scores with gate(h_art.to(fp32)),
// tokengate/e2e_gate/gate_module/gate_forward.py:1396-1407).
//
// HBM-bound. gate_score_stream_kernel: one warp per state row over a
// resident grid (one CTA of 32 warps per SM), each lane loading its 16-byte
// vectors of the row with non-allocating loads, w staged once per CTA in
// shared memory. (A bulk-copy form, rows streamed by the TMA engine into a
// shared-memory ring for consumer warps, measured 35.8 / 227 us for 1 / 8
// requests against 31.7 / 180 us for this one, and was replaced.)
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
};

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

// gate_score_stream_kernel: one warp per row over a resident grid (one CTA
// of 32 warps per SM, 16 for rows over 4 KB), each lane loading its NV
// 16-byte vectors of the row with non-allocating loads; w is staged once per
// CTA in shared memory (fp32, read by each lane as the same 8-element slices
// its vectors cover). The same arithmetic as the kernels above.
template <int NV>
__host__ __device__ constexpr int score_stream_threads() { return NV <= 8 ? 1024 : 512; }

template <int NV>
__global__ void __launch_bounds__(score_stream_threads<NV>(), 1) gate_score_stream_kernel(const ScoreParams p) {
  extern __shared__ __align__(16) float s_w[];  // NV * 256 floats
  for (int i = threadIdx.x; i < NV * 64; i += blockDim.x)
    reinterpret_cast<float4*>(s_w)[i] = __ldg(reinterpret_cast<const float4*>(p.w) + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int req = 0;
  for (int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < p.total_rows; g += n_warps) {
    while (g >= p.row_off[req + 1]) ++req;
    const __nv_bfloat16* row = p.h + (int64_t)req * p.h_sb + (int64_t)(p.begin[req] + (g - p.row_off[req])) * p.h_ss;
    uint4 hv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) hv[i] = ld_nc_v4(reinterpret_cast<const uint4*>(row + 8 * (lane + 32 * i)));
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float4 wa = reinterpret_cast<const float4*>(s_w)[2 * (lane + 32 * i)];
      const float4 wb = reinterpret_cast<const float4*>(s_w)[2 * (lane + 32 * i) + 1];
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint32_t hw[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc = __fmaf_rn(__uint_as_float(hw[e] << 16), wv[2 * e], acc);
        acc = __fmaf_rn(__uint_as_float(hw[e] & 0xFFFF0000u), wv[2 * e + 1], acc);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    if (lane == 0) p.out[(int64_t)req * p.out_sb + (g - p.row_off[req])] = tg_logsigmoid(acc);
  }
}

}  // namespace tg
