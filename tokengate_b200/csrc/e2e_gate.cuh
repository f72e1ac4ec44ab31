// The finalized TokenGate gate (E2EGate) on the prefill path: the scoring
// branch's readout and the per-layer Phase-2 bias / query-scale tables.
//
// branch_score_kernel — reference gate_branch_hs (tokengate/e2e_gate/
//   gate_module/gate_forward.py:491-524) with the absorbed readout: the branch
//   is a clone of the gate layer's SwiGLU MLP whose down_proj is one row
//   (e2e_gate_module.py:332-343 of build_gate_branch, gate_forward.py:330-340),
//   computed in bf16 by CastLinear (e2e_gate_module.py:125-135) and returned
//   as bf16 (gate_forward.py:521). Given the fused [gate | up] projection GU of
//   the LN2-normalised rows, one warp per row computes
//       act_k = bf16(bf16(silu(g_k)) * u_k)          (Qwen3MLP rounding points)
//       score = bf16(sum_k act_k * w_k)               (the 1-row down_proj)
//   Arithmetic contract (reproducible bit for bit on the host): lane l takes
//   the 8-element vectors i = l, l + 32, ... in order, elements e = 0..7 in
//   order, accumulating act * w with fused multiply-adds into one fp32
//   accumulator from 0; the 32 partials are combined by the xor butterfly
//   (16, 8, 4, 2, 1); silu(g) = g / (1 + exp(-g)) with IEEE division and the
//   IEEE-only tg_exp below; the bf16 result is stored as fp32 with -0
//   replaced by +0 (the selection score compares them equal). bf16(silu(g))
//   is read from a 65536-entry table of that same function over all bf16
//   patterns (built on the stream before each readout, staged per CTA in
//   shared memory), which takes the SiLU's ~30 instructions per element off
//   the issue path of an otherwise HBM-bound pass.
//
// branch_reduce_kernel — the fused form of the same readout: the branch GEMM
//   (gemm_pair.cuh, EPI_SWIGLU_READOUT) leaves one fp32 partial dot per row
//   and 64-column half tile; this kernel adds a row's partials in index order
//   and rounds to bf16. Same activations and rounding points, another fp32
//   summation order (and the GEMM's own [gate | up] accumulation order).
//
// phase2_tables_kernel — everything between the raw score and the attention
//   kernel's operands, for all Phase-2 layers in one launch:
//     rs    = rsqrt(mean_state(x^2) + eps)           E2EGate._seq_rms_norm_qwen
//     bn    = gain * (x * rs)                        (Qwen3RMSNorm(1), :338-343)
//     b     = bf16(bn * softplus(gate_scale)[l, h])  E2EGate.forward :348-385,
//                                                    build_gate_bias_vectorized
//                                                    (.to(bf16), :986-995)
//     r     = min(log(max(t+1, 2)) / log(max(p+1, 2)), 1)     _ssmax_ratio :574-585
//     s_eff = bf16(bf16(S_eff[l, h]) * bf16(r))      _ssmax_s_eff (qwen3_flex_
//                                                    attention.py:417-431)
//     sb    = bf16(mean_h s_eff)                     _phase2_q_bias :442-455
//     bias  = bf16(b * sb)   (0 * sb off the state, bf16(-1e9) * sb in pads)
//     q_scale = s_eff        (the attention kernel rounds q * q_scale to bf16,
//                             = the reference's q * s_eff in bf16)
//   Output layout (L', B, H, n_alloc) fp32 for both tables: layer l's slice is
//   the (B, H, S) bias / q-row-scale operand of the key-bias attention.
//   The variance reduction runs in a fixed order (four partial sums per thread
//   over 16-byte vectors, xor butterfly, warps in order) and is repeated
//   identically by every CTA of a request; CTAs split the slots, the requests
//   and groups of layers so that a few hundred CTAs share the writes.
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kBranchMaxReq = 128;
constexpr int kTablesMaxReq = 128;
constexpr int kTablesThreads = 256;
constexpr int kTablesMaxLH = 4096;  // L' * H entries staged in shared memory

struct BranchParams {
  const __nv_bfloat16* gu;  // row r of request b: gu + b * gu_sb + (begin[b] + r) * gu_ss
  int64_t gu_sb, gu_ss;
  int inter;                // gate half [0, inter), up half [inter, 2 inter)
  const __nv_bfloat16* w;   // (inter,) readout row
  float* out;
  int64_t out_sb;
  int B;
  int64_t total_rows;
  int begin[kBranchMaxReq];
  int64_t row_off[kBranchMaxReq + 1];
};

// exp(y) by Cody-Waite reduction y = k ln2 + r, |r| <= ln2/2, and a degree-7
// Taylor polynomial for exp(r), scaled by 2^k in two exact power-of-two steps;
// IEEE operations only. 0 below -104, +inf above the largest finite result.
__device__ __forceinline__ float tg_exp(float y) {
  if (y < -104.0f) return 0.0f;
  if (y > 88.72283935546875f) return __int_as_float(0x7f800000);
  const float kInvLn2 = 1.44269504088896341f;
  const float kLn2Hi = 0.693145751953125f;         // 0x3F317200
  const float kLn2Lo = 1.42860682030941723212e-6f;  // ln2 - kLn2Hi
  const float k = rintf(__fmul_rn(y, kInvLn2));
  float r = __fmaf_rn(-k, kLn2Hi, y);
  r = __fmaf_rn(-k, kLn2Lo, r);  // r = y - k ln2
  float q = 1.98412698412698413e-4f;  // 1/7!
  q = __fmaf_rn(q, r, 1.38888888888888889e-3f);
  q = __fmaf_rn(q, r, 8.33333333333333333e-3f);
  q = __fmaf_rn(q, r, 4.16666666666666667e-2f);
  q = __fmaf_rn(q, r, 1.66666666666666667e-1f);
  q = __fmaf_rn(q, r, 0.5f);
  q = __fmaf_rn(q, r, 1.0f);
  q = __fmaf_rn(q, r, 1.0f);
  const int ki = (int)k;  // [-150, 128]
  const int k1 = ki > 100 ? 100 : (ki < -100 ? -100 : ki);
  const int k2 = ki - k1;
  q = __fmul_rn(q, __int_as_float((127 + k1) << 23));
  if (k2 != 0) q = __fmul_rn(q, __int_as_float((127 + k2) << 23));
  return q;
}

__device__ __forceinline__ float tg_silu(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, tg_exp(-g)));
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// bf16(silu(g)) for every bf16 bit pattern g: the branch's activation takes
// only 2^16 values, so the IEEE-only SiLU is evaluated once per pattern
// (silu_lut_kernel, on the launching stream before every readout) and the
// readout looks it up in shared memory. Entry g holds the bf16 bits of
// bf16_round(tg_silu(g)), i.e. exactly the value the per-element evaluation
// produced, NaN patterns included.
constexpr int kSiluLutEntries = 1 << 16;
constexpr int kSiluLutBytes = kSiluLutEntries * 2;
constexpr int kBranchThreads = 1024;
__device__ __align__(16) uint16_t g_silu_bf16_lut[kSiluLutEntries];

__global__ void __launch_bounds__(256) silu_lut_kernel() {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;  // the grid covers 2^16 exactly
  g_silu_bf16_lut[i] = __bfloat16_as_ushort(__float2bfloat16_rn(tg_silu(__uint_as_float(i << 16))));
}

// act = bf16(bf16(silu(g)) * u) for the two bf16 lanes of a packed word; the
// activations of the low and high halves go to a0 / a1.
__device__ __forceinline__ void branch_act2(const uint16_t* lut, uint32_t gw, uint32_t uw, float& a0,
                                            float& a1) {
  const float s0 = __uint_as_float((uint32_t)lut[gw & 0xFFFFu] << 16);
  const float s1 = __uint_as_float((uint32_t)lut[gw >> 16] << 16);
  a0 = bf16_round(__fmul_rn(s0, __uint_as_float(uw << 16)));
  a1 = bf16_round(__fmul_rn(s1, __uint_as_float(uw & 0xFFFF0000u)));
}

// One CTA per SM (the table fills 128 KB of shared memory), one warp per row.
__global__ void __launch_bounds__(kBranchThreads, 1) branch_score_kernel(const BranchParams p) {
  extern __shared__ __align__(16) uint16_t s_lut[];
  {
    const uint4* src = reinterpret_cast<const uint4*>(g_silu_bf16_lut);
    uint4* dst = reinterpret_cast<uint4*>(s_lut);
    for (int i = threadIdx.x; i < kSiluLutBytes / 16; i += kBranchThreads) dst[i] = src[i];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nv = p.inter >> 8;  // 8-element vectors per lane
  int req = 0;
  for (int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < p.total_rows; g += n_warps) {
    while (g >= p.row_off[req + 1]) ++req;
    const int64_t r = g - p.row_off[req];
    const __nv_bfloat16* row = p.gu + (int64_t)req * p.gu_sb + (int64_t)(p.begin[req] + r) * p.gu_ss;
    const uint4* gp = reinterpret_cast<const uint4*>(row) + lane;
    const uint4* up = reinterpret_cast<const uint4*>(row + p.inter) + lane;
    const uint4* wp = reinterpret_cast<const uint4*>(p.w) + lane;
    float acc = 0.f;
    int i = 0;
    // four vectors of g and u in flight per lane
    for (; i + 4 <= nv; i += 4) {
      uint4 g4[4], u4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g4[j] = ld_nc_v4(gp + 32 * (i + j));
        u4[j] = ld_nc_v4(up + 32 * (i + j));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w4 = __ldg(wp + 32 * (i + j));
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g4[j]);
        const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u4[j]);
        const uint32_t* ww = reinterpret_cast<const uint32_t*>(&w4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a0, a1;
          branch_act2(s_lut, gw[e], uw[e], a0, a1);
          acc = __fmaf_rn(a0, __uint_as_float(ww[e] << 16), acc);
          acc = __fmaf_rn(a1, __uint_as_float(ww[e] & 0xFFFF0000u), acc);
        }
      }
    }
    for (; i < nv; ++i) {
      const uint4 g4 = ld_nc_v4(gp + 32 * i), u4 = ld_nc_v4(up + 32 * i), w4 = __ldg(wp + 32 * i);
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g4);
      const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u4);
      const uint32_t* ww = reinterpret_cast<const uint32_t*>(&w4);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a0, a1;
        branch_act2(s_lut, gw[e], uw[e], a0, a1);
        acc = __fmaf_rn(a0, __uint_as_float(ww[e] << 16), acc);
        acc = __fmaf_rn(a1, __uint_as_float(ww[e] & 0xFFFF0000u), acc);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    if (lane == 0) {
      const float s = bf16_round(acc);
      p.out[(int64_t)req * p.out_sb + r] = s == 0.0f ? 0.0f : s;
    }
  }
}

// Readout of the fused branch GEMM (gemm_pair EPI_SWIGLU_READOUT): score[r]
// = bf16(sum of partial[i][r] over i = 0..n_part-1 in index order), stored as
// fp32 with -0 replaced by +0. One thread per row; launched with programmatic
// stream serialization right after the GEMM that writes the partials.
struct BranchReduceParams {
  const float* partial;  // (n_part, ld_partial)
  int64_t ld_partial;
  int n_part;
  int64_t M;
  float* out;            // (M,)
};

__global__ void __launch_bounds__(256) branch_reduce_kernel(const BranchReduceParams p) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (r >= p.M) return;
  float acc = 0.f;
  for (int i = 0; i < p.n_part; ++i) acc = __fadd_rn(acc, p.partial[(int64_t)i * p.ld_partial + r]);
  const float s = bf16_round(acc);
  p.out[r] = s == 0.0f ? 0.0f : s;
}

struct TablesParams {
  const float* scores;  // request b, state token i: scores[b * s_sb + i]
  int64_t s_sb;
  const int64_t* keep;  // (B, n_alloc) kept positions, pads included
  int64_t keep_sb;
  const float* gate_scale;  // (L', H) softplus(gate_scale)
  const float* attn_scale;  // (L', H) softplus(attn_scale)
  float* bias;              // (L', B, H, n_alloc)
  float* q_scale;           // (L', B, H, n_alloc)
  int B, L, H, n_alloc;
  int layers_per_cta;
  float eps, gain;
  int n_state[kTablesMaxReq];
  int begin[kTablesMaxReq];
  int n_kept[kTablesMaxReq];
};

// grid (slot chunks of kTablesThreads, requests, layer groups): blockIdx.z
// covers layers [z * layers_per_cta, ...). Every CTA of a request computes the
// same rs (same loads, same order); the scores row is read from L2.
__global__ void __launch_bounds__(kTablesThreads) phase2_tables_kernel(const TablesParams p) {
  __shared__ float s_g[kTablesMaxLH];
  __shared__ float s_s[kTablesMaxLH];  // bf16(S_eff) as fp32
  __shared__ float s_warp[kTablesThreads / 32];
  __shared__ float s_rs;
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int l0 = blockIdx.z * p.layers_per_cta;
  const int l1 = min(p.L, l0 + p.layers_per_cta);
  for (int i = threadIdx.x; i < (l1 - l0) * p.H; i += kTablesThreads) {
    s_g[i] = p.gate_scale[l0 * p.H + i];
    s_s[i] = bf16_round(p.attn_scale[l0 * p.H + i]);
  }
  // ---- rs of request b: four independent partial sums per thread over
  // 16-byte vectors (scalar head / tail), combined in a fixed order
  const float* x = p.scores + (int64_t)b * p.s_sb;
  const int n = p.n_state[b];
  const int head = (int)(((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) >> 2);
  const int lead = head < n ? head : n;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if ((int)threadIdx.x < lead) a0 = __fmul_rn(x[threadIdx.x], x[threadIdx.x]);
  const float4* xv = reinterpret_cast<const float4*>(x + lead);
  const int nv = (n - lead) >> 2;
#pragma unroll 4
  for (int i = threadIdx.x; i < nv; i += kTablesThreads) {
    const float4 v = __ldg(xv + i);
    a0 = __fmaf_rn(v.x, v.x, a0);
    a1 = __fmaf_rn(v.y, v.y, a1);
    a2 = __fmaf_rn(v.z, v.z, a2);
    a3 = __fmaf_rn(v.w, v.w, a3);
  }
  for (int i = lead + 4 * nv + threadIdx.x; i < n; i += kTablesThreads) a1 = __fmaf_rn(x[i], x[i], a1);
  float acc = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if (lane == 0) s_warp[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.f;
    for (int w = 0; w < kTablesThreads / 32; ++w) sum = __fadd_rn(sum, s_warp[w]);
    const float var = __fmul_rn(sum, __frcp_rn((float)n));
    s_rs = rsqrtf(__fadd_rn(var, p.eps));
  }
  __syncthreads();
  const float rs = s_rs;

  const int t = blockIdx.x * kTablesThreads + threadIdx.x;
  if (t >= p.n_alloc) return;
  const int64_t pos = p.keep[(int64_t)b * p.keep_sb + t];
  const int begin = p.begin[b];
  // 0 state token, 1 kept non-state token, 2 pad slot
  const int kind = t >= p.n_kept[b] ? 2 : ((pos >= begin && pos < (int64_t)begin + n) ? 0 : 1);
  float bn = 0.f;
  if (kind == 0) bn = __fmul_rn(p.gain, __fmul_rn(x[pos - begin], rs));
  const float m = fmaxf((float)(t + 1), 2.0f);
  const float pp = fmaxf(__fadd_rn((float)pos, 1.0f), 2.0f);
  const float r = bf16_round(fminf(__fdiv_rn(logf(m), logf(pp)), 1.0f));
  const float inv_h = __frcp_rn((float)p.H);
  const float pad_b = bf16_round(-1e9f);
  const int64_t plane = (int64_t)p.B * p.H * p.n_alloc;
  for (int l = l0; l < l1; ++l) {
    const float* gl = s_g + (l - l0) * p.H;
    const float* sl = s_s + (l - l0) * p.H;
    float sum = 0.f;
    float* qrow = p.q_scale + l * plane + ((int64_t)b * p.H) * p.n_alloc + t;
    for (int h = 0; h < p.H; ++h) {
      const float se = bf16_round(__fmul_rn(sl[h], r));
      qrow[(int64_t)h * p.n_alloc] = se;
      sum = __fadd_rn(sum, se);
    }
    const float sb = bf16_round(__fmul_rn(sum, inv_h));
    float* brow = p.bias + l * plane + ((int64_t)b * p.H) * p.n_alloc + t;
    for (int h = 0; h < p.H; ++h) {
      const float base = kind == 0 ? bf16_round(__fmul_rn(bn, gl[h])) : (kind == 2 ? pad_b : 0.0f);
      brow[(int64_t)h * p.n_alloc] = bf16_round(__fmul_rn(base, sb));
    }
  }
}

}  // namespace tg
