// Fused elementwise glue of the Qwen3 decoder layers around the gated
// prefill's attention (HBM-bound; one pass over each tensor instead of the
// eager op chains). Each kernel keeps the rounding points of the
// transformers ops it replaces (modeling_qwen3: Qwen3RMSNorm, the residual
// adds of Qwen3DecoderLayer, apply_rotary_pos_emb, Qwen3MLP), which the
// reference runs through its patched attention module
// (tokengate/e2e_gate/attn/qwen3_flex_attention.py:539-551, :646-648):
//
//   add_rmsnorm   h <- bf16(h + delta);  x <- bf16(w * bf16(h * rsqrt(mean(h^2) + eps)))
//   qk_norm_rope  per q head and k head of the projections:
//                 y <- bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))
//                 x <- bf16(bf16(y * cos) + bf16(rotate_half(y) * sin))      (in place)
//   silu_mul      out <- bf16(bf16(silu(g)) * u) for a fused [g | u] row
//
// Reductions are fp32 in a fixed order (lane partials, xor butterfly), so
// they can differ from torch's reduction order in the last bit of the
// variance; everything else rounds exactly where the eager ops do.
#pragma once

#include "ptx.cuh"

namespace tg {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

struct RmsParams {
  const __nv_bfloat16* h_in;
  const __nv_bfloat16* delta;  // nullable: no residual add
  __nv_bfloat16* h_out;        // nullable when delta is null
  __nv_bfloat16* x_out;        // nullable: add only
  const __nv_bfloat16* w;
  int64_t rows;
  int64_t ld_h_in, ld_delta, ld_h_out, ld_x;  // row strides (elements)
  float eps;
  float inv_hidden;
};

// one warp per row; NV 16-byte vectors (8 elements) per lane, hidden = 256 * NV
template <int NV>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const RmsParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = warp_global; row < p.rows; row += n_warps) {
    uint4 hv[NV];
    const uint4* hin = reinterpret_cast<const uint4*>(p.h_in + row * p.ld_h_in);
#pragma unroll
    for (int i = 0; i < NV; ++i) hv[i] = ld_nc_v4(hin + lane + 32 * i);
    if (p.delta != nullptr) {
      const uint4* din = reinterpret_cast<const uint4*>(p.delta + row * p.ld_delta);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const uint4 dv = ld_nc_v4(din + lane + 32 * i);
        uint32_t* a = reinterpret_cast<uint32_t*>(&hv[i]);
        const uint32_t* d = reinterpret_cast<const uint32_t*>(&dv);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          a[e] = pack_bf16x2(bf16_lo(a[e]) + bf16_lo(d[e]), bf16_hi(a[e]) + bf16_hi(d[e]));
      }
      uint4* hout = reinterpret_cast<uint4*>(p.h_out + row * p.ld_h_out);
#pragma unroll
      for (int i = 0; i < NV; ++i) hout[lane + 32 * i] = hv[i];
    }
    if (p.x_out == nullptr) continue;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t* a = reinterpret_cast<const uint32_t*>(&hv[i]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16_lo(a[e]), hi = bf16_hi(a[e]);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss * p.inv_hidden + p.eps);
    const uint4* wv = reinterpret_cast<const uint4*>(p.w);
    uint4* xo = reinterpret_cast<uint4*>(p.x_out + row * p.ld_x);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint4 ww = __ldg(wv + lane + 32 * i);
      const uint32_t* a = reinterpret_cast<const uint32_t*>(&hv[i]);
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&ww);
      uint4 o;
      uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        ov[e] = pack_bf16x2(bf16_lo(w[e]) * round_bf16(bf16_lo(a[e]) * inv),
                            bf16_hi(w[e]) * round_bf16(bf16_hi(a[e]) * inv));
      xo[lane + 32 * i] = o;
    }
  }
}

struct QkRopeParams {
  __nv_bfloat16* q;            // (rows, n_q, 128), row stride ld_q
  __nv_bfloat16* k;            // (rows, n_k, 128), row stride ld_k
  int64_t rows;
  int64_t ld_q, ld_k;          // row strides (elements)
  int n_q, n_k;                // q heads and k heads to normalise + rotate
  int seq;                     // rows per batch entry (cos/sin are (B, seq, 128))
  const __nv_bfloat16* q_w;
  const __nv_bfloat16* k_w;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t cs_sb, cs_ss;        // cos/sin batch and row strides (elements)
  float eps;
};

// One half-warp per (row, head): lane l of the half holds elements 8l..8l+7
// (16-byte loads), its rotate-half partner elements (d +- 64) live in lane
// l ^ 8; each half-warp keeps two heads in flight per iteration.
__device__ __forceinline__ void qk_head(const QkRopeParams& p, int64_t item, int hl, bool active) {
  const int heads = p.n_q + p.n_k;
  const int64_t row = item / heads;
  const int hd = (int)(item - row * heads);
  const bool is_q = hd < p.n_q;
  const __nv_bfloat16* w = is_q ? p.q_w : p.k_w;
  __nv_bfloat16* base = is_q ? p.q + row * p.ld_q + (int64_t)hd * 128
                             : p.k + row * p.ld_k + (int64_t)(hd - p.n_q) * 128;
  uint4* xp = reinterpret_cast<uint4*>(base) + hl;
  uint4 xv = make_uint4(0u, 0u, 0u, 0u), cv = xv, sv = xv, wv = xv;
  if (active) {
    const int64_t b = row / p.seq, s = row - b * p.seq;
    xv = *xp;
    wv = __ldg(reinterpret_cast<const uint4*>(w) + hl);
    cv = __ldg(reinterpret_cast<const uint4*>(p.cos + b * p.cs_sb + s * p.cs_ss) + hl);
    sv = __ldg(reinterpret_cast<const uint4*>(p.sin + b * p.cs_sb + s * p.cs_ss) + hl);
  }
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
  float x[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    x[2 * e] = bf16_lo(xw[e]);
    x[2 * e + 1] = bf16_hi(xw[e]);
  }
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);  // within the half
  const float inv = rsqrtf(ss * (1.f / 128.f) + p.eps);
  const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
  const uint32_t* cw = reinterpret_cast<const uint32_t*>(&cv);
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(&sv);
  float y[8];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    y[2 * e] = round_bf16(bf16_lo(ww[e]) * round_bf16(x[2 * e] * inv));
    y[2 * e + 1] = round_bf16(bf16_hi(ww[e]) * round_bf16(x[2 * e + 1] * inv));
  }
  uint4 ov;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float o2[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float yy = y[2 * e + u];
      const float partner = __shfl_xor_sync(0xffffffffu, yy, 8);
      const float rot = hl < 8 ? -partner : partner;   // rotate_half: [-x2, x1]
      const float c = u ? bf16_hi(cw[e]) : bf16_lo(cw[e]);
      const float sn = u ? bf16_hi(sw[e]) : bf16_lo(sw[e]);
      o2[u] = round_bf16(round_bf16(yy * c) + round_bf16(rot * sn));
    }
    ow[e] = pack_bf16x2(o2[0], o2[1]);
  }
  if (active) *xp = ov;
}

__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkRopeParams p) {
  const int hl = threadIdx.x & 15;  // lane inside the half-warp
  const int64_t total = p.rows * (p.n_q + p.n_k);
  const int64_t half_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int64_t n_halves = ((int64_t)gridDim.x * blockDim.x) >> 4;
  // two items per iteration; the loop bound is uniform across the warp
  // (both halves iterate until every half of the warp is done)
  const int64_t warp_first = half_global & ~int64_t(1);
  for (int64_t base = warp_first; base < total; base += 2 * n_halves) {
    const int64_t i0 = base + (half_global & 1);
    const int64_t i1 = i0 + n_halves;
    qk_head(p, i0, hl, i0 < total);
    qk_head(p, i1, hl, i1 < total);
  }
}

struct SiluParams {
  const __nv_bfloat16* gu;  // (rows, 2 * inter): gate then up
  __nv_bfloat16* out;       // (rows, inter)
  int64_t rows;
  int64_t inter;            // multiple of 8
  int64_t ld_gu, ld_out;
};

__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  const int64_t vec_per_row = p.inter >> 3;
  const int64_t total = p.rows * vec_per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += stride) {
    const int64_t row = v / vec_per_row;
    const int64_t c = v - row * vec_per_row;
    const uint4* gp = reinterpret_cast<const uint4*>(p.gu + row * p.ld_gu) + c;
    const uint4 g4 = ld_nc_v4(gp);
    const uint4 u4 = ld_nc_v4(gp + vec_per_row);
    const uint32_t* g = reinterpret_cast<const uint32_t*>(&g4);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&u4);
    uint4 o4;
    uint32_t* o = reinterpret_cast<uint32_t*>(&o4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float g0 = bf16_lo(g[e]), g1 = bf16_hi(g[e]);
      const float a0 = round_bf16(g0 / (1.f + expf(-g0)));
      const float a1 = round_bf16(g1 / (1.f + expf(-g1)));
      o[e] = pack_bf16x2(a0 * bf16_lo(u[e]), a1 * bf16_hi(u[e]));
    }
    reinterpret_cast<uint4*>(p.out + row * p.ld_out)[c] = o4;
  }
}

}  // namespace tg
