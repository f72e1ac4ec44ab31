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

// One half-warp per (row, head): lane l of the half holds elements 4l..4l+3
// and their rotate-half partners 64+4l..64+4l+3 (two 8-byte loads), so the
// rotation needs no exchange between lanes; only the sum of squares is
// reduced across the half. Each half-warp works on two heads per iteration,
// with every load of both issued before any arithmetic.
struct QkItem {
  uint2 xl, xh, wl, wh, cl, ch, sl, sh;
  __nv_bfloat16* base;
  bool active;
};

__device__ __forceinline__ void qk_load(const QkRopeParams& p, int64_t item, int hl, bool active, QkItem& it) {
  const int heads = p.n_q + p.n_k;
  const int64_t row = active ? item / heads : 0;
  const int hd = active ? (int)(item - row * heads) : 0;
  const bool is_q = hd < p.n_q;
  const __nv_bfloat16* w = is_q ? p.q_w : p.k_w;
  it.base = is_q ? p.q + row * p.ld_q + (int64_t)hd * 128 : p.k + row * p.ld_k + (int64_t)(hd - p.n_q) * 128;
  it.active = active;
  const uint2 z = make_uint2(0u, 0u);
  it.xl = it.xh = it.wl = it.wh = it.cl = it.ch = it.sl = it.sh = z;
  if (active) {
    const int64_t b = row / p.seq, s = row - b * p.seq;
    const uint2* xp = reinterpret_cast<const uint2*>(it.base);
    it.xl = xp[hl];
    it.xh = xp[16 + hl];
    const uint2* wp = reinterpret_cast<const uint2*>(w);
    it.wl = __ldg(wp + hl);
    it.wh = __ldg(wp + 16 + hl);
    const uint2* cp = reinterpret_cast<const uint2*>(p.cos + b * p.cs_sb + s * p.cs_ss);
    const uint2* sp = reinterpret_cast<const uint2*>(p.sin + b * p.cs_sb + s * p.cs_ss);
    it.cl = __ldg(cp + hl);
    it.ch = __ldg(cp + 16 + hl);
    it.sl = __ldg(sp + hl);
    it.sh = __ldg(sp + 16 + hl);
  }
}

__device__ __forceinline__ float qk_sumsq(const QkItem& it) {
  const uint32_t v[4] = {it.xl.x, it.xl.y, it.xh.x, it.xh.y};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = bf16_lo(v[e]), c = bf16_hi(v[e]);
    ss = fmaf(a, a, ss);
    ss = fmaf(c, c, ss);
  }
  return ss;
}

__device__ __forceinline__ void qk_finish(const QkRopeParams& p, const QkItem& it, float ss, int hl) {
  const float inv = rsqrtf(ss * (1.f / 128.f) + p.eps);
  const uint32_t xl[2] = {it.xl.x, it.xl.y}, xh[2] = {it.xh.x, it.xh.y};
  const uint32_t wl[2] = {it.wl.x, it.wl.y}, wh[2] = {it.wh.x, it.wh.y};
  const uint32_t cl[2] = {it.cl.x, it.cl.y}, ch[2] = {it.ch.x, it.ch.y};
  const uint32_t sl[2] = {it.sl.x, it.sl.y}, sh[2] = {it.sh.x, it.sh.y};
  uint32_t ol[2], oh[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float lo[2], hi[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float xa = u ? bf16_hi(xl[e]) : bf16_lo(xl[e]);   // element d (< 64)
      const float xb = u ? bf16_hi(xh[e]) : bf16_lo(xh[e]);   // element d + 64
      const float wa = u ? bf16_hi(wl[e]) : bf16_lo(wl[e]);
      const float wb = u ? bf16_hi(wh[e]) : bf16_lo(wh[e]);
      const float ya = round_bf16(wa * round_bf16(xa * inv));
      const float yb = round_bf16(wb * round_bf16(xb * inv));
      const float ca = u ? bf16_hi(cl[e]) : bf16_lo(cl[e]);
      const float cb = u ? bf16_hi(ch[e]) : bf16_lo(ch[e]);
      const float sa = u ? bf16_hi(sl[e]) : bf16_lo(sl[e]);
      const float sb = u ? bf16_hi(sh[e]) : bf16_lo(sh[e]);
      // rotate_half: [-x2, x1]
      lo[u] = round_bf16(round_bf16(ya * ca) + round_bf16(-yb * sa));
      hi[u] = round_bf16(round_bf16(yb * cb) + round_bf16(ya * sb));
    }
    ol[e] = pack_bf16x2(lo[0], lo[1]);
    oh[e] = pack_bf16x2(hi[0], hi[1]);
  }
  if (it.active) {
    uint2* xp = reinterpret_cast<uint2*>(it.base);
    xp[hl] = make_uint2(ol[0], ol[1]);
    xp[16 + hl] = make_uint2(oh[0], oh[1]);
  }
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
    QkItem a, b;
    qk_load(p, i0, hl, i0 < total, a);
    qk_load(p, i1, hl, i1 < total, b);
    float sa = qk_sumsq(a), sb = qk_sumsq(b);
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {  // within the half
      sa += __shfl_xor_sync(0xffffffffu, sa, off);
      sb += __shfl_xor_sync(0xffffffffu, sb, off);
    }
    qk_finish(p, a, sa, hl);
    qk_finish(p, b, sb, hl);
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
