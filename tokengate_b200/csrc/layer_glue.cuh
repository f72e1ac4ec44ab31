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
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = warp_global; row < p.rows; row += n_warps) {
    uint4 hv[NV];
    const uint4* hin = reinterpret_cast<const uint4*>(p.h_in + row * p.ld_h_in);
#pragma unroll
    for (int i = 0; i < NV; ++i) hv[i] = ld_nc_v4(hin + lane + 32 * i);
    // up to hidden 2048 the gains are loaded with the row (one round trip
    // less on the few-row decode path); wider rows load them after the sum
    constexpr bool kEarlyW = NV <= 8;
    const uint4* wv = reinterpret_cast<const uint4*>(p.w);
    uint4 wgt[kEarlyW ? NV : 1];
    if (kEarlyW && p.x_out != nullptr) {
#pragma unroll
      for (int i = 0; i < (kEarlyW ? NV : 1); ++i) wgt[i] = __ldg(wv + lane + 32 * i);
    }
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
    uint4* xo = reinterpret_cast<uint4*>(p.x_out + row * p.ld_x);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint4 ww = kEarlyW ? wgt[kEarlyW ? i : 0] : __ldg(wv + lane + 32 * i);
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
  // decode append (k_cache nullable; one token per batch row, seq == 1): the
  // finished k heads and the v heads are also written to slot *slot_dev of
  // the (B, cap, n_k, 128) caches (batch stride kc_sb, slot stride kc_ss)
  const __nv_bfloat16* v;      // (rows, n_k, 128), row stride ld_v
  int64_t ld_v;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t kc_sb, kc_ss;
  const int64_t* slot_dev;
  int split;                   // warps per row: each takes every split-th group of 2 * kQkBatch heads
};

// One warp per row (with few rows, `split` warps per row, each taking every
// split-th group of heads): the row's cos / sin and the two norm gains are
// loaded once, then each half-warp takes every other head of the row, up to
// kQkBatch heads per half with every load issued before any arithmetic. Lane
// l of a half holds elements 4l..4l+3 of its head and their rotate-half
// partners 64+4l..64+4l+3 (two 8-byte loads), so the rotation needs no
// exchange between lanes; only the sum of squares is reduced across the half.
constexpr int kQkBatch = 4;

struct QkRow {
  uint2 cl, ch, sl, sh;  // cos / sin of this lane's elements
};

// rounds two floats to bf16 with one paired conversion
__device__ __forceinline__ void round_bf16x2(float& a, float& b) {
  const uint32_t w = pack_bf16x2(a, b);
  a = bf16_lo(w);
  b = bf16_hi(w);
}

__device__ __forceinline__ void qk_finish(const uint2 xl2, const uint2 xh2, const uint2 wl2, const uint2 wh2,
                                          const QkRow& cs, float ss, float eps, uint2& out_l, uint2& out_h) {
  const float inv = rsqrtf(ss * (1.f / 128.f) + eps);
  const uint32_t xl[2] = {xl2.x, xl2.y}, xh[2] = {xh2.x, xh2.y};
  const uint32_t wl[2] = {wl2.x, wl2.y}, wh[2] = {wh2.x, wh2.y};
  const uint32_t cl[2] = {cs.cl.x, cs.cl.y}, ch[2] = {cs.ch.x, cs.ch.y};
  const uint32_t sl[2] = {cs.sl.x, cs.sl.y}, sh[2] = {cs.sh.x, cs.sh.y};
  uint32_t ol[2], oh[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    // elements d, d + 1 (< 64) and their rotate-half partners d + 64, d + 65;
    // every rounding point of the eager ops, two values per conversion
    float ya0 = bf16_lo(xl[e]) * inv, ya1 = bf16_hi(xl[e]) * inv;
    float yb0 = bf16_lo(xh[e]) * inv, yb1 = bf16_hi(xh[e]) * inv;
    round_bf16x2(ya0, ya1);
    round_bf16x2(yb0, yb1);
    ya0 *= bf16_lo(wl[e]);
    ya1 *= bf16_hi(wl[e]);
    yb0 *= bf16_lo(wh[e]);
    yb1 *= bf16_hi(wh[e]);
    round_bf16x2(ya0, ya1);
    round_bf16x2(yb0, yb1);
    // rotate_half: [-x2, x1]
    float pc0 = ya0 * bf16_lo(cl[e]), pc1 = ya1 * bf16_hi(cl[e]);
    float ps0 = -yb0 * bf16_lo(sl[e]), ps1 = -yb1 * bf16_hi(sl[e]);
    float qc0 = yb0 * bf16_lo(ch[e]), qc1 = yb1 * bf16_hi(ch[e]);
    float qs0 = ya0 * bf16_lo(sh[e]), qs1 = ya1 * bf16_hi(sh[e]);
    round_bf16x2(pc0, pc1);
    round_bf16x2(ps0, ps1);
    round_bf16x2(qc0, qc1);
    round_bf16x2(qs0, qs1);
    ol[e] = pack_bf16x2(pc0 + ps0, pc1 + ps1);
    oh[e] = pack_bf16x2(qc0 + qs0, qc1 + qs1);
  }
  out_l = make_uint2(ol[0], ol[1]);
  out_h = make_uint2(oh[0], oh[1]);
}

__device__ __forceinline__ float qk_sumsq(const uint2 xl, const uint2 xh) {
  const uint32_t v[4] = {xl.x, xl.y, xh.x, xh.y};
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float a = bf16_lo(v[e]), c = bf16_hi(v[e]);
    ss = fmaf(a, a, ss);
    ss = fmaf(c, c, ss);
  }
  return ss;
}

// Launched with programmatic stream serialization (the norm gains are read
// after the wait too: a caller may have just written them).
__global__ void __launch_bounds__(256, 3) qk_norm_rope_kernel(const QkRopeParams p) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;    // lane inside the half-warp
  const int half = lane >> 4;  // heads half, half + 2, half + 4, ...
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int heads = p.n_q + p.n_k;
  const uint2* qwp = reinterpret_cast<const uint2*>(p.q_w);
  const uint2* kwp = reinterpret_cast<const uint2*>(p.k_w);
  const uint2 qwl = __ldg(qwp + hl), qwh = __ldg(qwp + 16 + hl);
  const uint2 kwl = __ldg(kwp + hl), kwh = __ldg(kwp + 16 + hl);
  const int64_t n_items = p.rows * p.split;
  for (int64_t item = warp_global; item < n_items; item += n_warps) {
    const int64_t row = p.split == 1 ? item : item / p.split;
    const int gsel = (int)(item - row * p.split);
    const int64_t b = row / p.seq, s = row - b * p.seq;
    QkRow cs;
    {
      const uint2* cp = reinterpret_cast<const uint2*>(p.cos + b * p.cs_sb + s * p.cs_ss);
      const uint2* sp = reinterpret_cast<const uint2*>(p.sin + b * p.cs_sb + s * p.cs_ss);
      cs.cl = __ldg(cp + hl);
      cs.ch = __ldg(cp + 16 + hl);
      cs.sl = __ldg(sp + hl);
      cs.sh = __ldg(sp + 16 + hl);
    }
    __nv_bfloat16* qrow = p.q + row * p.ld_q;
    __nv_bfloat16* krow = p.k + row * p.ld_k;
    __nv_bfloat16* kcrow = nullptr;
    __nv_bfloat16* vcrow = nullptr;
    if (p.k_cache != nullptr) {
      const int64_t slot = __ldg(p.slot_dev);
      kcrow = p.k_cache + row * p.kc_sb + slot * p.kc_ss;
      vcrow = p.v_cache + row * p.kc_sb + slot * p.kc_ss;
      // v heads: straight copy into the cache (by the row's first warp)
      const uint2* vrow = reinterpret_cast<const uint2*>(p.v + row * p.ld_v);
      for (int hd = half; gsel == 0 && hd < p.n_k; hd += 2) {
        const uint2 a = vrow[hd * 32 + hl], c = vrow[hd * 32 + 16 + hl];
        uint2* dst = reinterpret_cast<uint2*>(vcrow + (int64_t)hd * 128);
        dst[hl] = a;
        dst[16 + hl] = c;
      }
    }
    // the head loop is uniform across the warp (the shuffles need every lane)
    for (int h0 = gsel * 2 * kQkBatch; h0 < heads; h0 += p.split * 2 * kQkBatch) {
      uint2 xl[kQkBatch], xh[kQkBatch];
      float ss[kQkBatch];
#pragma unroll
      for (int i = 0; i < kQkBatch; ++i) {
        const int hd = h0 + 2 * i + half;
        xl[i] = xh[i] = make_uint2(0u, 0u);
        if (hd < heads) {
          const uint2* xp = reinterpret_cast<const uint2*>(
              hd < p.n_q ? qrow + (int64_t)hd * 128 : krow + (int64_t)(hd - p.n_q) * 128);
          xl[i] = xp[hl];
          xh[i] = xp[16 + hl];
        }
      }
#pragma unroll
      for (int i = 0; i < kQkBatch; ++i) ss[i] = qk_sumsq(xl[i], xh[i]);
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) {  // within the half
#pragma unroll
        for (int i = 0; i < kQkBatch; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], off);
      }
#pragma unroll
      for (int i = 0; i < kQkBatch; ++i) {
        const int hd = h0 + 2 * i + half;
        if (hd < heads) {
          const bool is_q = hd < p.n_q;
          uint2 ol, oh;
          qk_finish(xl[i], xh[i], is_q ? qwl : kwl, is_q ? qwh : kwh, cs, ss[i], p.eps, ol, oh);
          uint2* xp = reinterpret_cast<uint2*>(is_q ? qrow + (int64_t)hd * 128
                                                    : krow + (int64_t)(hd - p.n_q) * 128);
          xp[hl] = ol;
          xp[16 + hl] = oh;
          if (!is_q && kcrow != nullptr) {
            uint2* cp = reinterpret_cast<uint2*>(kcrow + (int64_t)(hd - p.n_q) * 128);
            cp[hl] = ol;
            cp[16 + hl] = oh;
          }
        }
      }
    }
  }
}

struct SiluParams {
  const __nv_bfloat16* gu;  // (rows, 2 * inter): gate then up
  __nv_bfloat16* out;       // (rows, inter)
  int64_t rows;
  int64_t inter;            // multiple of 8
  int64_t ld_gu, ld_out;
};

// One block per row at a time (grid-stride over rows), threads across the
// row's 16-byte vectors, up to kSiluUnroll vectors of gate and up loaded per
// thread before any arithmetic; no integer division per vector.
constexpr int kSiluUnroll = 4;

__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluParams p) {
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int vpr = (int)(p.inter >> 3);
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const uint4* gp = reinterpret_cast<const uint4*>(p.gu + row * p.ld_gu);
    uint4* op = reinterpret_cast<uint4*>(p.out + row * p.ld_out);
    for (int c0 = threadIdx.x; c0 < vpr; c0 += kSiluUnroll * 256) {
      uint4 g4[kSiluUnroll], u4[kSiluUnroll];
#pragma unroll
      for (int j = 0; j < kSiluUnroll; ++j) {
        const int c = c0 + j * 256;
        if (c < vpr) {
          g4[j] = ld_nc_v4(gp + c);
          u4[j] = ld_nc_v4(gp + vpr + c);
        }
      }
#pragma unroll
      for (int j = 0; j < kSiluUnroll; ++j) {
        const int c = c0 + j * 256;
        if (c < vpr) {
          const uint32_t* g = reinterpret_cast<const uint32_t*>(&g4[j]);
          const uint32_t* u = reinterpret_cast<const uint32_t*>(&u4[j]);
          uint4 o4;
          uint32_t* o = reinterpret_cast<uint32_t*>(&o4);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float g0 = bf16_lo(g[e]), g1 = bf16_hi(g[e]);
            float a0 = g0 / (1.f + expf(-g0));
            float a1 = g1 / (1.f + expf(-g1));
            round_bf16x2(a0, a1);
            o[e] = pack_bf16x2(a0 * bf16_lo(u[e]), a1 * bf16_hi(u[e]));
          }
          op[c] = o4;
        }
      }
    }
  }
}

}  // namespace tg
