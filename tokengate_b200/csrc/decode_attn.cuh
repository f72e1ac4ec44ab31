// Decode attention: one query token per (batch row, head) against the gated
// KV cache — the decode side of the reference's gated generation
// (tokengate/e2e_gate/decode/gate_decode.py:139-235, the folded Phase-2 form
// of qwen3_flex_attention.py:374-415 and :978-1116).
//
// Per (b, h):  out = softmax_j( scale * (q' . k_j) + m_j ) V
//   q'   = bf16(q * bf16(q_scale[b, h]))            (q_scale optional: the
//          per-step scaled-softmax query scale gamma * r of FormDecodeState)
//   m_j  = bias[b, h, j]  for prefix keys j < n_valid[b]
//          -inf           for prefix pad slots n_valid[b] <= j < n_prefix
//          0              for keys appended by decode, n_prefix <= j < n_keys
// The cache is (B, cap, Hkv, D) with the prefix (kept tokens, or the full
// Phase-1 cache below the gate) first and decode tokens appended after it.
//
// HBM-bound split-K design: a CTA takes one kv head of one row and a chunk
// of kDecKeys keys for all G query heads that share the kv head; thread t
// scores key t (its K row read once, q from shared memory), the CTA reduces
// the chunk's max and sum, then 8 stripes of 32 threads accumulate P V with
// 8-byte loads (each warp reads whole 256-byte V rows). One chunk writes the
// output directly; more chunks write (m, l, O) partials that a second kernel
// merges.
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kDecKeys = 256;
constexpr int kDecThreads = 256;
constexpr int kDecD = 128;
constexpr int kDecPart = 2 + kDecD;  // m, l, O[128] per (row, head, chunk)

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh;
  const float* q_scale;  // (B, Hq) nullable
  int64_t qs_sb;
  const __nv_bfloat16* k;
  int64_t k_sb, k_ss, k_sh;
  const __nv_bfloat16* v;
  int64_t v_sb, v_ss, v_sh;
  const float* bias;  // (B, Hq|1, n_prefix) nullable, score units
  int64_t bias_sb, bias_sh;
  const int32_t* n_valid;  // (B,)
  int n_prefix, n_keys;    // n_keys: the keys, or with n_keys_dev their upper bound (grid size)
  const int32_t* n_keys_dev;  // nullable: the actual key count, read on the device
  __nv_bfloat16* out;
  int64_t o_sb, o_sh;
  float* part;  // [B][Hq][n_chunks][kDecPart]
  int Hq, Hkv, n_chunks;
  float scale_log2;  // softmax_scale * log2(e)
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <int G>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(const DecodeParams p) {
  __shared__ float qs[G][kDecD];
  __shared__ float pr[G][kDecKeys];
  __shared__ float red[G][kDecThreads / 32];
  __shared__ float stat[2][G];
  __shared__ float obuf[kDecThreads / 32][G][kDecD];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int j0 = chunk * kDecKeys;
  const int n_keys = p.n_keys_dev != nullptr ? min(__ldg(p.n_keys_dev), p.n_keys) : p.n_keys;

  // q of the G heads on this kv head, scaled and rounded as the reference does
  for (int idx = t; idx < G * kDecD; idx += kDecThreads) {
    const int g = idx / kDecD, d = idx - g * kDecD, h = kvh * G + g;
    float qv = __bfloat162float(p.q[(int64_t)b * p.q_sb + (int64_t)h * p.q_sh + d]);
    if (p.q_scale != nullptr) qv = bf16r(qv * bf16r(p.q_scale[(int64_t)b * p.qs_sb + h]));
    qs[g][d] = qv;
  }
  __syncthreads();

  // ---- scores: thread t takes key j0 + t
  const int j = j0 + t;
  const int nv = __ldg(p.n_valid + b);
  const bool valid = j < n_keys && !(j < p.n_prefix && j >= nv);
  float sc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) sc[g] = 0.f;
  if (valid) {
    const uint4* kr = reinterpret_cast<const uint4*>(p.k + (int64_t)b * p.k_sb + (int64_t)j * p.k_ss +
                                                     (int64_t)kvh * p.k_sh);
#pragma unroll
    for (int c = 0; c < kDecD / 8; ++c) {
      const uint4 kv = __ldg(kr + c);
      const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float k0 = __uint_as_float(w[e] << 16), k1 = __uint_as_float(w[e] & 0xFFFF0000u);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          sc[g] = fmaf(qs[g][8 * c + 2 * e], k0, sc[g]);
          sc[g] = fmaf(qs[g][8 * c + 2 * e + 1], k1, sc[g]);
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (!valid) {
      sc[g] = -INFINITY;
    } else {
      float bj = 0.f;
      if (p.bias != nullptr && j < p.n_prefix)
        bj = __ldg(p.bias + (int64_t)b * p.bias_sb + (int64_t)(kvh * G + g) * p.bias_sh + j);
      sc[g] = sc[g] * p.scale_log2 + bj * 1.4426950408889634f;
    }
  }

  // ---- chunk max and sum per head
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = sc[g];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[g][warp] = m;
  }
  __syncthreads();
  if (t < G) {
    float m = red[t][0];
#pragma unroll
    for (int w = 1; w < kDecThreads / 32; ++w) m = fmaxf(m, red[t][w]);
    stat[0][t] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float m = stat[0][g];
    const float pv = (m == -INFINITY || sc[g] == -INFINITY) ? 0.f : exp2f(sc[g] - m);
    pr[g][t] = pv;
    float l = pv;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    sc[g] = l;
  }
  __syncthreads();  // red reused below
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) red[g][warp] = sc[g];
  }
  __syncthreads();
  if (t < G) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kDecThreads / 32; ++w) l += red[t][w];
    stat[1][t] = l;
  }

  // ---- P V: warp w takes keys j0 + w, j0 + w + 8, ...; lane l dims 4l..4l+3
  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  const int kend = min(kDecKeys, n_keys - j0);  // <= 0 for a chunk past the keys
  const __nv_bfloat16* vbase = p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh + 4 * lane;
#pragma unroll 8
  for (int kk = warp; kk < kend; kk += kDecThreads / 32) {
    const uint2 vv = __ldg(reinterpret_cast<const uint2*>(vbase + (int64_t)(j0 + kk) * p.v_ss));
    const float v0 = __uint_as_float(vv.x << 16), v1 = __uint_as_float(vv.x & 0xFFFF0000u);
    const float v2 = __uint_as_float(vv.y << 16), v3 = __uint_as_float(vv.y & 0xFFFF0000u);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pk = pr[g][kk];
      acc[g][0] = fmaf(pk, v0, acc[g][0]);
      acc[g][1] = fmaf(pk, v1, acc[g][1]);
      acc[g][2] = fmaf(pk, v2, acc[g][2]);
      acc[g][3] = fmaf(pk, v3, acc[g][3]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) obuf[warp][g][4 * lane + e] = acc[g][e];
  __syncthreads();

  // ---- sum the 8 stripes; one chunk: normalize and store, else a partial
  for (int idx = t; idx < G * kDecD; idx += kDecThreads) {
    const int g = idx / kDecD, d = idx - g * kDecD, h = kvh * G + g;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kDecThreads / 32; ++w) o += obuf[w][g][d];
    if (p.n_chunks == 1) {
      const float l = stat[1][g];
      p.out[(int64_t)b * p.o_sb + (int64_t)h * p.o_sh + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
    } else {
      float* rec = p.part + (((int64_t)b * p.Hq + h) * p.n_chunks + chunk) * kDecPart;
      rec[2 + d] = o;
      if (d == 0) {
        rec[0] = stat[0][g];
        rec[1] = stat[1][g];
      }
    }
  }
}

// Merges the chunks' (m, l, O) of one (b, h): 128 threads, one dim each.
__global__ void __launch_bounds__(kDecD) decode_combine_kernel(const DecodeParams p) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float* rec = p.part + ((int64_t)b * p.Hq + h) * p.n_chunks * kDecPart;
  float m = -INFINITY;
  for (int c = 0; c < p.n_chunks; ++c) m = fmaxf(m, rec[c * kDecPart]);
  float l = 0.f, o = 0.f;
  if (m != -INFINITY) {
    for (int c = 0; c < p.n_chunks; ++c) {
      const float mc = rec[c * kDecPart];
      if (mc == -INFINITY) continue;
      const float w = exp2f(mc - m);
      l = fmaf(w, rec[c * kDecPart + 1], l);
      o = fmaf(w, rec[c * kDecPart + 2 + d], o);
    }
  }
  p.out[(int64_t)b * p.o_sb + (int64_t)h * p.o_sh + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
}

}  // namespace tg
