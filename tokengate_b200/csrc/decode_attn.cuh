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
// of kDecKeys keys for all G query heads that share the kv head. It first
// streams the chunk's K and V rows into shared memory with asynchronous
// 16-byte copies (all of them in flight at once), then thread t scores key
// t from shared memory, the CTA reduces the chunk's max and sum, and 4
// stripes of 32 threads accumulate P V (each warp reads whole 256-byte V
// rows). One chunk writes the output directly; more chunks write (m, l, O)
// partials that a second kernel merges.
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kDecKeys = 128;     // keys per CTA, one per thread for the scores
constexpr int kDecThreads = 128;
constexpr int kDecD = 128;
constexpr int kDecPart = 4 + kDecD;  // m, l, 2 pad, O[128] per (row, head, chunk): 16-byte aligned records
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecRowBytes = kDecD * 2;
// dynamic shared memory: K chunk (16-byte pieces of row t at piece ^ (t & 15),
// so that thread t reading piece c of its row hits distinct banks across a
// quarter-warp), V chunk (rows in order), then the per-head scratch
constexpr int kDecSmK = 0;
constexpr int kDecSmV = kDecSmK + kDecKeys * kDecRowBytes;
constexpr int kDecSmRest = kDecSmV + kDecKeys * kDecRowBytes;
template <int G>
constexpr int dec_smem_bytes() {
  return kDecSmRest + (G * kDecD + G * kDecKeys + G * kDecWarps + 2 * G + kDecWarps * G * kDecD) * 4;
}

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
  float* part;  // [B][Hq][n_chunks][kDecPart], 16-byte aligned
  int Hq, Hkv, n_chunks;
  float scale_log2;  // softmax_scale * log2(e)
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Launched with programmatic stream serialization: before the wait for the
// kernel that appends this step's key, the chunk's prefix rows (those below
// n_prefix, allocated in every caller's cache) are only prefetched into L2,
// which cannot return stale data; q, the key count, every cache row, the
// bias and the outputs are read or written after the wait.
template <int G>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  float* qs = reinterpret_cast<float*>(dsm + kDecSmRest);   // [G][128]
  float* pr = qs + G * kDecD;                                 // [G][keys]
  float* red = pr + G * kDecKeys;                             // [G][warps]
  float* stat = red + G * kDecWarps;                          // [2][G]
  float* obuf = stat + 2 * G;                                 // [warps][G][128]

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int j0 = chunk * kDecKeys;
  if (j0 + t < p.n_prefix) {
    const int64_t j = j0 + t;
    prefetch_l2_bulk(p.k + (int64_t)b * p.k_sb + j * p.k_ss + (int64_t)kvh * p.k_sh, 256u);
    prefetch_l2_bulk(p.v + (int64_t)b * p.v_sb + j * p.v_ss + (int64_t)kvh * p.v_sh, 256u);
  }
  griddep_wait();
  griddep_launch_dependents();
  const int n_keys = p.n_keys_dev != nullptr ? min(__ldg(p.n_keys_dev), p.n_keys) : p.n_keys;
  const int kend = min(kDecKeys, n_keys - j0);  // keys of this chunk (<= 0: none)

  // ---- stream the chunk's K and V rows into shared memory (asynchronous)
  {
    const uint32_t sk = smem_u32(dsm + kDecSmK), sv = smem_u32(dsm + kDecSmV);
    const uint8_t* kb = reinterpret_cast<const uint8_t*>(p.k + (int64_t)b * p.k_sb + (int64_t)kvh * p.k_sh);
    const uint8_t* vb = reinterpret_cast<const uint8_t*>(p.v + (int64_t)b * p.v_sb + (int64_t)kvh * p.v_sh);
    for (int idx = t; idx < kDecKeys * 16; idx += kDecThreads) {
      const int key = idx >> 4, c = idx & 15;
      if (key < kend) {
        const int64_t j = j0 + key;
        cp_async16(sk + key * kDecRowBytes + ((c ^ (key & 15)) << 4), kb + j * p.k_ss * 2 + c * 16);
        cp_async16(sv + key * kDecRowBytes + (c << 4), vb + j * p.v_ss * 2 + c * 16);
      }
    }
    cp_async_commit();
  }
  // q of the G heads on this kv head, scaled and rounded as the reference does
  for (int idx = t; idx < G * kDecD; idx += kDecThreads) {
    const int g = idx / kDecD, d = idx - g * kDecD, h = kvh * G + g;
    float qv = __bfloat162float(p.q[(int64_t)b * p.q_sb + (int64_t)h * p.q_sh + d]);
    if (p.q_scale != nullptr) qv = bf16r(qv * bf16r(p.q_scale[(int64_t)b * p.qs_sb + h]));
    qs[g * kDecD + d] = qv;
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- scores: thread t takes key j0 + t
  const int j = j0 + t;
  const int nv = __ldg(p.n_valid + b);
  const bool valid = t < kend && !(j < p.n_prefix && j >= nv);
  float sc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) sc[g] = 0.f;
  if (valid) {
    const uint4* kr = reinterpret_cast<const uint4*>(dsm + kDecSmK + t * kDecRowBytes);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint4 kv = kr[c ^ (t & 15)];
      const uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float k0 = __uint_as_float(w[e] << 16), k1 = __uint_as_float(w[e] & 0xFFFF0000u);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          sc[g] = fmaf(qs[g * kDecD + 8 * c + 2 * e], k0, sc[g]);
          sc[g] = fmaf(qs[g * kDecD + 8 * c + 2 * e + 1], k1, sc[g]);
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
    if (lane == 0) red[g * kDecWarps + warp] = m;
  }
  __syncthreads();
  if (t < G) {
    float m = red[t * kDecWarps];
#pragma unroll
    for (int w = 1; w < kDecWarps; ++w) m = fmaxf(m, red[t * kDecWarps + w]);
    stat[t] = m;
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float m = stat[g];
    const float pv = (m == -INFINITY || sc[g] == -INFINITY) ? 0.f : exp2f(sc[g] - m);
    pr[g * kDecKeys + t] = pv;
    float l = pv;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    sc[g] = l;
  }
  __syncthreads();  // red reused below
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) red[g * kDecWarps + warp] = sc[g];
  }
  __syncthreads();
  if (t < G) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) l += red[t * kDecWarps + w];
    stat[G + t] = l;
  }

  // ---- P V from shared memory: warp w takes keys w, w + 4, ...; lane l dims 4l..4l+3
  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  const uint8_t* vs = dsm + kDecSmV + 8 * lane;
#pragma unroll 4
  for (int kk = warp; kk < kend; kk += kDecWarps) {
    const uint2 vv = *reinterpret_cast<const uint2*>(vs + kk * kDecRowBytes);
    const float v0 = __uint_as_float(vv.x << 16), v1 = __uint_as_float(vv.x & 0xFFFF0000u);
    const float v2 = __uint_as_float(vv.y << 16), v3 = __uint_as_float(vv.y & 0xFFFF0000u);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pk = pr[g * kDecKeys + kk];
      acc[g][0] = fmaf(pk, v0, acc[g][0]);
      acc[g][1] = fmaf(pk, v1, acc[g][1]);
      acc[g][2] = fmaf(pk, v2, acc[g][2]);
      acc[g][3] = fmaf(pk, v3, acc[g][3]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) obuf[(warp * G + g) * kDecD + 4 * lane + e] = acc[g][e];
  __syncthreads();

  // ---- sum the stripes; one chunk: normalize and store, else a partial
  for (int idx = t; idx < G * kDecD; idx += kDecThreads) {
    const int g = idx / kDecD, d = idx - g * kDecD, h = kvh * G + g;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) o += obuf[(w * G + g) * kDecD + d];
    if (p.n_chunks == 1) {
      const float l = stat[G + g];
      p.out[(int64_t)b * p.o_sb + (int64_t)h * p.o_sh + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
    } else {
      float* rec = p.part + (((int64_t)b * p.Hq + h) * p.n_chunks + chunk) * kDecPart;
      rec[4 + d] = o;
      if (d == 0) {
        rec[0] = stat[g];
        rec[1] = stat[G + g];
      }
    }
  }
}

// Merges the chunks' (m, l, O) of one (b, h): the chunks' max first, then
// each of 8 warps folds a stripe of chunks (lane l: dims 4l..4l+3, 16-byte
// loads), and the stripes are summed through shared memory.
constexpr int kCombThreads = 256;
__global__ void __launch_bounds__(kCombThreads) decode_combine_kernel(const DecodeParams p) {
  __shared__ float red[kCombThreads / 32];
  __shared__ float part_o[kCombThreads / 32][kDecD];
  __shared__ float part_l[kCombThreads / 32];
  griddep_wait();  // launched with programmatic stream serialization
  griddep_launch_dependents();
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* rec = p.part + ((int64_t)b * p.Hq + h) * p.n_chunks * kDecPart;
  float m = -INFINITY;
  for (int c = t; c < p.n_chunks; c += kCombThreads) m = fmaxf(m, rec[(int64_t)c * kDecPart]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < kCombThreads / 32; ++w) m = fmaxf(m, red[w]);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  float l = 0.f;
  if (m != -INFINITY) {
#pragma unroll 4
    for (int c = warp; c < p.n_chunks; c += kCombThreads / 32) {
      const float* r = rec + (int64_t)c * kDecPart;
      const float mc = r[0];
      if (mc == -INFINITY) continue;
      const float w = exp2f(mc - m);
      const float4 v = *reinterpret_cast<const float4*>(r + 4 + 4 * lane);
      l = fmaf(w, r[1], l);
      o.x = fmaf(w, v.x, o.x);
      o.y = fmaf(w, v.y, o.y);
      o.z = fmaf(w, v.z, o.z);
      o.w = fmaf(w, v.w, o.w);
    }
  }
  part_o[warp][4 * lane + 0] = o.x;
  part_o[warp][4 * lane + 1] = o.y;
  part_o[warp][4 * lane + 2] = o.z;
  part_o[warp][4 * lane + 3] = o.w;
  if (lane == 0) part_l[warp] = l;
  __syncthreads();
  if (t < kDecD) {
    float ot = 0.f, lt = 0.f;
#pragma unroll
    for (int w = 0; w < kCombThreads / 32; ++w) {
      ot += part_o[w][t];
      lt += part_l[w];
    }
    p.out[(int64_t)b * p.o_sb + (int64_t)h * p.o_sh + t] = __float2bfloat16_rn(lt > 0.f ? ot / lt : 0.f);
  }
}

}  // namespace tg
