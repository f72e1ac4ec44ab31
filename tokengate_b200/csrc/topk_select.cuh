// Top-K selection of state tokens and the kept-position list — radix select
// with the scores in registers: one CTA per request up to 8192 scores, a
// cluster of CTAs per request beyond (topk_select_cluster_kernel), the
// global-memory kernel past 8 x 32768.
//
// Reference semantics (tokengate/e2e_gate/gate_module/gate_forward.py):
//   topk = torch.topk(score, K_clamped).indices                   :84-99
//   keep = [0, start) ++ start + sort(topk) ++ [end, seq_len)        :1417-1421
//   gate_bias[:n_kept] = score at kept state tokens, 0 elsewhere;
//   gate_bias[n_kept:] = -1e9                                        :968-1036, :1463-1469
// with the order fixed as (score descending, index ascending), so among
// scores tied at the K-th value the lower indices are kept.
//
// Algorithm: scores are mapped to order-preserving uint32 keys; four 8-bit
// digit passes (MSB first, warp-aggregated shared-memory histograms) find the
// exact K-th key T and how many keys equal to T are taken. A compaction in
// index order then writes the selected positions already sorted: each thread
// owns a contiguous chunk, two block scans give its count of T-equal keys
// before it and its output offset.
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kTopkMaxReq = 64;
constexpr int kTopkThreads = 1024;
constexpr int kTopkRegKeys = 32;  // keys per thread held in registers (n_state <= 32768)

struct TopkParams {
  const float* scores;
  int64_t s_sb;
  int64_t* keep;
  int64_t keep_sb;
  void* bias_out;
  int64_t bias_sb;
  int bias_dtype;  // 0 fp32, 1 bf16
  int64_t* topk_local;
  int64_t tl_sb;
  int n_alloc;
  int n_state[kTopkMaxReq];
  int k[kTopkMaxReq];
  int begin[kTopkMaxReq];
  int seq_len[kTopkMaxReq];
};

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// inverse of order_key
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// exclusive block scan of one value per thread (kTopkThreads threads)
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = s_warp[lane];
    uint32_t wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += o;
    }
    s_warp[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const uint32_t res = s_warp[warp] + incl - v;
  __syncthreads();
  return res;
}

__device__ __forceinline__ void store_bias(const TopkParams& p, int b, int q, float v) {
  if (p.bias_out == nullptr) return;
  if (p.bias_dtype == 0)
    reinterpret_cast<float*>(p.bias_out)[(int64_t)b * p.bias_sb + q] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(p.bias_out)[(int64_t)b * p.bias_sb + q] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void topk_write_fixed(const TopkParams& p, int b, int begin, int K,
                                                 int end, int n_kept, int64_t* keep);

// Large requests (n_state > kTopkThreads * kTopkRegKeys): keys are re-read
// from global memory (L1/L2 resident) in every pass.
__global__ void __launch_bounds__(kTopkThreads, 1) topk_select_kernel(const TopkParams p) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_bin, s_need, s_total;

  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.n_state[b];
  const int K = p.k[b];
  const int begin = p.begin[b];
  const int end = begin + n;
  const int seq_len = p.seq_len[b];
  const int n_kept = begin + K + (seq_len - end);
  const float* sc = p.scores + (int64_t)b * p.s_sb;

  // ---- radix select: exact K-th largest key T and how many of T to take
  uint32_t prefix = 0, mask = 0, need = (uint32_t)K;
  const int n_iter = (n + kTopkThreads - 1) / kTopkThreads;
  for (int d = 3; d >= 0; --d) {
    const int shift = 8 * d;
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
    for (int it = 0; it < n_iter; ++it) {
      const int i = it * kTopkThreads + tid;
      uint32_t digit = 256;  // 256 = not a candidate
      if (i < n) {
        const uint32_t key = order_key(__ldg(sc + i));
        if ((key & mask) == prefix) digit = (key >> shift) & 255u;
      }
      const uint32_t peers = __match_any_sync(0xffffffffu, digit);
      if (digit < 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      // lane l owns bins 255-8l .. 248-8l (descending key order)
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = hist[255 - (lane * 8 + e)];
        sum += c[e];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const uint32_t excl = incl - sum;
      if (excl < need && need <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run + c[e] >= need) {
            s_bin = 255 - (lane * 8 + e);
            s_need = need - run;
            break;
          }
          run += c[e];
        }
      }
    }
    __syncthreads();
    prefix |= s_bin << shift;
    mask |= 255u << shift;
    need = s_need;
    __syncthreads();
  }
  const uint32_t T = prefix;

  // ---- compaction in index order
  const int chunk = (n + kTopkThreads - 1) / kTopkThreads;
  const int c0 = min(n, tid * chunk), c1 = min(n, c0 + chunk);
  uint32_t n_gt = 0, n_eq = 0;
  for (int i = c0; i < c1; ++i) {
    const uint32_t key = order_key(__ldg(sc + i));
    n_gt += key > T;
    n_eq += key == T;
  }
  const uint32_t eq_before = block_excl_scan(n_eq, s_warp, &s_total);
  const uint32_t take_eq =
      (need > eq_before) ? min(n_eq, need - eq_before) : 0u;  // T-equal keys this thread keeps
  const uint32_t n_sel = n_gt + take_eq;
  const uint32_t out_before = block_excl_scan(n_sel, s_warp, &s_total);

  int64_t* keep = p.keep + (int64_t)b * p.keep_sb;
  int64_t* tl = p.topk_local ? p.topk_local + (int64_t)b * p.tl_sb : nullptr;
  uint32_t rank = out_before, eq_seen = 0;
  for (int i = c0; i < c1; ++i) {
    const float x = __ldg(sc + i);
    const uint32_t key = order_key(x);
    bool sel = key > T;
    if (key == T) {
      sel = eq_seen < take_eq;
      ++eq_seen;
    }
    if (sel) {
      keep[begin + rank] = begin + i;
      if (tl) tl[rank] = i;
      store_bias(p, b, begin + (int)rank, x);
      ++rank;
    }
  }

  // ---- prefix, suffix and padding slots
  topk_write_fixed(p, b, begin, K, end, n_kept, keep);
}

// Prefix, suffix and padding slots of the kept list (everything but the
// selected state tokens).
__device__ __forceinline__ void topk_write_fixed(const TopkParams& p, int b, int begin, int K,
                                                 int end, int n_kept, int64_t* keep) {
  for (int q = threadIdx.x; q < p.n_alloc; q += kTopkThreads) {
    if (q < begin) {
      keep[q] = q;
      store_bias(p, b, q, 0.f);
    } else if (q >= begin + K && q < n_kept) {
      keep[q] = end + (q - begin - K);
      store_bias(p, b, q, 0.f);
    } else if (q >= n_kept) {
      keep[q] = 0;
      store_bias(p, b, q, -1e9f);
    }
  }
}

// Requests with n_state <= kTopkThreads * KPT: thread t owns the KPT
// consecutive scores [t*KPT, (t+1)*KPT), loaded once (16-byte loads when
// aligned) and kept in registers as order-preserving keys through the four
// digit passes and the index-order compaction.
template <int KPT>
__global__ void __launch_bounds__(kTopkThreads, 1) topk_select_reg_kernel(const TopkParams p) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_bin, s_need, s_total;

  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.n_state[b];
  const int K = p.k[b];
  const int begin = p.begin[b];
  const int end = begin + n;
  const int n_kept = begin + K + (p.seq_len[b] - end);
  const float* sc = p.scores + (int64_t)b * p.s_sb;
  const int i0 = tid * KPT;

  uint32_t key[KPT];
  const bool vec = ((reinterpret_cast<uintptr_t>(sc) & 15) == 0) && (i0 + KPT <= n);
  if (vec) {
#pragma unroll
    for (int e = 0; e < KPT; e += 4) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(sc + i0 + e));
      key[e] = order_key(f.x); key[e + 1] = order_key(f.y);
      key[e + 2] = order_key(f.z); key[e + 3] = order_key(f.w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < KPT; ++e) key[e] = order_key((i0 + e < n) ? __ldg(sc + i0 + e) : 0.f);
  }
  const int n_mine = max(0, min(KPT, n - i0));  // valid keys of this thread

  uint32_t prefix = 0, mask = 0, need = (uint32_t)K;
#pragma unroll 1
  for (int d = 3; d >= 0; --d) {
    const int shift = 8 * d;
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < KPT; ++e) {
      const uint32_t digit = (e < n_mine && (key[e] & mask) == prefix) ? (key[e] >> shift) & 255u : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, digit);
      if (digit < 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = hist[255 - (lane * 8 + e)];
        sum += c[e];
      }
      uint32_t incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const uint32_t excl = incl - sum;
      if (excl < need && need <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run + c[e] >= need) {
            s_bin = 255 - (lane * 8 + e);
            s_need = need - run;
            break;
          }
          run += c[e];
        }
      }
    }
    __syncthreads();
    prefix |= s_bin << shift;
    mask |= 255u << shift;
    need = s_need;
  }
  const uint32_t T = prefix;

  uint32_t n_gt = 0, n_eq = 0;
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    n_gt += (e < n_mine && key[e] > T);
    n_eq += (e < n_mine && key[e] == T);
  }
  const uint32_t eq_before = block_excl_scan(n_eq, s_warp, &s_total);
  const uint32_t take_eq = (need > eq_before) ? min(n_eq, need - eq_before) : 0u;
  const uint32_t out_before = block_excl_scan(n_gt + take_eq, s_warp, &s_total);

  int64_t* keep = p.keep + (int64_t)b * p.keep_sb;
  int64_t* tl = p.topk_local ? p.topk_local + (int64_t)b * p.tl_sb : nullptr;
  uint32_t rank = out_before, eq_seen = 0;
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    if (e < n_mine) {
      bool sel = key[e] > T;
      if (key[e] == T) {
        sel = eq_seen < take_eq;
        ++eq_seen;
      }
      if (sel) {
        keep[begin + rank] = begin + i0 + e;
        if (tl) tl[rank] = i0 + e;
        store_bias(p, b, begin + (int)rank, key_value(key[e]));
        ++rank;
      }
    }
  }
  topk_write_fixed(p, b, begin, K, end, n_kept, keep);
}

// A cluster of C = gridDim.x CTAs per request (grid (C, requests)), for
// requests past one CTA's registers (KPT = 32: up to kTopkMaxCluster x 32768
// scores) or to spread a 32 k request over four CTAs (KPT = 8). CTA r holds
// the scores [1024 KPT r, 1024 KPT (r + 1)) in registers as
// topk_select_reg_kernel holds its own. Each digit pass's histogram is the sum
// of the CTAs' shared-memory histograms, read through distributed shared
// memory in rank order, so every CTA takes the same decision; in the
// compaction, CTA r's offsets add the T-equal and selected counts of CTAs
// 0..r-1, keeping the index order of the whole request. Same results as the
// single-CTA kernels. Every CTA runs the same cluster barriers (none returns
// early), so each barrier completes.
constexpr int kTopkMaxCluster = 8;
template <int KPT>
__global__ void __launch_bounds__(kTopkThreads, 1) topk_select_cluster_kernel(const TopkParams p) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_warp[32];
  __shared__ uint32_t s_bin, s_need, s_total;
  __shared__ uint32_t s_cnt[2];  // this CTA's T-equal and above-T key counts
  __shared__ uint32_t s_off[2];  // T-equal and selected keys of the lower-rank CTAs

  const int C = (int)gridDim.x;
  const uint32_t rank_c = cluster_ctarank();
  const int b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.n_state[b];
  const int K = p.k[b];
  const int begin = p.begin[b];
  const int end = begin + n;
  const int n_kept = begin + K + (p.seq_len[b] - end);
  const float* sc = p.scores + (int64_t)b * p.s_sb;
  const int i0 = (int)rank_c * (kTopkThreads * KPT) + tid * KPT;

  uint32_t key[KPT];
  const bool vec = ((reinterpret_cast<uintptr_t>(sc) & 15) == 0) && (i0 + KPT <= n);
  if (vec) {
#pragma unroll
    for (int e = 0; e < KPT; e += 4) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(sc + i0 + e));
      key[e] = order_key(f.x); key[e + 1] = order_key(f.y);
      key[e + 2] = order_key(f.z); key[e + 3] = order_key(f.w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < KPT; ++e) key[e] = order_key((i0 + e < n) ? __ldg(sc + i0 + e) : 0.f);
  }
  const int n_mine = max(0, min(KPT, n - i0));

  uint32_t prefix = 0, mask = 0, need = (uint32_t)K;
#pragma unroll 1
  for (int d = 3; d >= 0; --d) {
    const int shift = 8 * d;
    if (tid < 256) hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < KPT; ++e) {
      const uint32_t digit = (e < n_mine && (key[e] & mask) == prefix) ? (key[e] >> shift) & 255u : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, digit);
      if (digit < 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[digit], __popc(peers));
    }
    cluster_sync_all();  // every CTA's histogram of this pass is complete
    if (warp == 0) {
      uint32_t c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t a = smem_u32(&hist[255 - (lane * 8 + e)]);
        uint32_t v = 0;
        for (int q = 0; q < C; ++q) v += ld_shared_cluster_u32(mapa_shared(a, (uint32_t)q));
        c[e] = v;
        sum += v;
      }
      uint32_t incl = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const uint32_t excl = incl - sum;
      if (excl < need && need <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run + c[e] >= need) {
            s_bin = 255 - (lane * 8 + e);
            s_need = need - run;
            break;
          }
          run += c[e];
        }
      }
    }
    cluster_sync_all();  // the remote reads are done before any CTA clears its histogram
    prefix |= s_bin << shift;
    mask |= 255u << shift;
    need = s_need;
  }
  const uint32_t T = prefix;

  uint32_t n_gt = 0, n_eq = 0;
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    n_gt += (e < n_mine && key[e] > T);
    n_eq += (e < n_mine && key[e] == T);
  }
  const uint32_t eq_local = block_excl_scan(n_eq, s_warp, &s_total);
  if (tid == 0) s_cnt[0] = s_total;
  (void)block_excl_scan(n_gt, s_warp, &s_total);
  if (tid == 0) s_cnt[1] = s_total;
  cluster_sync_all();  // every CTA's counts are published
  if (tid == 0) {
    uint32_t eq_b = 0, sel_b = 0;
    for (int q = 0; q < (int)rank_c; ++q) {
      const uint32_t E = ld_shared_cluster_u32(mapa_shared(smem_u32(&s_cnt[0]), (uint32_t)q));
      const uint32_t G = ld_shared_cluster_u32(mapa_shared(smem_u32(&s_cnt[1]), (uint32_t)q));
      const uint32_t take = need > eq_b ? min(E, need - eq_b) : 0u;
      sel_b += G + take;
      eq_b += E;
    }
    s_off[0] = eq_b;
    s_off[1] = sel_b;
  }
  cluster_sync_all();  // no CTA leaves while another still reads its counts
  const uint32_t eq_before = s_off[0] + eq_local;
  const uint32_t take_eq = (need > eq_before) ? min(n_eq, need - eq_before) : 0u;
  const uint32_t out_before = s_off[1] + block_excl_scan(n_gt + take_eq, s_warp, &s_total);

  int64_t* keep = p.keep + (int64_t)b * p.keep_sb;
  int64_t* tl = p.topk_local ? p.topk_local + (int64_t)b * p.tl_sb : nullptr;
  uint32_t rank = out_before, eq_seen = 0;
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    if (e < n_mine) {
      bool sel = key[e] > T;
      if (key[e] == T) {
        sel = eq_seen < take_eq;
        ++eq_seen;
      }
      if (sel) {
        keep[begin + rank] = begin + i0 + e;
        if (tl) tl[rank] = i0 + e;
        store_bias(p, b, begin + (int)rank, key_value(key[e]));
        ++rank;
      }
    }
  }
  if (rank_c == 0) topk_write_fixed(p, b, begin, K, end, n_kept, keep);
}

}  // namespace tg
