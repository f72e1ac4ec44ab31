// Causal GQA attention with an additive per-key bias — sm_100a forward kernel.
//
// Semantics follow the reference key-bias operator (softmax(scale*q.k + b)v,
// kernels/fa2bias/keybias.patch:387-461 and the FlexAttention score_mod
// tokengate/e2e_gate/attn/flex_attention_utils.py:174-198); the design is
// Blackwell-native:
//
//  * one CTA owns TWO 128-row query tiles that share one KV head: two heads
//    of a GQA group at the same rows (Hq/Hkv even), or two consecutive row
//    blocks of one head otherwise. K/V tiles are loaded once for both. In a
//    launch of about one wave the heaviest row blocks run one head per CTA
//    (tile 1 unused): those CTAs are the launch's span, and one tile's key
//    block costs ~1.8 us against ~2.0 for two.
//  * the key bias rides in the QK product: each K tile gets a 16-column
//    extension [b0_hi, b0_lo, b1_hi, b1_lo, 0...] (bias / scale split into two
//    bf16 that sum to it to ~16 bits) and each Q tile a constant one-hot
//    extension selecting its head's pair, so one extra K=16 MMA step adds
//    the bias in fp32 and the softmax never touches it;
//  * warp 8 streams Q/K/V through TMA (128-byte swizzle, no multicast) into a
//    2-stage ring and writes each K stage's bias extension (32-byte swizzle)
//    from the fp32 bias in global memory;
//  * warp 9 issues tcgen05.mma (M=128, N=128, K=16 steps): S_t = Q_t K^T
//    (+ bias step) into TMEM, then O_t += P_t V with P read straight from
//    TMEM (it overwrites the last 64 columns of S_t as packed bf16 pairs);
//  * warps 0-3 / 4-7 are the softmax warpgroups of tile 0 / tile 1: one TMEM
//    lane (= one query row) per thread, the 128-key row in registers,
//    p = 2^(S*scale*log2e - m) with one packed FFMA2 per pair and exp2 on the
//    MUFU. The running max m comes from the first key block's row max; later
//    blocks use it as it is (no max pass) and only take their true max, move
//    m and rescale O in TMEM when their row sum shows p above 2^16. Numerator
//    and denominator share the stale max, so the result is exact.
//  * TMEM: S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512) columns.
//
// Issue order of the MMA warp per key block j (tile 0, tile 1):
//   O0 += P0_j V_j ; S0 = Q0 K_{j+1} ; O1 += P1_j V_j ; S1 = Q1 K_{j+1}
// so each softmax warpgroup works while the tensor core runs the other
// tile's two MMAs. The tensor pipe executes one thread's MMAs in issue order,
// which is what makes writing S_t after the P_t V read safe.
#pragma once

#include "ptx.cuh"

namespace tg {

constexpr int kAttnBM = 128;
constexpr int kAttnBN = 128;
constexpr int kAttnD = 128;
constexpr int kAttnThreads = 384;  // 3 warpgroups: softmax 0, softmax 1, producer/MMA
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kAttnTileBytes = kAttnBM * kAttnD * 2;  // 32 KB: one Q/K/V tile
constexpr int kAttnHalfBytes = kAttnTileBytes / 2;    // 16 KB: 64 columns (one TMA box)
constexpr int kExtBytes = 128 * 32;                   // 4 KB: 128 rows x 16 bf16 extension
constexpr uint32_t kAttnPCol = 64;  // P_t (packed bf16 pairs) lives in columns [64, 128) of S_t

// dynamic shared memory layout (offsets from a 1024-byte aligned base)
constexpr int kSmQ = 0;                                  // 2 tiles
constexpr int kSmK = kSmQ + 2 * kAttnTileBytes;          // 2 stages
constexpr int kSmV = kSmK + 2 * kAttnTileBytes;          // 2 stages
constexpr int kSmKExt = kSmV + 2 * kAttnTileBytes;       // 2 stages: K bias extension
constexpr int kSmQExt = kSmKExt + 2 * kExtBytes;         // 2 tiles: Q one-hot extension
constexpr int kSmBar = kSmQExt + 2 * kExtBytes;
constexpr int kNumBars = 17;

// pairs q (0..31 per 64-key half) with (q & kAttnPolyMask) == kAttnPolyMask take
// exp2 on the FMA pipe (degree-3 polynomial) instead of the MUFU; a mask of
// -1 (the default) keeps every exp2 on the MUFU. Moving 1/8 or 1/4 of the
// pairs to the FMA pipe measured no faster on B200 (and slower with the key
// bias, whose variant then spills).
#ifndef TG_ATTN_POLY_MASK
#define TG_ATTN_POLY_MASK -1
#endif
constexpr int kAttnPolyMask = TG_ATTN_POLY_MASK;

constexpr int kSmTmemSlot = kSmBar + kNumBars * 8;
constexpr int kAttnSmemBytes = kSmTmemSlot + 16 + 1024;  // + alignment slack

// barrier indices
enum {
  BAR_Q = 0,
  BAR_K_FULL = 1,   // 2
  BAR_K_EMPTY = 3,  // 2
  BAR_V_FULL = 5,   // 2
  BAR_V_EMPTY = 7,  // 2
  BAR_S_FULL = 9,   // 2 (per tile)
  BAR_O_FULL = 11,  // 2 (per tile)
  BAR_MMA_DONE = 13,
  BAR_Q_READY = 14, // softmax warps scaled their Q rows (only with a row scale)
  BAR_P_FULL = 15   // 2 (per tile)
};

// device error bits
enum : unsigned int {
  ERR_ATTN_Q = 1u << 0,
  ERR_ATTN_K_EMPTY = 1u << 1,
  ERR_ATTN_V_EMPTY = 1u << 2,
  ERR_ATTN_K_FULL = 1u << 3,
  ERR_ATTN_V_FULL = 1u << 4,
  ERR_ATTN_P_FULL = 1u << 5,
  ERR_ATTN_S_FULL = 1u << 6,
  ERR_ATTN_O_FULL = 1u << 7,
  ERR_ATTN_DRAIN = 1u << 8,
  ERR_ATTN_Q_READY = 1u << 9,
};

struct AttnParams {
  const float* bias;
  int64_t bias_sb, bias_sh;
  const float* qscale;
  int64_t qs_sb, qs_sh;
  __nv_bfloat16* out;
  int64_t o_sb, o_ss, o_sh;
  float* lse;
  int64_t lse_sb, lse_sh;
  int B, Sq, Sk, Hq, Hkv, G;
  int pair_heads;  // 1: tiles are heads (2p, 2p+1) at one row block
  int causal;
  int n_mblocks;   // ceil(Sq / 128)
  int n_kblocks;   // ceil(Sk / 128)
  int heads_per_unit_row;  // pair_heads ? Hq/2 : Hq
  int n_single_rows;       // pair_heads: the heaviest row blocks run one head per CTA
  float scale;             // softmax_scale
  float scale_log2;        // softmax_scale * log2(e)
  unsigned int* err;
};

struct TileInfo {
  int head;
  int m0;
  int nblk;  // key blocks this tile needs (0 = tile unused)
};

// Work unit of this CTA. Units are numbered heavy rows first. With head
// pairs, the first n_single_rows * Hq units are the last n_single_rows row
// blocks, one head each (tile 1 unused), and the rest the other row blocks,
// two heads each: splitting the longest units shortens the launch's tail when
// it runs in about one wave.
__device__ __forceinline__ void attn_unit(const AttnParams& p, TileInfo (&ti)[2]) {
  int u = blockIdx.x;
  bool single = false;
  if (p.pair_heads) {
    const int n_single = p.n_single_rows * p.Hq;
    if (u < n_single) {
      single = true;
      const int h = u % p.Hq;
      const int mb = p.n_mblocks - 1 - u / p.Hq;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        ti[t].head = h;
        ti[t].m0 = mb * kAttnBM;
      }
    } else {
      u -= n_single;
      const int hp = u % p.heads_per_unit_row;
      const int mb = p.n_mblocks - p.n_single_rows - 1 - u / p.heads_per_unit_row;  // heavy rows first
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        ti[t].head = 2 * hp + t;
        ti[t].m0 = mb * kAttnBM;
      }
    }
  } else {
    const int h = u % p.heads_per_unit_row;
    const int n_pairs = (p.n_mblocks + 1) / 2;
    const int pr = n_pairs - 1 - u / p.heads_per_unit_row;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      ti[t].head = h;
      ti[t].m0 = (2 * pr + t) * kAttnBM;
    }
  }
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    if (ti[t].m0 >= p.Sq) {
      ti[t].nblk = 0;
    } else if (p.causal) {
      ti[t].nblk = min(p.n_kblocks, ti[t].m0 / kAttnBN + 1);
    } else {
      ti[t].nblk = p.n_kblocks;
    }
  }
  if (single) ti[1].nblk = 0;
}

// all lanes wait; the result is made warp-uniform
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, unsigned int* err,
                                          unsigned int code) {
  const bool ok = mbar_wait(bar, parity, err, code);
  return __all_sync(0xffffffffu, ok);
}

// byte offset of 16-byte chunk c (0/1) of row r in a 32-byte-swizzled tile
__device__ __forceinline__ uint32_t sw32_off(int r, int c) {
  return (uint32_t)r * 32u + ((uint32_t)(c ^ ((r >> 2) & 1)) << 4);
}

// byte offset of 16-byte chunk c (0..7) of row r in one 128-byte-swizzled
// 64-column half of a Q/K/V tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}

// (hi, lo) bf16 pair whose sum is v to ~16 bits; -inf -> (-inf, 0)
__device__ __forceinline__ uint32_t split_bf16x2(float v) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  const float hf = __bfloat162float(hi);
  const __nv_bfloat16 lo = __float2bfloat16_rn(isfinite(hf) ? v - hf : 0.f);
  return (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
}

// row max of the 128 raw logits a thread holds: eight independent 3-input
// max chains (their latency, not the instruction count, bounds this step),
// then a short tree
__device__ __forceinline__ float attn_row_max(const uint32_t (&sv)[128]) {
  float mxa[8];
#pragma unroll
  for (int a = 0; a < 8; ++a) mxa[a] = fmaxf(__uint_as_float(sv[2 * a]), __uint_as_float(sv[2 * a + 1]));
#pragma unroll
  for (int c = 16; c < 128; c += 16) {
#pragma unroll
    for (int a = 0; a < 8; ++a)
      mxa[a] = fmax3(mxa[a], __uint_as_float(sv[c + 2 * a]), __uint_as_float(sv[c + 2 * a + 1]));
  }
  return fmaxf(fmax3(mxa[0], mxa[1], mxa[2]), fmaxf(fmax3(mxa[3], mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
}

// p = 2^(S*c2 - m) for one row of 128 logits: one FFMA2 per pair and exp2 on
// the MUFU, except for the pairs the poly mask sends to the FMA pipe (clamped
// polynomial). P goes to TMEM as packed bf16 pairs, 32 keys per store
// (asynchronous stores: the caller waits before publishing); returns the row
// sum of the fp32 p.
__device__ __forceinline__ float attn_exp_store(const uint32_t (&sv)[128], float c2, float m, uint32_t tS) {
  const float2 c22 = make_float2(c2, c2);
  const float2 negm = make_float2(-m, -m);
  const float a_sat = c2 * (1.f / kPolyRange);
  const float b_sat = (-m - kPolyLo) * (1.f / kPolyRange);
  float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                  make_float2(0.f, 0.f)};
#pragma unroll
  for (int qt = 0; qt < 4; ++qt) {
    uint32_t pk[16];
#pragma unroll
    for (int qq = 0; qq < 16; ++qq) {
      const int q = (qt & 1) * 16 + qq;  // pair index inside its 64-key half
      const int c = qt * 32 + 2 * qq;
      float2 pp;
      if (kAttnPolyMask >= 0 && (q & kAttnPolyMask) == kAttnPolyMask) {
        pp = exp2_poly2_sat(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1]), a_sat, b_sat);
      } else {
        const float2 d = __ffma2_rn(make_float2(__uint_as_float(sv[c]), __uint_as_float(sv[c + 1])),
                                    c22, negm);
        pp.x = ex2_approx(d.x);
        pp.y = ex2_approx(d.y);
      }
      ls[q & 3] = __fadd2_rn(ls[q & 3], pp);
      pk[qq] = pack_bf16x2(pp.x, pp.y);
    }
    tmem_st16_async(tS + kAttnPCol + qt * 16, pk);
  }
  const float2 lsum = __fadd2_rn(__fadd2_rn(ls[0], ls[1]), __fadd2_rn(ls[2], ls[3]));
  return lsum.x + lsum.y;
}

template <bool kHasBias>
__global__ void __launch_bounds__(kAttnThreads, 1)
    keybias_attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + kSmQ, sK = sbase + kSmK, sV = sbase + kSmV;
  const uint32_t sKExt = sbase + kSmKExt, sQExt = sbase + kSmQExt;
  const uint32_t sBar = sbase + kSmBar;
  auto bar = [&](int i) { return sBar + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  constexpr bool has_bias = kHasBias;
  const bool has_qscale = p.qscale != nullptr;

  TileInfo ti[2];
  attn_unit(p, ti);
  const int kvh = ti[0].head / p.G;
  const int nblk = max(ti[0].nblk, ti[1].nblk);

  if (threadIdx.x == 0) {
    mbar_init(bar(BAR_Q), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(BAR_K_FULL + s), 1);
      mbar_init(bar(BAR_K_EMPTY + s), 1);
      mbar_init(bar(BAR_V_FULL + s), 1);
      mbar_init(bar(BAR_V_EMPTY + s), 1);
      mbar_init(bar(BAR_S_FULL + s), 1);
      mbar_init(bar(BAR_P_FULL + s), 4);
      mbar_init(bar(BAR_O_FULL + s), 1);
    }
    mbar_init(bar(BAR_MMA_DONE), 1);
    mbar_init(bar(BAR_Q_READY), 8);
    fence_mbar_init();
  }
  if (has_bias && threadIdx.x < 256) {
    // Q extension: row r of tile t holds ones in the columns of its head's
    // (hi, lo) pair: (2t, 2t+1) for a head pair, (0, 1) for two row blocks.
    // K extension: chunk 1 (columns 8..15) is zero in both stages; chunk 0
    // is rewritten per key block by the producer.
    const int t = threadIdx.x >> 7, r = threadIdx.x & 127;
    const int col = p.pair_heads ? 2 * t : 0;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    w[col >> 1] = 0x3F803F80u;  // two bf16 ones
    uint8_t* qe = smem + kSmQExt + t * kExtBytes;
    *reinterpret_cast<uint4*>(qe + sw32_off(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(qe + sw32_off(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
    uint8_t* ke = smem + kSmKExt + t * kExtBytes;  // t doubles as the stage here
    *reinterpret_cast<uint4*>(ke + sw32_off(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched with programmatic stream serialization: the prologue above
  // (barriers, the Q extension, TMEM) overlaps the previous kernel's drain;
  // Q/K/V, the bias and the row scale are read only after this wait.
  griddep_wait();
  griddep_launch_dependents();

  // Register split (launch: 384 threads x 168 = 64512): the two softmax
  // warpgroups take 192 each, the producer/MMA warpgroup keeps 120:
  // 2*128*192 + 128*120 = 64512 (no spills in either role or either bias
  // variant; the producer's bias-extension code needs more than 72). Each
  // role's code is dominated by its own setmaxnreg so the allocator gives it
  // that budget.
  if (warp >= kProducerWarp) {
  setmaxnreg_dec<120>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int nq = (ti[0].nblk > 0) + (ti[1].nblk > 0);
      mbar_arrive_expect_tx(bar(BAR_Q), nq * kAttnTileBytes);
      for (int t = 0; t < 2; ++t) {
        if (ti[t].nblk == 0) continue;
        const uint32_t dst = sQ + t * kAttnTileBytes;
        tma_load_4d(dst, &tm_q, bar(BAR_Q), 0, ti[t].head, ti[t].m0, b);
        tma_load_4d(dst + kAttnHalfBytes, &tm_q, bar(BAR_Q), 64, ti[t].head, ti[t].m0, b);
      }
    }
    const float inv_scale = 1.f / p.scale;
    const float* brow0 = has_bias ? p.bias + (int64_t)b * p.bias_sb + (int64_t)ti[0].head * p.bias_sh : nullptr;
    const float* brow1 = has_bias ? p.bias + (int64_t)b * p.bias_sb + (int64_t)ti[1].head * p.bias_sh : nullptr;
    int issued = 0;
    for (int j = 0; j < nblk; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      // this lane's four key rows of block j: bias of both tiles' heads
      float bv0[4], bv1[4];
      if (has_bias) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int key = j * kAttnBN + lane + 32 * u;
          bv0[u] = key < p.Sk ? __ldg(brow0 + key) : 0.f;
          bv1[u] = key < p.Sk ? __ldg(brow1 + key) : 0.f;
        }
      }
      if (!warp_wait(bar(BAR_K_EMPTY + s), ph ^ 1, p.err, ERR_ATTN_K_EMPTY)) break;
      if (has_bias) {
        uint8_t* ke = smem + kSmKExt + s * kExtBytes;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = lane + 32 * u;
          const uint32_t w0 = split_bf16x2(bv0[u] * inv_scale);
          const uint32_t w1 = p.pair_heads ? split_bf16x2(bv1[u] * inv_scale) : 0u;
          *reinterpret_cast<uint4*>(ke + sw32_off(r, 0)) = make_uint4(w0, w1, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) {
        const uint32_t dst = sK + s * kAttnTileBytes;
        mbar_arrive_expect_tx(bar(BAR_K_FULL + s), kAttnTileBytes);
        tma_load_4d(dst, &tm_k, bar(BAR_K_FULL + s), 0, kvh, j * kAttnBN, b);
        tma_load_4d(dst + kAttnHalfBytes, &tm_k, bar(BAR_K_FULL + s), 64, kvh, j * kAttnBN, b);
      }
      if (!warp_wait(bar(BAR_V_EMPTY + s), ph ^ 1, p.err, ERR_ATTN_V_EMPTY)) {
        issued = 2 * j + 1;
        break;
      }
      if (lane == 0) {
        const uint32_t dst = sV + s * kAttnTileBytes;
        mbar_arrive_expect_tx(bar(BAR_V_FULL + s), kAttnTileBytes);
        tma_load_4d(dst, &tm_v, bar(BAR_V_FULL + s), 0, kvh, j * kAttnBN, b);
        tma_load_4d(dst + kAttnHalfBytes, &tm_v, bar(BAR_V_FULL + s), 64, kvh, j * kAttnBN, b);
      }
      issued = 2 * j + 2;
    }
    // drain: make sure no TMA write is still in flight when the CTA retires
    // (only matters when a wait above gave up).
    {
      const int nk = (issued + 1) / 2;  // K loads issued
      const int nv = issued / 2;        // V loads issued
      for (int s = 0; s < 2; ++s) {
        // last use of stage s among the issued loads
        const int lastk = (nk - 1 - s) >= 0 ? ((nk - 1 - s) & ~1) + s : -1;
        const int lastv = (nv - 1 - s) >= 0 ? ((nv - 1 - s) & ~1) + s : -1;
        if (lastk >= 0) mbar_wait(bar(BAR_K_FULL + s), (lastk >> 1) & 1, p.err, ERR_ATTN_DRAIN);
        if (lastv >= 0) mbar_wait(bar(BAR_V_FULL + s), (lastv >> 1) & 1, p.err, ERR_ATTN_DRAIN);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs this code (descriptors and control flow stay
    // warp-uniform) and one elected lane issues each MMA and commit: issued
    // from a warp-converged loop a tcgen05.mma costs the issuer ~25 clocks,
    // from a single-lane branch ~49 (measured on B200), against 64 clocks of
    // tensor-pipe time per 128x128x16 step. The steady-state loop below
    // carries nothing but the MMAs, the waits they depend on and the commits
    // the other roles wait for.
    {
      constexpr uint32_t kIdescQK = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t kIdescPV = umma_idesc_bf16(128, 128, 0, 1);
      auto issue_qk = [&](int t, int s) {
        const uint32_t qa = sQ + t * kAttnTileBytes, ka = sK + s * kAttnTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kAttnHalfBytes + (kk & 3) * 32;
          if (elect_one())
            umma_ss(tmem + t * 128u, umma_desc_sw128(qa + off, 16, 1024),
                    umma_desc_sw128(ka + off, 16, 1024), kIdescQK, kk > 0);
        }
        if constexpr (kHasBias)
          if (elect_one())
            umma_ss(tmem + t * 128u, umma_desc_sw32(sQExt + t * kExtBytes, 16, 256),
                    umma_desc_sw32(sKExt + s * kExtBytes, 16, 256), kIdescQK, 1u);
      };
      auto issue_pv = [&](int t, int s, bool acc) {
        const uint32_t va = sV + s * kAttnTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if (elect_one())
            umma_ts(tmem + 256u + t * 128u, tmem + t * 128u + kAttnPCol + kk * 8,
                    umma_desc_sw128(va + kk * 2048, kAttnHalfBytes, 1024), kIdescPV,
                    (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = warp_wait(bar(BAR_Q), 0, p.err, ERR_ATTN_Q);
      if (ok && has_qscale) ok = warp_wait(bar(BAR_Q_READY), 0, p.err, ERR_ATTN_Q_READY);
      if (ok && nblk > 0) ok = warp_wait(bar(BAR_K_FULL + 0), 0, p.err, ERR_ATTN_K_FULL);
      if (ok && nblk > 0) {
        for (int t = 0; t < 2; ++t) {
          if (ti[t].nblk > 0) {
            issue_qk(t, 0);
            if (elect_one()) umma_commit(bar(BAR_S_FULL + t));
          }
        }
        if (elect_one()) umma_commit(bar(BAR_K_EMPTY + 0));
      }
      // steady state: both tiles need blocks j and j + 1
      const int nboth = min(ti[0].nblk, ti[1].nblk) - 1;
      int j = 0;
      for (; ok && j < nboth; ++j) {
        const int s = j & 1, s1 = s ^ 1;
        const uint32_t ph = (j >> 1) & 1, ph1 = ((j + 1) >> 1) & 1, pp = j & 1;
        if (!warp_wait(bar(BAR_V_FULL + s), ph, p.err, ERR_ATTN_V_FULL)) { ok = false; break; }
        if (!warp_wait(bar(BAR_P_FULL + 0), pp, p.err, ERR_ATTN_P_FULL)) { ok = false; break; }
        tc_fence_after();
        issue_pv(0, s, j > 0);
        if (!warp_wait(bar(BAR_K_FULL + s1), ph1, p.err, ERR_ATTN_K_FULL)) { ok = false; break; }
        issue_qk(0, s1);
        if (elect_one()) umma_commit(bar(BAR_S_FULL + 0));
        if (!warp_wait(bar(BAR_P_FULL + 1), pp, p.err, ERR_ATTN_P_FULL)) { ok = false; break; }
        tc_fence_after();
        issue_pv(1, s, j > 0);
        if (elect_one()) umma_commit(bar(BAR_V_EMPTY + s));
        issue_qk(1, s1);
        if (elect_one()) umma_commit(bar(BAR_S_FULL + 1));
        if (elect_one()) umma_commit(bar(BAR_K_EMPTY + s1));
      }
      // tail: the blocks where one tile has finished or no next block exists
      for (; ok && j < nblk; ++j) {
        const int s = j & 1, s1 = s ^ 1;
        const bool more = (j + 1) < nblk;
        if (!warp_wait(bar(BAR_V_FULL + s), (j >> 1) & 1, p.err, ERR_ATTN_V_FULL)) break;
        if (j < ti[0].nblk) {
          if (!warp_wait(bar(BAR_P_FULL + 0), j & 1, p.err, ERR_ATTN_P_FULL)) break;
          tc_fence_after();
          issue_pv(0, s, j > 0);
          if (j == ti[0].nblk - 1) {
            if (elect_one()) umma_commit(bar(BAR_O_FULL + 0));
          }
        }
        if (more) {
          if (!warp_wait(bar(BAR_K_FULL + s1), ((j + 1) >> 1) & 1, p.err, ERR_ATTN_K_FULL)) break;
          if (j + 1 < ti[0].nblk) {
            issue_qk(0, s1);
            if (elect_one()) umma_commit(bar(BAR_S_FULL + 0));
          }
        }
        if (j < ti[1].nblk) {
          if (!warp_wait(bar(BAR_P_FULL + 1), j & 1, p.err, ERR_ATTN_P_FULL)) break;
          tc_fence_after();
          issue_pv(1, s, j > 0);
          if (j == ti[1].nblk - 1) {
            if (elect_one()) umma_commit(bar(BAR_O_FULL + 1));
          }
        }
        if (elect_one()) umma_commit(bar(BAR_V_EMPTY + s));
        if (more) {
          if (j + 1 < ti[1].nblk) {
            issue_qk(1, s1);
            if (elect_one()) umma_commit(bar(BAR_S_FULL + 1));
          }
          if (elect_one()) umma_commit(bar(BAR_K_EMPTY + s1));
        }
      }
      // every MMA issued so far has completed before TMEM is released
      if (elect_one()) umma_commit(bar(BAR_MMA_DONE));
      warp_wait(bar(BAR_MMA_DONE), 0, p.err, ERR_ATTN_DRAIN);
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<192>();
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // row inside the tile == TMEM lane
    const TileInfo me = t ? ti[1] : ti[0];
    const int i = me.m0 + r;        // query index
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t tS = tmem + t * 128u + lane_off;
    const uint32_t tO = tmem + 256u + t * 128u + lane_off;
    bool ok = true;

    if (has_qscale) {
      // the Phase-2 query scale: q_row <- bf16(q_row * qs), in shared memory
      // before the first QK MMA (the reference scales q the same way)
      ok = warp_wait(bar(BAR_Q), 0, p.err, ERR_ATTN_Q);
      if (ok && me.nblk > 0) {
        const float qs = (i < p.Sq)
            ? __ldg(p.qscale + (int64_t)b * p.qs_sb + (int64_t)me.head * p.qs_sh + i) : 1.f;
        uint8_t* qt = smem + kSmQ + t * kAttnTileBytes;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4* ptr = reinterpret_cast<uint4*>(qt + hh * kAttnHalfBytes + sw128_off(r, c));
            uint4 v = *ptr;
            uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(w[e] << 16) * qs;
              const float hi = __uint_as_float(w[e] & 0xFFFF0000u) * qs;
              w[e] = pack_bf16x2(lo, hi);
            }
            *ptr = v;
          }
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_Q_READY));
    }

    const float c2 = p.scale_log2;   // raw logit -> log2 units
    float m_run = -INFINITY;         // running max, log2 units
    float l_run = 0.f;
    const int diag_blk = p.causal ? (me.m0 / kAttnBN) : -1;
    const int last_blk = me.nblk - 1;
    const int tail_keys = p.Sk - last_blk * kAttnBN;  // valid keys in the last block

    for (int j = 0; ok && j < me.nblk; ++j) {
      if (!warp_wait(bar(BAR_S_FULL + t), j & 1, p.err, ERR_ATTN_S_FULL)) { ok = false; break; }
      tc_fence_after();

      uint32_t sv[128];
      tmem_ld128(tS, sv);

      // masks: causal edge (keys past the query row) and keys past Sk
      const bool masked = j == diag_blk || (!p.causal && j == last_blk && tail_keys < kAttnBN);
      const int lim = (j == diag_blk) ? r : tail_keys - 1;
      if (masked) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c > lim) sv[c] = __float_as_uint(-INFINITY);
      }
      // block 0 sets the running max from its true row max (3-input max
      // chains); later blocks start optimistically from the running max and
      // only take the true max when their row sum shows that the logits
      // outgrew it (below)
      if (j == 0) m_run = attn_row_max(sv) * c2;
      float msub = (m_run == -INFINITY) ? 0.f : m_run;
      float lsum = attn_exp_store(sv, c2, msub, tS);

      // a row whose logits exceed the running max by more than ~16 in log2
      // units has a row sum above 2^16 (or inf): the warp then moves the max
      // for those rows, rescales O and recomputes P. Below that bound P and
      // the row sum carry the factor 2^(m_true - m_run) <= 2^16 in both the
      // numerator and the denominator, so the result is unchanged. O is
      // stable here because S_t(j) completing implies the P_t(j-1) V MMA,
      // issued earlier, completed too; P is only published after this.
      const bool grew = !(lsum <= 65536.f);
      if (__any_sync(0xffffffffu, grew)) {
        // P overwrote the logits of keys 64..127 in TMEM (still in registers:
        // they were consumed last); keys 0..63 are read back from TMEM
        {
          uint32_t h0[32], h1[32];
          tmem_ld32(tS, h0);
          tmem_ld32(tS + 32, h1);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = h0[e];
            sv[32 + e] = h1[e];
          }
          if (masked) {
#pragma unroll
            for (int c = 0; c < 64; ++c)
              if (c > lim) sv[c] = __float_as_uint(-INFINITY);
          }
        }
        const float m_new = fmaxf(m_run, attn_row_max(sv) * c2);
        float alpha = 1.f;
        if (grew && m_new > m_run) {
          alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - m_new);
          m_run = m_new;
        }
        l_run *= alpha;
        tmem_wait_st();  // the optimistic P stores land before they are replaced
        msub = (m_run == -INFINITY) ? 0.f : m_run;
        lsum = attn_exp_store(sv, c2, msub, tS);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(BAR_P_FULL + t));
      l_run += lsum;
    }

    if (ok && me.nblk > 0) {
      if (warp_wait(bar(BAR_O_FULL + t), 0, p.err, ERR_ATTN_O_FULL)) {
        tc_fence_after();
        const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
        const bool valid = i < p.Sq;
        __nv_bfloat16* orow =
            p.out + (int64_t)b * p.o_sb + (int64_t)i * p.o_ss + (int64_t)me.head * p.o_sh;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          uint4 w[4];
          uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
          for (int e = 0; e < 16; ++e)
            wp[e] = pack_bf16x2(__uint_as_float(o[2 * e]) * inv_l,
                                __uint_as_float(o[2 * e + 1]) * inv_l);
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e) dst[e] = w[e];
          }
        }
        if (valid && p.lse != nullptr) {
          const float lse2 = (l_run > 0.f) ? (m_run + __log2f(l_run)) : -INFINITY;
          p.lse[(int64_t)b * p.lse_sb + (int64_t)me.head * p.lse_sh + i] =
              lse2 * 0.6931471805599453f;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tg
