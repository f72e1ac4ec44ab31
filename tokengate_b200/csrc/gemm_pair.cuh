// Projection GEMMs of the Qwen3 decoder layer with their elementwise
// follow-ups in the epilogue — sm_100a, persistent CTA pairs (cta_group::2):
//
//  * EPI_SWIGLU, the MLP up-projection:
//      out[m, c] = bf16( bf16(silu(G[m, c])) * U[m, c] ),  c < inter,
//      G = bf16(x W_gate^T), U = bf16(x W_up^T), W = the fused [W_gate; W_up]
//    = modeling_qwen3.Qwen3MLP's act_fn(gate_proj(x)) * up_proj(x) in bf16;
//  * EPI_SWIGLU_READOUT, the finalized gate's scoring branch (the same
//    SwiGLU of its [W_gate; W_up] projection, silu by the IEEE-only tg_silu
//    as the branch readout computes it) folded into its one-row readout:
//      partial[2 nt + h][m] = sum over the tile's 64 columns c of half h of
//                             bf16(bf16(silu(G[m, c])) * U[m, c]) * w[c]
//    (fp32, fused multiply-adds in column order); branch_reduce_kernel adds
//    a row's partials in index order and rounds the score to bf16;
//  * EPI_QKV_ROPE, the attention input projection:
//      out[m, :] = [q heads | k heads | v heads] of bf16(x W_qkv^T), W = the
//      fused [W_q; W_k; W_v], with every q and k head RMS-normalised by its
//      q_norm / k_norm gains and rotated by the row's rotary cos / sin
//    = q_norm(q_proj(x)), k_norm(k_proj(x)), apply_rotary_pos_emb, v_proj(x).
// Both as the reference's decoder layers run them around the patched
// attention (tokengate/e2e_gate/attn/qwen3_flex_attention.py:539-551,
// :646-648). The rounding points are those of the eager chains (silu_mul and
// qk_norm_rope in layer_glue.cuh): the projection rounds to bf16, then every
// elementwise step rounds as the torch op does. The fp32 accumulation order of
// the projection is this kernel's own, so a projected value can differ from
// cuBLAS's in the last bf16 bit; silu uses the MUFU exp2 and reciprocal
// (swiglu_bf16) and the q/k sum of squares is summed in this kernel's order.
//
// A persistent grid of CTA pairs walks output tiles of 256 rows; tile t
// covers rows 256*(t / n_tiles_n) and column tile t % n_tiles_n, the columns
// of one row tile first, so the tiles in flight share x rows and the weight
// stays L2-resident. Per pair and tile one M=256 x N=256 fp32 accumulator:
// each CTA holds its own 128 x rows and 128 of the tile's 256 weight rows
// (the B operand's halves), and each CTA's TMEM holds all 256 columns of its
// 128 rows, so the epilogue needs no exchange:
//  * SwiGLU: rank 0 loads the tile's 128 W_gate rows and rank 1 the matching
//    128 W_up rows (columns 0..127 = G, 128..255 = U; 128 outputs per row);
//  * q/k/v: the tile is two consecutive heads (rank 0 the first, rank 1 the
//    second), each a row's whole 128 columns, so the RMS norm and the
//    rotate-half partners d, d + 64 stay inside one thread.
//
// Warps: 0-7 epilogue (warps w and w+4 share TMEM lanes: for SwiGLU they take
// 64 of the 128 outputs each, for q/k/v one head each), 8 TMA producer, 9 MMA
// issuer (rank 0). A ring of K=64 slices (32 KB per CTA per stage; 6 stages,
// 4 for q/k/v, which stages the tile's rotary rows in shared memory) feeds
// the MMAs; one elected lane issues a stage's 4 MMAs and 2 commits as
// one straight-line block; the accumulator is double-buffered in TMEM (2 x 256
// columns) so a tile's epilogue overlaps the next tile's main loop. Every
// wait is bounded.
#pragma once

#include "layer_glue.cuh"
#include "e2e_gate.cuh"

namespace tg {

constexpr int kGsThreads = 320;
constexpr int kGsProducerWarp = 8;
constexpr int kGsMmaWarp = 9;
constexpr int kGsBK = 64;                      // K per stage: one 128-byte swizzle atom of bf16
constexpr int kGsTileBytes = 128 * kGsBK * 2;  // 16 KB: 128 rows x 64 K of A or of B (one TMA box)
constexpr int kGsStageBytes = 2 * kGsTileBytes;

constexpr unsigned int ERR_GEMM = 1u << 14;

enum GemmEpilogue { EPI_SWIGLU = 0, EPI_QKV_ROPE = 1, EPI_SWIGLU_READOUT = 2 };

// Shared-memory layout per epilogue. The q/k/v epilogue stages each tile's
// 128 rotary cos / sin rows (256 B each, rows padded to 272 B so that the
// lanes of a warp, one row each, read 16 B per lane in 4 wavefronts) and the
// two norm gain vectors; it gives up two K stages for them (4 stages measured
// as fast in the main loop).
template <int kEpi>
struct GemmLayout {
  static constexpr bool kRope = kEpi == EPI_QKV_ROPE;
  static constexpr int kStages = kRope ? 4 : 6;
  static constexpr int kCsRow = 272;
  static constexpr int kSmCos = kStages * kGsStageBytes;
  static constexpr int kSmSin = kSmCos + (kRope ? 128 * kCsRow : 0);
  static constexpr int kSmGain = kSmSin + (kRope ? 128 * kCsRow : 0);  // q gains, then k gains
  static constexpr int kSmStage = kSmGain + (kRope ? 512 : 0);  // 8 epilogue warps x 2 KB
  static constexpr int kSmBar = kSmStage + 8 * 2048;
  // barriers
  static constexpr int kFull = 0;                   // rank 0, stages: both CTAs' A and B bytes
  static constexpr int kEmpty = kFull + kStages;    // both, stages: the stage's MMAs done
  static constexpr int kAccFull = kEmpty + kStages; // both, 2: a tile's accumulator complete
  static constexpr int kAccEmpty = kAccFull + 2;    // rank 0, 2, 16: both CTAs' epilogues read it
  static constexpr int kMmaDone = kAccEmpty + 2;    // rank 0, local
  static constexpr int kCsFull = kMmaDone + 1;      // local, 8: a tile's rotary rows staged
  static constexpr int kCsFree = kCsFull + 1;       // local, 8: the staged rows no longer read
  static constexpr int kCount = kCsFree + 1;
  static constexpr int kSmTmemSlot = kSmBar + kCount * 8;
  static constexpr int kSmemBytes = kSmTmemSlot + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 227 * 1024, "gemm_pair shared memory exceeds the per-CTA limit");
};

struct GemmPairParams {
  __nv_bfloat16* out;
  int64_t ld_out;
  int M, K;
  int n_tiles_n;   // column tiles
  int n_tiles_m;   // ceil(M / 256)
  int n_tiles;     // n_tiles_m * n_tiles_n
  int n_wide;      // tiles [0, n_wide) run whole (N = 256) in rounds over the clusters
  int n_narrow;    // items after them: half j = i & 1 (N = 128) of tile n_wide + i / 2, i < n_narrow
  int b_step;      // weight rows per column tile for rank 0 (SwiGLU 128, q/k/v 256)
  int b_rank1;     // rank 1's weight rows, offset from rank 0's (SwiGLU inter, q/k/v 128)
  int nb_step;     // narrow half j: rank 0's weight rows start at nt * b_step + j * nb_step
  int nb_rank1;    //   and rank 1's nb_rank1 after them (SwiGLU 64 / inter, q/k/v 128 / 64)
  // EPI_QKV_ROPE
  int n_q, n_k, n_heads;          // q heads, k heads, all heads (q + k + v)
  const __nv_bfloat16* q_w;       // (128,) q_norm gains
  const __nv_bfloat16* k_w;       // (128,) k_norm gains
  const __nv_bfloat16* cos;       // rotary cos / sin of row b*seq + s at b*cs_sb + s*cs_ss, 128 each
  const __nv_bfloat16* sin;
  int64_t cs_sb, cs_ss;
  int seq;
  float eps;
  // EPI_SWIGLU_READOUT
  const __nv_bfloat16* w_readout;  // (inter,) readout row
  float* partial;                  // (2 * n_tiles_n, ld_partial) per-half partial dots
  int64_t ld_partial;
  unsigned int* err;
};

// out = bf16(bf16(silu(g)) * u) for fp32 accumulators g and u (each first
// rounded to bf16, as a bf16 GEMM output is). silu(g) = g / (1 + 2^(-g log2 e))
// with the MUFU exp2 and reciprocal: a few fp32 ulps from the eager chain's
// expf and IEEE divide, so the bf16 silu equals the eager one except within
// those ulps of a bf16 rounding boundary (one bf16 ulp apart then). The
// exact forms cost ~20 instructions per element and slowed the main loop
// they run beside by 5-12 %.
__device__ __forceinline__ float swiglu_bf16(float g_acc, float u_acc) {
  const float g = round_bf16(g_acc);
  const float u = round_bf16(u_acc);
  const float e = ex2_approx(g * -1.4426950408889634f);
  const float a = round_bf16(__fdividef(g, 1.f + e));
  return a * u;
}

// Writes 32 consecutive bf16 of each of a warp's 32 rows (lane = row, vals =
// its 16 packed pairs) to gbase + row*ld: the warp transposes them through
// its 2 KB of shared memory (16-byte chunks XOR-swizzled by row so both
// passes take 4 wavefronts) so that each store instruction writes 64
// contiguous bytes of 8 rows instead of 16 bytes of 32 rows. Rows >= nvalid
// are not written.
__device__ __forceinline__ void store_rows_coalesced(const uint32_t (&vals)[16], uint8_t* stage,
                                                     __nv_bfloat16* gbase, int64_t ld, int nvalid, int lane) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *reinterpret_cast<uint4*>(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(vals[4 * k], vals[4 * k + 1], vals[4 * k + 2], vals[4 * k + 3]);
  __syncwarp();
  const int k = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = (lane >> 2) + 8 * i;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 64 + ((k ^ ((rr >> 1) & 3)) << 4));
    if (rr < nvalid) *reinterpret_cast<uint4*>(gbase + rr * ld + k * 8) = v;
  }
  __syncwarp();  // the buffer is rewritten by the next call
}

// The q/k/v epilogue of one row and one head (128 TMEM columns at tcol).
// q/k heads: x = bf16(acc); y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w);
// out[d] = bf16(bf16(y[d] cos[d]) + bf16(-y[d+64] sin[d])),
// out[d+64] = bf16(bf16(y[d+64] cos[d+64]) + bf16(y[d] sin[d+64])), d < 64
// (Qwen3RMSNorm and apply_rotary_pos_emb with rotate_half, as qk_finish in
// layer_glue.cuh rounds them), with the row's cos / sin and the gains read
// from shared memory. v heads: bf16(acc).
// gbase: the head's column 0 in the warp's first row; nvalid: rows of the
// warp's 32 below M.
__device__ __forceinline__ void qkv_rope_head(const GemmPairParams& p, uint32_t tcol, int hd,
                                              const uint8_t* cosr, const uint8_t* sinr, const uint8_t* gain,
                                              uint8_t* stage, __nv_bfloat16* gbase, int nvalid, int lane) {
  if (hd >= p.n_q + p.n_k) {
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32(tcol + c * 32, v);
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
      store_rows_coalesced(w, stage, gbase + c * 32, p.ld_out, nvalid, lane);
    }
    return;
  }
  // the head's 128 projected values, rounded to bf16 once (paired), and
  // their sum of squares
  uint32_t xp[64];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v[32];
    tmem_ld32(tcol + c * 32, v);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t w2 = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
      xp[c * 16 + e] = w2;
      const float a = bf16_lo(w2), b = bf16_hi(w2);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  const float inv = rsqrtf(ss * (1.f / 128.f) + p.eps);
  const uint8_t* wg = gain + (hd < p.n_q ? 0 : 256);
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t oa[16], ob[16];
#pragma unroll
    for (int q8 = 0; q8 < 4; ++q8) {
      const int b0 = (c * 32 + q8 * 8) * 2;  // byte offset of element d0 in a 128-element row
      const uint4 wl4 = *reinterpret_cast<const uint4*>(wg + b0);
      const uint4 wh4 = *reinterpret_cast<const uint4*>(wg + 128 + b0);
      const uint4 cl4 = *reinterpret_cast<const uint4*>(cosr + b0);
      const uint4 ch4 = *reinterpret_cast<const uint4*>(cosr + 128 + b0);
      const uint4 sl4 = *reinterpret_cast<const uint4*>(sinr + b0);
      const uint4 sh4 = *reinterpret_cast<const uint4*>(sinr + 128 + b0);
      const uint32_t wl[4] = {wl4.x, wl4.y, wl4.z, wl4.w}, wh[4] = {wh4.x, wh4.y, wh4.z, wh4.w};
      const uint32_t cl[4] = {cl4.x, cl4.y, cl4.z, cl4.w}, ch[4] = {ch4.x, ch4.y, ch4.z, ch4.w};
      const uint32_t sl[4] = {sl4.x, sl4.y, sl4.z, sl4.w}, sh[4] = {sh4.x, sh4.y, sh4.z, sh4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // elements d, d + 1 (d = 32c + 8 q8 + 2e < 64) and their rotate-half
        // partners d + 64, d + 65
        const uint32_t xa = xp[c * 16 + q8 * 4 + e], xb = xp[32 + c * 16 + q8 * 4 + e];
        float ya0 = bf16_lo(xa) * inv, ya1 = bf16_hi(xa) * inv;
        float yb0 = bf16_lo(xb) * inv, yb1 = bf16_hi(xb) * inv;
        round_bf16x2(ya0, ya1);
        round_bf16x2(yb0, yb1);
        ya0 *= bf16_lo(wl[e]);
        ya1 *= bf16_hi(wl[e]);
        yb0 *= bf16_lo(wh[e]);
        yb1 *= bf16_hi(wh[e]);
        round_bf16x2(ya0, ya1);
        round_bf16x2(yb0, yb1);
        float pc0 = ya0 * bf16_lo(cl[e]), pc1 = ya1 * bf16_hi(cl[e]);
        float ps0 = -yb0 * bf16_lo(sl[e]), ps1 = -yb1 * bf16_hi(sl[e]);
        float qc0 = yb0 * bf16_lo(ch[e]), qc1 = yb1 * bf16_hi(ch[e]);
        float qs0 = ya0 * bf16_lo(sh[e]), qs1 = ya1 * bf16_hi(sh[e]);
        round_bf16x2(pc0, pc1);
        round_bf16x2(ps0, ps1);
        round_bf16x2(qc0, qc1);
        round_bf16x2(qs0, qs1);
        oa[q8 * 4 + e] = pack_bf16x2(pc0 + ps0, pc1 + ps1);
        ob[q8 * 4 + e] = pack_bf16x2(qc0 + qs0, qc1 + qs1);
      }
    }
    store_rows_coalesced(oa, stage, gbase + c * 32, p.ld_out, nvalid, lane);
    store_rows_coalesced(ob, stage, gbase + 64 + c * 32, p.ld_out, nvalid, lane);
  }
}

// Work item k of cluster cid: its wide tiles cid, cid + n_clusters, ... below
// n_wide, then, when cid < n_narrow, one narrow item: half j = cid & 1 of
// tile n_wide + cid / 2. A launch whose last round would leave most CTA
// pairs idle runs that round's tiles as twice as many half-width items, each
// half the MMA time (j = -1 marks a wide tile). False past the last item.
__device__ __forceinline__ bool gemm_item(const GemmPairParams& p, int cid, int n_clusters, int k, int& t,
                                          int& j) {
  const int n_mine = cid < p.n_wide ? (p.n_wide - cid + n_clusters - 1) / n_clusters : 0;
  if (k < n_mine) {
    t = cid + k * n_clusters;
    j = -1;
    return true;
  }
  if (k == n_mine && cid < p.n_narrow) {
    t = p.n_wide + (cid >> 1);
    j = cid & 1;
    return true;
  }
  return false;
}

template <int kEpi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGsThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_w64, const GemmPairParams p) {
  using Lay = GemmLayout<kEpi>;
  constexpr int kStages = Lay::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sBar = sbase + Lay::kSmBar;
  auto bar = [&](int i) { return sBar + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::kSmTmemSlot);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t lbar0 = mapa_shared(sBar, 0);
  const uint32_t fbar0 = mapa_shared(sBar, 1);
  auto lbar = [&](int i) { return lbar0 + 8u * i; };
  auto fbar = [&](int i) { return fbar0 + 8u * i; };
  const int n_clusters = gridDim.x >> 1;
  const int cid = blockIdx.x >> 1;
  const int n_kb = p.K / kGsBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(Lay::kFull + s), 1);
      mbar_init(bar(Lay::kEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(Lay::kAccFull + b), 1);
      mbar_init(bar(Lay::kAccEmpty + b), 16);
    }
    mbar_init(bar(Lay::kMmaDone), 1);
    mbar_init(bar(Lay::kCsFull), 8);
    mbar_init(bar(Lay::kCsFree), 8);
    fence_mbar_init();
  }
  if (warp == kGsMmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched with programmatic stream serialization: the prologue above
  // (barriers, TMEM) overlaps the previous kernel's drain, and nothing that
  // kernel may write (x, the rotary rows, the gains) is read or written
  // before this wait. A CTA of this kernel and one of the attention kernel
  // cannot share an SM (shared memory), so TMEM is never contended.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == kGsProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      if (p.n_narrow > 0) tma_prefetch_desc(&tm_w64);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int t, j;
      for (int k = 0; ok && gemm_item(p, cid, n_clusters, k, t, j); ++k) {
        const int mt = t / p.n_tiles_n, nt = t - mt * p.n_tiles_n;
        const bool narrow = j >= 0;
        const int a_row = mt * 256 + (int)rank * 128;
        const int b_row = narrow ? nt * p.b_step + j * p.nb_step + (leader ? 0 : p.nb_rank1)
                                 : nt * p.b_step + (leader ? 0 : p.b_rank1);
        // both CTAs' A rows and B rows (64 per CTA for a narrow item)
        const uint32_t tx = narrow ? 2 * (kGsTileBytes + kGsTileBytes / 2) : 2 * kGsStageBytes;
        const CUtensorMap* tmb = narrow ? &tm_w64 : &tm_w;
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(bar(Lay::kEmpty + s), ph ^ 1u, p.err, ERR_GEMM)) { ok = false; break; }
          const uint32_t dst = sbase + s * kGsStageBytes;
          if (leader) mbar_arrive_expect_tx(bar(Lay::kFull + s), tx);
          tma_load_2d_pair(dst, &tm_x, lbar(Lay::kFull + s), kb * kGsBK, a_row);
          tma_load_2d_pair(dst + kGsTileBytes, tmb, lbar(Lay::kFull + s), kb * kGsBK, b_row);
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      // no load may still be in flight when the pair retires: the last
      // stages' EMPTY phases complete only after their FULL phases did
      for (int i = 0; ok && i < kStages; ++i) {
        if (!mbar_wait(bar(Lay::kEmpty + s), ph ^ 1u, p.err, ERR_GEMM)) break;
        if (++s == kStages) { s = 0; ph ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == kGsMmaWarp) {
    // ------------------------------------------------------------ MMA (rank 0)
    if (leader) {
      constexpr uint32_t kIdesc = umma_idesc_bf16(256, 256, 0, 0);
      constexpr uint32_t kIdescNarrow = umma_idesc_bf16(256, 128, 0, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int t, j;
      for (int it = 0; ok && gemm_item(p, cid, n_clusters, it, t, j); ++it) {
        const int buf = it & 1;
        const uint32_t idesc = j >= 0 ? kIdescNarrow : kIdesc;
        const uint32_t acc = tmem + (uint32_t)buf * 256u;
        // the epilogues of both CTAs have read this buffer's previous tile
        if (it >= 2 && !warp_wait(bar(Lay::kAccEmpty + buf), (uint32_t)((it >> 1) - 1) & 1u, p.err, ERR_GEMM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!warp_wait(bar(Lay::kFull + s), ph, p.err, ERR_GEMM)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + s * kGsStageBytes, sb = sa + kGsTileBytes;
          // one elected lane issues the stage's 4 MMAs and 2 commits as one
          // straight-line block: electing per MMA made the issue, not the
          // tensor core, the limit (1394 vs 1591 TFLOP/s at 32768 rows)
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kGsBK / 16; ++kk)
              umma_ss_pair(acc, umma_desc_sw128(sa + kk * 32, 16, 1024), umma_desc_sw128(sb + kk * 32, 16, 1024),
                           idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(lbar(Lay::kEmpty + s));
            umma_commit_pair(fbar(Lay::kEmpty + s));
          }
          __syncwarp();
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        if (elect_one()) {
          umma_commit_pair(lbar(Lay::kAccFull + buf));
          umma_commit_pair(fbar(Lay::kAccFull + buf));
        }
      }
      if (elect_one()) umma_commit_pair(lbar(Lay::kMmaDone));
      warp_wait(bar(Lay::kMmaDone), 0, p.err, ERR_GEMM);
    }
    __syncwarp();
  } else if (warp < kGsProducerWarp) {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;           // TMEM lanes 32*sub..
    const int half = warp >> 2;         // SwiGLU: outputs 64*half..; q/k/v: head 2*nt + half
    const int r = sub * 32 + lane;      // row of this CTA's 128
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const int etid = warp * 32 + lane;  // 0..255 over the epilogue warps
    if constexpr (Lay::kRope) {
      // the q and k norm gains, once (visible to the other warps through the
      // first staged tile's kCsFull barrier)
      if (warp == 0) {
        const __nv_bfloat16* src = lane < 16 ? p.q_w + lane * 8 : p.k_w + (lane - 16) * 8;
        *reinterpret_cast<uint4*>(smem + Lay::kSmGain + lane * 16) = __ldg(reinterpret_cast<const uint4*>(src));
      }
    }
    int n_staged = 0;
    int t, j;
    for (int it = 0; gemm_item(p, cid, n_clusters, it, t, j); ++it) {
      const int buf = it & 1;
      const int mt = t / p.n_tiles_n, nt = t - mt * p.n_tiles_n;
      // A wide tile: warp half h takes outputs 64h.. (SwiGLU; G in TMEM columns
      // 64h.., U in 128 + 64h..) or head 2 nt + h (q/k/v, columns 128h..). A
      // narrow item j holds 128 columns (G 0..63, U 64..127, or one head),
      // which half 0 takes as a wide tile's half j would; half 1 only keeps
      // the barrier protocol.
      const bool narrow = j >= 0;
      const int part = narrow ? j : half;               // the wide tile's half this warp computes
      const bool active = !narrow || half == 0;
      const uint32_t gcol = narrow ? 0u : (uint32_t)half * 64u;
      const uint32_t ucol = narrow ? 64u : 128u + (uint32_t)half * 64u;
      const int64_t row0 = (int64_t)mt * 256 + (int)rank * 128 + sub * 32;  // the warp's first row
      const int64_t left = (int64_t)p.M - row0;
      const int nvalid = left <= 0 ? 0 : (left >= 32 ? 32 : (int)left);
      uint8_t* stage = smem + Lay::kSmStage + warp * 2048;
      // q/k tiles: stage this CTA's 128 rotary cos / sin rows (4096 16-byte
      // chunks, 16 per thread, coalesced along each row) while the
      // accumulator is still being computed
      const bool rope = Lay::kRope && 2 * nt + (narrow ? j : 0) < p.n_q + p.n_k;
      if (rope) {
        if (n_staged > 0 &&
            !warp_wait(bar(Lay::kCsFree), (uint32_t)(n_staged - 1) & 1u, p.err, ERR_GEMM))
          break;
#pragma unroll 4
        for (int jj = 0; jj < 16; ++jj) {
          const int q = etid + 256 * jj;          // 0..4095: cos chunks, then sin chunks
          const int tab = q >> 11, rr = (q >> 4) & 127, ch = q & 15;
          int64_t grow = (int64_t)mt * 256 + (int)rank * 128 + rr;
          if (grow >= p.M) grow = p.M - 1;        // rows past M: any valid row
          const int64_t bq = grow / p.seq, sq = grow - bq * p.seq;
          const __nv_bfloat16* src = (tab ? p.sin : p.cos) + bq * p.cs_sb + sq * p.cs_ss + ch * 8;
          cp_async16(sbase + (tab ? Lay::kSmSin : Lay::kSmCos) + rr * Lay::kCsRow + ch * 16, src);
        }
        cp_async_commit();
      }
      if (!warp_wait(bar(Lay::kAccFull + buf), (uint32_t)(it >> 1) & 1u, p.err, ERR_GEMM)) break;
      tc_fence_after();
      if (rope) {
        cp_async_wait_all();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(Lay::kCsFull));
        if (!warp_wait(bar(Lay::kCsFull), (uint32_t)n_staged & 1u, p.err, ERR_GEMM)) break;
      }
      if constexpr (kEpi == EPI_SWIGLU_READOUT) {
        // this row's 64 SwiGLU activations of the tile's half, dotted with
        // the readout row in column order
        const int col0 = nt * 128 + part * 64;
        const uint32_t tacc = tmem + lane_off + (uint32_t)buf * 256u;
        float dot = 0.f;
#pragma unroll 1
        for (int c = 0; active && c < 2; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(tacc + gcol + c * 32, g);
          tmem_ld32(tacc + ucol + c * 32, u);
          const uint4* wv = reinterpret_cast<const uint4*>(p.w_readout + col0 + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 w4 = __ldg(wv + q);
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int k = q * 8 + e;
              const float gb = round_bf16(__uint_as_float(g[k]));
              const float ub = round_bf16(__uint_as_float(u[k]));
              const float a = round_bf16(__fmul_rn(round_bf16(tg_silu(gb)), ub));
              const float wk = (e & 1) ? bf16_hi(ww[e >> 1]) : bf16_lo(ww[e >> 1]);
              dot = __fmaf_rn(a, wk, dot);
            }
          }
        }
        if (active && lane < nvalid) p.partial[(int64_t)(2 * nt + part) * p.ld_partial + row0 + lane] = dot;
      } else if constexpr (kEpi == EPI_SWIGLU) {
        const int col0 = nt * 128 + part * 64;
        const uint32_t tacc = tmem + lane_off + (uint32_t)buf * 256u;
#pragma unroll 1
        for (int c = 0; active && c < 2; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(tacc + gcol + c * 32, g);
          tmem_ld32(tacc + ucol + c * 32, u);
          uint32_t wv[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            wv[e] = pack_bf16x2(swiglu_bf16(__uint_as_float(g[2 * e]), __uint_as_float(u[2 * e])),
                                swiglu_bf16(__uint_as_float(g[2 * e + 1]), __uint_as_float(u[2 * e + 1])));
          store_rows_coalesced(wv, stage, p.out + row0 * p.ld_out + col0 + c * 32, p.ld_out, nvalid, lane);
        }
      } else {
        const int hd = 2 * nt + part;
        if (active && hd < p.n_heads)
          qkv_rope_head(p, tmem + lane_off + (uint32_t)buf * 256u + (narrow ? 0u : (uint32_t)half * 128u), hd,
                        smem + Lay::kSmCos + r * Lay::kCsRow, smem + Lay::kSmSin + r * Lay::kCsRow,
                        smem + Lay::kSmGain, stage, p.out + row0 * p.ld_out + (int64_t)hd * 128, nvalid, lane);
        if (rope) {
          // this warp no longer reads the staged rows
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(Lay::kCsFree));
          ++n_staged;
        }
      }
      // this CTA's half of the buffer is read: rank 0's MMA warp may reuse it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(lbar(Lay::kAccEmpty + buf));
    }
    if constexpr (Lay::kRope) cp_async_wait_all();  // no staging copy outlives the CTA (error exits)
  }

  tc_fence_before();
  cluster_sync_all();  // both CTAs done with TMEM and shared memory
  if (warp == kGsMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace tg
