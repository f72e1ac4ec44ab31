// Qwen3 MLP up-projection with the SwiGLU epilogue fused — sm_100a:
//
//   out[m, c] = bf16( bf16(silu(G[m, c])) * U[m, c] ),   c < inter,
//   G = bf16(x W_gate^T), U = bf16(x W_up^T)
//
// the product of modeling_qwen3.Qwen3MLP's act_fn(gate_proj(x)) * up_proj(x)
// in bf16, as the reference's decoder layers run it (tokengate/e2e_gate/
// attn/qwen3_flex_attention.py:646-648 call the model's MLP unchanged). The
// rounding points are those of the eager chain (silu_mul in layer_glue.cuh):
// the projections round to bf16, silu runs in fp32 and rounds, the product
// rounds. The fp32 accumulation order of the projections is this kernel's
// own, so G and U can differ from cuBLAS's in the last bf16 bit, and silu
// uses the MUFU exp2 and reciprocal (swiglu_bf16 below).
//
// W is the layer's fused [W_gate; W_up] (2*inter x K, row-major), read in
// place. A persistent grid of CTA pairs (clusters of 2, cta_group::2) walks
// output tiles of 256 rows x 128 columns; tile t covers rows
// 256*(t / n_tiles_n) and columns 128*(t % n_tiles_n), so the tiles in flight
// share x rows and the weight stays L2-resident. Per pair and tile one
// M=256 x N=256 accumulator: rank 0's shared memory holds the 128 W_gate rows
// of the tile, rank 1's the matching 128 W_up rows, each CTA its own 128 x
// rows; in each CTA's TMEM, columns 0..127 are G and 128..255 are U of its
// 128 rows, so the epilogue pairs them without any exchange.
//
// Warps: 0-7 epilogue (warps w and w+4 share TMEM lanes and take 64 of the
// 128 output columns each), 8 TMA producer, 9 MMA issuer (rank 0). A
// 6-stage ring of K=64 slices (32 KB per CTA per stage) feeds the MMAs; the
// accumulator is double-buffered in TMEM (2 x 256 columns) so a tile's
// epilogue overlaps the next tile's main loop. Every wait is bounded.
#pragma once

#include "layer_glue.cuh"

namespace tg {

constexpr int kGsThreads = 320;
constexpr int kGsProducerWarp = 8;
constexpr int kGsMmaWarp = 9;
constexpr int kGsStages = 6;
constexpr int kGsBK = 64;                      // K per stage: one 128-byte swizzle atom of bf16
constexpr int kGsTileBytes = 128 * kGsBK * 2;  // 16 KB: 128 rows x 64 K of A or of B (one TMA box)
constexpr int kGsStageBytes = 2 * kGsTileBytes;

enum {
  GB_FULL = 0,                         // rank 0, stages: both CTAs' A and B bytes
  GB_EMPTY = GB_FULL + kGsStages,      // both, stages: the stage's MMAs done
  GB_ACC_FULL = GB_EMPTY + kGsStages,  // both, 2: a tile's accumulator complete
  GB_ACC_EMPTY = GB_ACC_FULL + 2,      // rank 0, 2, 16: both CTAs' epilogues read it
  GB_MMA_DONE = GB_ACC_EMPTY + 2,      // rank 0, local
  GB_COUNT = GB_MMA_DONE + 1
};
constexpr int kGsSmBar = kGsStages * kGsStageBytes;
constexpr int kGsSmTmemSlot = kGsSmBar + GB_COUNT * 8;
constexpr int kGsSmemBytes = kGsSmTmemSlot + 16 + 1024;  // + alignment slack
static_assert(kGsSmemBytes <= 227 * 1024, "gemm_swiglu shared memory exceeds the per-CTA limit");

constexpr unsigned int ERR_GEMM = 1u << 14;

struct GemmSwigluParams {
  __nv_bfloat16* out;
  int64_t ld_out;
  int M, K, inter;
  int n_tiles_n;   // inter / 128
  int n_tiles_m;   // ceil(M / 256)
  int n_tiles;     // ceil(M / 256) * n_tiles_n
  unsigned int* err;
};

// Output tile t -> (row tile, column tile): the columns of one row tile
// first, so the tiles in flight share x rows and the whole weight stays
// L2-resident (grouping G row tiles per column sweep measured no faster).
__device__ __forceinline__ void gs_tile(const GemmSwigluParams& p, int t, int& mt, int& nt) {
  mt = t / p.n_tiles_n;
  nt = t % p.n_tiles_n;
}

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

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGsThreads, 1)
    gemm_swiglu_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w, const GemmSwigluParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sBar = sbase + kGsSmBar;
  auto bar = [&](int i) { return sBar + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kGsSmTmemSlot);
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
    for (int s = 0; s < kGsStages; ++s) {
      mbar_init(bar(GB_FULL + s), 1);
      mbar_init(bar(GB_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(GB_ACC_FULL + b), 1);
      mbar_init(bar(GB_ACC_EMPTY + b), 16);
    }
    mbar_init(bar(GB_MMA_DONE), 1);
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

  if (warp == kGsProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = cid; ok && t < p.n_tiles; t += n_clusters) {
        int mt, nt;
        gs_tile(p, t, mt, nt);
        const int a_row = mt * 256 + (int)rank * 128;
        const int b_row = nt * 128 + (leader ? 0 : p.inter);  // W_gate / W_up rows
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(bar(GB_EMPTY + s), ph ^ 1u, p.err, ERR_GEMM)) { ok = false; break; }
          const uint32_t dst = sbase + s * kGsStageBytes;
          if (leader) mbar_arrive_expect_tx(bar(GB_FULL + s), 2 * kGsStageBytes);
          tma_load_2d_pair(dst, &tm_x, lbar(GB_FULL + s), kb * kGsBK, a_row);
          tma_load_2d_pair(dst + kGsTileBytes, &tm_w, lbar(GB_FULL + s), kb * kGsBK, b_row);
          if (++s == kGsStages) { s = 0; ph ^= 1u; }
        }
      }
      // no load may still be in flight when the pair retires: the last
      // stages' EMPTY phases complete only after their FULL phases did
      for (int i = 0; ok && i < kGsStages; ++i) {
        if (!mbar_wait(bar(GB_EMPTY + s), ph ^ 1u, p.err, ERR_GEMM)) break;
        if (++s == kGsStages) { s = 0; ph ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == kGsMmaWarp) {
    // ------------------------------------------------------------ MMA (rank 0)
    if (leader) {
      constexpr uint32_t kIdesc = umma_idesc_bf16(256, 256, 0, 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int it = 0;
      for (int t = cid; ok && t < p.n_tiles; t += n_clusters, ++it) {
        const int buf = it & 1;
        const uint32_t acc = tmem + (uint32_t)buf * 256u;
        // the epilogues of both CTAs have read this buffer's previous tile
        if (it >= 2 && !warp_wait(bar(GB_ACC_EMPTY + buf), (uint32_t)((it >> 1) - 1) & 1u, p.err, ERR_GEMM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!warp_wait(bar(GB_FULL + s), ph, p.err, ERR_GEMM)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = sbase + s * kGsStageBytes, sb = sa + kGsTileBytes;
          // one elected lane issues the stage's 4 MMAs and 2 commits as one
          // straight-line block: electing per MMA made the issue, not the
          // tensor core, the limit (1394 vs 1591 TFLOP/s at 32768 rows)
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < kGsBK / 16; ++kk)
              umma_ss_pair(acc, umma_desc_sw128(sa + kk * 32, 16, 1024), umma_desc_sw128(sb + kk * 32, 16, 1024),
                           kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
            umma_commit_pair(lbar(GB_EMPTY + s));
            umma_commit_pair(fbar(GB_EMPTY + s));
          }
          __syncwarp();
          if (++s == kGsStages) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        if (elect_one()) {
          umma_commit_pair(lbar(GB_ACC_FULL + buf));
          umma_commit_pair(fbar(GB_ACC_FULL + buf));
        }
      }
      if (elect_one()) umma_commit_pair(lbar(GB_MMA_DONE));
      warp_wait(bar(GB_MMA_DONE), 0, p.err, ERR_GEMM);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;           // TMEM lanes 32*sub..
    const int half = warp >> 2;         // output columns 64*half..
    const int r = sub * 32 + lane;      // row of this CTA's 128
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    int it = 0;
    for (int t = cid; t < p.n_tiles; t += n_clusters, ++it) {
      const int buf = it & 1;
      if (!warp_wait(bar(GB_ACC_FULL + buf), (uint32_t)(it >> 1) & 1u, p.err, ERR_GEMM)) break;
      tc_fence_after();
      int mt, nt;
      gs_tile(p, t, mt, nt);
      const int64_t row = (int64_t)mt * 256 + (int)rank * 128 + r;
      const int col0 = nt * 128 + half * 64;
      const uint32_t tacc = tmem + lane_off + (uint32_t)buf * 256u + (uint32_t)half * 64u;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t g[32], u[32];
        tmem_ld32(tacc + c * 32, g);
        tmem_ld32(tacc + 128 + c * 32, u);
        uint4 w[4];
        uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
        for (int e = 0; e < 16; ++e)
          wp[e] = pack_bf16x2(swiglu_bf16(__uint_as_float(g[2 * e]), __uint_as_float(u[2 * e])),
                              swiglu_bf16(__uint_as_float(g[2 * e + 1]), __uint_as_float(u[2 * e + 1])));
        if (row < p.M) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + row * p.ld_out + col0 + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[e] = w[e];
        }
      }
      // this CTA's half of the buffer is read: rank 0's MMA warp may reuse it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(lbar(GB_ACC_EMPTY + buf));
    }
  }

  tc_fence_before();
  cluster_sync_all();  // both CTAs done with TMEM and shared memory
  if (warp == kGsMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace tg
