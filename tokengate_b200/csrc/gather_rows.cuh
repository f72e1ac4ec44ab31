// Compaction of kept rows: hidden states, below-gate K/V rows (any number of
// tensors in one launch). Replaces the per-request advanced indexing and
// index_select + pad of the reference prefill
// (tokengate/e2e_gate/gate_module/gate_forward.py:1443-1461, :1491-1522).
//
// HBM-bound copy. Two kernels:
//  * gather_rows_bulk_kernel (rows up to kGatherStageMax bytes): the TMA
//    engine moves the rows. One warp per CTA walks a contiguous range of
//    (request, tensor, row) units; its lane 0 issues bulk global->shared
//    copies of whole rows (one per segment) into a ring of stages, each
//    completing on its own mbarrier, and kGatherLag rows later the bulk
//    shared->global copies of the same stage to the destination row, so
//    ~kGatherLag rows per CTA are in flight with no per-vector instructions;
//  * gather_rows_kernel (fallback for longer rows): one warp per unit, lanes
//    moving 16-byte vectors with non-allocating loads, four in flight per
//    lane before the stores.
// Rows at or past the request's n_valid are zero-filled, as the reference's
// zero-initialised / F.pad-ed outputs are.
#pragma once

#include "ptx.cuh"
#include "../../include/tokengate_b200.h"

namespace tg {

constexpr int kGatherMaxReq = 64;
constexpr int kGatherStages = 16;        // ring stages per CTA (bulk kernel)
constexpr int kGatherLag = 8;            // rows loaded ahead of their stores
constexpr int kGatherStageMax = 10240;   // longest row (bytes) the bulk kernel stages
constexpr unsigned int ERR_GATHER = 1u << 12;

struct GatherParams {
  tg_gather_tensor t[TG_MAX_GATHER_TENSORS];
  int n_tensors;
  const int64_t* idx;
  int64_t idx_sb;
  int n_rows;
  int B;
  int n_valid[kGatherMaxReq];
  int stage_bytes;        // bulk kernel: bytes of one ring stage (>= the longest row)
  int64_t units_per_cta;  // bulk kernel: contiguous units per CTA
  unsigned int* err;
};

// shared-memory bytes of the bulk kernel for a given stage size
__host__ __device__ constexpr int gather_bulk_smem(int stage_bytes) {
  return kGatherStages * stage_bytes + kGatherStages * 8 + kGatherStages * 32;
}

__global__ void __launch_bounds__(32) gather_rows_bulk_kernel(const GatherParams p) {
  extern __shared__ __align__(128) uint8_t g_smem[];
  struct Pending {
    char* dst;
    int64_t seg_stride;
    int seg_bytes, n_seg;
  };
  const int lane = threadIdx.x;
  const uint32_t sbase = smem_u32(g_smem);
  const uint32_t bars = sbase + kGatherStages * p.stage_bytes;
  Pending* pend = reinterpret_cast<Pending*>(g_smem + kGatherStages * p.stage_bytes + kGatherStages * 8);
  if (lane == 0) {
    for (int k = 0; k < kGatherStages; ++k) mbar_init(bars + 8u * k, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int64_t per_req = (int64_t)p.n_tensors * p.n_rows;
  const int64_t total = per_req * p.B;
  const int64_t u0 = (int64_t)blockIdx.x * p.units_per_cta;
  const int64_t u1 = u0 + p.units_per_cta < total ? u0 + p.units_per_cta : total;
  int nl = 0, ns = 0;          // rows loaded / stored (valid rows only; lane 0's counts)
  uint32_t inflight = 0;       // stages whose load has not been seen to land (lane 0)
  bool ok = true;
  // lane 0: bulk store of the oldest loaded row once its load has landed
  auto store_next = [&]() {
    const int k = ns % kGatherStages;
    if (ok) {
      if (mbar_wait(bars + 8u * k, (uint32_t)(ns / kGatherStages) & 1u, p.err, ERR_GATHER)) {
        inflight &= ~(1u << k);
        const Pending& q = pend[k];
        for (int sg = 0; sg < q.n_seg; ++sg)
          bulk_store(q.dst + sg * q.seg_stride, sbase + k * p.stage_bytes + sg * q.seg_bytes, q.seg_bytes);
      } else {
        ok = false;
      }
    }
    bulk_commit();  // one group per row (empty once a wait has given up)
    ++ns;
  };
  // units fit 32 bits here (the host checks), so the decode divides in 32 bits
  const uint32_t per_req32 = (uint32_t)per_req, n_rows32 = (uint32_t)p.n_rows;
  auto decode = [&](int64_t u, int& b, int& ti, int& r) {
    const uint32_t uu = (uint32_t)u;
    b = (int)(uu / per_req32);
    const uint32_t rem = uu - (uint32_t)b * per_req32;
    ti = (int)(rem / n_rows32);
    r = (int)(rem - (uint32_t)ti * n_rows32);
  };
  for (int64_t c0 = u0; c0 < u1; c0 += 32) {
    // each lane fetches the source row of one of the next 32 units, so the
    // issuing lane never waits on an index load per row
    int64_t my_src = 0;
    if (c0 + lane < u1) {
      int b, ti, r;
      decode(c0 + lane, b, ti, r);
      if (r < p.n_valid[b]) my_src = __ldg(p.idx + (int64_t)b * p.idx_sb + r);
    }
    const int cn = (int)(u1 - c0 < 32 ? u1 - c0 : 32);
    for (int j = 0; j < cn; ++j) {
      const int64_t src_row = __shfl_sync(0xffffffffu, my_src, j);
      int b, ti, r;
      decode(c0 + j, b, ti, r);
      const tg_gather_tensor& T = p.t[ti];
      char* dst = static_cast<char*>(T.dst) + b * T.dst_batch_stride + (int64_t)r * T.dst_row_stride;
      if (r >= p.n_valid[b]) {  // pad row: zeros from the whole warp
        const int seg_vecs = (int)(T.seg_bytes >> 4);
        for (int v = lane; v < seg_vecs * T.n_seg; v += 32) {
          const int sg = v / seg_vecs, o = v - sg * seg_vecs;
          reinterpret_cast<uint4*>(dst + sg * T.dst_seg_stride)[o] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      if (lane == 0) {
        if (nl - ns == kGatherLag) store_next();
        // reusing stage k: its previous row (load nl - kGatherStages) was
        // stored; of the ns committed groups at most ns - 1 - (nl -
        // kGatherStages) = kGatherStages - kGatherLag may still be reading
        if (nl >= kGatherStages) bulk_wait_read<kGatherStages - kGatherLag>();
        const int k = nl % kGatherStages;
        const char* src = static_cast<const char*>(T.src) + b * T.src_batch_stride + src_row * T.src_row_stride;
        pend[k] = Pending{dst, T.dst_seg_stride, (int)T.seg_bytes, T.n_seg};
        if (ok) {
          mbar_arrive_expect_tx(bars + 8u * k, (uint32_t)(T.seg_bytes * T.n_seg));
          for (int sg = 0; sg < T.n_seg; ++sg)
            bulk_load(sbase + k * p.stage_bytes + sg * (uint32_t)T.seg_bytes, src + sg * T.src_seg_stride,
                      (uint32_t)T.seg_bytes, bars + 8u * k);
          inflight |= 1u << k;
        } else {
          mbar_arrive(bars + 8u * k);  // keeps the stage's phase count; nothing is copied
        }
        ++nl;
      }
    }
  }
  if (lane == 0) {
    while (ns < nl) store_next();
    bulk_wait<0>();  // every store has written global memory before the CTA retires
    // after a wait that gave up: wait (bounded) for loads still landing in
    // shared memory before the CTA's shared memory is released
    for (int k = 0; k < kGatherStages && inflight; ++k) {
      if (!(inflight & (1u << k))) continue;
      int last = nl - 1 - ((nl - 1 - k) % kGatherStages + kGatherStages) % kGatherStages;
      mbar_wait(bars + 8u * k, (uint32_t)(last / kGatherStages) & 1u, p.err, ERR_GATHER);
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t per_req = (int64_t)p.n_tensors * p.n_rows;
  const int64_t total = per_req * p.B;

  for (int64_t w = warp_global; w < total; w += n_warps) {
    const int b = (int)(w / per_req);
    const int64_t rem = w - (int64_t)b * per_req;
    const int ti = (int)(rem / p.n_rows);
    const int r = (int)(rem - (int64_t)ti * p.n_rows);
    const tg_gather_tensor& T = p.t[ti];
    const bool valid = r < p.n_valid[b];
    const int64_t src_row = valid ? __ldg(p.idx + (int64_t)b * p.idx_sb + r) : 0;
    const char* src = static_cast<const char*>(T.src) + b * T.src_batch_stride + src_row * T.src_row_stride;
    char* dst = static_cast<char*>(T.dst) + b * T.dst_batch_stride + (int64_t)r * T.dst_row_stride;
    const int seg_vecs = (int)(T.seg_bytes >> 4);
    const int n_vec = seg_vecs * T.n_seg;
    int v = lane;
    for (; v + 96 < n_vec; v += 128) {
      uint4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int vv = v + 32 * u;
        const int sg = vv / seg_vecs, o = vv - sg * seg_vecs;
        x[u] = valid ? ld_nc_v4(reinterpret_cast<const uint4*>(src + sg * T.src_seg_stride) + o)
                     : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int vv = v + 32 * u;
        const int sg = vv / seg_vecs, o = vv - sg * seg_vecs;
        reinterpret_cast<uint4*>(dst + sg * T.dst_seg_stride)[o] = x[u];
      }
    }
    for (; v < n_vec; v += 32) {
      const int sg = v / seg_vecs, o = v - sg * seg_vecs;
      const uint4 x = valid ? ld_nc_v4(reinterpret_cast<const uint4*>(src + sg * T.src_seg_stride) + o)
                            : make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(dst + sg * T.dst_seg_stride)[o] = x;
    }
  }
}

}  // namespace tg
