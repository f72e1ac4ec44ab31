// Compaction of kept rows: hidden states, below-gate K/V rows (any number of
// tensors in one launch). Replaces the per-request advanced indexing and
// index_select + pad of the reference prefill
// (tokengate/e2e_gate/gate_module/gate_forward.py:1443-1461, :1491-1522).
//
// HBM-bound copy: one warp per (request, tensor, row); lanes move 16-byte
// vectors with non-allocating loads, eight in flight per lane before the
// stores for single-segment rows (four for segmented ones). Rows at or past the request's n_valid are zero-filled, as the
// reference's zero-initialised / F.pad-ed outputs are.
#pragma once

#include "ptx.cuh"
#include "../../include/tokengate_b200.h"

namespace tg {

constexpr int kGatherMaxReq = 64;

struct GatherParams {
  tg_gather_tensor t[TG_MAX_GATHER_TENSORS];
  int n_tensors;
  const int64_t* idx;
  int64_t idx_sb;
  int n_rows;
  int B;
  int n_valid[kGatherMaxReq];
};

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
    if (T.n_seg == 1) {
      // one contiguous segment (token-major tensors): eight vectors in flight
      // per lane, no segment arithmetic
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      for (; v + 224 < n_vec; v += 256) {
        uint4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) x[u] = valid ? ld_nc_v4(s4 + v + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 8; ++u) d4[v + 32 * u] = x[u];
      }
      for (; v + 96 < n_vec; v += 128) {
        uint4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = valid ? ld_nc_v4(s4 + v + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 4; ++u) d4[v + 32 * u] = x[u];
      }
      for (; v < n_vec; v += 32) d4[v] = valid ? ld_nc_v4(s4 + v) : make_uint4(0, 0, 0, 0);
      continue;
    }
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
