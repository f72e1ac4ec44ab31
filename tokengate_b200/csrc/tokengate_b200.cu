// C ABI of the tokengate_b200 kernels (declared in include/tokengate_b200.h).
//
// One translation unit: the kernels live in the .cuh files included below,
// so the library has a single device error word and no relocatable device
// code. Host code here validates arguments, encodes TMA tensor maps through
// the driver entry point (no libcuda link), and launches on the caller's
// stream. Nothing here allocates device memory.
#include <cstdio>
#include <cstring>
#include <cstdarg>
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <tuple>
#include <vector>

#include "../../include/tokengate_b200.h"
#include "ptx.cuh"
#include "keybias_attn.cuh"
#include "gemm_pair.cuh"
#include "gate_score.cuh"
#include "topk_select.cuh"
#include "gather_rows.cuh"
#include "layer_glue.cuh"
#include "e2e_gate.cuh"
#include "decode_attn.cuh"
#include "gemv.cuh"

// Bit flags set by kernels whose bounded waits gave up (see ptx.cuh).
__device__ unsigned int g_tg_device_error = 0;

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned int* g_err_ptr[kMaxDevices] = {};
bool g_attn_attr_set[kMaxDevices] = {};
bool g_dec_attr_set[kMaxDevices] = {};

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

int64_t resident_blocks(int64_t needed, int per_sm) {
  const int64_t cap = (int64_t)sm_count() * per_sm;
  return needed < cap ? (needed < 1 ? 1 : needed) : cap;
}

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device
// (`flags` is the kernel's own array), so launches inside a stream capture
// issue no attribute calls.
template <typename Kern>
cudaError_t smem_limit_once(Kern kern, int bytes, bool (&flags)[kMaxDevices], int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (flags[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) flags[dev] = true;
  return e;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(TG_ERR_UNSUPPORTED, "device index %d", *dev);
  return TG_OK;
}

// Device address of g_tg_device_error on the current device.
int device_error_ptr(unsigned int** out) {
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_tg_device_error);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_tg_device_error)");
    g_err_ptr[dev] = static_cast<unsigned int*>(p);
  }
  *out = g_err_ptr[dev];
  return TG_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) cached = (EncodeTiledFn)p;
  });
  if (cached == nullptr)
    return fail(TG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(err));
  *fn = cached;
  return TG_OK;
}

// (B, S, H, 128) bf16 tensor with element strides -> 4-D map over (d, h, s, b),
// box (64, 1, 128, 1), 128-byte swizzle, zero fill out of bounds.
int encode_bshd(CUtensorMap* map, const void* base, int B, int S, int H, int64_t sb, int64_t ss,
                int64_t sh, const char* name) {
  EncodeTiledFn enc = nullptr;
  int st = get_encode_fn(&enc);
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(TG_ERR_ALIGNMENT, "%s: base address not 16-byte aligned", name);
  if (B == 1) sb = ss * S;  // unused coordinate: any legal stride
  if (H == 1) sh = 128;
  const int64_t bytes[3] = {sh * 2, ss * 2, sb * 2};
  for (int i = 0; i < 3; ++i)
    if (bytes[i] <= 0 || (bytes[i] & 15) != 0 || bytes[i] >= (int64_t(1) << 40))
      return fail(TG_ERR_ALIGNMENT,
                  "%s: head/row/batch strides (%lld, %lld, %lld elements) must be positive "
                  "multiples of 8",
                  name, (long long)sh, (long long)ss, (long long)sb);
  cuuint64_t dims[4] = {128, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)bytes[0], (cuuint64_t)bytes[1], (cuuint64_t)bytes[2]};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TG_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return TG_OK;
}

// (rows, cols) row-major bf16 matrix with row stride ld (elements) -> 2-D map
// over (col, row), box (64, box_rows), 128-byte swizzle, zero fill out of
// bounds.
int encode_2d_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld,
                   int box_rows, const char* name) {
  EncodeTiledFn enc = nullptr;
  int st = get_encode_fn(&enc);
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(TG_ERR_ALIGNMENT, "%s: base address not 16-byte aligned", name);
  if (ld < cols || (ld & 7) != 0)
    return fail(TG_ERR_ALIGNMENT, "%s: row stride %lld must be >= %lld and a multiple of 8", name,
                (long long)ld, (long long)cols);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TG_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return TG_OK;
}

}  // namespace

namespace {
// Launch with programmatic stream serialization, for the kernels of the
// layer chains (layer glue, projections, attention, decode attention, gemv):
// the kernel may start
// while the previous kernel on the stream drains, and waits on the device
// (griddep_wait) before it touches anything that kernel writes. Under a
// stream capture this becomes a programmatic edge of the graph.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

constexpr int kGemvMaxSmem = 200 * 1024;  // the rows of x in shared memory: BT * K * 2 bytes at most

// One gemv launch: the kernel's shared-memory limit is raised once per device
// (not per launch, so launches inside a stream capture issue no attribute
// calls); two CTAs of 8 warps per SM, or fewer when there are fewer rows.
template <int BT, bool SW, int NB>
cudaError_t launch_gemv_nb(const tg::GemvParams& p, cudaStream_t s, int dev) {
  static bool attr_set[kMaxDevices] = {};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(tg::gemv_kernel<BT, SW, NB>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvMaxSmem);
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  const int smem = BT * p.K * 2;
  const int64_t groups = (p.N + tg::kGemvWarps - 1) / tg::kGemvWarps;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(groups, 2LL * sm_count()));
  return launch_pdl(tg::gemv_kernel<BT, SW, NB>, dim3((unsigned)blocks), dim3(tg::kGemvThreads), (size_t)smem, s,
                    p);
}

// the plain form with at most 4 rows and K of 16 slices or more loads a
// whole row per batch; everything else 8 slices
template <int BT, bool SW>
cudaError_t launch_gemv(const tg::GemvParams& p, cudaStream_t s, int dev) {
  if constexpr (!SW && BT <= 4) {
    if (p.K / 256 >= 16 && p.K / 256 <= tg::kGemvLongBatch)
      return launch_gemv_nb<BT, SW, tg::kGemvLongBatch>(p, s, dev);
  }
  return launch_gemv_nb<BT, SW, tg::kGemvBatch>(p, s, dev);
}
}  // namespace

namespace {
// One launch of the CTA-pair GEMM (gemm_pair.cuh): x (M, K) row stride ld_x
// against the weight rows (w_rows, K) row stride ld_w, the params' epilogue
// fields already set. Persistent: one CTA pair per SM pair, or fewer when
// there are fewer tiles.
template <int kEpi>
int launch_gemm_pair(const void* x, int64_t ld_x, const void* w, int64_t w_rows, int64_t ld_w,
                     tg::GemmPairParams& p, void* stream, const char* name) {
  CUtensorMap tx, tw, tw64;
  int st;
  if ((st = encode_2d_bf16(&tx, x, p.M, p.K, ld_x, 128, name))) return st;
  if ((st = encode_2d_bf16(&tw, w, w_rows, p.K, ld_w, 128, name))) return st;
  if ((st = encode_2d_bf16(&tw64, w, w_rows, p.K, ld_w, 64, name))) return st;  // narrow items' B halves
  p.n_tiles_m = (p.M + 255) / 256;
  const int64_t n_tiles = (int64_t)p.n_tiles_m * p.n_tiles_n;
  if (n_tiles > INT32_MAX) return fail(TG_ERR_UNSUPPORTED, "%s: too many tiles", name);
  p.n_tiles = (int)n_tiles;
  // Rounds of one tile per CTA pair; when the last round would fill at most
  // half the pairs, its tiles run as two half-width items each (half the
  // MMA time per item, the same accumulation order per output).
  const int64_t pairs = std::max<int64_t>(1, sm_count() / 2);
  const int64_t full = n_tiles / pairs * pairs, rest = n_tiles - full;
  int64_t clusters;
  if (rest > 0 && 2 * rest <= pairs) {
    p.n_wide = (int)full;
    p.n_narrow = (int)(2 * rest);
    clusters = full > 0 ? pairs : 2 * rest;
  } else {
    p.n_wide = (int)n_tiles;
    p.n_narrow = 0;
    clusters = std::min<int64_t>(n_tiles, pairs);
  }
  if ((st = device_error_ptr(&p.err))) return st;
  int dev;
  if ((st = current_device(&dev))) return st;
  static bool attr_set[kMaxDevices] = {};
  cudaError_t e = smem_limit_once(tg::gemm_pair_kernel<kEpi>, tg::GemmLayout<kEpi>::kSmemBytes, attr_set, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm_pair smem)");
  e = launch_pdl(tg::gemm_pair_kernel<kEpi>, dim3((unsigned)(2 * clusters)), dim3(tg::kGsThreads),
                 (size_t)tg::GemmLayout<kEpi>::kSmemBytes, static_cast<cudaStream_t>(stream), tx, tw, tw64, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, name);
  return TG_OK;
}

// How many of the heaviest row blocks of a causal head-pair launch run one
// head per CTA. A list-scheduling model of the launch: CTAs go out in unit
// order (batch-major as the grid is) to the SM that frees first, one CTA per
// SM, and a CTA costs kFix + key blocks * (kPair for two heads, kSingle for
// one), in microseconds: kFix and kPair from a global-timer trace of the
// S=2768 launch, kSingle fitted to launches with 0..8 single-head rows
// (S=2768: 51, 51, 49, 47, 48, 51, 55, 62 us; S=4096: 0 rows fastest).
// Launches of more than two waves of head pairs keep 0 (their tail is a
// small share). Memoised per shape.
int attn_single_rows(int n_mblocks, int Hq, int B, int sms) {
  constexpr double kFix = 5.3, kPair = 2.0, kSingle = 1.8;
  const int64_t pair_ctas = (int64_t)n_mblocks * (Hq / 2) * B;
  if (n_mblocks < 2 || pair_ctas > 2LL * sms) return 0;
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> memo;
  const auto key = std::make_tuple(n_mblocks, Hq, B, sms);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
  }
  auto span = [&](int T) {
    std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
    for (int i = 0; i < sms; ++i) free_at.push(0.0);
    double end = 0.0;
    auto put = [&](double cost) {
      const double t = free_at.top() + cost;
      free_at.pop();
      free_at.push(t);
      end = t > end ? t : end;
    };
    for (int b = 0; b < B; ++b) {
      for (int mb = n_mblocks - 1; mb >= n_mblocks - T; --mb)
        for (int h = 0; h < Hq; ++h) put(kFix + kSingle * (mb + 1));
      for (int mb = n_mblocks - T - 1; mb >= 0; --mb)
        for (int h = 0; h < Hq / 2; ++h) put(kFix + kPair * (mb + 1));
    }
    return end;
  };
  const int t_max = n_mblocks - 1 < 64 ? n_mblocks - 1 : 64;
  std::vector<double> sp(t_max + 1);
  double best = 1e300;
  for (int T = 0; T <= t_max; ++T) {
    sp[T] = span(T);
    best = sp[T] < best ? sp[T] : best;
  }
  // Among the counts within 0.5 % of the shortest span: the largest whose
  // CTAs still fit in one wave (idle SMs make the extra CTAs free; measured
  // at 868 and 1268 keys: 174 / 283 TFLOP/s with 1 row, 184-188 / 297-298
  // with 3-8), else the smallest.
  int best_t = -1;
  for (int T = 0; T <= t_max; ++T) {
    const int64_t ctas = (int64_t)B * ((int64_t)(n_mblocks - T) * (Hq / 2) + (int64_t)T * Hq);
    if (sp[T] <= best * 1.005 && ctas <= sms) best_t = T;
  }
  if (best_t < 0)
    for (int T = 0; T <= t_max && best_t < 0; ++T)
      if (sp[T] <= best * 1.005) best_t = T;
  std::lock_guard<std::mutex> lk(mu);
  memo[key] = best_t;
  return best_t;
}
}  // namespace

extern "C" {

int tg_abi_version(void) { return TG_ABI_VERSION; }

const char* tg_last_error(void) { return g_last_error; }

int tg_find_state_span(const int64_t* ids, int64_t n, int64_t start_id, int64_t end_id, int64_t* first_start,
                       int64_t* first_end, int64_t* n_start, int64_t* n_end) {
  if (n < 0 || (n > 0 && ids == nullptr) || first_start == nullptr || first_end == nullptr || n_start == nullptr ||
      n_end == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "find_state_span: NULL argument or n=%lld", (long long)n);
  // one pass: counts of both sentinels (branch-free, vectorisable), then the
  // first position of each, searched only when it occurs
  int64_t cs = 0, ce = 0;
  for (int64_t i = 0; i < n; ++i) {
    cs += ids[i] == start_id;
    ce += ids[i] == end_id;
  }
  int64_t fs = -1, fe = -1;
  for (int64_t i = 0; cs > 0 && i < n; ++i)
    if (ids[i] == start_id) { fs = i; break; }
  for (int64_t i = 0; ce > 0 && i < n; ++i)
    if (ids[i] == end_id) { fe = i; break; }
  *first_start = fs;
  *first_end = fe;
  *n_start = cs;
  *n_end = ce;
  return TG_OK;
}

int tg_device_error(void* stream, unsigned int* flags_out, int clear) {
  if (flags_out == nullptr) return fail(TG_ERR_INVALID_ARGUMENT, "flags_out is NULL");
  unsigned int* dptr;
  int st = device_error_ptr(&dptr);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(flags_out, dptr, sizeof(unsigned int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (clear) {
    e = cudaMemsetAsync(dptr, 0, sizeof(unsigned int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  return TG_OK;
}

int tg_keybias_attn_fwd(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k,
                        int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb,
                        int64_t v_ss, int64_t v_sh, const float* bias, int64_t bias_sb,
                        int64_t bias_sh, const float* q_row_scale, int64_t qs_sb, int64_t qs_sh,
                        void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, float* lse,
                        int64_t lse_sb, int64_t lse_sh, int B, int Sq, int Sk, int Hq, int Hkv,
                        int D, float softmax_scale, int causal, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "q, k, v and out must be non-NULL");
  if (B < 1 || Sq < 1 || Sk < 1 || Hq < 1 || Hkv < 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "empty problem: B=%d Sq=%d Sk=%d Hq=%d Hkv=%d", B, Sq, Sk,
                Hq, Hkv);
  if (B > 65535) return fail(TG_ERR_UNSUPPORTED, "B=%d exceeds 65535", B);
  if (D != 128) return fail(TG_ERR_UNSUPPORTED, "head_dim %d not served (only 128)", D);
  if (Hq % Hkv != 0)
    return fail(TG_ERR_INVALID_ARGUMENT, "query heads %d not a multiple of kv heads %d", Hq, Hkv);
  if (causal && Sq != Sk)
    return fail(TG_ERR_INVALID_ARGUMENT, "causal attention needs Sq == Sk (got %d, %d)", Sq, Sk);
  if (!(softmax_scale > 0.f)) return fail(TG_ERR_INVALID_ARGUMENT, "softmax_scale must be > 0");
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (o_ss & 7) || (o_sh & 7) || (o_sb & 7))
    return fail(TG_ERR_ALIGNMENT, "out: base 16-byte aligned and strides multiples of 8 needed");

  CUtensorMap tq, tk, tv;
  int st;
  if ((st = encode_bshd(&tq, q, B, Sq, Hq, q_sb, q_ss, q_sh, "q"))) return st;
  if ((st = encode_bshd(&tk, k, B, Sk, Hkv, k_sb, k_ss, k_sh, "k"))) return st;
  if ((st = encode_bshd(&tv, v, B, Sk, Hkv, v_sb, v_ss, v_sh, "v"))) return st;

  tg::AttnParams p;
  memset(&p, 0, sizeof(p));
  p.bias = bias;
  p.bias_sb = bias_sb;
  p.bias_sh = bias_sh;
  p.qscale = q_row_scale;
  p.qs_sb = qs_sb;
  p.qs_sh = qs_sh;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_sb = o_sb;
  p.o_ss = o_ss;
  p.o_sh = o_sh;
  p.lse = lse;
  p.lse_sb = lse_sb;
  p.lse_sh = lse_sh;
  p.B = B;
  p.Sq = Sq;
  p.Sk = Sk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.pair_heads = (p.G % 2 == 0) ? 1 : 0;
  p.causal = causal ? 1 : 0;
  p.n_mblocks = (Sq + tg::kAttnBM - 1) / tg::kAttnBM;
  p.n_kblocks = (Sk + tg::kAttnBN - 1) / tg::kAttnBN;
  p.heads_per_unit_row = p.pair_heads ? Hq / 2 : Hq;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  if ((st = device_error_ptr(&p.err))) return st;

  p.n_single_rows = (p.pair_heads && p.causal) ? attn_single_rows(p.n_mblocks, Hq, B, sm_count()) : 0;
  const int64_t units =
      p.pair_heads ? (int64_t)(p.n_mblocks - p.n_single_rows) * (Hq / 2) + (int64_t)p.n_single_rows * Hq
                   : (int64_t)((p.n_mblocks + 1) / 2) * Hq;
  if (units > 0x7fffffff) return fail(TG_ERR_UNSUPPORTED, "problem too large");

  int dev;
  if ((st = current_device(&dev))) return st;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_attn_attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(tg::keybias_attn_fwd_kernel<true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           tg::kAttnSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tg::keybias_attn_fwd_kernel<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kAttnSmemBytes);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(attention smem)");
      g_attn_attr_set[dev] = true;
    }
  }
  dim3 grid((unsigned)units, (unsigned)B);
  cudaError_t e = p.bias != nullptr
      ? launch_pdl(tg::keybias_attn_fwd_kernel<true>, grid, dim3(tg::kAttnThreads), (size_t)tg::kAttnSmemBytes,
                   static_cast<cudaStream_t>(stream), tq, tk, tv, p)
      : launch_pdl(tg::keybias_attn_fwd_kernel<false>, grid, dim3(tg::kAttnThreads), (size_t)tg::kAttnSmemBytes,
                   static_cast<cudaStream_t>(stream), tq, tk, tv, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "keybias attention launch");
  return TG_OK;
}

int tg_gate_score(const void* hidden, int64_t h_sb, int64_t h_ss, int hidden_dim, const float* w,
                  int B, const int32_t* row_begin, const int32_t* row_count, float* scores,
                  int64_t s_sb, void* stream) {
  if (hidden == nullptr || w == nullptr || scores == nullptr || row_begin == nullptr ||
      row_count == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "NULL argument");
  if (B < 1) return fail(TG_ERR_INVALID_ARGUMENT, "B=%d", B);
  const int nv = hidden_dim / 256;
  if (hidden_dim % 256 != 0 ||
      !(nv == 1 || nv == 2 || nv == 4 || nv == 8 || nv == 10 || nv == 16 || nv == 20))
    return fail(TG_ERR_UNSUPPORTED,
                "hidden_dim %d not served (256, 512, 1024, 2048, 2560, 4096, 5120)", hidden_dim);
  if ((reinterpret_cast<uintptr_t>(hidden) & 15) || (h_ss & 7) || (h_sb & 7) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return fail(TG_ERR_ALIGNMENT, "hidden rows and w must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tg::kScoreMaxReq) {
    const int nb = B - b0 < tg::kScoreMaxReq ? B - b0 : tg::kScoreMaxReq;
    tg::ScoreParams p;
    memset(&p, 0, sizeof(p));
    p.h = static_cast<const __nv_bfloat16*>(hidden) + (int64_t)b0 * h_sb;
    p.h_sb = h_sb;
    p.h_ss = h_ss;
    p.w = w;
    p.out = scores + (int64_t)b0 * s_sb;
    p.out_sb = s_sb;
    p.B = nb;
    p.row_off[0] = 0;
    for (int i = 0; i < nb; ++i) {
      if (row_begin[b0 + i] < 0 || row_count[b0 + i] < 0)
        return fail(TG_ERR_INVALID_ARGUMENT, "negative row range for request %d", b0 + i);
      p.begin[i] = row_begin[b0 + i];
      p.row_off[i + 1] = p.row_off[i] + row_count[b0 + i];
    }
    p.total_rows = p.row_off[nb];
    if (p.total_rows == 0) continue;
    // one CTA of one warp per row at a time per SM, rows grid-strided
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    void (*kern)(const tg::ScoreParams) = nullptr;
    int smem = 0, threads = 0;
    cudaError_t e = cudaSuccess;
    switch (nv) {
#define TG_SCORE_CASE(NV)                                                              \
      case NV: {                                                                       \
        static bool attr_set[kMaxDevices] = {};                                        \
        kern = tg::gate_score_stream_kernel<NV>;                                       \
        smem = NV * 256 * (int)sizeof(float);                                          \
        threads = tg::score_stream_threads<NV>();                                      \
        e = smem_limit_once(kern, smem, attr_set, dev);                                \
        break;                                                                         \
      }
      TG_SCORE_CASE(1)
      TG_SCORE_CASE(2)
      TG_SCORE_CASE(4)
      TG_SCORE_CASE(8)
      TG_SCORE_CASE(10)
      TG_SCORE_CASE(16)
      TG_SCORE_CASE(20)
#undef TG_SCORE_CASE
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gate score smem)");
    const int64_t warps_per_cta = threads / 32;
    const int64_t want = (p.total_rows + warps_per_cta - 1) / warps_per_cta;
    const int64_t blocks = want < sms ? want : sms;
    kern<<<(unsigned)blocks, threads, smem, s>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gate score launch");
  }
  return TG_OK;
}

int tg_topk_select(const float* scores, int64_t s_sb, int B, const int32_t* n_state,
                   const int32_t* k, const int32_t* state_begin, const int32_t* seq_len,
                   int n_alloc, int64_t* keep, int64_t keep_sb, void* bias_out, int64_t bias_sb,
                   int bias_dtype, int64_t* topk_local, int64_t tl_sb, void* stream) {
  if (scores == nullptr || keep == nullptr || n_state == nullptr || k == nullptr ||
      state_begin == nullptr || seq_len == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "NULL argument");
  if (B < 1 || n_alloc < 1) return fail(TG_ERR_INVALID_ARGUMENT, "B=%d n_alloc=%d", B, n_alloc);
  if (bias_out != nullptr && bias_dtype != 0 && bias_dtype != 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "bias_dtype %d (0 = fp32, 1 = bf16)", bias_dtype);
  for (int b = 0; b < B; ++b) {
    const int n = n_state[b], kk = k[b], s0 = state_begin[b], L = seq_len[b];
    if (n < 1 || kk < 1 || kk > n)
      return fail(TG_ERR_INVALID_ARGUMENT, "request %d: need 1 <= k (%d) <= n_state (%d)", b, kk, n);
    if (s0 < 0 || s0 + n > L)
      return fail(TG_ERR_INVALID_ARGUMENT, "request %d: state [%d, %d) outside seq_len %d", b, s0,
                  s0 + n, L);
    const int n_kept = s0 + kk + (L - s0 - n);
    if (n_kept > n_alloc)
      return fail(TG_ERR_INVALID_ARGUMENT, "request %d: n_kept %d exceeds n_alloc %d", b, n_kept,
                  n_alloc);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tg::kTopkMaxReq) {
    const int nb = B - b0 < tg::kTopkMaxReq ? B - b0 : tg::kTopkMaxReq;
    tg::TopkParams p;
    memset(&p, 0, sizeof(p));
    p.scores = scores + (int64_t)b0 * s_sb;
    p.s_sb = s_sb;
    p.keep = keep + (int64_t)b0 * keep_sb;
    p.keep_sb = keep_sb;
    p.bias_dtype = bias_dtype;
    p.bias_sb = bias_sb;
    if (bias_out != nullptr)
      p.bias_out = static_cast<char*>(bias_out) + (int64_t)b0 * bias_sb * (bias_dtype ? 2 : 4);
    p.topk_local = topk_local ? topk_local + (int64_t)b0 * tl_sb : nullptr;
    p.tl_sb = tl_sb;
    p.n_alloc = n_alloc;
    for (int i = 0; i < nb; ++i) {
      p.n_state[i] = n_state[b0 + i];
      p.k[i] = k[b0 + i];
      p.begin[i] = state_begin[b0 + i];
      p.seq_len[i] = seq_len[b0 + i];
    }
    int n_max = 0;
    for (int i = 0; i < nb; ++i) n_max = p.n_state[i] > n_max ? p.n_state[i] : n_max;
    // a cluster of CTAs per request, each holding 1024 * kpt scores in registers
    auto launch_cluster = [&](auto kern, int kpt) {
      const int per = tg::kTopkThreads * kpt;
      const unsigned C = (unsigned)((n_max + per - 1) / per);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(C, (unsigned)nb);
      cfg.blockDim = dim3(tg::kTopkThreads);
      cfg.stream = s;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = C;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, kern, p);
    };
    cudaError_t el = cudaSuccess;
    if (n_max <= tg::kTopkThreads * 8)
      tg::topk_select_reg_kernel<8><<<nb, tg::kTopkThreads, 0, s>>>(p);
    else if (n_max <= tg::kTopkThreads * tg::kTopkRegKeys)
      el = launch_cluster(tg::topk_select_cluster_kernel<8>, 8);  // 2-4 CTAs of 8192 scores
    else if (n_max <= tg::kTopkMaxCluster * tg::kTopkThreads * tg::kTopkRegKeys)
      el = launch_cluster(tg::topk_select_cluster_kernel<tg::kTopkRegKeys>, tg::kTopkRegKeys);
    else
      tg::topk_select_kernel<<<nb, tg::kTopkThreads, 0, s>>>(p);
    if (el != cudaSuccess) return cuda_fail(el, "top-k cluster launch");
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "top-k launch");
  }
  return TG_OK;
}

int tg_gather_rows(const tg_gather_tensor* tensors, int n_tensors, const int64_t* idx,
                   int64_t idx_sb, int B, int n_rows, const int32_t* n_valid, void* stream) {
  if (tensors == nullptr || idx == nullptr || n_valid == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "NULL argument");
  if (n_tensors < 1 || n_tensors > TG_MAX_GATHER_TENSORS)
    return fail(TG_ERR_INVALID_ARGUMENT, "n_tensors %d (1..%d)", n_tensors, TG_MAX_GATHER_TENSORS);
  if (B < 1 || n_rows < 0) return fail(TG_ERR_INVALID_ARGUMENT, "B=%d n_rows=%d", B, n_rows);
  if (n_rows == 0) return TG_OK;
  for (int i = 0; i < n_tensors; ++i) {
    const tg_gather_tensor& t = tensors[i];
    if (t.src == nullptr || t.dst == nullptr)
      return fail(TG_ERR_INVALID_ARGUMENT, "tensor %d: NULL pointer", i);
    if (t.n_seg < 1 || t.seg_bytes < 16)
      return fail(TG_ERR_INVALID_ARGUMENT, "tensor %d: n_seg %d seg_bytes %lld", i, t.n_seg,
                  (long long)t.seg_bytes);
    const int64_t m = (reinterpret_cast<uintptr_t>(t.src) | reinterpret_cast<uintptr_t>(t.dst) |
                       t.src_batch_stride | t.src_row_stride | t.src_seg_stride |
                       t.dst_batch_stride | t.dst_row_stride | t.dst_seg_stride | t.seg_bytes);
    if (m & 15) return fail(TG_ERR_ALIGNMENT, "tensor %d: addresses/strides/seg_bytes not 16-byte multiples", i);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tg::kGatherMaxReq) {
    const int nb = B - b0 < tg::kGatherMaxReq ? B - b0 : tg::kGatherMaxReq;
    tg::GatherParams p;
    memset(&p, 0, sizeof(p));
    for (int i = 0; i < n_tensors; ++i) {
      p.t[i] = tensors[i];
      p.t[i].src = static_cast<const char*>(tensors[i].src) + (int64_t)b0 * tensors[i].src_batch_stride;
      p.t[i].dst = static_cast<char*>(tensors[i].dst) + (int64_t)b0 * tensors[i].dst_batch_stride;
    }
    p.n_tensors = n_tensors;
    p.idx = idx + (int64_t)b0 * idx_sb;
    p.idx_sb = idx_sb;
    p.n_rows = n_rows;
    p.B = nb;
    for (int i = 0; i < nb; ++i) {
      if (n_valid[b0 + i] < 0 || n_valid[b0 + i] > n_rows)
        return fail(TG_ERR_INVALID_ARGUMENT, "n_valid[%d]=%d outside [0, %d]", b0 + i,
                    n_valid[b0 + i], n_rows);
      p.n_valid[i] = n_valid[b0 + i];
    }
    int sms = 148;
    {
      int dev = 0;
      if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int64_t warps = (int64_t)nb * n_tensors * n_rows;
    int64_t blocks = (warps + 7) / 8;
    if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;  // two resident waves, grid-stride rows
    tg::gather_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  }
  return TG_OK;
}

int tg_add_rmsnorm(const void* h_in, int64_t ld_h_in, const void* delta, int64_t ld_delta,
                   void* h_out, int64_t ld_h_out, void* x_out, int64_t ld_x, const void* weight,
                   int64_t rows, int hidden, float eps, void* stream) {
  if (h_in == nullptr || (delta != nullptr && h_out == nullptr) || (x_out != nullptr && weight == nullptr))
    return fail(TG_ERR_INVALID_ARGUMENT, "add_rmsnorm: NULL argument");
  if (delta == nullptr && x_out == nullptr) return fail(TG_ERR_INVALID_ARGUMENT, "add_rmsnorm: nothing to do");
  if (rows < 0) return fail(TG_ERR_INVALID_ARGUMENT, "add_rmsnorm: rows=%lld", (long long)rows);
  const int nv = hidden / 256;
  if (hidden % 256 != 0 || !(nv == 1 || nv == 2 || nv == 4 || nv == 8 || nv == 10 || nv == 16 || nv == 20))
    return fail(TG_ERR_UNSUPPORTED, "add_rmsnorm: hidden %d not served", hidden);
  const uintptr_t m = reinterpret_cast<uintptr_t>(h_in) | reinterpret_cast<uintptr_t>(delta) |
                      reinterpret_cast<uintptr_t>(h_out) | reinterpret_cast<uintptr_t>(x_out) |
                      reinterpret_cast<uintptr_t>(weight);
  if ((m & 15) || ((ld_h_in | ld_delta | ld_h_out | ld_x) & 7))
    return fail(TG_ERR_ALIGNMENT, "add_rmsnorm: pointers 16-byte aligned, strides multiples of 8 needed");
  if (rows == 0) return TG_OK;
  tg::RmsParams p;
  p.h_in = static_cast<const __nv_bfloat16*>(h_in);
  p.delta = static_cast<const __nv_bfloat16*>(delta);
  p.h_out = static_cast<__nv_bfloat16*>(h_out);
  p.x_out = static_cast<__nv_bfloat16*>(x_out);
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.rows = rows;
  p.ld_h_in = ld_h_in;
  p.ld_delta = ld_delta;
  p.ld_h_out = ld_h_out;
  p.ld_x = ld_x;
  p.eps = eps;
  p.inv_hidden = 1.f / (float)hidden;
  const int64_t blocks = resident_blocks((rows + 7) / 8, 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)blocks), block(256);
  cudaError_t e;
  switch (nv) {
    case 1: e = launch_pdl(tg::add_rmsnorm_kernel<1>, grid, block, 0, s, p); break;
    case 2: e = launch_pdl(tg::add_rmsnorm_kernel<2>, grid, block, 0, s, p); break;
    case 4: e = launch_pdl(tg::add_rmsnorm_kernel<4>, grid, block, 0, s, p); break;
    case 8: e = launch_pdl(tg::add_rmsnorm_kernel<8>, grid, block, 0, s, p); break;
    case 10: e = launch_pdl(tg::add_rmsnorm_kernel<10>, grid, block, 0, s, p); break;
    case 16: e = launch_pdl(tg::add_rmsnorm_kernel<16>, grid, block, 0, s, p); break;
    default: e = launch_pdl(tg::add_rmsnorm_kernel<20>, grid, block, 0, s, p); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "add_rmsnorm launch");
  return TG_OK;
}

namespace {
struct AppendArgs {
  const void* v;
  int64_t ld_v;
  void* k_cache;
  void* v_cache;
  int64_t kc_sb, kc_ss;
  const int64_t* slot_dev;
};
}  // namespace

static int qk_norm_rope_impl(void* q, int64_t ld_q, int n_q_heads, void* k, int64_t ld_k, int n_k_heads,
                             int64_t rows, int seq, const void* q_norm_w, const void* k_norm_w,
                             const void* cos, const void* sin, int64_t cs_sb, int64_t cs_ss, int head_dim,
                             float eps, const AppendArgs* append, void* stream) {
  if (q == nullptr || k == nullptr || q_norm_w == nullptr || k_norm_w == nullptr || cos == nullptr ||
      sin == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "qk_norm_rope: NULL argument");
  if (head_dim != 128) return fail(TG_ERR_UNSUPPORTED, "qk_norm_rope: head_dim %d (only 128)", head_dim);
  if (rows < 0 || n_q_heads < 0 || n_k_heads < 0 || seq < 1 || (rows % seq) != 0)
    return fail(TG_ERR_INVALID_ARGUMENT, "qk_norm_rope: rows %lld must be a multiple of seq %d",
                (long long)rows, seq);
  if (ld_q < (int64_t)n_q_heads * 128 || ld_k < (int64_t)n_k_heads * 128)
    return fail(TG_ERR_INVALID_ARGUMENT, "qk_norm_rope: row strides shorter than the heads");
  const uintptr_t m = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                      reinterpret_cast<uintptr_t>(q_norm_w) | reinterpret_cast<uintptr_t>(k_norm_w) |
                      reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin);
  if ((m & 15) || ((ld_q | ld_k | cs_sb | cs_ss) & 7))
    return fail(TG_ERR_ALIGNMENT, "qk_norm_rope: pointers 16-byte aligned, strides multiples of 8 needed");
  if (rows == 0 || n_q_heads + n_k_heads == 0) return TG_OK;
  tg::QkRopeParams p;
  p.q = static_cast<__nv_bfloat16*>(q);
  p.k = static_cast<__nv_bfloat16*>(k);
  p.rows = rows;
  p.ld_q = ld_q;
  p.ld_k = ld_k;
  p.n_q = n_q_heads;
  p.n_k = n_k_heads;
  p.seq = seq;
  p.q_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  p.k_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.cs_sb = cs_sb;
  p.cs_ss = cs_ss;
  p.eps = eps;
  p.v = nullptr;
  p.ld_v = 0;
  p.k_cache = p.v_cache = nullptr;
  p.kc_sb = p.kc_ss = 0;
  p.slot_dev = nullptr;
  if (append != nullptr) {
    p.v = static_cast<const __nv_bfloat16*>(append->v);
    p.ld_v = append->ld_v;
    p.k_cache = static_cast<__nv_bfloat16*>(append->k_cache);
    p.v_cache = static_cast<__nv_bfloat16*>(append->v_cache);
    p.kc_sb = append->kc_sb;
    p.kc_ss = append->kc_ss;
    p.slot_dev = append->slot_dev;
  }
  // one warp per row; with few rows (decode) one warp per group of
  // 2 * kQkBatch heads of a row, so the heads are not done one group after another
  const int groups = (n_q_heads + n_k_heads + 2 * tg::kQkBatch - 1) / (2 * tg::kQkBatch);
  p.split = rows <= 64 ? groups : 1;
  const int64_t blocks = resident_blocks((rows * p.split + 7) / 8, 8);
  cudaError_t e = launch_pdl(tg::qk_norm_rope_kernel, dim3((unsigned)blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) return cuda_fail(e, "qk_norm_rope launch");
  return TG_OK;
}

int tg_qk_norm_rope(void* q, int64_t ld_q, int n_q_heads, void* k, int64_t ld_k, int n_k_heads,
                    int64_t rows, int seq, const void* q_norm_w, const void* k_norm_w,
                    const void* cos, const void* sin, int64_t cs_sb, int64_t cs_ss, int head_dim,
                    float eps, void* stream) {
  return qk_norm_rope_impl(q, ld_q, n_q_heads, k, ld_k, n_k_heads, rows, seq, q_norm_w, k_norm_w, cos, sin,
                           cs_sb, cs_ss, head_dim, eps, nullptr, stream);
}

int tg_qk_norm_rope_append(void* q, int64_t ld_q, int n_q_heads, void* k, int64_t ld_k, int n_k_heads,
                           const void* v, int64_t ld_v, int64_t rows, const void* q_norm_w,
                           const void* k_norm_w, const void* cos, const void* sin, int64_t cs_sb,
                           int64_t cs_ss, int head_dim, float eps, void* k_cache, void* v_cache,
                           int64_t cache_sb, int64_t cache_ss, const int64_t* slot_dev, void* stream) {
  if (v == nullptr || k_cache == nullptr || v_cache == nullptr || slot_dev == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: v, caches and slot must be non-NULL");
  if (ld_v < (int64_t)n_k_heads * 128 || cache_ss < (int64_t)n_k_heads * 128)
    return fail(TG_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: v row / cache slot strides shorter than the heads");
  if (((reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_cache) |
        reinterpret_cast<uintptr_t>(v_cache)) & 15) || ((ld_v | cache_sb | cache_ss) & 7))
    return fail(TG_ERR_ALIGNMENT, "qk_norm_rope_append: v and caches 16-byte aligned, strides multiples of 8");
  AppendArgs ap{v, ld_v, k_cache, v_cache, cache_sb, cache_ss, slot_dev};
  return qk_norm_rope_impl(q, ld_q, n_q_heads, k, ld_k, n_k_heads, rows, 1, q_norm_w, k_norm_w, cos, sin,
                           cs_sb, cs_ss, head_dim, eps, &ap, stream);
}

int tg_silu_mul(const void* gu, int64_t ld_gu, void* out, int64_t ld_out, int64_t rows, int64_t inter,
                void* stream) {
  if (gu == nullptr || out == nullptr) return fail(TG_ERR_INVALID_ARGUMENT, "silu_mul: NULL argument");
  if (rows < 0 || inter < 8 || (inter & 7)) return fail(TG_ERR_INVALID_ARGUMENT, "silu_mul: inter %lld must be a positive multiple of 8", (long long)inter);
  if (ld_gu < 2 * inter || ld_out < inter) return fail(TG_ERR_INVALID_ARGUMENT, "silu_mul: strides too short");
  if (((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(out)) & 15) || ((ld_gu | ld_out) & 7))
    return fail(TG_ERR_ALIGNMENT, "silu_mul: pointers 16-byte aligned, strides multiples of 8 needed");
  if (rows == 0) return TG_OK;
  tg::SiluParams p;
  p.gu = static_cast<const __nv_bfloat16*>(gu);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.rows = rows;
  p.inter = inter;
  p.ld_gu = ld_gu;
  p.ld_out = ld_out;
  if (inter / 8 > (int64_t)INT32_MAX) return fail(TG_ERR_UNSUPPORTED, "silu_mul: inter %lld", (long long)inter);
  const int64_t blocks = resident_blocks(rows, 8);   // a block per row at a time
  cudaError_t e = launch_pdl(tg::silu_mul_kernel, dim3((unsigned)blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), p);
  if (e != cudaSuccess) return cuda_fail(e, "silu_mul launch");
  return TG_OK;
}

int tg_gemm_swiglu(const void* x, int64_t ld_x, const void* w_gu, int64_t ld_w, void* out,
                   int64_t ld_out, int64_t M, int K, int inter, void* stream) {
  if (M < 0 || K < 1 || inter < 1) return fail(TG_ERR_INVALID_ARGUMENT, "gemm_swiglu: M=%lld K=%d inter=%d",
                                               (long long)M, K, inter);
  if (M == 0) return TG_OK;  // empty input: nothing to read or write
  if (x == nullptr || w_gu == nullptr || out == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemm_swiglu: NULL argument");
  if (K % tg::kGsBK != 0) return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu: K=%d must be a multiple of %d", K, tg::kGsBK);
  if (inter % 128 != 0) return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu: inter=%d must be a multiple of 128", inter);
  if (M > (int64_t)INT32_MAX - 256) return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu: M=%lld too large", (long long)M);
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (ld_out & 7) || ld_out < inter)
    return fail(TG_ERR_ALIGNMENT, "gemm_swiglu: out 16-byte aligned, row stride >= inter and a multiple of 8");
  tg::GemmPairParams p;
  memset(&p, 0, sizeof(p));
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.M = (int)M;
  p.K = K;
  p.n_tiles_n = inter / 128;
  p.b_step = 128;     // rank 0: W_gate rows 128*nt..; rank 1: the W_up rows inter + 128*nt..
  p.b_rank1 = inter;
  p.nb_step = 64;     // narrow half j: W_gate rows 128*nt + 64*j.. and the matching W_up rows
  p.nb_rank1 = inter;
  return launch_gemm_pair<tg::EPI_SWIGLU>(x, ld_x, w_gu, 2 * (int64_t)inter, ld_w, p, stream, "gemm_swiglu");
}

int tg_gemm_swiglu_readout(const void* x, int64_t ld_x, const void* w_gu, int64_t ld_w, const void* w_readout,
                           float* partial, float* scores, int64_t M, int K, int inter, void* stream) {
  if (M < 0 || K < 1 || inter < 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemm_swiglu_readout: M=%lld K=%d inter=%d", (long long)M, K, inter);
  if (M == 0) return TG_OK;
  if (x == nullptr || w_gu == nullptr || w_readout == nullptr || partial == nullptr || scores == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemm_swiglu_readout: NULL argument");
  if (K % tg::kGsBK != 0)
    return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu_readout: K=%d must be a multiple of %d", K, tg::kGsBK);
  if (inter % 128 != 0)
    return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu_readout: inter=%d must be a multiple of 128", inter);
  if (M > (int64_t)INT32_MAX - 256)
    return fail(TG_ERR_UNSUPPORTED, "gemm_swiglu_readout: M=%lld too large", (long long)M);
  if (reinterpret_cast<uintptr_t>(w_readout) & 15)
    return fail(TG_ERR_ALIGNMENT, "gemm_swiglu_readout: w_readout must be 16-byte aligned");
  tg::GemmPairParams p;
  memset(&p, 0, sizeof(p));
  p.M = (int)M;
  p.K = K;
  p.n_tiles_n = inter / 128;
  p.b_step = 128;  // as gemm_swiglu: rank 0 the W_gate rows, rank 1 the matching W_up rows
  p.b_rank1 = inter;
  p.nb_step = 64;
  p.nb_rank1 = inter;
  p.w_readout = static_cast<const __nv_bfloat16*>(w_readout);
  p.partial = partial;
  p.ld_partial = M;
  int st = launch_gemm_pair<tg::EPI_SWIGLU_READOUT>(x, ld_x, w_gu, 2 * (int64_t)inter, ld_w, p, stream,
                                                    "gemm_swiglu_readout");
  if (st) return st;
  tg::BranchReduceParams r;
  r.partial = partial;
  r.ld_partial = M;
  r.n_part = inter / 64;
  r.M = M;
  r.out = scores;
  cudaError_t e = launch_pdl(tg::branch_reduce_kernel, dim3((unsigned)((M + 255) / 256)), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), r);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "branch_reduce launch");
  return TG_OK;
}

int tg_gemm_qkv_rope(const void* x, int64_t ld_x, const void* w_qkv, int64_t ld_w, void* out, int64_t ld_out,
                     int64_t M, int K, int n_q_heads, int n_k_heads, const void* q_norm_w, const void* k_norm_w,
                     const void* cos, const void* sin, int64_t cs_sb, int64_t cs_ss, int seq, float eps,
                     void* stream) {
  if (M < 0 || K < 1 || n_q_heads < 1 || n_k_heads < 1 || seq < 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: M=%lld K=%d heads %d/%d seq=%d", (long long)M, K,
                n_q_heads, n_k_heads, seq);
  if (M == 0) return TG_OK;
  if (x == nullptr || w_qkv == nullptr || out == nullptr || q_norm_w == nullptr || k_norm_w == nullptr ||
      cos == nullptr || sin == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: NULL argument");
  if (K % tg::kGsBK != 0) return fail(TG_ERR_UNSUPPORTED, "gemm_qkv_rope: K=%d must be a multiple of %d", K, tg::kGsBK);
  if (M % seq != 0) return fail(TG_ERR_INVALID_ARGUMENT, "gemm_qkv_rope: M=%lld rows not whole sequences of %d",
                                (long long)M, seq);
  if (M > (int64_t)INT32_MAX - 256) return fail(TG_ERR_UNSUPPORTED, "gemm_qkv_rope: M=%lld too large", (long long)M);
  const int n_heads = n_q_heads + 2 * n_k_heads;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (ld_out & 7) || ld_out < (int64_t)n_heads * 128)
    return fail(TG_ERR_ALIGNMENT, "gemm_qkv_rope: out 16-byte aligned, row stride >= heads*128, a multiple of 8");
  if (((reinterpret_cast<uintptr_t>(q_norm_w) | reinterpret_cast<uintptr_t>(k_norm_w) |
        reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15) || ((cs_sb | cs_ss) & 7))
    return fail(TG_ERR_ALIGNMENT, "gemm_qkv_rope: gains and cos/sin 16-byte aligned, cos/sin strides multiples of 8");
  tg::GemmPairParams p;
  memset(&p, 0, sizeof(p));
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.M = (int)M;
  p.K = K;
  p.n_tiles_n = (n_heads + 1) / 2;   // two heads per column tile
  p.b_step = 256;                     // rank 0: head 2*nt, rank 1: head 2*nt + 1
  p.b_rank1 = 128;
  p.nb_step = 128;                    // narrow half j: head 2*nt + j, rank 0 its rows 0..63,
  p.nb_rank1 = 64;                    // rank 1 its rows 64..127
  p.n_q = n_q_heads;
  p.n_k = n_k_heads;
  p.n_heads = n_heads;
  p.q_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  p.k_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.cs_sb = cs_sb;
  p.cs_ss = cs_ss;
  p.seq = seq;
  p.eps = eps;
  return launch_gemm_pair<tg::EPI_QKV_ROPE>(x, ld_x, w_qkv, (int64_t)n_heads * 128, ld_w, p, stream,
                                            "gemm_qkv_rope");
}

int tg_branch_score(const void* gu, int64_t gu_sb, int64_t gu_ss, int inter, const void* w_row,
                    int B, const int32_t* row_begin, const int32_t* row_count, float* scores,
                    int64_t s_sb, void* stream) {
  if (gu == nullptr || w_row == nullptr || scores == nullptr || row_begin == nullptr ||
      row_count == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "branch_score: NULL argument");
  if (B < 1) return fail(TG_ERR_INVALID_ARGUMENT, "branch_score: B=%d", B);
  if (inter < 256 || inter % 256 != 0)
    return fail(TG_ERR_UNSUPPORTED, "branch_score: inter %d must be a positive multiple of 256", inter);
  if (gu_ss < 2 * (int64_t)inter)
    return fail(TG_ERR_INVALID_ARGUMENT, "branch_score: row stride %lld shorter than 2*inter",
                (long long)gu_ss);
  if (((reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(w_row)) & 15) || (gu_ss & 7) ||
      (gu_sb & 7))
    return fail(TG_ERR_ALIGNMENT, "branch_score: rows and w_row must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t all_rows = 0;
  for (int b = 0; b < B; ++b) {
    if (row_begin[b] < 0 || row_count[b] < 0)
      return fail(TG_ERR_INVALID_ARGUMENT, "branch_score: negative row range for request %d", b);
    all_rows += row_count[b];
  }
  if (all_rows == 0) return TG_OK;
  int dev, st;
  if ((st = current_device(&dev))) return st;
  static bool attr_set[kMaxDevices] = {};
  cudaError_t ea = smem_limit_once(tg::branch_score_kernel, tg::kSiluLutBytes, attr_set, dev);
  if (ea != cudaSuccess) return cuda_fail(ea, "cudaFuncSetAttribute(branch_score smem)");
  // the SiLU table, rebuilt on this stream (2^16 evaluations) so that every
  // readout, captured or not, finds it complete
  tg::silu_lut_kernel<<<tg::kSiluLutEntries / 256, 256, 0, s>>>();
  ea = cudaGetLastError();
  if (ea != cudaSuccess) return cuda_fail(ea, "silu_lut launch");
  for (int b0 = 0; b0 < B; b0 += tg::kBranchMaxReq) {
    const int nb = B - b0 < tg::kBranchMaxReq ? B - b0 : tg::kBranchMaxReq;
    tg::BranchParams p;
    memset(&p, 0, sizeof(p));
    p.gu = static_cast<const __nv_bfloat16*>(gu) + (int64_t)b0 * gu_sb;
    p.gu_sb = gu_sb;
    p.gu_ss = gu_ss;
    p.inter = inter;
    p.w = static_cast<const __nv_bfloat16*>(w_row);
    p.out = scores + (int64_t)b0 * s_sb;
    p.out_sb = s_sb;
    p.B = nb;
    p.row_off[0] = 0;
    for (int i = 0; i < nb; ++i) {
      p.begin[i] = row_begin[b0 + i];
      p.row_off[i + 1] = p.row_off[i] + row_count[b0 + i];
    }
    p.total_rows = p.row_off[nb];
    if (p.total_rows == 0) continue;
    const int64_t blocks = resident_blocks((p.total_rows + 31) / 32, 1);  // 32 rows per CTA at a time
    tg::branch_score_kernel<<<(unsigned)blocks, tg::kBranchThreads, tg::kSiluLutBytes, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "branch_score launch");
  }
  return TG_OK;
}

int tg_phase2_tables(const float* scores, int64_t s_sb, int B, const int32_t* state_begin,
                     const int32_t* n_state, const int64_t* keep, int64_t keep_sb,
                     const int32_t* n_kept, int n_alloc, const float* gate_scale,
                     const float* attn_scale, int n_layers, int n_heads, float eps, float gain,
                     float* bias, float* q_scale, void* stream) {
  if (scores == nullptr || state_begin == nullptr || n_state == nullptr || keep == nullptr ||
      n_kept == nullptr || gate_scale == nullptr || attn_scale == nullptr || bias == nullptr ||
      q_scale == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "phase2_tables: NULL argument");
  if (B < 1 || n_alloc < 1 || n_layers < 1 || n_heads < 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "phase2_tables: B=%d n_alloc=%d n_layers=%d n_heads=%d", B,
                n_alloc, n_layers, n_heads);
  if ((int64_t)n_layers * n_heads > tg::kTablesMaxLH)
    return fail(TG_ERR_UNSUPPORTED, "phase2_tables: n_layers * n_heads = %lld exceeds %d",
                (long long)n_layers * n_heads, tg::kTablesMaxLH);
  if (!(eps >= 0.f)) return fail(TG_ERR_INVALID_ARGUMENT, "phase2_tables: eps must be >= 0");
  for (int b = 0; b < B; ++b) {
    if (n_state[b] < 1 || state_begin[b] < 0)
      return fail(TG_ERR_INVALID_ARGUMENT, "phase2_tables: request %d: state [%d, +%d)", b,
                  state_begin[b], n_state[b]);
    if (n_kept[b] < 1 || n_kept[b] > n_alloc)
      return fail(TG_ERR_INVALID_ARGUMENT, "phase2_tables: request %d: n_kept %d outside [1, %d]", b,
                  n_kept[b], n_alloc);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int b0 = 0; b0 < B; b0 += tg::kTablesMaxReq) {
    const int nb = B - b0 < tg::kTablesMaxReq ? B - b0 : tg::kTablesMaxReq;
    tg::TablesParams p;
    memset(&p, 0, sizeof(p));
    p.scores = scores + (int64_t)b0 * s_sb;
    p.s_sb = s_sb;
    p.keep = keep + (int64_t)b0 * keep_sb;
    p.keep_sb = keep_sb;
    p.gate_scale = gate_scale;
    p.attn_scale = attn_scale;
    // the tables keep the full batch's layout; this launch writes its requests
    p.bias = bias + (int64_t)b0 * n_heads * n_alloc;
    p.q_scale = q_scale + (int64_t)b0 * n_heads * n_alloc;
    p.B = B;  // plane stride of the output
    p.L = n_layers;
    p.H = n_heads;
    p.n_alloc = n_alloc;
    p.eps = eps;
    p.gain = gain;
    for (int i = 0; i < nb; ++i) {
      p.n_state[i] = n_state[b0 + i];
      p.begin[i] = state_begin[b0 + i];
      p.n_kept[i] = n_kept[b0 + i];
    }
    // layer groups: about 3 CTAs per SM in total, at least one layer per CTA
    const int64_t chunks = (n_alloc + tg::kTablesThreads - 1) / tg::kTablesThreads;
    const int64_t target = 3LL * sm_count();
    int64_t groups = (target + chunks * nb - 1) / (chunks * nb);
    if (groups > n_layers) groups = n_layers;
    if (groups < 1) groups = 1;
    p.layers_per_cta = (int)((n_layers + groups - 1) / groups);
    groups = (n_layers + p.layers_per_cta - 1) / p.layers_per_cta;
    dim3 grid((unsigned)chunks, (unsigned)nb, (unsigned)groups);
    tg::phase2_tables_kernel<<<grid, tg::kTablesThreads, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "phase2_tables launch");
  }
  return TG_OK;
}

// Fixed device scratch for tg_decode_attn_noalloc (each GPU that loads the
// library holds it until the process exits).
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB
static __device__ __align__(256) float g_tg_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];
float* g_noalloc_ptr[kMaxDevices] = {};

namespace {
int decode_chunks(int n_keys) { return (n_keys + tg::kDecKeys - 1) / tg::kDecKeys; }
}  // namespace

int tg_decode_attn_workspace(int B, int Hq, int n_keys, size_t* bytes) {
  if (bytes == nullptr) return fail(TG_ERR_INVALID_ARGUMENT, "bytes must be non-NULL");
  *bytes = 0;
  if (B < 1 || Hq < 1 || n_keys < 1)
    return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn_workspace: B=%d Hq=%d n_keys=%d", B, Hq, n_keys);
  const int nc = decode_chunks(n_keys);
  if (nc > 1) *bytes = (size_t)B * Hq * nc * tg::kDecPart * sizeof(float);
  return TG_OK;
}

int tg_decode_attn(const void* q, int64_t q_sb, int64_t q_sh, const float* q_scale, int64_t qs_sb,
                   const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb,
                   int64_t v_ss, int64_t v_sh, const float* bias, int64_t bias_sb, int64_t bias_sh,
                   const int32_t* n_valid, int n_prefix, int n_keys, void* out, int64_t o_sb, int64_t o_sh,
                   void* workspace, size_t workspace_bytes, int B, int Hq, int Hkv, int D,
                   float softmax_scale, void* stream) {
  return tg_decode_attn_ex(q, q_sb, q_sh, q_scale, qs_sb, k, k_sb, k_ss, k_sh, v, v_sb, v_ss, v_sh, bias,
                           bias_sb, bias_sh, n_valid, n_prefix, n_keys, nullptr, out, o_sb, o_sh, workspace,
                           workspace_bytes, B, Hq, Hkv, D, softmax_scale, stream);
}

int tg_decode_attn_ex(const void* q, int64_t q_sb, int64_t q_sh, const float* q_scale, int64_t qs_sb,
                      const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb,
                      int64_t v_ss, int64_t v_sh, const float* bias, int64_t bias_sb, int64_t bias_sh,
                      const int32_t* n_valid, int n_prefix, int n_keys, const int32_t* n_keys_dev, void* out,
                      int64_t o_sb, int64_t o_sh, void* workspace, size_t workspace_bytes, int B, int Hq,
                      int Hkv, int D, float softmax_scale, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || n_valid == nullptr)
    return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn: q, k, v, out and n_valid must be non-NULL");
  if (B < 1 || B > 65535 || Hq < 1 || Hkv < 1 || n_keys < 1 || n_prefix < 0 || n_prefix > n_keys)
    return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn: B=%d Hq=%d Hkv=%d n_prefix=%d n_keys=%d", B, Hq, Hkv,
                n_prefix, n_keys);
  if (D != 128) return fail(TG_ERR_UNSUPPORTED, "decode_attn: head_dim %d not served (only 128)", D);
  if (Hq % Hkv != 0)
    return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn: query heads %d not a multiple of kv heads %d", Hq, Hkv);
  const int G = Hq / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(TG_ERR_UNSUPPORTED, "decode_attn: %d query heads per kv head (1, 2, 4 or 8 served)", G);
  if (!(softmax_scale > 0.f)) return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn: softmax_scale must be > 0");
  if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) ||
      ((k_sb | k_ss | k_sh | v_sb | v_ss | v_sh) & 7))
    return fail(TG_ERR_ALIGNMENT, "decode_attn: k and v 16-byte aligned with strides multiples of 8 elements");
  const int nc = decode_chunks(n_keys);
  if (nc > 1) {
    const size_t need = (size_t)B * Hq * nc * tg::kDecPart * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(TG_ERR_INVALID_ARGUMENT, "decode_attn: workspace of %zu bytes, %zu needed", workspace_bytes,
                  need);
    if (reinterpret_cast<uintptr_t>(workspace) & 15)
      return fail(TG_ERR_ALIGNMENT, "decode_attn: workspace must be 16-byte aligned");
  }
  tg::DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.q_scale = q_scale;
  p.qs_sb = qs_sb;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.k_sb = k_sb;
  p.k_ss = k_ss;
  p.k_sh = k_sh;
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.v_sb = v_sb;
  p.v_ss = v_ss;
  p.v_sh = v_sh;
  p.bias = bias;
  p.bias_sb = bias_sb;
  p.bias_sh = bias_sh;
  p.n_valid = n_valid;
  p.n_prefix = n_prefix;
  p.n_keys = n_keys;
  p.n_keys_dev = n_keys_dev;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.part = static_cast<float*>(workspace);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.n_chunks = nc;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dec_attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(tg::decode_attn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           tg::dec_smem_bytes<1>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tg::decode_attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 tg::dec_smem_bytes<2>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tg::decode_attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 tg::dec_smem_bytes<4>());
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tg::decode_attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 tg::dec_smem_bytes<8>());
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode attention smem)");
      g_dec_attr_set[dev] = true;
    }
  }
  dim3 grid((unsigned)nc, (unsigned)Hkv, (unsigned)B);
  const dim3 block(tg::kDecThreads);
  cudaError_t e;
  switch (G) {
    case 1: e = launch_pdl(tg::decode_attn_kernel<1>, grid, block, tg::dec_smem_bytes<1>(), s, p); break;
    case 2: e = launch_pdl(tg::decode_attn_kernel<2>, grid, block, tg::dec_smem_bytes<2>(), s, p); break;
    case 4: e = launch_pdl(tg::decode_attn_kernel<4>, grid, block, tg::dec_smem_bytes<4>(), s, p); break;
    default: e = launch_pdl(tg::decode_attn_kernel<8>, grid, block, tg::dec_smem_bytes<8>(), s, p); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "decode_attn launch");
  if (nc > 1) {
    e = launch_pdl(tg::decode_combine_kernel, dim3((unsigned)Hq, (unsigned)B), dim3(tg::kCombThreads), 0, s, p);
    if (e != cudaSuccess) return cuda_fail(e, "decode_attn combine launch");
  }
  return TG_OK;
}


int tg_gemv(const void* x, int64_t ld_x, const void* w, int64_t ld_w, void* y, int64_t ld_y, int B, int N, int K,
            int swiglu, void* stream) {
  if (x == nullptr || w == nullptr || y == nullptr) return fail(TG_ERR_INVALID_ARGUMENT, "gemv: NULL argument");
  if (B < 1 || B > 8 || N < 1 || K < 256 || (K % 256) != 0)
    return fail(TG_ERR_UNSUPPORTED, "gemv: B=%d (1..8 served), N=%d, K=%d (a multiple of 256 served)", B, N, K);
  if (ld_x < K || ld_w < K || ld_y < N)
    return fail(TG_ERR_INVALID_ARGUMENT, "gemv: row strides shorter than the rows");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) || ((ld_x | ld_w) & 7))
    return fail(TG_ERR_ALIGNMENT, "gemv: x and w 16-byte aligned with row strides multiples of 8");
  if ((size_t)((B <= 1) ? 1 : (B <= 2) ? 2 : (B <= 4) ? 4 : 8) * K * 2 > (size_t)kGemvMaxSmem)
    return fail(TG_ERR_UNSUPPORTED, "gemv: %d rows of K=%d do not fit shared memory", B, K);
  tg::GemvParams p;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ld_x = ld_x;
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.ld_w = ld_w;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ld_y = ld_y;
  p.B = B;
  p.N = N;
  p.K = K;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  cudaError_t e;
  if (swiglu) {
    e = B <= 1 ? launch_gemv<1, true>(p, s, dev) : B <= 2 ? launch_gemv<2, true>(p, s, dev)
        : B <= 4 ? launch_gemv<4, true>(p, s, dev) : launch_gemv<8, true>(p, s, dev);
  } else {
    e = B <= 1 ? launch_gemv<1, false>(p, s, dev) : B <= 2 ? launch_gemv<2, false>(p, s, dev)
        : B <= 4 ? launch_gemv<4, false>(p, s, dev) : launch_gemv<8, false>(p, s, dev);
  }
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return TG_OK;
}

int tg_decode_attn_noalloc(const void* q, int64_t q_sb, int64_t q_sh, const float* q_scale, int64_t qs_sb,
                           const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh, const void* v,
                           int64_t v_sb, int64_t v_ss, int64_t v_sh, const float* bias, int64_t bias_sb,
                           int64_t bias_sh, const int32_t* n_valid, int n_prefix, int n_keys, void* out,
                           int64_t o_sb, int64_t o_sh, int B, int Hq, int Hkv, int D, float softmax_scale,
                           void* stream) {
  // The key-chunk partials go to the library's fixed per-device buffer
  // instead of a caller workspace. Its device address is looked up once per
  // device, with that device current, on the first call made there.
  size_t need = 0;
  int st = tg_decode_attn_workspace(B, Hq, n_keys, &need);
  if (st) return st;
  if (need > kNoAllocScratchBytes)
    return fail(TG_ERR_INVALID_ARGUMENT,
                "decode_attn_noalloc: B=%d Hq=%d n_keys=%d needs %zu bytes of scratch, more than the fixed "
                "%zu-byte buffer; use tg_decode_attn with a workspace",
                B, Hq, n_keys, need, kNoAllocScratchBytes);
  int dev;
  if ((st = current_device(&dev))) return st;
  float* scratch;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      // the scratch address is resolved on a device's first call, which a
      // stream capture cannot record: refuse instead of invalidating it
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cs) == cudaSuccess &&
          cs != cudaStreamCaptureStatusNone)
        return fail(TG_ERR_INVALID_ARGUMENT,
                    "decode_attn_noalloc: the first call on a device must come before any stream capture "
                    "(it resolves the scratch buffer's address); make one call outside the capture first");
      void* ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_tg_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
      g_noalloc_ptr[dev] = static_cast<float*>(ptr);
    }
    scratch = g_noalloc_ptr[dev];
  }
  return tg_decode_attn(q, q_sb, q_sh, q_scale, qs_sb, k, k_sb, k_ss, k_sh, v, v_sb, v_ss, v_sh, bias, bias_sb,
                        bias_sh, n_valid, n_prefix, n_keys, out, o_sb, o_sh, scratch, kNoAllocScratchBytes, B,
                        Hq, Hkv, D, softmax_scale, stream);
}

}  // extern "C"
