/*
 * CPU ORACLE — test infrastructure only, never a product path.
 *
 * Plain-C restatement of the integer/byte and fixed-order fp32 parts of the
 * reference gated prefill, used by tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline leg to check the CUDA kernels:
 *
 *   oracle_gate_score   logsigmoid(w . h) of the synthetic linear gate
 *                       (reference: b_scores = gate(h_art.to(fp32)),
 *                        tokengate/e2e_gate/gate_module/gate_forward.py:1396-1407,
 *                        with the fp32 readout fixture of
 *                        tests/inference/test_prefill_memory.py:18-33 plus
 *                        the log-sigmoid of the gate-scoring workload);
 *   oracle_topk_select  torch.topk + keep-list + Phase-2 bias row
 *                       (gate_forward.py:84-99, :1409-1421, :968-1036, :1463-1469),
 *                       ordering (score desc, index asc);
 *   oracle_branch_score the finalized gate's scoring-branch readout
 *                       bf16(sum_k bf16(bf16(silu(g_k)) * u_k) * w_k) over a
 *                       fused [gate | up] row (gate_branch_hs,
 *                       gate_forward.py:491-524, absorbed 1-row down_proj
 *                       :330-340, Qwen3MLP rounding points), in the kernel's
 *                       fixed order, silu with the IEEE-only exp below.
 *
 * The scorer fixes one summation order (documented in the kernel source):
 * 32 lane partials, lane l summing elements 8*(l+32*i)+e for i, e ascending
 * with fused multiply-adds, then an xor butterfly; logsigmoid evaluated with
 * IEEE +,-,*,/,fma only (Cody-Waite exp, atanh-series log1p). Compiled with
 * -ffp-contract=off so every operation rounds exactly as written.
 * Parity of this restatement with the reference's own float path is pinned
 * by tests/test_oracle.py against tests/golden/ (reference-generated).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float u32_as_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* exp(-a), a >= 0: a = k ln2 - r, |r| <= ln2/2, degree-7 Taylor for exp(r) */
static float exp_neg(float a) {
  if (a > 104.0f) return 0.0f;
  const float kInvLn2 = 1.44269504088896341f;
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.42860682030941723212e-6f;
  const float k = rintf(a * kInvLn2);
  float r = fmaf(k, kLn2Hi, -a);
  r = fmaf(k, kLn2Lo, r);
  float q = 1.98412698412698413e-4f;
  q = fmaf(q, r, 1.38888888888888889e-3f);
  q = fmaf(q, r, 8.33333333333333333e-3f);
  q = fmaf(q, r, 4.16666666666666667e-2f);
  q = fmaf(q, r, 1.66666666666666667e-1f);
  q = fmaf(q, r, 0.5f);
  q = fmaf(q, r, 1.0f);
  q = fmaf(q, r, 1.0f);
  int ki = (int)k;
  int k1 = ki > 100 ? 100 : ki;
  int k2 = ki - k1;
  q = q * u32_as_f32((uint32_t)(127 - k1) << 23);
  if (k2 > 0) q = q * u32_as_f32((uint32_t)(127 - k2) << 23);
  return q;
}

/* log1p(x), x in [0, 1] */
static float log1p_unit(float x) {
  if (x < 2.44140625e-4f) {
    float s = fmaf(x, 0.333333333333333333f, -0.5f);
    s = s * x;
    return fmaf(s, x, x);
  }
  const float u = 1.0f + x;
  const float corr = (x - (u - 1.0f)) / u;
  float m = u, j = 0.0f;
  if (u > 1.41421356237309505f) {
    m = u * 0.5f;
    j = 1.0f;
  }
  const float f = (m - 1.0f) / (m + 1.0f);
  const float f2 = f * f;
  float s = 7.69230769230769231e-2f;
  s = fmaf(s, f2, 9.09090909090909091e-2f);
  s = fmaf(s, f2, 1.11111111111111111e-1f);
  s = fmaf(s, f2, 1.42857142857142857e-1f);
  s = fmaf(s, f2, 2.0e-1f);
  s = fmaf(s, f2, 3.33333333333333333e-1f);
  s = s * f2;
  const float two_f = 2.0f * f;
  const float logm = fmaf(two_f, s, two_f);
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.42860682030941723212e-6f;
  const float lo = fmaf(j, kLn2Lo, logm + corr);
  return fmaf(j, kLn2Hi, lo);
}

float oracle_logsigmoid(float z) {
  const float a = fabsf(z);
  const float e = exp_neg(a);
  const float l = log1p_unit(e);
  return fminf(z, 0.0f) - l;
}

/* scores[r] = logsigmoid(w . h[r]) for r < n_rows; h is bf16 bits, row stride in elements */
void oracle_gate_score(const uint16_t* h, int64_t row_stride, int64_t n_rows, int hidden,
                       const float* w, float* scores) {
  const int nv = hidden / 256;
  float part[32];
  for (int64_t r = 0; r < n_rows; ++r) {
    const uint16_t* row = h + r * row_stride;
    for (int l = 0; l < 32; ++l) {
      float acc = 0.0f;
      for (int i = 0; i < nv; ++i) {
        const int base = 8 * (l + 32 * i);
        for (int e = 0; e < 8; ++e) acc = fmaf(bf16_to_f32(row[base + e]), w[base + e], acc);
      }
      part[l] = acc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
      float nxt[32];
      for (int l = 0; l < 32; ++l) nxt[l] = part[l] + part[l ^ off];
      memcpy(part, nxt, sizeof(part));
    }
    scores[r] = oracle_logsigmoid(part[0]);
  }
}

static uint32_t order_key(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct {
  uint32_t key;
  int32_t idx;
} key_idx;

static int cmp_desc_key_asc_idx(const void* a, const void* b) {
  const key_idx* x = (const key_idx*)a;
  const key_idx* y = (const key_idx*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx);
}

static int cmp_i32(const void* a, const void* b) {
  const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return x < y ? -1 : (x > y);
}

/*
 * One request. keep: n_alloc int64 (pads 0); bias (nullable): n_alloc fp32
 * (score at kept state tokens, 0 at prefix/suffix, -1e9 pads);
 * topk_local (nullable): k int64 ascending. Returns n_kept, or -1 on bad args.
 */
int64_t oracle_topk_select(const float* scores, int n_state, int k, int state_begin, int seq_len,
                           int n_alloc, int64_t* keep, float* bias, int64_t* topk_local) {
  if (n_state < 1 || k < 1 || k > n_state || state_begin < 0 || state_begin + n_state > seq_len)
    return -1;
  const int state_end = state_begin + n_state;
  const int n_kept = state_begin + k + (seq_len - state_end);
  if (n_kept > n_alloc) return -1;
  key_idx* ki = (key_idx*)malloc(sizeof(key_idx) * (size_t)n_state);
  int32_t* sel = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
  if (!ki || !sel) {
    free(ki);
    free(sel);
    return -1;
  }
  for (int i = 0; i < n_state; ++i) {
    ki[i].key = order_key(scores[i]);
    ki[i].idx = i;
  }
  qsort(ki, (size_t)n_state, sizeof(key_idx), cmp_desc_key_asc_idx);
  for (int i = 0; i < k; ++i) sel[i] = ki[i].idx;
  qsort(sel, (size_t)k, sizeof(int32_t), cmp_i32);
  int q = 0;
  for (int p = 0; p < state_begin; ++p, ++q) {
    keep[q] = p;
    if (bias) bias[q] = 0.0f;
  }
  for (int i = 0; i < k; ++i, ++q) {
    keep[q] = state_begin + sel[i];
    if (bias) bias[q] = scores[sel[i]];
    if (topk_local) topk_local[i] = sel[i];
  }
  for (int p = state_end; p < seq_len; ++p, ++q) {
    keep[q] = p;
    if (bias) bias[q] = 0.0f;
  }
  for (; q < n_alloc; ++q) {
    keep[q] = 0;
    if (bias) bias[q] = -1e9f;
  }
  free(ki);
  free(sel);
  return n_kept;
}


/* ---------------------------------------------------------------- finalized gate */

/* bf16 round-to-nearest-even of a finite fp32 value, returned as fp32 */
static float bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x; /* inf / nan pass through */
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  return u32_as_f32(u);
}

/* exp(y): y = k ln2 + r, |r| <= ln2/2, degree-7 Taylor for exp(r), 2^k in two
 * exact steps; 0 below -104, +inf above the largest finite result */
static float exp_any(float y) {
  if (y < -104.0f) return 0.0f;
  if (y > 88.72283935546875f) return u32_as_f32(0x7f800000u);
  const float kInvLn2 = 1.44269504088896341f;
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.42860682030941723212e-6f;
  const float k = rintf(y * kInvLn2);
  float r = fmaf(-k, kLn2Hi, y);
  r = fmaf(-k, kLn2Lo, r);
  float q = 1.98412698412698413e-4f;
  q = fmaf(q, r, 1.38888888888888889e-3f);
  q = fmaf(q, r, 8.33333333333333333e-3f);
  q = fmaf(q, r, 4.16666666666666667e-2f);
  q = fmaf(q, r, 1.66666666666666667e-1f);
  q = fmaf(q, r, 0.5f);
  q = fmaf(q, r, 1.0f);
  q = fmaf(q, r, 1.0f);
  const int ki = (int)k;
  const int k1 = ki > 100 ? 100 : (ki < -100 ? -100 : ki);
  const int k2 = ki - k1;
  q = q * u32_as_f32((uint32_t)(127 + k1) << 23);
  if (k2 != 0) q = q * u32_as_f32((uint32_t)(127 + k2) << 23);
  return q;
}

float oracle_silu(float g) { return g / (1.0f + exp_any(-g)); }

/* rows x [g (inter) | u (inter)] bf16 with row stride ld (elements); w: bf16 (inter,) */
void oracle_branch_score(const uint16_t* gu, int64_t ld, int64_t rows, int inter, const uint16_t* w,
                         float* out) {
  const int nv = inter / 256;
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* g = gu + r * ld;
    const uint16_t* u = g + inter;
    float part[32];
    for (int lane = 0; lane < 32; ++lane) {
      float acc = 0.0f;
      for (int i = 0; i < nv; ++i) {
        for (int e = 0; e < 8; ++e) {
          const int k = 8 * (lane + 32 * i) + e;
          const float s = bf16_round(oracle_silu(bf16_to_f32(g[k])));
          const float a = bf16_round(s * bf16_to_f32(u[k]));
          acc = fmaf(a, bf16_to_f32(w[k]), acc);
        }
      }
      part[lane] = acc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
      float nxt[32];
      for (int lane = 0; lane < 32; ++lane) nxt[lane] = part[lane] + part[lane ^ off];
      memcpy(part, nxt, sizeof(part));
    }
    const float sc = bf16_round(part[0]);
    out[r] = sc == 0.0f ? 0.0f : sc;
  }
}
