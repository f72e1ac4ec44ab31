/*
 * tokengate_b200 — C ABI of the B200 (sm_100a) gated-prefill kernels.
 *
 * Plain pointers, sizes and strides; no framework types. Every entry point:
 *   - returns TG_OK (0) or a tg_status code; tg_last_error() gives a message
 *     for the calling thread's most recent failure;
 *   - is asynchronous on `stream` (a cudaStream_t passed as void*; NULL is the
 *     legacy default stream) and allocates no device memory: the caller owns
 *     every buffer;
 *   - runs on the device that is current on the calling thread, which must be
 *     the device holding the buffers.
 * Kernels whose internal waits give up (see tg_device_error) record a flag on
 * the device instead of hanging; the host can read it after synchronising.
 *
 * Strides are in ELEMENTS unless the name says bytes.
 */
#ifndef TOKENGATE_B200_H
#define TOKENGATE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TG_ABI_VERSION 1

typedef enum {
  TG_OK = 0,
  TG_ERR_INVALID_ARGUMENT = 1, /* a shape, count or pointer is invalid   */
  TG_ERR_UNSUPPORTED = 2,      /* valid, but not served (e.g. head_dim)  */
  TG_ERR_ALIGNMENT = 3,        /* a pointer or stride breaks alignment   */
  TG_ERR_CUDA = 4              /* a CUDA runtime/driver call failed      */
} tg_status;

/* ABI stamp (TG_ABI_VERSION of the built library). Mirrors the loader's ABI
 * check of the reference extension (kernels/fa2bias/site_path.py:6-8,
 * kernels/fa2bias/keybias.py:29-37). */
int tg_abi_version(void);

/* Message of the calling thread's last failed call ("" if none). */
const char* tg_last_error(void);

/* Host-side scan of a prompt's ids for the state-span sentinels
 * (split_state_span, tokengate/e2e_gate/gate_module/gate_forward.py:664-689):
 * counts of start_id / end_id in ids[0, n) and the first position of each
 * (-1 when absent). A valid span has exactly one of each, start first. No
 * device work; ids is host memory. */
int tg_find_state_span(const int64_t* ids, int64_t n, int64_t start_id, int64_t end_id, int64_t* first_start,
                       int64_t* first_end, int64_t* n_start, int64_t* n_end);

/* Reads the device-side error word of the current device (bit flags set by a
 * kernel whose bounded wait timed out; 0 = none). Synchronises `stream`.
 * clear != 0 resets the word to 0 afterwards. */
int tg_device_error(void* stream, unsigned int* flags_out, int clear);

/*
 * Causal GQA attention with an additive per-key bias, forward.
 *
 * Replaces the reference key-bias operator
 *   torch.ops.recursive_kvs.fa2_keybias_fwd(q, k, v, bias_raw, scale, causal)
 *   (kernels/fa2bias/keybias.py:40-45; wrapper flash_attn_key_bias :85-87;
 *    kernel kernels/fa2bias/keybias.patch:276-461)
 * and the FlexAttention key-bias score_mod path
 *   (tokengate/e2e_gate/attn/flex_attention_utils.py:174-198, :233-287).
 *
 *   out[b,i,h,:] = sum_j softmax_j( softmax_scale * qs[b,h,i] * q[b,i,h,:].k[b,j,g,:]
 *                                   + bias[b,h,j] ) * v[b,j,g,:],   g = h / (Hq/Hkv)
 *   j <= i when causal (then Sq must equal Sk).
 *   lse[b,h,i] = log sum_j exp(...)  (natural log, fp32)
 *
 * The bias is in score units (what the flex score_mod adds), i.e. the
 * reference's bias_raw * softmax_scale. bias_sh == 0 broadcasts one row over
 * all heads (the reference's scalar (S,)/(B,S) layouts); bias_sb == 0
 * broadcasts over the batch. Finite large negative values (the reference pads
 * with -1e9) are treated as ordinary finite biases.
 *
 * q: (B, Sq, Hq, D) bf16 with strides (q_sb, q_ss, q_sh, 1); k, v likewise
 * with Sk, Hkv. Only D == 128 is served. Bases 16-byte aligned and the batch,
 * row and head strides multiples of 8 elements (TMA).
 * bias: fp32, (B, Hq, Sk) with strides (bias_sb, bias_sh, 1), nullable.
 * q_row_scale: fp32, (B, Hq, Sq) with strides (qs_sb, qs_sh, 1), nullable:
 *   the per-row query scale of the Phase-2 prologue
 *   (tokengate/e2e_gate/attn/qwen3_flex_attention.py:433-473).
 * out: bf16 (B, Sq, Hq, D) strides (o_sb, o_ss, o_sh, 1).
 * lse: fp32 (B, Hq, Sq) strides (lse_sb, lse_sh, 1), nullable.
 */
int tg_keybias_attn_fwd(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                        const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                        const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                        const float* bias, int64_t bias_sb, int64_t bias_sh,
                        const float* q_row_scale, int64_t qs_sb, int64_t qs_sh,
                        void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                        float* lse, int64_t lse_sb, int64_t lse_sh,
                        int B, int Sq, int Sk, int Hq, int Hkv, int D,
                        float softmax_scale, int causal, void* stream);

/*
 * Gate scorer: score[b, r] = logsigmoid( sum_e float(h[b, row_begin[b]+r, e]) * w[e] )
 * for r < row_count[b].
 *
 * Replaces the synthetic linear gate's scoring of the state span,
 *   b_scores = gate(h_art.to(fp32))  with a fp32 1-wide readout + logsigmoid
 *   (tokengate/e2e_gate/gate_module/gate_forward.py:1396-1407; fixture shape
 *    of tests/inference/test_prefill_memory.py:18-33).
 * The dot product has a fixed summation order and logsigmoid is computed
 * with IEEE operations only, so results are reproducible bit for bit.
 *
 * hidden: bf16 (B, S, hidden_dim), strides (h_sb, h_ss, 1); hidden_dim one of
 * 256, 512, 1024, 2048, 2560, 4096, 5120; rows 16-byte aligned.
 * w: fp32 (hidden_dim,). row_begin / row_count: HOST arrays of B ints.
 * scores: fp32 (B, >= max row_count), batch stride s_sb.
 */
int tg_gate_score(const void* hidden, int64_t h_sb, int64_t h_ss, int hidden_dim,
                  const float* w, int B, const int32_t* row_begin, const int32_t* row_count,
                  float* scores, int64_t s_sb, void* stream);

/*
 * Top-K selection and the kept-position list.
 *
 * Replaces, per request b, the selection and keep-list construction
 *   K_clamped = max(1, min(K, n_art)); topk = torch.topk(score, K_clamped)
 *   keep = [0, start) ++ start + sort(topk) ++ [end, seq_len)
 *   (tokengate/e2e_gate/gate_module/gate_forward.py:84-99, :1409-1421)
 * and the Phase-2 bias row and padding
 *   gate_bias[b, :n_kept] = score at kept state tokens, 0 elsewhere;
 *   gate_bias[b, n_kept:] = -1e9   (:968-1036, :1463-1469).
 * Ordering contract: by (score descending, index ascending), so ties at the
 * K-th value keep the lower indices. Scores are compared as IEEE floats
 * (-0.0 < +0.0; NaNs are not supported).
 *
 * scores: fp32 (B, >= n_state[b]), batch stride s_sb.
 * n_state, k, state_begin, seq_len: HOST arrays of B ints; k is K_clamped
 * (1 <= k <= n_state). n_kept[b] = state_begin + k + (seq_len - state_begin - n_state)
 * must be <= n_alloc.
 * keep: int64 (B, n_alloc), batch stride keep_sb: kept ORIGINAL positions in
 *   ascending order, slots >= n_kept set to 0.
 * bias_out (nullable): (B, n_alloc) in bias_dtype (0 = fp32, 1 = bf16),
 *   batch stride bias_sb.
 * topk_local (nullable): int64 (B, >= k), batch stride tl_sb: the selected
 *   state-relative indices in ascending order.
 */
int tg_topk_select(const float* scores, int64_t s_sb, int B, const int32_t* n_state,
                   const int32_t* k, const int32_t* state_begin, const int32_t* seq_len,
                   int n_alloc, int64_t* keep, int64_t keep_sb, void* bias_out, int64_t bias_sb,
                   int bias_dtype, int64_t* topk_local, int64_t tl_sb, void* stream);

/*
 * Compaction: gather kept rows of several tensors in one launch.
 *
 * Replaces hs_pruned[b, :n] = hidden_states[b, keep]
 *   (tokengate/e2e_gate/gate_module/gate_forward.py:1443-1461)
 * and the below-gate K/V gathers of prefill_batch_for_decode
 *   (index_select + pad, :1491-1522; B=1 form prune_kv_cache :1078-1097).
 *
 * For each tensor t, request b < B and row r < n_rows:
 *   r <  n_valid[b]: dst row r <- src row idx[b, r]
 *   r >= n_valid[b]: dst row r <- zeros
 * A row is n_seg segments of seg_bytes at seg_stride (one segment for a
 * (B, S, ...) token-major tensor, one per head for a (B, H, S, D) one).
 * Addresses, strides and seg_bytes must be multiples of 16 bytes.
 * idx: int64 device array (B, >= n_rows), batch stride idx_sb; every index
 * used must be in range for the source (the caller's contract).
 * n_valid: HOST array of B ints. At most TG_MAX_GATHER_TENSORS tensors.
 */
#define TG_MAX_GATHER_TENSORS 16
typedef struct {
  const void* src;
  void* dst;
  int64_t src_batch_stride; /* bytes */
  int64_t src_row_stride;   /* bytes */
  int64_t src_seg_stride;   /* bytes */
  int64_t dst_batch_stride; /* bytes */
  int64_t dst_row_stride;   /* bytes */
  int64_t dst_seg_stride;   /* bytes */
  int64_t seg_bytes;
  int32_t n_seg;
  int32_t reserved;
} tg_gather_tensor;

int tg_gather_rows(const tg_gather_tensor* tensors, int n_tensors, const int64_t* idx,
                   int64_t idx_sb, int B, int n_rows, const int32_t* n_valid, void* stream);

/*
 * Decoder-layer glue (the fused layer prologues). Each replaces an
 * eager op chain of the transformers Qwen3 layer that the reference runs
 * around its patched attention (tokengate/e2e_gate/attn/qwen3_flex_attention.py:
 * 539-551 q/k projections + q_norm/k_norm + apply_rotary_pos_emb, :646-648
 * o_proj; transformers Qwen3DecoderLayer residual adds, Qwen3RMSNorm,
 * Qwen3MLP), keeping its bf16 rounding points. bf16 tensors, 16-byte aligned
 * rows, strides in elements.
 */

/* h_out = bf16(h_in + delta) (skipped when delta is NULL; h_out may alias
 * h_in); x_out = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) with h the
 * updated row (skipped when x_out is NULL). hidden: 256 * {1,2,4,8,10,16,20}. */
int tg_add_rmsnorm(const void* h_in, int64_t ld_h_in, const void* delta, int64_t ld_delta,
                   void* h_out, int64_t ld_h_out, void* x_out, int64_t ld_x, const void* weight,
                   int64_t rows, int hidden, float eps, void* stream);

/* In place on the q projection (rows x n_q_heads x 128, row stride ld_q) and
 * the k projection (rows x n_k_heads x 128, row stride ld_k) of `rows`
 * tokens: every head (head_dim 128) is RMS-normalised with its norm weight,
 * then rotated: x = bf16(bf16(y*cos) + bf16(rotate_half(y)*sin)).
 * cos/sin: (B, seq, 128) bf16 with batch/row strides cs_sb/cs_ss; rows = B*seq. */
int tg_qk_norm_rope(void* q, int64_t ld_q, int n_q_heads, void* k, int64_t ld_k, int n_k_heads,
                    int64_t rows, int seq, const void* q_norm_w, const void* k_norm_w,
                    const void* cos, const void* sin, int64_t cs_sb, int64_t cs_ss, int head_dim,
                    float eps, void* stream);

/* tg_qk_norm_rope for one decode token per row (seq == 1) that also
 * appends it to the layer's caches: the finished k heads and the v heads
 * (rows x n_k_heads x 128, row stride ld_v) are written to slot *slot_dev
 * (device int64) of k_cache / v_cache, (B = rows, cap, n_k_heads, 128) with
 * batch stride cache_sb and slot stride cache_ss. One launch instead of
 * three per layer and decode step (the reference's DynamicCache.update in
 * the decode layers, tokengate/e2e_gate/attn/qwen3_flex_attention.py:395-398). */
int tg_qk_norm_rope_append(void* q, int64_t ld_q, int n_q_heads, void* k, int64_t ld_k, int n_k_heads,
                           const void* v, int64_t ld_v, int64_t rows, const void* q_norm_w,
                           const void* k_norm_w, const void* cos, const void* sin, int64_t cs_sb,
                           int64_t cs_ss, int head_dim, float eps, void* k_cache, void* v_cache,
                           int64_t cache_sb, int64_t cache_ss, const int64_t* slot_dev, void* stream);

/* out[r, :] = bf16(bf16(silu(g)) * u) for a fused row [g (inter) | u (inter)]. */
int tg_silu_mul(const void* gu, int64_t ld_gu, void* out, int64_t ld_out, int64_t rows, int64_t inter,
                void* stream);

/* The Qwen3 MLP up-projection with the SwiGLU fused into its epilogue:
 *   out[m, c] = bf16(bf16(silu(G[m, c])) * U[m, c]),  G = bf16(x W_gate^T), U = bf16(x W_up^T)
 * for m < M, c < inter: act_fn(gate_proj(x)) * up_proj(x) of the decoder
 * layers the reference runs (tokengate/e2e_gate/attn/qwen3_flex_attention.py:
 * 646-648, modeling_qwen3.Qwen3MLP), replacing the bf16 GEMM into [G | U]
 * and tg_silu_mul. A persistent tcgen05 GEMM of CTA pairs.
 * x: bf16 (M, K) row stride ld_x; w_gu: bf16 (2*inter, K) = [W_gate; W_up]
 * row stride ld_w; out: bf16 (M, inter) row stride ld_out. K a multiple of
 * 64, inter a multiple of 128; bases 16-byte aligned, strides multiples of 8.
 * M == 0 returns TG_OK without touching the pointers. */
int tg_gemm_swiglu(const void* x, int64_t ld_x, const void* w_gu, int64_t ld_w, void* out,
                   int64_t ld_out, int64_t M, int K, int inter, void* stream);

/* The decoder layer's attention input projection with the q/k RMSNorm and
 * RoPE fused into its epilogue:
 *   out[m, :] = [q heads | k heads | v heads] of bf16(x W_qkv^T), every q and
 *   k head y <- bf16(w * bf16(y * rsqrt(mean(y^2) + eps))), then rotated:
 *   y <- bf16(bf16(y * cos) + bf16(rotate_half(y) * sin)) at row m's cos/sin;
 *   v heads as projected.
 * = q_norm(q_proj(x)), k_norm(k_proj(x)), apply_rotary_pos_emb and v_proj(x)
 * of the decoder layers the reference runs (tokengate/e2e_gate/attn/
 * qwen3_flex_attention.py:539-551), replacing a bf16 GEMM into [q | k | v]
 * and tg_qk_norm_rope. A persistent tcgen05 GEMM of CTA pairs.
 * x: bf16 (M, K) row stride ld_x; w_qkv: bf16 ((n_q + 2*n_k)*128, K) =
 * [W_q; W_k; W_v] row stride ld_w; out: bf16 (M, (n_q + 2*n_k)*128) row
 * stride ld_out; q_norm_w / k_norm_w: bf16 (128,); cos / sin: bf16, the 128
 * values of row m = b*seq + s at b*cs_sb + s*cs_ss (M a multiple of seq).
 * K a multiple of 64; pointers 16-byte aligned, strides multiples of 8.
 * M == 0 returns TG_OK without touching the pointers. */
int tg_gemm_qkv_rope(const void* x, int64_t ld_x, const void* w_qkv, int64_t ld_w, void* out, int64_t ld_out,
                     int64_t M, int K, int n_q_heads, int n_k_heads, const void* q_norm_w, const void* k_norm_w,
                     const void* cos, const void* sin, int64_t cs_sb, int64_t cs_ss, int seq, float eps,
                     void* stream);

/*
 * a4 (finalized gate) — readout of the scoring branch:
 *   score[b, r] = bf16( sum_k bf16(bf16(silu(g_k)) * u_k) * w[k] ),  stored as fp32
 * over the fused [gate | up] projection row GU[b, row_begin[b] + r] = [g | u]
 * of the LN2-normalised gate-layer boundary, for r < row_count[b].
 *
 * Replaces the scoring branch of the finalized E2EGate,
 *   gate_branch_hs -> br(z) with the absorbed 1-row down_proj
 *   (tokengate/e2e_gate/gate_module/gate_forward.py:491-524, :330-340),
 *   computed in bf16 by CastLinear (e2e_gate_module.py:125-135) and returned
 *   as bf16 (gate_forward.py:521), then cast to the gate's fp32 (:1402-1405).
 * The dot product has a fixed order and silu uses IEEE operations only, so the
 * result is reproducible bit for bit; -0 is stored as +0. bf16(silu(g)) is
 * read from a table of all 65536 bf16 patterns held in the library's device
 * memory (128 KB per device), which each call rewrites on `stream` before its
 * readout: overlapping calls on different streams write the same values.
 *
 * gu: bf16 (B, S, >= 2*inter), strides (gu_sb, gu_ss, 1), rows 16-byte aligned;
 * inter a multiple of 256. w_row: bf16 (inter,), 16-byte aligned.
 * row_begin / row_count: HOST arrays of B ints. scores: fp32, batch stride s_sb.
 */
int tg_branch_score(const void* gu, int64_t gu_sb, int64_t gu_ss, int inter, const void* w_row,
                    int B, const int32_t* row_begin, const int32_t* row_count, float* scores,
                    int64_t s_sb, void* stream);

/*
 * a4 (finalized gate), fused — the scoring branch from the LN2-normalised
 * rows themselves: the [gate | up] projection GEMM with the SwiGLU and the
 * readout row in its epilogue, so the projection never reaches memory:
 *   score[m] = bf16( sum_c bf16(bf16(silu(G[m, c])) * U[m, c]) * w_readout[c] )
 *   G = bf16(x W_gate^T), U = bf16(x W_up^T), silu with IEEE operations only
 * (the activations of tg_branch_score, on this GEMM's own projection). The
 * epilogue leaves one fp32 partial dot per row and 64-column half tile in
 * `partial`; a second kernel on the same stream adds a row's partials in
 * index order and rounds to bf16 (-0 stored as +0). The projection's and the
 * dot's fp32 summation orders are this kernel's own: against the GEMM +
 * tg_branch_score chain a score can differ in its last bf16 bits.
 * Same operation as the reference's gate_branch_hs -> br(z)
 * (tokengate/e2e_gate/gate_module/gate_forward.py:491-524, :330-340).
 *
 * x: bf16 (M, K) row stride ld_x (the state rows of one request);
 * w_gu: bf16 (2*inter, K) = [W_gate; W_up] row stride ld_w; w_readout: bf16
 * (inter,), 16-byte aligned; partial: caller workspace of (inter/64) * M
 * floats; scores: fp32 (M,). K a multiple of 64, inter a multiple of 128.
 * M == 0 returns TG_OK without touching the pointers.
 */
int tg_gemm_swiglu_readout(const void* x, int64_t ld_x, const void* w_gu, int64_t ld_w, const void* w_readout,
                           float* partial, float* scores, int64_t M, int K, int inter, void* stream);

/*
 * The finalized gate's Phase-2 operands of every biased layer
 * from the raw branch scores, in one launch. For request b, kept slot t
 * (position p = keep[b, t]), Phase-2 layer l and head h:
 *   rs      = rsqrt(mean over the state span of score^2 + eps)
 *   b       = bf16(gain * (score[p - state_begin] * rs) * gate_scale[l, h])  (state tokens)
 *   r       = bf16(min(log(max(t + 1, 2)) / log(max(p + 1, 2)), 1))
 *   q_scale[l, b, h, t] = s = bf16(bf16(attn_scale[l, h]) * r)
 *   bias[l, b, h, t]    = bf16(x * bf16(mean_h s)),  x = b on kept state tokens,
 *                         0 on kept non-state tokens, bf16(-1e9) for t >= n_kept[b]
 * gate_scale / attn_scale are the EFFECTIVE (softplus-applied) (L', H) fp32 tables.
 *
 * Replaces E2EGate.forward's sequence RMSNorm x softplus(gate_scale)
 *   (tokengate/e2e_gate/gate_module/e2e_gate_module.py:327-385),
 *   build_gate_bias_vectorized + the -1e9 pads (gate_forward.py:968-1000,
 *   :1463-1469), _ssmax_ratio (:574-585), the per-layer slicing of
 *   _apply_gate_bias (:588-660) and the scaled-softmax prologue
 *   _ssmax_s_eff / _phase2_q_bias (tokengate/e2e_gate/attn/
 *   qwen3_flex_attention.py:417-473).
 *
 * scores: fp32 (B, >= n_state[b]), batch stride s_sb, state token i at i.
 * keep: int64 (B, >= n_alloc), batch stride keep_sb (pads included).
 * state_begin / n_state / n_kept: HOST arrays of B ints.
 * bias / q_scale: fp32 (n_layers, B, n_heads, n_alloc), contiguous; layer l's
 * slice is the (B, H, S) bias / q_row_scale operand of tg_keybias_attn_fwd.
 * n_layers * n_heads <= 4096.
 */
int tg_phase2_tables(const float* scores, int64_t s_sb, int B, const int32_t* state_begin,
                     const int32_t* n_state, const int64_t* keep, int64_t keep_sb,
                     const int32_t* n_kept, int n_alloc, const float* gate_scale,
                     const float* attn_scale, int n_layers, int n_heads, float eps, float gain,
                     float* bias, float* q_scale, void* stream);

/*
 * Decode attention (the decode side of the gated generation): one
 * query token per (batch row, head) against the gated KV cache.
 *
 * Replaces the decode step's attention of the reference's gated generation,
 *   generate_batch (tokengate/e2e_gate/decode/gate_decode.py:139-235) with
 *   FormDecodeState's folded Phase-2 form
 *   (tokengate/e2e_gate/attn/qwen3_flex_attention.py:374-415, :978-1116):
 *   out[b,h,:] = sum_j softmax_j( softmax_scale * (q'[b,h,:] . k[b,j,g,:]) + m[b,h,j] ) v[b,j,g,:]
 *   q' = bf16(q * bf16(q_scale[b,h]))  (q_scale nullable: the per-step
 *        scaled-softmax query scale gamma * r; no scaling when NULL)
 *   m  = bias[b,h,j] for j < n_valid[b]; -inf for n_valid[b] <= j < n_prefix
 *        (pad slots); 0 for n_prefix <= j < n_keys (tokens appended by decode).
 *
 * q: (B, Hq, D) bf16 strides (q_sb, q_sh, 1); k, v: (B, cap >= n_keys, Hkv,
 * D) bf16 strides (k_sb, k_ss, k_sh, 1) — 16-byte aligned with strides
 * multiples of 8. bias: fp32
 * (B, Hq|1, n_prefix) strides (bias_sb, bias_sh, 1) in score units,
 * nullable. n_valid: device int32 (B,). out: (B, Hq, D) bf16. Only D == 128
 * and Hq / Hkv in {1, 2, 4, 8}. workspace: device scratch of
 * tg_decode_attn_workspace bytes (0 when n_keys <= 128), 16-byte aligned;
 * calls sharing it must not overlap on the GPU.
 */
int tg_decode_attn(const void* q, int64_t q_sb, int64_t q_sh,
                   const float* q_scale, int64_t qs_sb,
                   const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                   const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                   const float* bias, int64_t bias_sb, int64_t bias_sh,
                   const int32_t* n_valid, int n_prefix, int n_keys,
                   void* out, int64_t o_sb, int64_t o_sh,
                   void* workspace, size_t workspace_bytes,
                   int B, int Hq, int Hkv, int D, float softmax_scale, void* stream);

/* tg_decode_attn with the key count read on the device: n_keys_dev
 * (device int32, nullable) holds the keys to attend, at most n_keys, which
 * then sizes the grid and the workspace. Lets one launch, captured once,
 * serve decode steps whose cache grows by one key per step. Same reference
 * interface as tg_decode_attn. */
int tg_decode_attn_ex(const void* q, int64_t q_sb, int64_t q_sh,
                      const float* q_scale, int64_t qs_sb,
                      const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                      const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                      const float* bias, int64_t bias_sb, int64_t bias_sh,
                      const int32_t* n_valid, int n_prefix, int n_keys, const int32_t* n_keys_dev,
                      void* out, int64_t o_sb, int64_t o_sh,
                      void* workspace, size_t workspace_bytes,
                      int B, int Hq, int Hkv, int D, float softmax_scale, void* stream);

/* Decode projections: y[b, :] = x[b, :] W^T for B <= 8 rows (the
 * decode step's tokens), x (B, K) bf16 row stride ld_x, W (N, K) bf16
 * row-major row stride ld_w, y (B, N) bf16 row stride ld_y; K a multiple of
 * 256; x and W 16-byte aligned with row strides multiples of 8. With swiglu
 * != 0, W is the fused [gate; up] weight of 2N rows and
 * y[b, j] = bf16(bf16(silu(bf16(g))) * bf16(u)) with g, u rows j and N + j —
 * the decode layer's gate/up projection and SwiGLU in one pass.
 * Replaces the decode step's projections (nn.Linear under the layers of
 * tokengate/e2e_gate/decode/gate_decode.py:199-219) for small batches. */
int tg_gemv(const void* x, int64_t ld_x, const void* w, int64_t ld_w, void* y, int64_t ld_y,
            int B, int N, int K, int swiglu, void* stream);

/* Scratch bytes tg_decode_attn needs (0: one key chunk, none). */
int tg_decode_attn_workspace(int B, int Hq, int n_keys, size_t* bytes);

/*
 * tg_decode_attn for callers that cannot allocate device memory where they
 * call it: a host runtime that binds this library over its FFI while owning
 * the GPU's memory pool itself (so the binding has no allocator to hand a
 * workspace from), or code on a path where a cudaMalloc is not allowed (it
 * can synchronize the device, or the memory budget was fixed up front).
 * Same arguments and results as tg_decode_attn without the workspace: the
 * key-chunk partials go to a fixed 8 MiB buffer the library keeps on every
 * GPU that loads it, until the process exits. Nothing is allocated. A
 * problem needing more than 8 MiB of scratch (B * Hq * ceil(n_keys / 128) *
 * 528 bytes) is rejected with TG_ERR_INVALID_ARGUMENT. The first call on a
 * device looks up the buffer's device address: make it before any stream
 * capture on that device (a first call inside a capture returns
 * TG_ERR_INVALID_ARGUMENT and leaves the capture intact). All calls share the one buffer: calls that
 * overlap on the GPU race and must be serialized by the caller. No
 * counterpart in the reference.
 */
int tg_decode_attn_noalloc(const void* q, int64_t q_sb, int64_t q_sh,
                           const float* q_scale, int64_t qs_sb,
                           const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                           const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                           const float* bias, int64_t bias_sb, int64_t bias_sh,
                           const int32_t* n_valid, int n_prefix, int n_keys,
                           void* out, int64_t o_sb, int64_t o_sh,
                           int B, int Hq, int Hkv, int D, float softmax_scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TOKENGATE_B200_H */
