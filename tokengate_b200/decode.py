"""Gated generation: the prefill, then greedy decode over the gated KV cache.

Mirrors the reference's one generation implementation, generate_batch
(tokengate/e2e_gate/decode/gate_decode.py:87-260), with its decode-side
contracts:

  * the cache layout the prefill leaves: layers above the gate hold the
    kept tokens (B, max_n_kept) with rows shorter than max_n_kept padded at
    the end, layers at and below the gate their full padded Phase-1 cache
    (B, max prompt length) — or the kept tokens with prune_below_gate;
    decoded tokens are appended after that prefix (:139-165);
  * the pad-slot mask: prefix slots past each row's valid length are never
    attended (:141-150, :152-164);
  * the folded Phase-2 softmax form (FormDecodeState,
    qwen3_flex_attention.py:978-1116): above the gate, every prefix key keeps
    the additive bias the prefill gave it (for the finalized gate the
    per-head bias times the head-mean scaled-softmax factor of the key's own
    ratio), decoded keys get none, and each decode query is scaled by
    gamma_h * r with r = min(log(max(n_kept + 1 + step, 2)) /
    log(max(pos + 1, 2)), 1) in float32, cast to bf16 (:374-415, :1089-1101);
    phase2_form=False is the plain decode (no bias, no query scale);
  * RoPE at the original positions: the first decode token sits one past
    the last kept position (:137-138);
  * stop when every row's last token is EOS; answers cut at the first EOS.

Each decode step runs the fused layer ops (residual add + RMSNorm, one
[q; k; v] projection, q/k RMSNorm + RoPE, the tg_decode_attn kernel over
the cache, o projection, SwiGLU MLP) and the head.
"""
import time
from dataclasses import dataclass
from typing import List, Optional, Sequence, Union

import torch
import torch.nn.functional as F

from . import ops
from .layers import fused_weights
from .prefill import prefill_batch_for_decode


@dataclass
class GateGenerateResult:
    token_ids: List[List[int]]  # generated ids per row, through the first EOS inclusive
    n_gen: List[int]            # generated tokens per row before the first EOS
    n_kepts: List[int]
    kept_pos: torch.Tensor      # (B, max_n_kept) original positions, on the device
    K_clampeds: List[int]
    prefill_s: float
    decode_s: float
    steps: int                  # decode steps run (batch-wide)


def _sync(device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def _proj(x: torch.Tensor, w: torch.Tensor, swiglu: bool = False, gemv: bool = True) -> torch.Tensor:
    """A decode-step projection of the (B, 1, K) rows: the tg_gemv kernel
    where it beats cuBLAS on B200 (measured: every projection at B <= 2, the
    layer projections at B <= 4; its CUDA-core FMAs fall behind cuBLAS's
    tensor cores beyond that, first on the 151936-row lm_head), cuBLAS
    otherwise or when gemv is False."""
    B, _, Kd = x.shape
    if gemv and Kd % 256 == 0 and (B <= 2 or (B <= _GEMV_LAYER_MAX_B and w.shape[0] < 32768)):
        return ops.gemv(x.view(B, Kd), w, swiglu=swiglu).view(B, 1, -1)
    y = F.linear(x, w)
    return ops.silu_mul(y) if swiglu else y


# the largest batch whose layer projections (fewer than 32768 output rows)
# run on tg_gemv (measured on B200: at B = 6 and 8 the decode step is
# 8-15 % slower with them there than on cuBLAS)
_GEMV_LAYER_MAX_B = 4


class _DecodeCache:
    """Per-layer K/V with room for the decoded tokens: the prefill's prefix
    copied to the front, decode tokens appended after it."""

    def __init__(self, cache, n_layers: int, extra: int):
        self.k, self.v, self.width = [], [], []
        for i in range(n_layers):
            k, v = cache.layers[i].k_tok, cache.layers[i].v_tok
            B, W, Hkv, D = k.shape
            kb = torch.empty((B, W + extra, Hkv, D), dtype=k.dtype, device=k.device)
            vb = torch.empty_like(kb)
            kb[:, :W].copy_(k)
            vb[:, :W].copy_(v)
            self.k.append(kb)
            self.v.append(vb)
            self.width.append(W)


@torch.no_grad()
def generate_batch(model, gate, prompt_ids_list: Sequence, article_starts: Sequence[int],
                   article_ends: Sequence[int], gate_layer: int, max_kept_prefill_tokens,
                   max_new_tokens: int, *, eos_token_id: Optional[int] = None,
                   phase2_form: bool = True, prune_below_gate: bool = False,
                   streamer=None, forced_tokens: Optional[torch.Tensor] = None,
                   logits_out: Optional[list] = None, use_graph: bool = True,
                   use_gemv: bool = True) -> GateGenerateResult:
    """Gated prefill + greedy decode of up to max_new_tokens tokens per row.

    forced_tokens: (B, max_new_tokens - 1) ids fed to the decode steps in
    place of the previous step's argmax (teacher forcing, to score a given
    continuation);
    logits_out: a list that receives each decode step's (B, vocab) fp32 logits;
    use_graph: replay the decode step as one CUDA graph after the first
    (eager) step — the state a step reads (token, position, append slot, key
    count) lives in device buffers the step itself advances; use_gemv: the
    decode projections on the tg_gemv kernel (False: cuBLAS)."""
    if max_new_tokens < 1:
        raise ValueError("max_new_tokens must be positive")
    device = next(model.parameters()).device
    inner = model.model
    n_layers = len(inner.layers)
    st: dict = {}
    _sync(device)
    t0 = time.perf_counter()
    first, cache, kept_pos, n_kepts, K_cl = prefill_batch_for_decode(
        model, gate, prompt_ids_list, article_starts, article_ends, gate_layer,
        max_kept_prefill_tokens, prune_below_gate=prune_below_gate, fused=True, decode_state=st)
    _sync(device)
    prefill_s = time.perf_counter() - t0
    B = first.shape[0]
    if streamer is not None:
        streamer.put(first.detach().cpu())
    gen = [first]
    steps = 0
    t1 = time.perf_counter()
    if max_new_tokens > 1:
        fw = fused_weights(model)
        lens = st["lens"]
        dc = _DecodeCache(cache, n_layers, max_new_tokens - 1)
        del cache
        n_kept_dev = torch.tensor(n_kepts, dtype=torch.int32, device=device)
        valid_below = n_kept_dev if prune_below_gate else torch.tensor(lens, dtype=torch.int32, device=device)
        last = torch.tensor([n - 1 for n in n_kepts], device=device)
        next_pos = kept_pos[torch.arange(B, device=device), last] + 1            # (B,)
        n_p2 = n_layers - 1 - gate_layer
        bias = st["bias"] if phase2_form else [None] * n_p2
        qs_all = None
        if phase2_form and st["gamma"] is not None:
            # the per-step query scale of every Phase-2 layer, computed as
            # FormDecodeState.step does (float32 on the device)
            s_idx = torch.arange(max_new_tokens - 1, device=device, dtype=torch.float32)[:, None]
            m = (n_kept_dev.float()[None, :] + 1 + s_idx).clamp(min=2.0)               # (steps, B)
            pp = (next_pos.float()[None, :] + s_idx + 1.0).clamp(min=2.0)
            r = (torch.log(m) / torch.log(pp)).clamp(max=1.0)
            gam = st["gamma"].float()                                                   # (L', H)
            qs_all = (gam[None, :, None, :] * r[:, None, :, None]).contiguous()        # (steps, L', B, H)
        lw0 = fw[0]
        nq, nkv, D = lw0.n_q, lw0.n_kv, lw0.head_dim
        # step state on the device, so that one captured step serves every
        # step: the token, its position, each cache's append slot and key count
        cur = first.clone()
        wb, w2 = dc.width[0], dc.width[n_layers - 1]
        extra = max_new_tokens - 1
        # the counters one step advances, one add each: the two caches' append
        # slots and the step index (int64), the two key counts (int32)
        ctr = torch.tensor([wb, w2, 0], dtype=torch.int64, device=device)
        slot_b, slot_2, step_idx = ctr[0:1], ctr[1:2], ctr[2:3]
        nkc = torch.tensor([wb + 1, w2 + 1], dtype=torch.int32, device=device)
        nk_b, nk_2 = nkc[0:1], nkc[1:2]
        # the rotary cos / sin of every decode position, made once by the
        # model's own rotary embedding (elementwise in the position, so equal
        # to making them step by step); a step gathers its row
        step_pos = next_pos.view(B, 1) + torch.arange(extra, device=device).view(1, extra)      # (B, extra)
        like = torch.empty((B, 1, 1), dtype=inner.embed_tokens.weight.dtype, device=device)
        cos_t, sin_t = inner.rotary_emb(like, step_pos)
        rot = torch.stack((cos_t, sin_t), dim=2)                                                 # (B, extra, 2, D)
        qs_cur = torch.empty_like(qs_all[0]) if qs_all is not None else None
        lg_buf = torch.empty((B, model.lm_head.weight.shape[0]), dtype=torch.float32, device=device)

        def step_body():
            h = inner.embed_tokens(cur)                                               # (B, 1, H)
            r = rot.index_select(1, step_idx)                                         # (B, 1, 2, D)
            cos, sin = r[:, :, 0], r[:, :, 1]
            delta = None
            for i in range(n_layers):
                lw = fw[i]
                below = i <= gate_layer
                h, x = ops.add_rmsnorm(h, delta, lw.in_w, lw.eps, h_out=h if delta is not None else None)
                qkv = _proj(x, lw.wqkv, gemv=use_gemv).view(B, 1, nq + 2 * nkv, D)
                q = qkv[:, :, :nq]
                k = qkv[:, :, nq:nq + nkv]
                v = qkv[:, :, nq + nkv:]
                ops.qk_norm_rope_append(q, k, v, lw.q_norm_w, lw.k_norm_w, cos, sin, lw.qk_eps,
                                        dc.k[i], dc.v[i], slot_b if below else slot_2)
                W = dc.width[i]
                if below:
                    a = ops.decode_attention(q[:, 0], dc.k[i], dc.v[i], valid_below, W, W + extra,
                                             n_keys_dev=nk_b)
                else:
                    li = i - gate_layer - 1
                    a = ops.decode_attention(q[:, 0], dc.k[i], dc.v[i], n_kept_dev, W, W + extra,
                                             bias=bias[li], q_scale=qs_cur[li] if qs_cur is not None else None,
                                             n_keys_dev=nk_2)
                o = _proj(a.view(B, 1, nq * D), lw.wo, gemv=use_gemv)
                h, x2 = ops.add_rmsnorm(h, o, lw.post_w, lw.eps, h_out=h)
                delta = _proj(_proj(x2, lw.wgu, swiglu=True, gemv=use_gemv), lw.wdown, gemv=use_gemv)
            _, hn = ops.add_rmsnorm(h, delta, inner.norm.weight, float(inner.norm.variance_epsilon))
            lg = _proj(hn, model.lm_head.weight, gemv=use_gemv)[:, -1]
            lg_buf.copy_(lg)
            cur.copy_(lg.argmax(-1, keepdim=True))
            ctr.add_(1)
            nkc.add_(1)

        graph = None
        eos_seen = torch.zeros(B, dtype=torch.bool, device=device)
        for step in range(extra):
            if eos_token_id is not None:
                eos_seen |= cur[:, 0] == eos_token_id
                if bool(eos_seen.all()):
                    break
            if forced_tokens is not None:
                cur.copy_(forced_tokens[:, step:step + 1].to(device=device, dtype=cur.dtype))
            if qs_cur is not None:
                qs_cur.copy_(qs_all[step])
            if graph is None and use_graph and step > 0:
                # the first step ran eagerly (library handles, kernel attributes);
                # capture the same body once, replay it for the rest
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    step_body()
            if graph is not None:
                graph.replay()
            else:
                step_body()
            if logits_out is not None:
                logits_out.append(lg_buf.clone())
            nxt = cur.clone()
            if streamer is not None:
                streamer.put(nxt.detach().cpu())
            gen.append(nxt)
            steps += 1
        del graph
    _sync(device)
    decode_s = time.perf_counter() - t1
    if streamer is not None:
        streamer.end()
    allg = torch.cat(gen, dim=1).cpu().tolist()
    token_ids, n_gen = [], []
    for row in allg:
        if eos_token_id is not None and eos_token_id in row:
            end = row.index(eos_token_id)
            token_ids.append(row[:end + 1])
            n_gen.append(end)
        else:
            token_ids.append(row)
            n_gen.append(len(row))
    return GateGenerateResult(token_ids, n_gen, list(n_kepts), kept_pos, list(K_cl), prefill_s, decode_s, steps)
