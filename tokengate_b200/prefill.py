"""Batched gated prefill on the B200 kernels.

Same control flow and return contract as the reference
  prefill_batch_for_decode(model, gate, prompt_ids_list, article_starts,
                           article_ends, gate_layer, K, prune_below_gate=False)
  -> (first_tokens (B,1), cache, kept_positions (B, max_n_kept), n_kepts, K_clampeds)
(tokengate/e2e_gate/gate_module/gate_forward.py:1269-1579):

  Phase 1   layers 0..L on the right-padded full prompts, causal attention
            (the tcgen05 kernel with no bias);
  score     one gate_score launch over every request's state rows;
  select    one topk_select launch: K_clamped = max(1, min(K, n_state)),
            kept positions (prefix, sorted top-K, suffix) and the Phase-2 bias
            row (score at kept state tokens, 0 elsewhere, -1e9 pads);
  compact   one gather launch for the hidden rows (+ the below-gate K/V rows
            of every layer <= L when prune_below_gate);
  Phase 2   layers L+1..N-1 on the kept tokens with the key bias, RoPE at the
            ORIGINAL positions;
  head      final norm of each request's last kept row -> lm_head -> argmax.

With the finalized gate (E2EGate, a scoring branch attached) the gate layer
is split at its attention residual a_j (split_gate_layer_mlp, :345-357):
Phase 1 ends with layer L's attention half; the branch (LN2 -> fused
[gate | up] GEMM -> branch_score readout) scores each request's state rows;
selection is top-K of the raw score, which orders exactly like the
reference's aggregate (a positive scaling of it; ties in one are ties in the
other); phase2_tables builds every Phase-2 layer's per-head bias and
scaled-softmax query scale in one launch; the gate layer's MLP runs on the
kept rows at Phase-2 entry (gate_layer_mlp, :420-435).

The reference's per-request Python loop for scoring/selection/gather and its
host-side index construction are replaced by three batched launches; no host
synchronisation happens between Phase 1 and the head.
"""
import array
import weakref
from typing import List, Optional, Sequence, Union

import torch

from . import ops
from .gate import e2e_kernel_weights, is_e2e_gate, readout_vector
from .layers import fused_weights, layer_attention, layer_forward, layer_mlp
from .model import PrefillCache, set_attn_scale_for_layers, set_gate_bias_for_layers

# Phase-2 length bucket (the reference's set_phase2_bucket, gate_forward.py:531-546):
# None = exact max_n_kept.
_PHASE2_BUCKET: Optional[int] = None


def set_phase2_bucket(n: Optional[int]) -> None:
    global _PHASE2_BUCKET
    _PHASE2_BUCKET = None if n is None else int(n)


# Phase 2 of the fused path through one CUDA graph per shape (tokengate_b200.
# phase2_graph; the reference's _PHASE2_GRAPHS mode, gate_forward.py:531-546,
# :1528-1530). Off by default: the returned cache then aliases the graph's
# buffers until the next prefill of the same shape.
_PHASE2_GRAPHS = False


def set_phase2_graphs(enabled: bool) -> None:
    global _PHASE2_GRAPHS
    _PHASE2_GRAPHS = bool(enabled)


# rows per scoring-branch GEMM: bounds the [gate | up] workspace (rows x 2*inter bf16)
_BRANCH_CHUNK = 32768

# The finalized gate's branch as one fused GEMM (ops.gemm_swiglu_readout: the
# SwiGLU and the readout row in the projection's epilogue) where its shapes
# allow; False runs the projection GEMM and the branch_score readout, whose
# scores are reproducible bit for bit from that projection.
_BRANCH_FUSED = True


def set_branch_fused(enabled: bool) -> None:
    global _BRANCH_FUSED
    _BRANCH_FUSED = bool(enabled)


def _branch_scores(ew, x2: torch.Tensor, starts: Sequence[int], n_state: Sequence[int]) -> torch.Tensor:
    """Raw scores of the finalized gate's branch over each request's state rows.

    x2: (B, S, H) bf16 = post_attention_layernorm(a_j) of the gate layer. Each
    request's state rows are contiguous, so the branch runs on them directly
    (no gather): the fused GEMM (SwiGLU + readout epilogue) per request, or
    the [gate | up] GEMM in chunks of _BRANCH_CHUNK rows followed by the
    branch_score readout. Returns fp32 (B, max n_state)."""
    B = x2.shape[0]
    scores = torch.empty((B, max(n_state)), dtype=torch.float32, device=x2.device)
    inter = ew.w_row.shape[0]
    fused = _BRANCH_FUSED and inter % 128 == 0 and x2.shape[-1] % 64 == 0
    for b in range(B):
        if fused:
            ops.gemm_swiglu_readout(x2[b, starts[b]:starts[b] + n_state[b]], ew.wgu, ew.w_row, out=scores[b])
            continue
        for c0 in range(0, n_state[b], _BRANCH_CHUNK):
            c1 = min(n_state[b], c0 + _BRANCH_CHUNK)
            gu = torch.nn.functional.linear(x2[b, starts[b] + c0:starts[b] + c1], ew.wgu)
            ops.branch_score(gu.unsqueeze(0), ew.w_row, [0], [c1 - c0], out=scores[b:b + 1, c0:])
    return scores


# Phase 1's rotary tables: cos / sin of positions 0..S-1 depend only on the
# rotary module and S, so the fused path computes them once per (module, S,
# device, dtype) and reuses them (expanded over the batch) on later prefills.
_PHASE1_ROPE: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()
_PHASE1_ROPE_MAX = 4


def _phase1_rope(rotary_emb, hidden: torch.Tensor, S: int, B: int):
    key = (S, hidden.device, hidden.dtype)
    per_mod = _PHASE1_ROPE.setdefault(rotary_emb, {})
    hit = per_mod.get(key)
    if hit is None:
        pos = torch.arange(S, device=hidden.device).unsqueeze(0)
        cos, sin = rotary_emb(hidden[:1, :S], pos)
        if len(per_mod) >= _PHASE1_ROPE_MAX:
            per_mod.pop(next(iter(per_mod)))
        hit = per_mod[key] = (cos.contiguous(), sin.contiguous())
    cos, sin = hit
    return cos.expand(B, -1, -1), sin.expand(B, -1, -1)


def _ids_to_device(prompt_ids_list, device) -> torch.Tensor:
    B = len(prompt_ids_list)
    if B == 1 and torch.is_tensor(prompt_ids_list[0]):
        return prompt_ids_list[0].to(device=device, dtype=torch.long, non_blocking=True).reshape(1, -1)
    if all(torch.is_tensor(x) and x.device == torch.device(device) for x in prompt_ids_list):
        # ids already on the GPU (a serving loop's tokens): right-pad there
        lens = [int(x.numel()) for x in prompt_ids_list]
        out = torch.zeros(B, max(lens), dtype=torch.long, device=device)
        for b, x in enumerate(prompt_ids_list):
            out[b, :lens[b]] = x.reshape(-1)
        return out
    lens = [len(x) for x in prompt_ids_list]
    host = torch.zeros(B, max(lens), dtype=torch.long, pin_memory=torch.cuda.is_available())
    for b, ids in enumerate(prompt_ids_list):
        if torch.is_tensor(ids):
            host[b, :lens[b]] = ids
        else:   # list of ints -> int64 buffer without per-element tensor conversion
            host[b, :lens[b]] = torch.frombuffer(array.array("q", ids), dtype=torch.long)
    return host.to(device, non_blocking=True)


@torch.no_grad()
def prefill_batch_for_decode(model: torch.nn.Module, gate, prompt_ids_list: Sequence,
                             article_starts: Sequence[int], article_ends: Sequence[int],
                             gate_layer: int, K: Union[int, Sequence[int]],
                             prune_below_gate: bool = False, fused: Optional[bool] = None,
                             decode_state: Optional[dict] = None):
    """fused: run the decoder layers through the fused glue kernels
    (tokengate_b200.layers); None picks it whenever the gate has no learned
    attention scale. False runs the transformers layers with the patched
    attention module (the reference's structure).

    decode_state: a dict to receive what the decode side folds from this
    prefill (the reference reads the same values from the layers' bias /
    scale attributes, qwen3_flex_attention.py:978-1057): 'bias', one fp32
    (B, H|1, max_n_kept) Phase-2 key bias per layer above the gate;
    'gamma', the (L', H) fp32 scaled-softmax gains or None; 'lens'. Fused
    path only."""
    B = len(prompt_ids_list)
    if B < 1:
        raise ValueError("empty batch")
    if len(article_starts) != B or len(article_ends) != B:
        raise ValueError("one article start/end per prompt")
    inner = model.model
    n_layers = len(inner.layers)
    if not 0 <= gate_layer < n_layers - 1:
        raise ValueError(f"gate_layer {gate_layer} must leave at least one Phase-2 layer")
    device = next(model.parameters()).device
    lens = [int(x.numel()) if torch.is_tensor(x) else len(x) for x in prompt_ids_list]
    starts = [int(s) for s in article_starts]
    ends = [int(e) for e in article_ends]
    for b in range(B):
        if not 0 <= starts[b] < ends[b] <= lens[b]:
            raise ValueError(f"request {b}: state span [{starts[b]}, {ends[b]}) invalid for length {lens[b]}")
    max_seq_len = max(lens)
    e2e = is_e2e_gate(gate)
    has_attn_scale = hasattr(gate, "attn_scale_eff") and not getattr(gate, "_baseline_no_bias_scale", False)
    if fused is None:
        fused = e2e or not has_attn_scale
    if e2e:
        if not fused:
            raise NotImplementedError("the finalized gate is served by the fused layer path (fused=True)")
        if getattr(gate, "selection_mode", "topk") != "topk" or getattr(gate, "random_topk", False):
            raise NotImplementedError("only top-K selection is served by the B200 selection kernel")
        if getattr(gate, "_baseline_no_bias_scale", False):
            raise NotImplementedError("the selection-only baseline mode of the finalized gate is not served")
        if gate.n_layers_bias != n_layers - 1 - gate_layer:
            raise ValueError(f"n_layers_bias mismatch: gate has {gate.n_layers_bias} layer slots, the model "
                             f"has {n_layers - 1 - gate_layer} layers above gate_layer={gate_layer}")
        if gate.n_heads != model.config.num_attention_heads:
            raise ValueError(f"gate has {gate.n_heads} heads, the model {model.config.num_attention_heads} "
                             f"query heads (the bias is per Phase-2 query head)")
        ew = e2e_kernel_weights(gate, device)
    elif fused and has_attn_scale:
        raise NotImplementedError("the fused layer path serves gates without a learned attention scale")
    fw = fused_weights(model) if fused else None

    # ---- Phase 1
    ids = _ids_to_device(prompt_ids_list, device)
    set_gate_bias_for_layers(model, 0, gate_layer + 1, None)
    hidden = inner.embed_tokens(ids)
    cache = PrefillCache(n_layers)
    x2 = None
    pe = None
    if fused:
        cos, sin = rope1 = _phase1_rope(inner.rotary_emb, hidden, max_seq_len, B)
        delta = None
        for i in range(gate_layer if e2e else gate_layer + 1):
            hidden, delta = layer_forward(fw[i], hidden, delta, cos, sin, cache, i)
        if e2e:   # Phase 1 ends at the gate layer's attention residual a_j
            hidden, x2 = layer_attention(fw[gate_layer], hidden, delta, cos, sin, cache, gate_layer)
        else:
            hidden, _ = ops.add_rmsnorm(hidden, delta, None, 0.0, h_out=hidden, want_x=False)
        del delta, cos, sin
    else:
        position_ids = torch.arange(max_seq_len, device=device).unsqueeze(0).expand(B, -1)
        pe = inner.rotary_emb(hidden, position_ids)
        for i in range(gate_layer + 1):
            hidden = inner.layers[i](hidden, attention_mask=None, position_ids=position_ids,
                                     past_key_values=cache, use_cache=True, position_embeddings=pe)
    del pe

    # ---- score + select
    n_state = [e - s for s, e in zip(starts, ends)]
    if e2e:
        scores = _branch_scores(ew, x2, starts, n_state)
        del x2
    else:
        w = readout_vector(gate, hidden.shape[-1], device)
        scores = ops.gate_score(hidden, w, starts, n_state)
    Ks = list(K) if isinstance(K, (list, tuple)) else [K] * B
    K_clampeds = [max(1, min(int(Ks[b]), n_state[b])) for b in range(B)]
    n_kepts = [starts[b] + K_clampeds[b] + (lens[b] - ends[b]) for b in range(B)]
    max_n_kept = max(n_kepts)
    n_alloc = max_n_kept if _PHASE2_BUCKET is None else -(-max_n_kept // _PHASE2_BUCKET) * _PHASE2_BUCKET
    if e2e:
        # every aggregate 0 when all first-layer scales are 0: index order decides
        sel = torch.zeros_like(scores) if ew.degenerate else scores
        kept_positions, bias_row, _ = ops.topk_select(sel, n_state, K_clampeds, starts, lens, n_alloc,
                                                      bias_dtype=None)
        bias_tab, qs_tab = ops.phase2_tables(scores, starts, n_state, kept_positions, n_kepts,
                                             ew.gate_scale, ew.attn_scale, ew.eps, ew.gain)
    else:
        kept_positions, bias_row, _ = ops.topk_select(scores, n_state, K_clampeds, starts, lens,
                                                      n_alloc, bias_dtype=hidden.dtype)

    # ---- compact
    H = hidden.shape[-1]
    hs_pruned = torch.empty((B, n_alloc, H), dtype=hidden.dtype, device=device)
    specs = [ops.gather_spec_rows(hidden, hs_pruned, 1)]
    if prune_below_gate:
        pruned_kv = []
        for li in range(gate_layer + 1):
            lc = cache.layers[li]
            kd = lc.k_tok.new_empty((B, max_n_kept) + tuple(lc.k_tok.shape[2:]))
            vd = lc.v_tok.new_empty((B, max_n_kept) + tuple(lc.v_tok.shape[2:]))
            specs.append(ops.gather_spec_rows(lc.k_tok, kd, 1))
            specs.append(ops.gather_spec_rows(lc.v_tok, vd, 1))
            pruned_kv.append((kd, vd))
    if prune_below_gate and max_n_kept != n_alloc:
        # below-gate caches are max_n_kept wide (reference: pad to max_n_kept); one launch per width
        ops.gather_rows(specs[:1], kept_positions, n_kepts, n_alloc, device)
        ops.gather_rows(specs[1:], kept_positions, n_kepts, max_n_kept, device)
    else:
        ops.gather_rows(specs, kept_positions, n_kepts, n_alloc, device)
    if prune_below_gate:
        for li, (kd, vd) in enumerate(pruned_kv):
            cache.layers[li].k_tok, cache.layers[li].v_tok = kd, vd
    del hidden, scores

    # ---- Phase 2
    if fused:
        # the kept positions' rotary rows, gathered from Phase 1's table of
        # positions 0..S-1 (the same values the rotary module gives them; pad
        # slots hold position 0, so every row is gathered)
        D = rope1[0].shape[-1]
        cos2 = torch.empty((B, n_alloc, D), dtype=rope1[0].dtype, device=device)
        sin2 = torch.empty_like(cos2)
        ops.gather_rows([ops.gather_spec_rows(rope1[0], cos2, 1), ops.gather_spec_rows(rope1[1], sin2, 1)],
                        kept_positions, [n_alloc] * B, n_alloc, device)
        pe2 = (cos2, sin2)
        del rope1
    else:
        pe2 = inner.rotary_emb(hs_pruned, kept_positions)
    # pinned source, asynchronous copy: a pageable one would synchronise the stream
    last_valid = torch.tensor([n - 1 for n in n_kepts], dtype=torch.long,
                              pin_memory=torch.cuda.is_available()).to(device, non_blocking=True)
    rows = torch.arange(B, device=device)
    graphed = None
    if fused and _PHASE2_GRAPHS:
        from .phase2_graph import run_phase2
        cos2, sin2 = pe2
        if e2e:
            graphed = run_phase2(model, fw, gate_layer, hs_pruned, cos2, sin2, bias_tab, qs_tab, cache, True)
        else:
            graphed = run_phase2(model, fw, gate_layer, hs_pruned, cos2, sin2,
                                 bias_row.float().unsqueeze(1), None, cache, False)
    if graphed is not None:
        hs_pruned, delta = graphed
        h_last = hs_pruned[rows, last_valid]
        _, hs_last = ops.add_rmsnorm(h_last, delta[rows, last_valid], inner.norm.weight,
                                     float(inner.norm.variance_epsilon))
    elif e2e:
        cos2, sin2 = pe2
        # Phase-2 entry: the gate layer's own MLP on the kept rows (zero pad rows stay zero)
        _, x2p = ops.add_rmsnorm(hs_pruned, None, fw[gate_layer].post_w, fw[gate_layer].eps)
        delta = layer_mlp(fw[gate_layer], x2p)
        del x2p
        for i in range(gate_layer + 1, n_layers):
            li = i - gate_layer - 1
            hs_pruned, delta = layer_forward(fw[i], hs_pruned, delta, cos2, sin2, cache, i,
                                             gate_bias=bias_tab[li], q_row_scale=qs_tab[li])
        h_last = hs_pruned[rows, last_valid]
        _, hs_last = ops.add_rmsnorm(h_last, delta[rows, last_valid], inner.norm.weight,
                                     float(inner.norm.variance_epsilon))
    elif fused:
        # The reference hands the bf16 bias to every layer and each converts it to
        # fp32 (_bias_bhs); converting once here gives the same values.
        bias3 = bias_row.float().unsqueeze(1)               # (B, 1, n_alloc): one row for all heads
        cos2, sin2 = pe2
        delta = None
        for i in range(gate_layer + 1, n_layers):
            hs_pruned, delta = layer_forward(fw[i], hs_pruned, delta, cos2, sin2, cache, i,
                                             gate_bias=bias3)
        # final residual add + norm only on the rows the head reads
        h_last = hs_pruned[rows, last_valid]
        _, hs_last = ops.add_rmsnorm(h_last, delta[rows, last_valid], inner.norm.weight,
                                     float(inner.norm.variance_epsilon))
    else:
        # the bias in the model dtype, scaled there by an attention scale as the
        # reference's is; _bias_bhs widens it to fp32 for the kernel
        set_gate_bias_for_layers(model, gate_layer + 1, n_layers, bias_row, per_head=False)
        attn_scale = gate.attn_scale_eff() if has_attn_scale else None
        set_attn_scale_for_layers(model, gate_layer + 1, n_layers, attn_scale)
        for i in range(gate_layer + 1, n_layers):
            hs_pruned = inner.layers[i](hs_pruned, attention_mask=None, position_ids=kept_positions,
                                        past_key_values=cache, use_cache=True, position_embeddings=pe2)
        hs_last = inner.norm(hs_pruned[rows, last_valid])

    if decode_state is not None:
        if not fused:
            raise NotImplementedError("decode_state is filled by the fused layer path")
        if e2e:
            decode_state["bias"] = [bias_tab[li][:, :, :max_n_kept] for li in range(n_layers - 1 - gate_layer)]
            decode_state["gamma"] = ew.attn_scale
        else:
            row = bias_row[:, :max_n_kept].float().unsqueeze(1)
            decode_state["bias"] = [row] * (n_layers - 1 - gate_layer)
            decode_state["gamma"] = None
        decode_state["lens"] = lens

    # ---- head
    first_tokens = model.lm_head(hs_last).argmax(-1, keepdim=True)
    if n_alloc != max_n_kept:
        for i in range(gate_layer + 1, n_layers):
            lc = cache.layers[i]
            lc.k_tok = lc.k_tok[:, :max_n_kept]
            lc.v_tok = lc.v_tok[:, :max_n_kept]
        kept_positions = kept_positions[:, :max_n_kept]
    return first_tokens, cache, kept_positions, n_kepts, K_clampeds
