"""CPU ORACLE (test infrastructure and the benchmark's CPU baseline legs only):
the reference's CPU torch paths for the key-bias attention op and for the
gate-scoring / selection / compaction ops, restated so they can be timed on
a machine where the reference checkout is absent.

  flex_keybias_attention  flex_attention_gate_bias (tokengate/e2e_gate/attn/
        flex_attention_utils.py:233-287): the scalar-per-key or per-head
        score_mod (:174-198) adds the bias to each score, a causal block mask
        (get_causal_block_mask) keeps keys <= query, GQA inside the op
        (enable_gqa, :201-210). Called through torch's FlexAttention WITHOUT
        torch.compile: compiled FlexAttention on the CPU fails in this torch
        build (an Inductor cpp_micro_gemm assertion), so on the CPU the
        reference's path runs torch's unfused implementation, which
        materialises the score matrix.
  sdpa_causal             sdpa_compat.sdpa_causal (tokengate/e2e_gate/attn/
        sdpa_compat.py:6-37): GQA by repeating K/V heads, query chunks of 128
        rows against the key prefix they can see, the bias plus a causal -inf
        in an additive mask, F.scaled_dot_product_attention.
  gate_select_compact     the reference's per-request torch ops between the
        phases: scores = logsigmoid(linear(h_state.float())) (gate_forward.py:
        1396-1407), torch.topk of K_clamped = max(1, min(K, n_state)) scores
        (:84-99, :1409-1410), the sorted keep list [0, start) ++ start +
        sort(topk) ++ [end, len) (:1417-1421), the advanced-index gather of the
        kept hidden rows (:1443-1461) and index_select of the below-gate K/V
        rows (:1491-1522).

Inputs follow the reference's layouts: Q/K/V (B, H, S, D); gate_bias (S,),
(B, S), (S, H) or (B, S, H).
"""
from typing import Dict, List, Sequence

import torch
import torch.nn.functional as F

_BLOCK_MASKS: Dict[tuple, object] = {}


def _causal_block_mask(S: int):
    from torch.nn.attention.flex_attention import create_block_mask
    key = (S,)
    if key not in _BLOCK_MASKS:
        _BLOCK_MASKS[key] = create_block_mask(lambda b, h, q, kv: q >= kv, None, None, S, S, device="cpu")
    return _BLOCK_MASKS[key]


def flex_keybias_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, gate_bias: torch.Tensor,
                           per_head: bool = False) -> torch.Tensor:
    """Causal attention + additive per-key bias through torch FlexAttention (uncompiled)."""
    import warnings
    from torch.nn.attention.flex_attention import flex_attention
    S = Q.shape[2]
    bias = gate_bias
    if per_head:
        mod = (lambda s, b, h, q, kv: s + bias[kv, h]) if bias.dim() == 2 else \
              (lambda s, b, h, q, kv: s + bias[b, kv, h])
    else:
        mod = (lambda s, b, h, q, kv: s + bias[kv]) if bias.dim() == 1 else \
              (lambda s, b, h, q, kv: s + bias[b, kv])
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")   # torch warns that the uncompiled path is unfused
        return flex_attention(Q, K, V, score_mod=mod, block_mask=_causal_block_mask(S),
                              enable_gqa=K.shape[1] != Q.shape[1])


def _bias_bhs(gate_bias: torch.Tensor, per_head: bool, B: int, H: int, S: int) -> torch.Tensor:
    """Any reference gate_bias layout -> (B, H, S) (flex_attention_utils.py:686-695)."""
    b = gate_bias
    if b.dim() == 1 or (b.dim() == 2 and not per_head):
        b = b.reshape(1, -1, 1) if b.dim() == 1 else b[:, :, None]
    elif b.dim() == 2:
        b = b[None]
    return b.permute(0, 2, 1).expand(B, H, S)


def sdpa_causal(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, gate_bias=None, per_head: bool = False,
                chunk_size: int = 128) -> torch.Tensor:
    """Chunked exact causal attention with an optional additive key bias."""
    B, H, S, _ = Q.shape
    groups = H // K.shape[1]
    if groups > 1:
        K = K.repeat_interleave(groups, dim=1)
        V = V.repeat_interleave(groups, dim=1)
    bias = None if gate_bias is None else _bias_bhs(gate_bias, per_head, B, H, S).unsqueeze(-2)
    out = []
    for c0 in range(0, S, chunk_size):
        c1 = min(c0 + chunk_size, S)
        allowed = torch.arange(c1)[None, :] <= torch.arange(c0, c1)[:, None]
        mask = torch.zeros((c1 - c0, c1), dtype=Q.dtype)
        if bias is not None:
            mask = mask + bias[..., :c1].to(Q.dtype)
        mask = mask.masked_fill(~allowed, float("-inf"))
        out.append(F.scaled_dot_product_attention(Q[:, :, c0:c1], K[:, :, :c1], V[:, :, :c1], attn_mask=mask))
    return torch.cat(out, dim=2)


def gate_select_compact(hidden: torch.Tensor, w: torch.Tensor, start: int, end: int, K: int,
                        kv: Sequence[torch.Tensor] = ()) -> dict:
    """One request: hidden (S, H) in the model dtype, w (H,) fp32, kv a list of
    (Hkv, S, D) below-gate K/V tensors. Returns the scores, the kept positions,
    the compacted hidden rows and K/V rows."""
    seq = hidden.shape[0]
    scores = F.logsigmoid(F.linear(hidden[start:end].float(), w.view(1, -1))).view(-1)
    kc = max(1, min(int(K), end - start))
    top = torch.topk(scores, kc).indices
    keep = torch.cat([torch.arange(start), start + torch.sort(top).values, torch.arange(end, seq)])
    h_kept = hidden[keep]
    kv_kept: List[torch.Tensor] = [t.index_select(1, keep) for t in kv]
    return dict(scores=scores, keep=keep, hidden=h_kept, kv=kv_kept, K_clamped=kc)
