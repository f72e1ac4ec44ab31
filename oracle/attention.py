"""CPU ORACLE (test infrastructure): causal GQA attention with a per-key bias.

Restates, in float64 numpy, the reference's exact compatibility path
  tokengate/e2e_gate/attn/sdpa_compat.py:6-37  (sdpa_causal: bias added to the
  scaled logits, causal -inf mask, softmax, @ V, GQA by repeating K/V heads)
and the FlexAttention score_mod it must agree with
  tokengate/e2e_gate/attn/flex_attention_utils.py:174-198  (score + bias[b, kv]
  or bias[b, kv, h]),
with the bias layouts of _bias_bhs (flex_attention_utils.py:686-695).
"""
import numpy as np


def bias_bhs(gate_bias, per_head: bool, B: int, H: int, S: int) -> np.ndarray:
    """Any reference gate_bias layout -> (B, H, S) float64.

    (S,) and (B, S) are scalar-per-key; (S, H) and (B, S, H) are per head
    (flex_attention_utils.py:686-695).
    """
    b = np.asarray(gate_bias, dtype=np.float64)
    if b.ndim == 1 or (b.ndim == 2 and not per_head):
        b = b.reshape(1, -1, 1) if b.ndim == 1 else b[:, :, None]
    elif b.ndim == 2:
        b = b[None]
    if b.shape[-2] != S:
        raise ValueError(f"gate_bias covers {b.shape[-2]} tokens, K/V {S}")
    return np.broadcast_to(np.transpose(b, (0, 2, 1)), (B, H, S))


def keybias_attention(q, k, v, bias_bhs_=None, scale=None, causal=True, rows=None,
                      q_row_scale=None):
    """out (B, n_rows, Hq, D), lse (B, Hq, n_rows) in float64.

    q: (B, Sq, Hq, D), k/v: (B, Sk, Hkv, D) (token-major, as the kernel reads
    them); bias_bhs_: (B, Hq, Sk) score-unit bias or None; rows: query indices
    to evaluate (default all); q_row_scale: (B, Hq, Sq) or None (multiplies
    the row's logits before the bias, the fused Phase-2 query scale).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    G = Hq // Hkv
    if scale is None:
        scale = D ** -0.5
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    out = np.zeros((B, len(rows), Hq, D))
    lse = np.zeros((B, Hq, len(rows)))
    keys = np.arange(Sk)
    for b in range(B):
        for h in range(Hq):
            kh = k[b, :, h // G]
            vh = v[b, :, h // G]
            for c0 in range(0, len(rows), 256):
                rr = rows[c0:c0 + 256]
                s = (q[b, rr, h] @ kh.T) * scale
                if q_row_scale is not None:
                    s = s * np.asarray(q_row_scale, dtype=np.float64)[b, h, rr][:, None]
                if bias_bhs_ is not None:
                    s = s + np.asarray(bias_bhs_, dtype=np.float64)[b, h][None, :]
                if causal:
                    s = np.where(keys[None, :] <= rr[:, None], s, -np.inf)
                m = s.max(axis=1, keepdims=True)
                p = np.exp(s - m)
                l = p.sum(axis=1, keepdims=True)
                out[b, c0:c0 + len(rr), h] = (p @ vh) / l
                lse[b, h, c0:c0 + len(rr)] = (m + np.log(l))[:, 0]
    return out, lse
