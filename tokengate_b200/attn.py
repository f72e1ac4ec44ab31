"""Attention operator surface of the gated prefill, served by the B200 kernel.

Mirrors the reference dispatch functions (same names, argument meaning and
error behaviour):
  attention_causal(Q, K, V, backend)                      flex_attention_utils.py:477-495
  attention_gate_bias(Q, K, V, gate_bias, per_head, backend)   :498-517
  _bias_bhs(gate_bias, per_head, B, H, S)                 :686-695
Q, K, V are (B, heads, S, D) tensors — in the reference they are the
transposed views of (B, S, heads, D) projections (qwen3_flex_attention.py:
539-541) and are passed to the kernel as they are, strides and all.

There is one backend, "b200" (the tcgen05 key-bias kernel). The reference's
default name "fa2-bias" (and "fa2" in GATE_ATTN), which named the FA2 key-bias
kernel this one replaces, is accepted as an alias. Any other name raises:
no multi-backend dispatch and no CPU fallback.
"""
import torch

from .keybias import keybias_attention_bhsd

BACKEND = "b200"
CAUSAL_BACKENDS = ("b200",)
BIAS_BACKENDS = ("b200",)
_ALIASES = {"fa2-bias": "b200", "flash": "b200", "b200": "b200"}

# name -> (causal backend, gate-bias backend), as the reference's GATE_ATTN
# (qwen3_flex_attention.py:1158-1171); "fa2" was the reference's default.
GATE_ATTN = {
    "b200": ("b200", "b200"),
    "fa2": ("b200", "b200"),
}


def resolve_backend(name: str, causal: bool) -> str:
    to = _ALIASES.get(name)
    if to is None:
        kind = "causal" if causal else "gate-bias"
        options = CAUSAL_BACKENDS if causal else BIAS_BACKENDS
        raise ValueError(f"{kind} attention backend {name!r} not in {options} "
                         f"(aliases: {sorted(k for k in _ALIASES if k != 'b200')})")
    return to


def _bias_bhs(gate_bias: torch.Tensor, per_head: bool, B: int, H: int, S: int) -> torch.Tensor:
    """gate_bias in any of its layouts -> fp32 broadcastable to (B, H, S).

    (S,) / (B, S) scalar per key -> (1|B, 1, S); (S, H) / (B, S, H) per head
    -> (1|B, H, S). The reference expands to (B, H, S); the kernel reads the
    broadcast (zero-stride) dims directly, so nothing is materialised beyond
    the fp32 cast.
    """
    b = gate_bias
    if b.dim() == 1 or (b.dim() == 2 and not per_head):
        b = b.reshape(1, 1, -1) if b.dim() == 1 else b.unsqueeze(1)        # (B|1, 1, S)
    elif b.dim() == 2:
        b = b.t().unsqueeze(0)                                             # (1, H, S)
    elif b.dim() == 3:
        b = b.permute(0, 2, 1)                                             # (B, H, S)
    else:
        raise ValueError(f"gate_bias must be 1-3 dimensional, got {tuple(gate_bias.shape)}")
    if b.shape[-1] != S:
        raise ValueError(f"gate_bias covers {b.shape[-1]} tokens, K/V {S}")
    if b.shape[0] not in (1, B) or b.shape[1] not in (1, H):
        raise ValueError(f"gate_bias {tuple(gate_bias.shape)} does not match B={B}, H={H}")
    b = b.float()
    if b.stride(-1) != 1:
        b = b.contiguous()
    return b


def _gqa_check(Q, K):
    if Q.shape[1] % K.shape[1] != 0:
        raise ValueError(f"query heads {Q.shape[1]} not a multiple of kv heads {K.shape[1]}")


def attention_causal(Q, K, V, backend: str = BACKEND) -> torch.Tensor:
    """Causal attention (Phase 1, or any layer with no gate bias set). (B, H, S, D) in and out."""
    resolve_backend(backend, causal=True)
    _gqa_check(Q, K)
    return keybias_attention_bhsd(Q, K, V, None, None)


def attention_gate_bias(Q, K, V, gate_bias, per_head: bool, backend: str = BACKEND,
                        q_row_scale=None) -> torch.Tensor:
    """Causal attention plus the gate's additive key bias (Phase 2).

    gate_bias: (S,) / (B, S) scalar-per-token, or (S, H) / (B, S, H) per head,
    already scaled by whatever attn_scale the caller applies (as in the
    reference). q_row_scale (optional, fp32 broadcastable to (B, H, S)) is the
    per-row query scale of the scaled-softmax Phase-2 form, fused into the
    kernel instead of materialising q * s_eff.
    """
    resolve_backend(backend, causal=False)
    _gqa_check(Q, K)
    B, H, S, _ = Q.shape
    b = _bias_bhs(gate_bias, per_head, B, H, K.shape[2])
    return keybias_attention_bhsd(Q, K, V, b, q_row_scale)
