"""torch custom op around the key-bias attention kernel.

Mirrors the reference op and wrapper (kernels/fa2bias/keybias.py:40-49, :85-87):
  torch.ops.recursive_kvs.fa2_keybias_fwd(q, k, v, bias_raw, scale, causal) -> (out, lse)
  flash_attn_key_bias(q, k, v, key_bias, softmax_scale, causal=True)
with q/k/v in (B, S, heads, D) layout. The reference passes bias_raw =
key_bias / scale to FA2, which adds it before scaling; this kernel takes the
bias in score units directly (what the FlexAttention score_mod adds), so
flash_attn_key_bias hands key_bias through unchanged. A fake (meta) kernel is
registered so torch.compile and CUDA-graph capture can trace the op.
"""
from typing import Optional

import torch

from . import ops


@torch.library.custom_op("tokengate_b200::keybias_fwd", mutates_args=())
def keybias_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, bias: Optional[torch.Tensor],
                scale: float, causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    out, lse = ops.keybias_attention(q, k, v, bias=bias, softmax_scale=scale, causal=causal,
                                     return_lse=True)
    return out, lse


@keybias_fwd.register_fake
def _keybias_fwd_fake(q, k, v, bias, scale, causal):
    return (q.new_empty(q.shape), q.new_empty((q.shape[0], q.shape[2], q.shape[1]), dtype=torch.float32))


def flash_attn_key_bias(q, k, v, key_bias, softmax_scale, causal=True):
    """(B, S, H, D) q/k/v, key_bias broadcastable to (B, H, S) in score units -> out (B, S, H, D)."""
    b = None if key_bias is None else key_bias.float()
    if b is not None and b.stride(-1) != 1:
        b = b.contiguous()
    return keybias_fwd(q, k, v, b, float(softmax_scale), bool(causal))[0]


def keybias_attention_bhsd(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                           bias_bhs: Optional[torch.Tensor],
                           q_row_scale: Optional[torch.Tensor]) -> torch.Tensor:
    """(B, H, S, D) views in and out, causal, scale D^-0.5 (the reference's Phase-2 call)."""
    D = Q.shape[-1]
    q, k, v = Q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2)
    if q_row_scale is None:
        out = keybias_fwd(q, k, v, bias_bhs, D ** -0.5, True)[0]
    else:
        out = ops.keybias_attention(q, k, v, bias=bias_bhs, softmax_scale=D ** -0.5, causal=True,
                                    q_row_scale=q_row_scale)
    return out.transpose(1, 2)
