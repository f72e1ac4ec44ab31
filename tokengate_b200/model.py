"""Qwen3 attention patched onto the B200 kernel, and the prefill KV cache.

Mirrors the reference's patched module and per-layer setters
(tokengate/e2e_gate/attn/qwen3_flex_attention.py):
  patch_model_with_flex_attention(model)              :924-975
  set_gate_bias_for_layers(model, start, end, bias, per_head)   :1128-1155
  set_attn_scale_for_layers / set_ssmax_ratio_for_layers
  set_attention_backends_for_layers(model, gate_attn)  :1174-1193
  Qwen3FlexAttention.forward / _phase2_q_bias          :433-652
and the store-first prefill cache (tokengate/e2e_gate/attn/kv_cache.py:17-37).

The patched forward keeps Q/K/V token-major, (B, S, heads, D), end to end:
the kernel reads that layout natively, so no transpose or contiguous copy is
made, and the cache stores K/V token-major (its `.keys` / `.values` expose
the reference's (B, heads, S, D) view of the same memory).
"""
from typing import List, Optional

import torch

from . import attn as _attn

try:  # transformers >= 5
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Attention
except ImportError:  # pragma: no cover - transformers is a hard dependency of the host side
    Qwen3Attention = None


class _CacheLayer:
    __slots__ = ("k_tok", "v_tok")

    def __init__(self):
        self.k_tok = None   # (B, S, Hkv, D)
        self.v_tok = None

    @property
    def keys(self) -> Optional[torch.Tensor]:
        """(B, Hkv, S, D) view, the layout the reference's cache exposes."""
        return None if self.k_tok is None else self.k_tok.transpose(1, 2)

    @property
    def values(self) -> Optional[torch.Tensor]:
        return None if self.v_tok is None else self.v_tok.transpose(1, 2)

    @keys.setter
    def keys(self, t):
        self.k_tok = None if t is None else t.transpose(1, 2)

    @values.setter
    def values(self, t):
        self.v_tok = None if t is None else t.transpose(1, 2)


class PrefillCache:
    """Per-layer K/V of one prefill. The first update of a layer stores the
    tensor itself (no copy, as kv_cache.py:17-26); later updates append along
    the sequence."""

    def __init__(self, n_layers: int):
        self.layers: List[_CacheLayer] = [_CacheLayer() for _ in range(n_layers)]

    def update_tok(self, k: torch.Tensor, v: torch.Tensor, layer_idx: int):
        """k, v token-major (B, S, Hkv, D); returns the layer's full token-major K, V."""
        lc = self.layers[layer_idx]
        if lc.k_tok is None:
            lc.k_tok, lc.v_tok = k, v
        else:
            lc.k_tok = torch.cat([lc.k_tok, k], dim=1)
            lc.v_tok = torch.cat([lc.v_tok, v], dim=1)
        return lc.k_tok, lc.v_tok

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """transformers Cache interface: (B, Hkv, S, D) in and out."""
        k, v = self.update_tok(key_states.transpose(1, 2), value_states.transpose(1, 2), layer_idx)
        return k.transpose(1, 2), v.transpose(1, 2)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        lc = self.layers[layer_idx]
        return 0 if lc.k_tok is None else lc.k_tok.shape[1]


def _rope_tok(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding on (B, S, H, D) with cos/sin (B, S, D) (rotate-half convention)."""
    cos = cos.unsqueeze(2)
    sin = sin.unsqueeze(2)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


def _phase2_q_scale_and_bias(self, B: int, S: int, dtype):
    """(q_row_scale (B|1, H|1, S) fp32 or None, bias) per the reference's
    _phase2_q_bias / _ssmax_s_eff (qwen3_flex_attention.py:417-473) at its
    rounding points: the scales are formed in the query dtype (attn_scale and
    the ssmax ratio cast to it, their product rounded to it), the kernel rounds
    q * q_row_scale to bf16 exactly as the reference's q * s_eff is rounded,
    and the bias is scaled in its own dtype."""
    per_head = getattr(self, "_gate_per_head", False)
    bias = self.gate_bias
    if self.attn_scale is not None and getattr(self, "ssmax_ratio", None) is not None:
        gamma = self.attn_scale.to(dtype)
        r = self.ssmax_ratio.to(dtype)
        if r.dim() == 1:
            r = r.unsqueeze(0).expand(B, -1)
        g = gamma.view(1, -1, 1) if gamma.numel() > 1 else gamma.reshape(1, 1, 1)
        s_eff = g * r.unsqueeze(1)                                    # (B, H|1, S) in dtype
        if bias is not None:
            sb = s_eff.mean(dim=1) if s_eff.shape[1] > 1 else s_eff[:, 0]   # (B, S)
            bias = bias * (sb.unsqueeze(-1) if bias.dim() == 3 else sb[0].unsqueeze(-1)
                           if bias.dim() == 2 else sb[0])
        return s_eff.float().contiguous(), bias
    if self.attn_scale is not None:
        scale = self.attn_scale.to(dtype)
        if scale.numel() == 1:
            return scale.float().reshape(1, 1, 1).expand(1, 1, S).contiguous(), bias * scale
        qs = scale.float().view(1, -1, 1).expand(1, scale.numel(), S).contiguous()
        if per_head:
            bias = bias * scale.view(*([1] * (bias.dim() - 1)), -1)
        else:
            bias = bias * scale.mean()
        return qs, bias
    return None, bias


def _patched_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                     past_key_values=None, **kwargs):
    if "past_key_value" in kwargs:
        past_key_values = kwargs.pop("past_key_value")
    if hidden_states.dim() != 3:
        raise ValueError(f"hidden_states should be (batch, seq, hidden), got {tuple(hidden_states.shape)}")
    B, S, _ = hidden_states.shape
    D = self.head_dim
    if S == 1:
        raise NotImplementedError("token-by-token decode is outside the B200 prefill path")
    if attention_mask is not None:
        raise ValueError("the B200 prefill path takes no attention_mask: causal masking is in the "
                         "kernel and padding is encoded as gate_bias = -1e9")
    q = self.q_norm(self.q_proj(hidden_states).view(B, S, -1, D))
    k = self.k_norm(self.k_proj(hidden_states).view(B, S, -1, D))
    v = self.v_proj(hidden_states).view(B, S, -1, D)
    cos, sin = position_embeddings
    q = _rope_tok(q, cos, sin)
    k = _rope_tok(k, cos, sin)
    if past_key_values is not None:
        if isinstance(past_key_values, PrefillCache):
            k, v = past_key_values.update_tok(k, v, self.layer_idx)
        else:
            kk, vv = past_key_values.update(k.transpose(1, 2), v.transpose(1, 2), self.layer_idx)
            k, v = kk.transpose(1, 2), vv.transpose(1, 2)
    if k.shape[1] != S:
        raise ValueError("prefill attention expects aligned query and key lengths")
    Qv, Kv, Vv = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)   # (B, H, S, D) views
    if self.gate_bias is not None:
        backend = self.attn_backend_bias
        qs, bias = _phase2_q_scale_and_bias(self, B, S, q.dtype)
        out = _attn.attention_gate_bias(Qv, Kv, Vv, bias, getattr(self, "_gate_per_head", False),
                                        backend=backend, q_row_scale=qs)
    else:
        out = _attn.attention_causal(Qv, Kv, Vv, backend=self.attn_backend_causal)
    out = out.transpose(1, 2).reshape(B, S, -1)     # (B, S, H*D) — already contiguous
    return self.o_proj(out), None


def _set_gate_bias(self, bias: Optional[torch.Tensor], per_head: bool = False):
    self.gate_bias = bias
    self._gate_per_head = bool(per_head) if bias is not None else False


def _set_attn_scale(self, scale: Optional[torch.Tensor]):
    self.attn_scale = scale


def _set_ssmax_ratio(self, ratio: Optional[torch.Tensor]):
    self.ssmax_ratio = ratio


def full_attn_layer_indices(model) -> List[int]:
    return [i for i, layer in enumerate(model.model.layers) if hasattr(layer, "self_attn")]


def rope_inv_freq_fp32(model: torch.nn.Module) -> None:
    """Give every rotary embedding of `model` float32 inverse frequencies.

    transformers builds them in float32 and computes the rotary angles
    position * inv_freq in float32 (Qwen3RotaryEmbedding.forward). A
    `model.to(torch.bfloat16)` casts these buffers too; bf16 keeps 8
    significant bits, so the angle of frequency f at position p moves by up to
    ~p * f * 2^-9 radians: wrong rotations from a few hundred positions on
    (whole turns at 32k). A model loaded with from_pretrained(dtype=bf16), as
    the reference loads it, keeps them in float32; this restores that for
    models cast after construction, recomputing them from the config."""
    for mod in model.modules():
        inv = getattr(mod, "inv_freq", None)
        if not isinstance(inv, torch.Tensor) or inv.dtype == torch.float32 or not hasattr(mod, "config"):
            continue
        rope_type = getattr(mod, "rope_type", "default")
        if rope_type == "default" and hasattr(mod, "compute_default_rope_parameters"):
            fresh, _ = mod.compute_default_rope_parameters(mod.config, inv.device)
        else:
            from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
            fresh, _ = ROPE_INIT_FUNCTIONS[rope_type](mod.config, inv.device)
        mod.inv_freq = fresh.to(torch.float32)
        if isinstance(getattr(mod, "original_inv_freq", None), torch.Tensor):
            mod.original_inv_freq = fresh.to(torch.float32).clone()


def patch_model(model: torch.nn.Module) -> torch.nn.Module:
    """Route every Qwen3 attention module of `model` through the B200 kernel
    (the reference's patch_model_with_flex_attention, qwen3_flex_attention.py:924);
    the rotary inverse frequencies are kept in float32 (rope_inv_freq_fp32)."""
    rope_inv_freq_fp32(model)
    idx = full_attn_layer_indices(model)
    if not idx:
        raise ValueError("patch_model: no full-attention layers found in model")
    for i in idx:
        a = model.model.layers[i].self_attn
        if Qwen3Attention is not None and not isinstance(a, Qwen3Attention):
            raise NotImplementedError(f"layer {i}: attention class {type(a).__name__!r} is not "
                                      f"served (Qwen3Attention only)")
        if a.head_dim != 128:
            raise NotImplementedError(f"head_dim {a.head_dim}: the B200 kernel serves 128")
        a.gate_bias = None
        a._gate_per_head = False
        a.attn_scale = None
        a.ssmax_ratio = None
        a.attn_backend_causal = _attn.BACKEND
        a.attn_backend_bias = _attn.BACKEND
        a.forward = _patched_forward.__get__(a, type(a))
        a.set_gate_bias = _set_gate_bias.__get__(a, type(a))
        a.set_attn_scale = _set_attn_scale.__get__(a, type(a))
        a.set_ssmax_ratio = _set_ssmax_ratio.__get__(a, type(a))
    model._full_attn_layer_indices = idx
    return model


# the reference's name for the same operation
patch_model_with_flex_attention = patch_model


def set_gate_bias_for_layers(model, start_layer: int, end_layer: int,
                             gate_bias: Optional[torch.Tensor], per_head: bool = False) -> None:
    for i in range(start_layer, end_layer):
        a = getattr(model.model.layers[i], "self_attn", None)
        if a is not None and hasattr(a, "set_gate_bias"):
            a.set_gate_bias(gate_bias, per_head=per_head)


def set_attn_scale_for_layers(model, start_layer: int, end_layer: int,
                              scale: Optional[torch.Tensor]) -> None:
    for i in range(start_layer, end_layer):
        a = getattr(model.model.layers[i], "self_attn", None)
        if a is not None and hasattr(a, "set_attn_scale"):
            a.set_attn_scale(scale)


def set_ssmax_ratio_for_layers(model, start_layer: int, end_layer: int,
                               ratio: Optional[torch.Tensor]) -> None:
    for i in range(start_layer, end_layer):
        a = getattr(model.model.layers[i], "self_attn", None)
        if a is not None and hasattr(a, "set_ssmax_ratio"):
            a.set_ssmax_ratio(ratio)


def set_attention_backends_for_layers(model, gate_attn: str) -> None:
    """Pick the kernels per GATE_ATTN name (qwen3_flex_attention.py:1174-1193)."""
    if gate_attn not in _attn.GATE_ATTN:
        raise ValueError(f"gate_attn {gate_attn!r} not in {sorted(_attn.GATE_ATTN)}")
    causal, bias = _attn.GATE_ATTN[gate_attn]
    for i in model._full_attn_layer_indices:
        a = model.model.layers[i].self_attn
        a.attn_backend_causal = causal
        a.attn_backend_bias = bias
