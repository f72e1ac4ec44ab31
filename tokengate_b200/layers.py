"""Fused Qwen3 decoder layer for the gated prefill: the layer prologues and glue as fused kernels.

The transformers Qwen3DecoderLayer the reference runs (with its attention
patched, tokengate/e2e_gate/attn/qwen3_flex_attention.py:475-652) issues ~30
elementwise kernels per layer around 7 GEMMs. Here one layer is

    h, x  = add_rmsnorm(h, delta_prev, input_layernorm)     # residual add + RMSNorm
    qkv   = rope(qk_norm(x @ [Wq; Wk; Wv]^T))               # one tcgen05 GEMM, q/k RMSNorm + RoPE in its epilogue
    a     = keybias_attention(q, k, v, gate bias)           # tcgen05 kernel
    h, x2 = add_rmsnorm(h, a @ Wo^T, post_attention_layernorm)
    act   = silu(x2 @ Wgate^T) * (x2 @ Wup^T)               # one tcgen05 GEMM, SwiGLU in its epilogue
    delta = act @ Wdown^T                                   # added by the next layer

with the module's own weights: the q/k/v and gate/up weights are
concatenated once and the modules' parameters re-pointed to views of the
concatenation, so nothing is duplicated and the model stays usable through
transformers. Q, K and V are views of the fused [q | k | v] projection; the
prefill cache keeps the K/V views (and with them the buffer's q part: one
GEMM instead of two costs that memory, ~11 MB per layer at 2768 tokens).
The [q | k | v] projection runs through tg_gemm_qkv_rope (the q/k RMSNorm
and RoPE in its epilogue) and the [gate | up] projection through
tg_gemm_swiglu (the SwiGLU in its epilogue), so neither the unnormalised
q/k nor the 2*intermediate-wide projection reaches HBM. Shapes they do not
serve (hidden not a multiple of 64, an intermediate size not a multiple of
128) take cuBLAS and the qk_norm_rope / silu_mul kernels.
"""
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops


class FusedLayerWeights:
    """Views of one Qwen3DecoderLayer's parameters in the fused layout."""

    def __init__(self, layer):
        a, m = layer.self_attn, layer.mlp
        for lin in (a.q_proj, a.k_proj, a.v_proj, a.o_proj, m.gate_proj, m.up_proj, m.down_proj):
            if lin.bias is not None:
                raise NotImplementedError("projection biases are not served by the fused layer")
        cfg = a.config
        self.head_dim = a.head_dim
        if self.head_dim != 128:
            raise NotImplementedError(f"head_dim {self.head_dim}: the B200 kernels serve 128")
        self.n_q = cfg.num_attention_heads
        self.n_kv = cfg.num_key_value_heads
        self.eps = float(layer.input_layernorm.variance_epsilon)
        self.qk_eps = float(a.q_norm.variance_epsilon)
        self.wqkv = self._fuse(a.q_proj, a.k_proj, a.v_proj)
        self.wgu = self._fuse(m.gate_proj, m.up_proj)
        self.wo = a.o_proj.weight
        self.wdown = m.down_proj.weight
        self.in_w = layer.input_layernorm.weight
        self.post_w = layer.post_attention_layernorm.weight
        self.q_norm_w = a.q_norm.weight
        self.k_norm_w = a.k_norm.weight
        self.inter = m.gate_proj.weight.shape[0]
        # shapes the fused projection kernels serve (K a multiple of 64, inter of 128)
        self.swiglu_fused = self.inter % 128 == 0 and self.wgu.shape[1] % 64 == 0
        self.qkv_fused = self.wqkv.shape[1] % 64 == 0

    @staticmethod
    def _fuse(*lins):
        ws = [l.weight for l in lins]
        base = ws[0]
        # already fused (an earlier call re-pointed them as consecutive views of
        # one buffer): reuse that buffer
        offs, expect = [], base.storage_offset()
        for w in ws:
            offs.append(w.storage_offset() == expect and w.is_contiguous()
                        and w.untyped_storage().data_ptr() == base.untyped_storage().data_ptr())
            expect += w.numel()
        if all(offs):
            total = sum(w.shape[0] for w in ws)
            return base.new_empty(0).set_(base.untyped_storage(), base.storage_offset(),
                                          (total, base.shape[1]))
        fused = torch.cat([w.detach() for w in ws], dim=0).contiguous()
        off = 0
        for l, w in zip(lins, ws):
            n = w.shape[0]
            l.weight.data = fused[off:off + n]
            off += n
        return fused


def fused_weights(model):
    """Per-layer fused weight views, built once and cached on the model."""
    fw = getattr(model, "_tg_fused", None)
    if fw is None:
        fw = [FusedLayerWeights(layer) for layer in model.model.layers]
        model._tg_fused = fw
    return fw


def layer_attention(lw: FusedLayerWeights, h: torch.Tensor, delta: Optional[torch.Tensor],
                    cos: torch.Tensor, sin: torch.Tensor, cache, layer_idx: int,
                    gate_bias: Optional[torch.Tensor] = None,
                    q_row_scale: Optional[torch.Tensor] = None):
    """The attention half of a decoder layer, up to the token-mixer residual.

    h: (B, S, H) residual stream (updated in place when delta is given);
    delta: the previous layer's MLP output or None. Returns (a, x2): a = the
    residual after attention (the reference's a_j boundary of the split gate
    layer, gate_forward.py:398-418) and x2 = post_attention_layernorm(a)."""
    B, S, H = h.shape
    h, x = ops.add_rmsnorm(h, delta, lw.in_w, lw.eps, h_out=h if delta is not None else None)
    if lw.qkv_fused:
        qkv = ops.gemm_qkv_rope(x, lw.wqkv, lw.n_q, lw.n_kv, lw.q_norm_w, lw.k_norm_w, cos, sin, lw.qk_eps)
    else:
        qkv = F.linear(x, lw.wqkv).view(B, S, lw.n_q + 2 * lw.n_kv, lw.head_dim)
    q = qkv[:, :, :lw.n_q]
    k = qkv[:, :, lw.n_q:lw.n_q + lw.n_kv]
    v = qkv[:, :, lw.n_q + lw.n_kv:]
    if not lw.qkv_fused:
        ops.qk_norm_rope(q, k, lw.q_norm_w, lw.k_norm_w, cos, sin, lw.qk_eps)
    if cache is not None:
        k, v = cache.update_tok(k, v, layer_idx)
    a = ops.keybias_attention(q, k, v, bias=gate_bias, causal=True, q_row_scale=q_row_scale)
    o = F.linear(a.view(B, S, -1), lw.wo)
    return ops.add_rmsnorm(h, o, lw.post_w, lw.eps, h_out=h)


def layer_mlp(lw: FusedLayerWeights, x2: torch.Tensor) -> torch.Tensor:
    """The MLP half on post_attention_layernorm output x2: returns the MLP output
    (not yet added to the residual)."""
    if lw.swiglu_fused:
        act = ops.gemm_swiglu(x2, lw.wgu, lw.inter)
    else:
        act = ops.silu_mul(F.linear(x2, lw.wgu))
    return F.linear(act, lw.wdown)


def layer_forward(lw: FusedLayerWeights, h: torch.Tensor, delta: Optional[torch.Tensor],
                  cos: torch.Tensor, sin: torch.Tensor, cache, layer_idx: int,
                  gate_bias: Optional[torch.Tensor] = None,
                  q_row_scale: Optional[torch.Tensor] = None):
    """One decoder layer. h: (B, S, H) residual stream (updated in place when
    delta is given); delta: the previous layer's MLP output or None. Returns
    (h, delta') with delta' this layer's MLP output, not yet added."""
    h, x2 = layer_attention(lw, h, delta, cos, sin, cache, layer_idx, gate_bias, q_row_scale)
    return h, layer_mlp(lw, x2)
