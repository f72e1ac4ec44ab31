"""CPU ORACLE (test infrastructure): gated generation — prefill, then greedy
decode over the gated KV cache — in float32 torch on the CPU.

Restates, independently of tokengate_b200's modules, the reference's
generate_batch (tokengate/e2e_gate/decode/gate_decode.py:87-260) with the
folded Phase-2 form of FormDecodeState / decode_phase2_layer_tensors
(tokengate/e2e_gate/attn/qwen3_flex_attention.py:374-415, :978-1116):
  * caches: layers at and below the gate keep the full padded Phase-1 K/V
    (width = longest prompt), layers above it the kept tokens (width =
    max_n_kept); decoded tokens are appended; prefix slots past a row's valid
    length are masked (:139-165);
  * above the gate each prefix key keeps the additive bias the prefill gave
    it (finalized gate: the per-head bias times the head-mean s_eff of the
    key's own ratio; linear gate: the score row), decoded keys none; with the
    finalized gate the decode query is scaled by gamma_h * r_dec,
    r_dec = min(log(max(n_kept + 1 + step, 2)) / log(max(pos + 1, 2)), 1);
  * the first decode token sits one past the last kept position, then +1
    per step; greedy argmax; stop when every row's last token is EOS.
The prefill part follows oracle/prefill.py (same control flow, same
restated math) but keeps each layer's post-RoPE K and V.
"""
from typing import Sequence

import numpy as np
import torch

from . import gate_e2e as ge
from .prefill import _mlp_half, _rms, _rope_cos_sin, _rot_half, _attention, weights_fp32
from .select import topk_indices


def _attn_half_kv(h, p, cfg, cos, sin, bias_bs, q_scale=None):
    """oracle.prefill._attn_half that also returns the layer's K and V."""
    B, S, _ = h.shape
    D = cfg["head_dim"]
    eps = cfg["rms_norm_eps"]
    x = _rms(h, p["input_layernorm.weight"], eps)
    q = (x @ p["self_attn.q_proj.weight"].T).view(B, S, -1, D)
    k = (x @ p["self_attn.k_proj.weight"].T).view(B, S, -1, D)
    v = (x @ p["self_attn.v_proj.weight"].T).view(B, S, -1, D)
    q = _rms(q, p["self_attn.q_norm.weight"], eps)
    k = _rms(k, p["self_attn.k_norm.weight"], eps)
    c, s_ = cos[:, :, None, :], sin[:, :, None, :]
    q = q * c + _rot_half(q) * s_
    k = k * c + _rot_half(k) * s_
    a = _attention(q, k, v, bias_bs, q_scale=q_scale).reshape(B, S, -1)
    return h + a @ p["self_attn.o_proj.weight"].T, k, v


def _decode_attention(q, K, V, add_mask):
    """q (B, Hq, D); K/V (B, N, Hkv, D); add_mask (B, Hq|1, N) with -inf for
    masked keys. Returns (B, Hq, D)."""
    B, Hq, D = q.shape
    G = Hq // K.shape[2]
    kk = K.repeat_interleave(G, dim=2).permute(0, 2, 3, 1)    # (B, Hq, D, N)
    vv = V.repeat_interleave(G, dim=2).permute(0, 2, 1, 3)    # (B, Hq, N, D)
    s = (q[:, :, None, :] @ kk)[:, :, 0] * (D ** -0.5) + add_mask
    return (torch.softmax(s, dim=-1)[:, :, None, :] @ vv)[:, :, 0]


def gated_generate(model, gate, prompt_ids_list: Sequence[Sequence[int]], starts: Sequence[int],
                   ends: Sequence[int], gate_layer: int, K, max_new_tokens: int, *,
                   e2e: bool = False, phase2_form: bool = True, eos_token_id=None,
                   weights=None, bias_bf16: bool = True, forced_tokens=None) -> dict:
    """gate: the fp32 readout vector (linear gate) or, with e2e=True, the dict
    oracle.prefill.gated_prefill_e2e takes. forced_tokens (B, max_new_tokens - 1):
    fed to the decode steps in place of the previous argmax (teacher forcing). Returns
    dict(tokens (list per row, through the first EOS), logits (steps x (B,
    vocab) fp32; [0] is the prefill's), n_kepts, kept_positions)."""
    layers, g, cfg = weights if weights is not None else weights_fp32(model)
    eps = cfg["rms_norm_eps"]
    D = cfg["head_dim"]
    B = len(prompt_ids_list)
    lens = [len(x) for x in prompt_ids_list]
    S = max(lens)
    ids = torch.zeros(B, S, dtype=torch.long)
    for b, x in enumerate(prompt_ids_list):
        ids[b, :lens[b]] = torch.as_tensor(list(x), dtype=torch.long)
    h = g["embed"][ids]
    pos = torch.arange(S).unsqueeze(0).expand(B, -1)
    cos, sin = _rope_cos_sin(pos, D, cfg["rope_theta"])
    kc, vc = [None] * cfg["n_layers"], [None] * cfg["n_layers"]
    Ks = list(K) if isinstance(K, (list, tuple)) else [K] * B

    # ---- Phase 1 (the finalized gate splits the gate layer at its attention residual)
    n_full = gate_layer if e2e else gate_layer + 1
    for i in range(n_full):
        h, kc[i], vc[i] = _attn_half_kv(h, layers[i], cfg, cos, sin, None)
        h = _mlp_half(h, layers[i], cfg)
    if e2e:
        h, kc[gate_layer], vc[gate_layer] = _attn_half_kv(h, layers[gate_layer], cfg, cos, sin, None)

    # ---- score, select, compact (oracle/prefill.py)
    kept, n_kepts, K_cl = [], [], []
    if e2e:
        z = _rms(h, layers[gate_layer]["post_attention_layernorm.weight"], eps)
        wg, wu, w_row = (torch.as_tensor(np.asarray(gate[k]), dtype=torch.float32) for k in ("wg", "wu", "w_row"))
        gs = np.asarray(gate["gate_scale_eff"], dtype=np.float32)
        at = torch.as_tensor(np.asarray(gate["attn_scale_eff"], dtype=np.float32))
        bs = []
        for b in range(B):
            zb = z[b, starts[b]:ends[b]]
            raw = ((torch.nn.functional.silu(zb @ wg.T) * (zb @ wu.T)) @ w_row).numpy()
            bb = ge.e2e_bias(raw, gs, gate["eps"], gate["gain"])
            kc_b = max(1, min(int(Ks[b]), len(raw)))
            top = torch.as_tensor(ge.select(ge.aggregate(bb), kc_b), dtype=torch.long)
            kept.append(torch.cat([torch.arange(starts[b]), starts[b] + top, torch.arange(ends[b], lens[b])]))
            bs.append(bb)
            n_kepts.append(len(kept[-1]))
            K_cl.append(kc_b)
    else:
        w64 = gate.detach().double().reshape(-1).cpu()
        scores = []
        for b in range(B):
            sc = torch.nn.functional.logsigmoid(h[b, starts[b]:ends[b]].double() @ w64).float()
            kc_b = max(1, min(int(Ks[b]), ends[b] - starts[b]))
            top = torch.as_tensor(topk_indices(sc.numpy(), kc_b), dtype=torch.long)
            kept.append(torch.cat([torch.arange(starts[b]), starts[b] + top, torch.arange(ends[b], lens[b])]))
            scores.append(sc)
            n_kepts.append(len(kept[-1]))
            K_cl.append(kc_b)
    W2 = max(n_kepts)
    hp = torch.zeros(B, W2, h.shape[-1])
    kp = torch.zeros(B, W2, dtype=torch.long)
    for b in range(B):
        hp[b, :n_kepts[b]] = h[b, kept[b]]
        kp[b, :n_kepts[b]] = kept[b]
    cos2, sin2 = _rope_cos_sin(kp, D, cfg["rope_theta"])
    n_p2 = cfg["n_layers"] - 1 - gate_layer
    biases, gammas = [], None
    if e2e:
        Lp, Hg = gs.shape
        base = torch.zeros(B, W2, Lp, Hg)
        for b in range(B):
            st = kept[b][starts[b]:starts[b] + K_cl[b]] - starts[b]
            base[b, starts[b]:starts[b] + K_cl[b]] = torch.as_tensor(bs[b])[st]
            base[b, n_kepts[b]:] = -1e9
        hp = _mlp_half(hp, layers[gate_layer], cfg)
        r = torch.as_tensor(ge.ssmax_ratio(kp.numpy()))
        gammas = at
        for li, i in enumerate(range(gate_layer + 1, cfg["n_layers"])):
            s_eff = at[li].view(1, -1, 1) * r[:, None, :]
            sb = s_eff.mean(dim=1)
            bias = (base[:, :, li, :] * sb[:, :, None]).permute(0, 2, 1)       # (B, Hg, W2)
            biases.append(bias)
            hp, kc[i], vc[i] = _attn_half_kv(hp, layers[i], cfg, cos2, sin2, bias, q_scale=s_eff)
            hp = _mlp_half(hp, layers[i], cfg)
    else:
        bias = torch.full((B, W2), -1e9)
        for b in range(B):
            bias[b, :n_kepts[b]] = 0.0
            bias[b, starts[b]:starts[b] + K_cl[b]] = scores[b][kept[b][starts[b]:starts[b] + K_cl[b]] - starts[b]]
        if bias_bf16:
            bias = bias.to(torch.bfloat16).float()
        for i in range(gate_layer + 1, cfg["n_layers"]):
            biases.append(bias[:, None, :])
            hp, kc[i], vc[i] = _attn_half_kv(hp, layers[i], cfg, cos2, sin2, bias)
            hp = _mlp_half(hp, layers[i], cfg)
    last = torch.stack([_rms(hp[b, n_kepts[b] - 1], g["norm"], eps) for b in range(B)])
    logits = [last @ g["lm_head"].T]
    cur = logits[0].argmax(-1)
    gen = [cur]

    # ---- decode
    Hq = layers[0]["self_attn.q_proj.weight"].shape[0] // D
    valid_below = torch.as_tensor(lens)
    valid_p2 = torch.as_tensor(n_kepts)
    next_pos = torch.stack([kp[b, n_kepts[b] - 1] for b in range(B)]) + 1
    eos = torch.zeros(B, dtype=torch.bool)
    widths = [kc[i].shape[1] for i in range(cfg["n_layers"])]    # prefix width per layer
    for step in range(max_new_tokens - 1):
        if eos_token_id is not None:
            eos |= cur == eos_token_id
            if bool(eos.all()):
                break
        if forced_tokens is not None:
            cur = torch.as_tensor(forced_tokens)[:, step].long()
        x = g["embed"][cur][:, None, :]                                        # (B, 1, H)
        c1, s1 = _rope_cos_sin(next_pos[:, None], D, cfg["rope_theta"])
        for i in range(cfg["n_layers"]):
            p = layers[i]
            xn = _rms(x, p["input_layernorm.weight"], eps)
            q = (xn @ p["self_attn.q_proj.weight"].T).view(B, 1, -1, D)
            k = (xn @ p["self_attn.k_proj.weight"].T).view(B, 1, -1, D)
            v = (xn @ p["self_attn.v_proj.weight"].T).view(B, 1, -1, D)
            q = _rms(q, p["self_attn.q_norm.weight"], eps)
            k = _rms(k, p["self_attn.k_norm.weight"], eps)
            c, s_ = c1[:, :, None, :], s1[:, :, None, :]
            q = (q * c + _rot_half(q) * s_)[:, 0]                             # (B, Hq, D)
            k = k * c + _rot_half(k) * s_
            W = widths[i]
            kc[i] = torch.cat([kc[i], k], dim=1)
            vc[i] = torch.cat([vc[i], v], dim=1)
            n = kc[i].shape[1]
            mask = torch.zeros(B, 1, n)
            valid = valid_below if i <= gate_layer else valid_p2
            for b in range(B):
                mask[b, :, int(valid[b]):W] = float("-inf")
            if i > gate_layer and phase2_form:
                li = i - gate_layer - 1
                mask = mask.expand(B, Hq, n).clone() if biases[li].shape[1] > 1 else mask
                mask[:, :, :W] = mask[:, :, :W] + biases[li]
                if gammas is not None:
                    m_ = (valid_p2.float() + 1 + step).clamp(min=2.0)
                    pp = (next_pos.float() + 1.0).clamp(min=2.0)
                    r_dec = (torch.log(m_) / torch.log(pp)).clamp(max=1.0)         # (B,)
                    q = q * (gammas[li][None, :] * r_dec[:, None])[:, :, None]
            a = _decode_attention(q, kc[i], vc[i], mask).reshape(B, 1, -1)
            x = x + a @ p["self_attn.o_proj.weight"].T
            x = _mlp_half(x, p, cfg)
        lg = _rms(x[:, 0], g["norm"], eps) @ g["lm_head"].T
        logits.append(lg)
        cur = lg.argmax(-1)
        gen.append(cur)
        next_pos = next_pos + 1
    allg = torch.stack(gen, dim=1).tolist()
    tokens = []
    for row in allg:
        if eos_token_id is not None and eos_token_id in row:
            row = row[:row.index(eos_token_id) + 1]
        tokens.append(row)
    return dict(tokens=tokens, logits=logits, n_kepts=n_kepts, kept_positions=[k.tolist() for k in kept])
