"""CPU ORACLE (test infrastructure): the gated prefill in float32 torch on the CPU.

Restates, independently of tokengate_b200's modules:
  * the reference control flow prefill_batch_for_decode
    (tokengate/e2e_gate/gate_module/gate_forward.py:1269-1579): right-padded
    Phase 1 over layers 0..L, scoring of each request's state span
    (:1396-1407), K_clamped = max(1, min(K, n_art)) (:1409-1410), selection +
    sorted keep list (:84-99, :1417-1421), gather of kept hidden rows with
    original positions (:1443-1461), Phase-2 gate bias = score at kept state
    tokens, 0 elsewhere, -1e9 pads (:968-1036, :1463-1469), Phase 2 over
    layers L+1..N-1 with RoPE at the kept positions (:1528-1553), head on the
    last kept row (:1555-1562);
  * the Qwen3 decoder math the reference runs through transformers
    (RMSNorm, q/k RMSNorm, rotate-half RoPE, causal attention with the
    additive key bias as in sdpa_compat.py:6-37, SwiGLU MLP, tied or untied
    lm_head).
Scores are logsigmoid(w . h) with h the float32 layer-L output, evaluated in
float64 and rounded to float32; selection by (score desc, index asc).
"""
import time
from typing import Dict, List, Sequence

import torch

from .select import topk_indices


def _rms(x, w, eps):
    v = x.pow(2).mean(-1, keepdim=True)
    return w * (x * torch.rsqrt(v + eps))


def _rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    f = positions.to(torch.float64)[..., None] * inv            # (B, S, D/2)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float(), emb.sin().float()


def _rot_half(x):
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def _attention(q, k, v, bias_bs, chunk=256, q_scale=None):
    """q (B,S,Hq,D), k/v (B,S,Hkv,D) fp32, bias_bs (B,S) or (B,Hq,S) or None; causal.
    q_scale (B,Hq|1,S) multiplies each query row (the scaled-softmax prologue)."""
    B, S, Hq, D = q.shape
    G = Hq // k.shape[2]
    kk = k.repeat_interleave(G, dim=2).permute(0, 2, 3, 1)     # (B, Hq, D, S)
    vv = v.repeat_interleave(G, dim=2).permute(0, 2, 1, 3)     # (B, Hq, S, D)
    qq = q.permute(0, 2, 1, 3)                                 # (B, Hq, S, D)
    if q_scale is not None:
        qq = qq * q_scale[..., None]
    out = torch.empty_like(qq)
    keys = torch.arange(S)
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        # a query chunk sees the key prefix [0, c1) only (causal)
        s = (qq[:, :, c0:c1] @ kk[..., :c1]) * (D ** -0.5)
        if bias_bs is not None:
            s = s + (bias_bs[:, None, None, :c1] if bias_bs.dim() == 2 else bias_bs[:, :, None, :c1])
        s = s.masked_fill(keys[None, None, None, :c1] > torch.arange(c0, c1)[None, None, :, None],
                          float("-inf"))
        out[:, :, c0:c1] = torch.softmax(s, dim=-1) @ vv[:, :, :c1]
    return out.permute(0, 2, 1, 3)


def _attention_sdpa_compat(q, k, v, bias_bs, q_scale=None):
    """The reference's CPU attention path, sdpa_compat.sdpa_causal (query
    chunks of 128 rows, F.scaled_dot_product_attention with an additive
    bias + causal mask), on (B, S, H, D) tensors; scalar-per-key bias (B, S)."""
    from .cpu_paths import sdpa_causal
    if q_scale is not None or (bias_bs is not None and bias_bs.dim() != 2):
        raise ValueError("the sdpa_compat path here takes a (B, S) bias and no query scale")
    o = sdpa_causal(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), bias_bs, per_head=False)
    return o.transpose(1, 2)


def _layer(h, p: Dict[str, torch.Tensor], cfg, cos, sin, bias_bs, q_scale=None, attn=None):
    return _mlp_half(_attn_half(h, p, cfg, cos, sin, bias_bs, q_scale, attn), p, cfg)


def _attn_half(h, p: Dict[str, torch.Tensor], cfg, cos, sin, bias_bs, q_scale=None, attn=None):
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
    a = (attn or _attention)(q, k, v, bias_bs, q_scale=q_scale).reshape(B, S, -1)
    return h + a @ p["self_attn.o_proj.weight"].T


def _mlp_half(h, p: Dict[str, torch.Tensor], cfg):
    eps = cfg["rms_norm_eps"]
    x = _rms(h, p["post_attention_layernorm.weight"], eps)
    g = x @ p["mlp.gate_proj.weight"].T
    u = x @ p["mlp.up_proj.weight"].T
    h = h + (torch.nn.functional.silu(g) * u) @ p["mlp.down_proj.weight"].T
    return h


def weights_fp32(model) -> (dict, dict):
    """(per-layer param dicts, globals) as float32 CPU tensors, plus a config dict."""
    sd = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    c = model.config
    cfg = dict(head_dim=c.head_dim, rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_parameters["rope_theta"]
               if getattr(c, "rope_parameters", None) else c.rope_theta,
               n_layers=c.num_hidden_layers)
    layers = []
    for i in range(c.num_hidden_layers):
        pre = f"model.layers.{i}."
        layers.append({k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)})
    g = dict(embed=sd["model.embed_tokens.weight"], norm=sd["model.norm.weight"],
             lm_head=sd.get("lm_head.weight", sd["model.embed_tokens.weight"]))
    return layers, g, cfg


def gated_prefill(model, w_gate: torch.Tensor, prompt_ids_list: Sequence[Sequence[int]],
                  starts: Sequence[int], ends: Sequence[int], gate_layer: int, K,
                  weights=None, bias_bf16: bool = False, kept_override=None) -> dict:
    """Returns dict(first_tokens (B,), kept_positions list, n_kepts, K_clampeds,
    logits (B, vocab) fp32, scores list, phase1_hidden (B, S, H),
    selected_positions list).

    bias_bf16: round the Phase-2 bias to bfloat16, as the reference does when
    the model runs in bf16 (gate_bias_batched has the hidden dtype, :1450).
    kept_override: per request, the kept positions Phase 2 runs on instead of
    this oracle's own selection (prefix, K_clamped state tokens, suffix, in
    ascending order; the bias is this oracle's score at those state tokens).
    The oracle's own selection is returned as selected_positions either way,
    so one call gives both the selection to compare and Phase-2 logits on
    another implementation's kept rows."""
    layers, g, cfg = weights if weights is not None else weights_fp32(model)
    B = len(prompt_ids_list)
    lens = [len(x) for x in prompt_ids_list]
    S = max(lens)
    ids = torch.zeros(B, S, dtype=torch.long)
    for b, x in enumerate(prompt_ids_list):
        ids[b, :lens[b]] = torch.as_tensor(list(x), dtype=torch.long)
    h = g["embed"][ids]
    pos = torch.arange(S).unsqueeze(0).expand(B, -1)
    cos, sin = _rope_cos_sin(pos, cfg["head_dim"], cfg["rope_theta"])
    for i in range(gate_layer + 1):
        h = _layer(h, layers[i], cfg, cos, sin, None)
    w64 = w_gate.detach().double().reshape(-1).cpu()
    Ks = list(K) if isinstance(K, (list, tuple)) else [K] * B
    kept, scores, n_kepts, K_cl, selected = [], [], [], [], []
    for b in range(B):
        n_art = ends[b] - starts[b]
        sc = torch.nn.functional.logsigmoid(h[b, starts[b]:ends[b]].double() @ w64).float()
        kc = max(1, min(int(Ks[b]), n_art))
        top = torch.as_tensor(topk_indices(sc.numpy(), kc), dtype=torch.long)
        keep = torch.cat([torch.arange(starts[b]), starts[b] + top, torch.arange(ends[b], lens[b])])
        selected.append(keep.tolist())
        if kept_override is not None:
            keep = torch.as_tensor(list(kept_override[b]), dtype=torch.long)
            if len(keep) != len(selected[-1]):
                raise ValueError(f"request {b}: kept_override has {len(keep)} positions, "
                                 f"the selection {len(selected[-1])}")
        kept.append(keep)
        scores.append(sc)
        n_kepts.append(len(keep))
        K_cl.append(kc)
    n_alloc = max(n_kepts)
    hp = torch.zeros(B, n_alloc, h.shape[-1])
    kp = torch.zeros(B, n_alloc, dtype=torch.long)
    bias = torch.full((B, n_alloc), -1e9)
    for b in range(B):
        n = n_kepts[b]
        hp[b, :n] = h[b, kept[b]]
        kp[b, :n] = kept[b]
        bias[b, :n] = 0.0
        bias[b, starts[b]:starts[b] + K_cl[b]] = scores[b][kept[b][starts[b]:starts[b] + K_cl[b]] - starts[b]]
    if bias_bf16:
        bias = bias.to(torch.bfloat16).float()
    phase1_hidden = h
    cos2, sin2 = _rope_cos_sin(kp, cfg["head_dim"], cfg["rope_theta"])
    for i in range(gate_layer + 1, cfg["n_layers"]):
        hp = _layer(hp, layers[i], cfg, cos2, sin2, bias)
    last = torch.stack([_rms(hp[b, n_kepts[b] - 1], g["norm"], cfg["rms_norm_eps"]) for b in range(B)])
    logits = last @ g["lm_head"].T
    return dict(first_tokens=logits.argmax(-1), kept_positions=[k.tolist() for k in kept],
                n_kepts=n_kepts, K_clampeds=K_cl, logits=logits, scores=scores,
                phase1_hidden=phase1_hidden, bias=bias, selected_positions=selected)


def gated_prefill_e2e(model, gate: dict, prompt_ids_list: Sequence[Sequence[int]],
                      starts: Sequence[int], ends: Sequence[int], gate_layer: int, K,
                      weights=None) -> dict:
    """The gated prefill with the finalized gate, float32 on the CPU.

    gate: dict(wg (inter, H), wu (inter, H), w_row (inter,), gate_scale_eff (L', Hg),
    attn_scale_eff (L', Hg), eps, gain) — fp32 tensors/arrays. Restates the split
    gate layer (attention half in Phase 1, gate_forward.py:345-418; its MLP on the
    kept rows at Phase-2 entry, :420-435, :1481-1483), the branch score
    (:491-524), E2EGate.forward / aggregate (e2e_gate_module.py:348-399), the
    selection on the aggregate, the per-layer per-head bias and the
    scaled-softmax query scale of every Phase-2 layer (:588-660,
    qwen3_flex_attention.py:417-473) in float32 arithmetic.
    Returns dict(first_tokens, kept_positions, n_kepts, K_clampeds, logits, raw_scores).
    """
    import numpy as np
    from . import gate_e2e as ge
    layers, g, cfg = weights if weights is not None else weights_fp32(model)
    B = len(prompt_ids_list)
    lens = [len(x) for x in prompt_ids_list]
    S = max(lens)
    ids = torch.zeros(B, S, dtype=torch.long)
    for b, x in enumerate(prompt_ids_list):
        ids[b, :lens[b]] = torch.as_tensor(list(x), dtype=torch.long)
    h = g["embed"][ids]
    pos = torch.arange(S).unsqueeze(0).expand(B, -1)
    cos, sin = _rope_cos_sin(pos, cfg["head_dim"], cfg["rope_theta"])
    for i in range(gate_layer):
        h = _layer(h, layers[i], cfg, cos, sin, None)
    h = _attn_half(h, layers[gate_layer], cfg, cos, sin, None)          # a_j
    z = _rms(h, layers[gate_layer]["post_attention_layernorm.weight"], cfg["rms_norm_eps"])
    wg, wu, w_row = (torch.as_tensor(np.asarray(gate[k]), dtype=torch.float32) for k in ("wg", "wu", "w_row"))
    gs = np.asarray(gate["gate_scale_eff"], dtype=np.float32)
    at = torch.as_tensor(np.asarray(gate["attn_scale_eff"], dtype=np.float32))
    Ks = list(K) if isinstance(K, (list, tuple)) else [K] * B
    kept, raws, bs, n_kepts, K_cl = [], [], [], [], []
    for b in range(B):
        zb = z[b, starts[b]:ends[b]]
        raw = ((torch.nn.functional.silu(zb @ wg.T) * (zb @ wu.T)) @ w_row).numpy()
        bb = ge.e2e_bias(raw, gs, gate["eps"], gate["gain"])                 # (n, L', Hg)
        kc = max(1, min(int(Ks[b]), len(raw)))
        top = torch.as_tensor(ge.select(ge.aggregate(bb), kc), dtype=torch.long)
        keep = torch.cat([torch.arange(starts[b]), starts[b] + top, torch.arange(ends[b], lens[b])])
        kept.append(keep)
        raws.append(raw)
        bs.append(bb)
        n_kepts.append(len(keep))
        K_cl.append(kc)
    n_alloc = max(n_kepts)
    Lp, Hg = gs.shape
    hp = torch.zeros(B, n_alloc, h.shape[-1])
    kp = torch.zeros(B, n_alloc, dtype=torch.long)
    base = torch.zeros(B, n_alloc, Lp, Hg)
    for b in range(B):
        n = n_kepts[b]
        hp[b, :n] = h[b, kept[b]]
        kp[b, :n] = kept[b]
        st = kept[b][starts[b]:starts[b] + K_cl[b]] - starts[b]
        base[b, starts[b]:starts[b] + K_cl[b]] = torch.as_tensor(bs[b])[st]
        base[b, n:] = -1e9
    hp = _mlp_half(hp, layers[gate_layer], cfg)                         # gate layer MLP on kept rows
    r = torch.as_tensor(ge.ssmax_ratio(kp.numpy()))                     # (B, n_alloc)
    cos2, sin2 = _rope_cos_sin(kp, cfg["head_dim"], cfg["rope_theta"])
    for li, i in enumerate(range(gate_layer + 1, cfg["n_layers"])):
        s_eff = at[li].view(1, -1, 1) * r[:, None, :]                   # (B, Hg, n)
        sb = s_eff.mean(dim=1)                                          # (B, n)
        bias = (base[:, :, li, :] * sb[:, :, None]).permute(0, 2, 1)    # (B, Hg, n)
        hp = _layer(hp, layers[i], cfg, cos2, sin2, bias, q_scale=s_eff)
    last = torch.stack([_rms(hp[b, n_kepts[b] - 1], g["norm"], cfg["rms_norm_eps"]) for b in range(B)])
    logits = last @ g["lm_head"].T
    return dict(first_tokens=logits.argmax(-1), kept_positions=[k.tolist() for k in kept],
                n_kepts=n_kepts, K_clampeds=K_cl, logits=logits, raw_scores=raws)


def prefill_by_parts(weights, ids: Sequence[int], start: int, end: int, gate_layer: int, K: int,
                     w_gate: torch.Tensor, bias_bf16: bool = True, attention: str = "sdpa_compat") -> dict:
    """One request's gated prefill on the CPU, timed by parts, for a CPU
    baseline at a prompt length the whole run would take minutes at.

    Runs, once each and in order, the parts gated_prefill runs: the token
    embedding, ONE Phase-1 layer (layer 0) on the full prompt, the scoring /
    selection / compaction of the state span on that layer's output, ONE
    Phase-2 layer (layer gate_layer + 1) on the kept rows with the key bias
    and the kept positions' RoPE, and the head. Every Phase-1 layer has the
    same shapes and work (as does every Phase-2 layer), so the whole prefill
    takes embed + (gate_layer + 1) * phase1_layer + select + (n_layers -
    gate_layer - 1) * phase2_layer + head; that sum is returned as total_s,
    with each part's seconds. attention: "sdpa_compat" runs the attention
    the way the reference does on a CPU (its sdpa_compat chunks), "oracle"
    this module's float32 restatement."""
    attn = _attention_sdpa_compat if attention == "sdpa_compat" else _attention
    layers, g, cfg = weights
    S = len(ids)
    t = {}
    t0 = time.perf_counter()
    h = g["embed"][torch.as_tensor(list(ids), dtype=torch.long)][None]
    pos = torch.arange(S)[None]
    cos, sin = _rope_cos_sin(pos, cfg["head_dim"], cfg["rope_theta"])
    t["embed"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    h = _layer(h, layers[0], cfg, cos, sin, None, attn=attn)
    t["phase1_layer"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    w64 = w_gate.detach().double().reshape(-1).cpu()
    sc = torch.nn.functional.logsigmoid(h[0, start:end].double() @ w64).float()
    kc = max(1, min(int(K), end - start))
    top = torch.as_tensor(topk_indices(sc.numpy(), kc), dtype=torch.long)
    keep = torch.cat([torch.arange(start), start + top, torch.arange(end, S)])
    hp = h[:, keep]
    bias = torch.zeros(1, len(keep))
    bias[0, start:start + kc] = sc[top]
    if bias_bf16:
        bias = bias.to(torch.bfloat16).float()
    cos2, sin2 = _rope_cos_sin(keep[None], cfg["head_dim"], cfg["rope_theta"])
    t["select"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    hp = _layer(hp, layers[gate_layer + 1], cfg, cos2, sin2, bias, attn=attn)
    t["phase2_layer"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    last = _rms(hp[0, -1], g["norm"], cfg["rms_norm_eps"])
    (last @ g["lm_head"].T).argmax()
    t["head"] = time.perf_counter() - t0
    n1 = gate_layer + 1
    n2 = cfg["n_layers"] - n1
    total = t["embed"] + n1 * t["phase1_layer"] + t["select"] + n2 * t["phase2_layer"] + t["head"]
    return dict(parts_s=t, total_s=total, n_kept=len(keep), phase1_layers=n1, phase2_layers=n2)
