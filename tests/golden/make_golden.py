"""Generate the golden fixtures of tests/golden/ by running the REFERENCE's own code.

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py <reference checkout>

Runs on CPU in the container that has the reference checkout (it does not
exist on the GPU box, so the fixtures are committed). Every output below
comes from reference functions, imported unmodified:

  attn_sdpa_small.npz   sdpa_compat.sdpa_causal on the shapes of
                        tests/attention/test_sdpa_compat.py:10-36 (fp32,
                        kv heads 1/2/4, bias layouts (S,), (B,S), (S,H), (B,S,H));
  attn_d128.npz         flex_attention_utils.flex_attention_gate_bias (the
                        FlexAttention key-bias path, run uncompiled: torch's
                        compiled CPU path fails in this container) and
                        sdpa_causal at head_dim 128 with GQA, a per-head bias
                        with -1e9 pads and a scalar bias;
  select.npz            gate_forward._select_indices (torch.topk), the keep
                        list as prefill_batch_for_decode builds it
                        (gate_forward.py:1417-1421) and
                        build_gate_bias_vectorized + -1e9 pads;
  prefill_tiny.npz      gate_forward.prefill_batch_for_decode on a tiny
                        random-init Qwen3 (head_dim 128) with backend "sdpa"
                        and a linear log-sigmoid gate fixture; first tokens,
                        kept positions, n_kept, last-row logits;
  e2e_gate_ckpt.pt      e2e_gate_module.save_gate of a small finalized
                        E2EGate (d_model 32, 4 heads, 3 bias layers, branch
                        inter 256) — the checkpoint format load_gate reads;
  e2e_gate.npz          that gate's forward / aggregate on bf16-valued raw
                        scores, _select_indices on the aggregate,
                        build_gate_bias_vectorized (bf16), _ssmax_ratio and
                        Qwen3FlexAttention._phase2_q_bias per layer in bf16
                        (s_eff and the scaled bias), and the branch readout
                        br(z) in bf16 with its fused [gate | up] projection;
  prefill_e2e_tiny.npz  prefill_batch_for_decode with a finalized E2EGate
                        (built by E2EGate + set_qk_norm_scales +
                        build_gate_branch, then seeded readout / scales) on a
                        4-layer tiny Qwen3, backend "sdpa".
"""
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def _bf16_grid(t):
    return t.to(torch.bfloat16).float()


def gen_attn_sdpa_small():
    from tokengate.e2e_gate.attn.sdpa_compat import sdpa_causal
    torch.manual_seed(7)
    B, H, S, D = 2, 4, 19, 8
    out = {}
    for kvh in (1, 2, 4):
        q = torch.randn(B, H, S, D)
        k = torch.randn(B, kvh, S, D)
        v = torch.randn_like(k)
        out[f"kv{kvh}_q"], out[f"kv{kvh}_k"], out[f"kv{kvh}_v"] = q.numpy(), k.numpy(), v.numpy()
        for tag, shape, per_head in (("none", None, False), ("s", (S,), False), ("bs", (B, S), False),
                                     ("sh", (S, H), True), ("bsh", (B, S, H), True)):
            bias = torch.randn(*shape) if shape else None
            o = sdpa_causal(q, k, v, bias, per_head, 7)
            out[f"kv{kvh}_{tag}_out"] = o.numpy()
            if bias is not None:
                out[f"kv{kvh}_{tag}_bias"] = bias.numpy()
    _save("attn_sdpa_small.npz", **out)


def gen_attn_d128():
    from tokengate.e2e_gate.attn import flex_attention_utils as fau
    from torch.nn.attention.flex_attention import flex_attention as flex_eager
    from tokengate.e2e_gate.attn.sdpa_compat import sdpa_causal
    fau.flex_attention = flex_eager  # the compiled CPU path fails here; run the same op uncompiled
    g = torch.Generator().manual_seed(1234)
    B, H, Hkv, S, D = 1, 4, 2, 136, 128
    q = _bf16_grid(torch.randn(B, H, S, D, generator=g) * 0.5)
    k = _bf16_grid(torch.randn(B, Hkv, S, D, generator=g) * 0.5)
    v = _bf16_grid(torch.randn(B, Hkv, S, D, generator=g))
    bias_h = torch.randn(S, H, generator=g) * 2.0
    bias_h[-16:] = -1e9
    bias_s = torch.nn.functional.logsigmoid(torch.randn(S, generator=g) * 2.0)
    bits = lambda t: t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    out = dict(q_bf16=bits(q), k_bf16=bits(k), v_bf16=bits(v), bias_h=bias_h.numpy(),
               bias_s=bias_s.numpy())
    out["flex_h"] = fau.flex_attention_gate_bias(q, k, v, bias_h, per_head=True).numpy()
    out["flex_s"] = fau.flex_attention_gate_bias(q, k, v, bias_s, per_head=False).numpy()
    out["flex_causal"] = fau.flex_attention_causal(q, k, v).numpy()
    out["sdpa_h"] = sdpa_causal(q, k, v, bias_h, True).numpy()
    _save("attn_d128.npz", **out)


class _TopKGate:
    selection_mode = "topk"
    random_topk = False


def gen_select():
    from tokengate.e2e_gate.gate_module.gate_forward import _select_indices, build_gate_bias_vectorized
    g = torch.Generator().manual_seed(99)
    cases = []
    out = {}
    for ci, (n, start, suffix) in enumerate(((1000, 37, 21), (3000, 512, 256), (64, 0, 5))):
        scores = torch.nn.functional.logsigmoid(torch.randn(n, generator=g) * 2.0)
        seq_len = start + n + suffix
        end = start + n
        out[f"c{ci}_scores"] = scores.numpy()
        for K in (1, 10, n // 3, n - 1, n, n + 50):
            Kc = max(1, min(K, n))
            topk_local = _select_indices(scores, Kc, _TopKGate())
            keep = torch.cat([torch.arange(start), start + torch.sort(topk_local).values,
                              torch.arange(end, seq_len)])
            n_kept = keep.shape[0]
            n_alloc = n_kept + 3
            b_pruned = build_gate_bias_vectorized(scores, topk_local, start, end, keep, seq_len,
                                                  torch.float32)
            bias = torch.zeros(n_alloc)
            bias[:n_kept] = b_pruned
            bias[n_kept:] = -1e9
            # the K-th and (K+1)-th scores must differ, else torch.topk's pick is arbitrary
            srt = torch.sort(scores, descending=True).values
            margin = float(srt[Kc - 1] - srt[Kc]) if Kc < n else float("inf")
            key = f"c{ci}_K{K}"
            out[key + "_topk"] = torch.sort(topk_local).values.numpy()
            out[key + "_keep"] = keep.numpy()
            out[key + "_bias"] = bias.numpy()
            cases.append(dict(case=ci, n=n, start=start, seq_len=seq_len, K=K, K_clamped=Kc,
                              n_kept=n_kept, n_alloc=n_alloc, key=key, margin=margin))
    out["cases_json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)
    _save("select.npz", **out)


class LinLogSigGateFixture(torch.nn.Module):
    """DeterministicGate (tests/inference/test_prefill_memory.py:18-33) with log-sigmoid applied."""
    n_layers_bias = 0
    selection_mode = "topk"

    def __init__(self, hidden, seed):
        super().__init__()
        self.gate_branch = None
        self.readout = torch.nn.Linear(hidden, 1, bias=False)
        with torch.no_grad():
            self.readout.weight.copy_(torch.randn(1, hidden, generator=torch.Generator().manual_seed(seed))
                                      * hidden ** -0.5)

    def forward(self, hidden):
        return torch.nn.functional.logsigmoid(self.readout(hidden)).squeeze(-1)

    def aggregate(self, scores):
        return scores


TINY = dict(hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=4,
            num_key_value_heads=2, head_dim=128, vocab_size=1000, rope_theta=1e6,
            tie_word_embeddings=False)
TINY_SEED = 17
TINY_GATE_SEED = 18


def tiny_model():
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM
    cfg = Qwen3Config(**TINY)
    cfg._attn_implementation = "eager"
    torch.manual_seed(TINY_SEED)
    return Qwen3ForCausalLM(cfg).eval()


def weights_digest(model) -> str:
    h = hashlib.sha256()
    for name, p in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def gen_prefill_tiny():
    from tokengate.e2e_gate.attn.qwen3_flex_attention import (patch_model_with_flex_attention,
                                                              set_attention_backends_for_layers)
    from tokengate.e2e_gate.gate_module import gate_forward as gf
    model = tiny_model()
    digest = weights_digest(model)
    patch_model_with_flex_attention(model)
    set_attention_backends_for_layers(model, "sdpa")
    gate = LinLogSigGateFixture(TINY["hidden_size"], TINY_GATE_SEED)
    g = torch.Generator().manual_seed(5)
    lens = [300, 257]
    prompts = [torch.randint(0, TINY["vocab_size"], (n,), generator=g).tolist() for n in lens]
    starts, ends, K = [20, 33], [280, 200], 40
    logits_seen = []
    h = model.lm_head.register_forward_hook(lambda m, a, o: logits_seen.append(o.detach().clone()))
    try:
        first, cache, kept, n_kepts, K_cl = gf.prefill_batch_for_decode(
            model, gate, prompts, starts, ends, 1, K)
    finally:
        h.remove()
    out = dict(prompt0=np.array(prompts[0]), prompt1=np.array(prompts[1]), starts=np.array(starts),
               ends=np.array(ends), K=np.array(K), first_tokens=first.numpy()[:, 0],
               kept=kept.numpy(), n_kepts=np.array(n_kepts), K_clampeds=np.array(K_cl),
               logits=logits_seen[-1].numpy(),
               gate_w=gate.readout.weight.detach().numpy()[0],
               meta_json=np.frombuffer(json.dumps(dict(tiny=TINY, seed=TINY_SEED, gate_seed=TINY_GATE_SEED,
                                                       weights_sha256=digest, gate_layer=1)).encode(),
                                       dtype=np.uint8))
    _save("prefill_tiny.npz", **out)


E2E_SEED = 20261012
TINY_E2E = dict(TINY, num_hidden_layers=4)


def e2e_seeded_params(gate, seed):
    """Deterministic non-trivial readout row and per-(layer, head) scales.

    The folded readout row is zero-initialised by build_gate_branch, so it is
    drawn here (std 0.05, as tests/inference/test_bench_batched_equivalence.py
    does), and gate_scale / attn_scale get a seeded perturbation so that layers
    and heads differ."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        dp = gate.gate_branch.down_proj.weight
        dp.copy_(torch.randn(dp.shape, generator=g) * 0.05)
        gate.gate_scale.add_(torch.randn(gate.gate_scale.shape, generator=g) * 0.3)
        gate.attn_scale.add_(torch.randn(gate.attn_scale.shape, generator=g) * 0.3)


def state_digest(sd) -> str:
    h = hashlib.sha256()
    for name, p in sorted(sd.items()):
        h.update(name.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def gen_e2e_gate():
    from types import SimpleNamespace
    from transformers.models.qwen3.modeling_qwen3 import Qwen3MLP
    from tokengate.e2e_gate.attn.qwen3_flex_attention import Qwen3FlexAttention
    from tokengate.e2e_gate.gate_module import gate_forward as gf
    from tokengate.e2e_gate.gate_module.e2e_gate_module import E2EGate, save_gate, to_cast_linears
    d_model, n_heads, n_lb, inter = 32, 4, 3, 256
    torch.manual_seed(3)
    gate = E2EGate(d_model=d_model, n_heads=n_heads, n_layers_bias=n_lb)
    br = Qwen3MLP(SimpleNamespace(hidden_size=d_model, intermediate_size=inter, hidden_act="silu"))
    br.down_proj = torch.nn.Linear(inter, 1, bias=False)
    gate.gate_branch = to_cast_linears(br)
    with torch.no_grad():
        for lin in (br.gate_proj, br.up_proj):
            lin.weight.copy_(torch.randn(lin.weight.shape) * d_model ** -0.5)
        gate.gate_scale.copy_(torch.randn(n_lb, n_heads))
    e2e_seeded_params(gate, 11)
    gate = gate.float().eval()
    path = os.path.join(HERE, "e2e_gate_ckpt.pt")
    save_gate(gate, path, metadata={"gate_layer": 1, "base_model": "synthetic"})
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")

    g = torch.Generator().manual_seed(21)
    out = dict(n_heads=np.array(n_heads), n_layers_bias=np.array(n_lb))
    bits = lambda t: t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    # raw scores as the prefill hands them to the gate: bf16 branch outputs cast to fp32
    n_art, start, suffix = 300, 17, 9
    seq_len = start + n_art + suffix
    raw = (torch.randn(n_art, 1, generator=g) * 0.7).to(torch.bfloat16).float()
    with torch.no_grad():
        b = gate(raw)
        agg = gate.aggregate(b)
    out.update(raw=raw.numpy()[:, 0], b=b.numpy(), agg=agg.numpy())
    cases = []
    keeps, biases = [], []
    for K in (1, 40, 150, n_art):
        topk_local = gf._select_indices(agg, K, gate)
        keep = torch.cat([torch.arange(start), start + torch.sort(topk_local).values,
                          torch.arange(start + n_art, seq_len)])
        bp = gf.build_gate_bias_vectorized(b, topk_local, start, start + n_art, keep, seq_len,
                                           torch.bfloat16)
        srt = torch.sort(agg, descending=True).values
        margin = float(srt[K - 1] - srt[K]) if K < n_art else float("inf")
        out[f"K{K}_topk"] = torch.sort(topk_local).values.numpy()
        out[f"K{K}_keep"] = keep.numpy()
        out[f"K{K}_bias"] = bits(bp)
        cases.append(dict(K=K, n_kept=int(keep.shape[0]), margin=margin))
        keeps.append(keep)
        biases.append(bp)
    # batched Phase-2 operands: the four cases as one batch, padded to n_alloc
    B = len(keeps)
    n_alloc = max(k.shape[0] for k in keeps) + 5
    kept_positions = torch.zeros(B, n_alloc, dtype=torch.long)
    gate_bias = torch.zeros(B, n_alloc, n_lb, n_heads, dtype=torch.bfloat16)
    for i, (k, bp) in enumerate(zip(keeps, biases)):
        kept_positions[i, :k.shape[0]] = k
        gate_bias[i, :k.shape[0]] = bp
        gate_bias[i, k.shape[0]:] = -1e9
    r = gf._ssmax_ratio(kept_positions)
    out.update(kept_positions=kept_positions.numpy(), ssmax_ratio=r.numpy(),
               gate_bias_batched=bits(gate_bias))
    q = torch.randn(B, n_heads, n_alloc, 8, generator=g).to(torch.bfloat16)
    eff = gate.attn_scale_eff()
    for l in range(n_lb):
        ns = SimpleNamespace(attn_scale=eff[l], ssmax_ratio=r, gate_bias=gate_bias[..., l, :],
                             _gate_per_head=True)
        q_for, bias_for, s_eff = Qwen3FlexAttention._phase2_q_bias(ns, q)
        out[f"L{l}_s_eff"] = bits(s_eff)            # (B, H, n_alloc)
        out[f"L{l}_bias"] = bits(bias_for)          # (B, n_alloc, H)
    out["q"] = bits(q)
    out["cases_json"] = np.frombuffer(json.dumps(cases).encode(), dtype=np.uint8)
    # branch readout on bf16 rows, as gate_branch_hs computes it (absorbed, no residual)
    z = torch.randn(64, d_model, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        score = gate.gate_branch(z)                 # CastLinear: bf16 compute
        gu = torch.cat([torch.nn.functional.linear(z, br.gate_proj.weight.to(torch.bfloat16)),
                        torch.nn.functional.linear(z, br.up_proj.weight.to(torch.bfloat16))], dim=-1)
    out.update(z=bits(z), gu=bits(gu), branch_score=bits(score[:, 0]),
               readout_row=bits(br.down_proj.weight[0]))
    _save("e2e_gate.npz", **out)


def tiny_e2e_model():
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM
    cfg = Qwen3Config(**TINY_E2E)
    cfg._attn_implementation = "eager"
    torch.manual_seed(TINY_SEED)
    return Qwen3ForCausalLM(cfg).eval()


def gen_prefill_e2e_tiny():
    from tokengate.e2e_gate.attn.qwen3_flex_attention import (patch_model_with_flex_attention,
                                                              set_attention_backends_for_layers)
    from tokengate.e2e_gate.gate_module import gate_forward as gf
    from tokengate.e2e_gate.gate_module.e2e_gate_module import E2EGate
    model = tiny_e2e_model()
    digest = weights_digest(model)
    patch_model_with_flex_attention(model)
    set_attention_backends_for_layers(model, "sdpa")
    gate_layer = 1
    n_lb = TINY_E2E["num_hidden_layers"] - 1 - gate_layer
    gate = E2EGate(d_model=TINY_E2E["hidden_size"], n_heads=TINY_E2E["num_attention_heads"],
                   n_layers_bias=n_lb).float()
    gate.set_qk_norm_scales(model, gate_layer)
    gf.build_gate_branch(model, gate, gate_layer)
    e2e_seeded_params(gate, E2E_SEED)
    gate.eval()
    g = torch.Generator().manual_seed(6)
    lens = [300, 257]
    prompts = [torch.randint(0, TINY_E2E["vocab_size"], (n,), generator=g).tolist() for n in lens]
    starts, ends, K = [20, 33], [280, 200], 40
    logits_seen = []
    h = model.lm_head.register_forward_hook(lambda m, a, o: logits_seen.append(o.detach().clone()))
    try:
        with torch.no_grad():
            first, cache, kept, n_kepts, K_cl = gf.prefill_batch_for_decode(
                model, gate, prompts, starts, ends, gate_layer, K)
    finally:
        h.remove()
    out = dict(prompt0=np.array(prompts[0]), prompt1=np.array(prompts[1]), starts=np.array(starts),
               ends=np.array(ends), K=np.array(K), first_tokens=first.numpy()[:, 0],
               kept=kept.numpy(), n_kepts=np.array(n_kepts), K_clampeds=np.array(K_cl),
               logits=logits_seen[-1].numpy(),
               meta_json=np.frombuffer(json.dumps(dict(
                   tiny=TINY_E2E, seed=TINY_SEED, e2e_seed=E2E_SEED, weights_sha256=digest,
                   gate_sha256=state_digest(gate.state_dict()), gate_layer=gate_layer)).encode(),
                   dtype=np.uint8))
    _save("prefill_e2e_tiny.npz", **out)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else None
    if ref:
        sys.path.insert(0, ref)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gen_attn_sdpa_small()
    gen_attn_d128()
    gen_select()
    gen_prefill_tiny()
    gen_e2e_gate()
    gen_prefill_e2e_tiny()


if __name__ == "__main__":
    main()
