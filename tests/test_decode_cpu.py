"""The decode oracle (oracle/decode.py) on CPU: its first step is the prefill
oracle's, its plain limit is transformers' own causal LM, and batching with
ragged prompts changes nothing (the pad slots are masked)."""
import importlib.util
import os

import numpy as np
import pytest
import torch

import oracle.decode as odec
import oracle.prefill as opre
from tokengate_b200.gate import synthetic_e2e_gate

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


@pytest.fixture(scope="module")
def tiny():
    mg = _mg()
    model = mg.tiny_model()
    return dict(mg=mg, model=model, weights=opre.weights_fp32(model))


def _prompts(vocab, lens, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g).tolist() for n in lens]


def e2e_gate_dict(gate):
    br = gate.gate_branch
    return dict(wg=br.gate_proj.weight.detach(), wu=br.up_proj.weight.detach(),
                w_row=br.down_proj.weight.detach()[0],
                gate_scale_eff=torch.nn.functional.softplus(gate.gate_scale).detach(),
                attn_scale_eff=gate.attn_scale_eff().detach(), eps=1e-6, gain=1.0)


def test_first_step_is_the_prefill_oracle(tiny):
    model, w = tiny["model"], tiny["weights"]
    prompts = _prompts(1000, [300, 257], 5)
    gw = torch.randn(512, generator=torch.Generator().manual_seed(3)) * 0.05
    out = odec.gated_generate(model, gw, prompts, [20, 33], [280, 200], 1, 40, 3, weights=w)
    ref = opre.gated_prefill(model, gw, prompts, [20, 33], [280, 200], 1, 40, weights=w, bias_bf16=True)
    assert torch.equal(out["logits"][0], ref["logits"])
    assert [t[0] for t in out["tokens"]] == ref["first_tokens"].tolist()
    assert out["n_kepts"] == ref["n_kepts"] and len(out["tokens"][0]) == 3


def test_first_step_is_the_prefill_oracle_e2e():
    mg = _mg()
    model = mg.tiny_e2e_model()
    w = opre.weights_fp32(model)
    gate = synthetic_e2e_gate(model, 1, device="cpu")
    gp = e2e_gate_dict(gate)
    prompts = _prompts(1000, [300, 257], 6)
    out = odec.gated_generate(model, gp, prompts, [20, 33], [280, 200], 1, 40, 3, e2e=True, weights=w)
    ref = opre.gated_prefill_e2e(model, gp, prompts, [20, 33], [280, 200], 1, 40, weights=w)
    assert torch.equal(out["logits"][0], ref["logits"])
    assert out["n_kepts"] == ref["n_kepts"]


def test_plain_limit_is_the_causal_lm(tiny):
    """Zero gate, the whole prompt as the state span, K = all, plain decode:
    every Phase-2 key carries the same bias (softmax-invariant) and nothing is
    pruned, so the gated generation must be the model's own greedy decode —
    checked against transformers' float32 forward of prompt + continuation."""
    model, w = tiny["model"], tiny["weights"]
    prompt = _prompts(1000, [150], 7)[0]
    n = len(prompt)
    out = odec.gated_generate(model, torch.zeros(512), [prompt], [0], [n], 1, n, 5,
                              phase2_form=False, weights=w)
    toks = out["tokens"][0]
    with torch.no_grad():
        full = model(torch.tensor([prompt + toks[:-1]])).logits[0].float()
    for s in range(5):
        ref = full[n - 1 + s]
        assert (out["logits"][s][0] - ref).abs().max().item() <= 2e-3, s


def test_batched_ragged_equals_single(tiny):
    model, w = tiny["model"], tiny["weights"]
    prompts = _prompts(1000, [300, 211], 8)
    starts, ends = [20, 10], [280, 190]
    gw = torch.randn(512, generator=torch.Generator().manual_seed(4)) * 0.05
    forced = torch.randint(0, 1000, (2, 4), generator=torch.Generator().manual_seed(9))
    both = odec.gated_generate(model, gw, prompts, starts, ends, 1, 30, 5, weights=w, forced_tokens=forced)
    for b in range(2):
        one = odec.gated_generate(model, gw, [prompts[b]], [starts[b]], [ends[b]], 1, 30, 5, weights=w,
                                  forced_tokens=forced[b:b + 1])
        for s in range(5):
            assert (both["logits"][s][b] - one["logits"][s][0]).abs().max().item() <= 1e-4, (b, s)
