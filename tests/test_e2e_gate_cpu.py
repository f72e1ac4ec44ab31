"""The finalized gate (E2EGate) on the CPU: checkpoint compatibility, the module
mirror and the oracle, each against the reference's own outputs in
tests/golden/ (e2e_gate_ckpt.pt written by the reference's save_gate;
e2e_gate.npz and prefill_e2e_tiny.npz from its E2EGate, _select_indices,
build_gate_bias_vectorized, _ssmax_ratio, _phase2_q_bias, gate_branch_hs and
prefill_batch_for_decode).

Tolerances: bf16 quantities (the Phase-2 bias and query scale, the branch
score) are compared bit for bit; fp32 intermediates that pass through
transcendental functions or long reductions (softplus, the sequence RMS, the
ssmax ratio) within 4 ulp.
"""
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

from oracle import gate_e2e as ge
from oracle import prefill as opre
from tokengate_b200.gate import E2EGate, load_gate, save_gate, synthetic_e2e_gate

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


@pytest.fixture(scope="module")
def fx():
    z = np.load(os.path.join(GOLD, "e2e_gate.npz"))
    gate, meta = load_gate(os.path.join(GOLD, "e2e_gate_ckpt.pt"))
    return z, gate, meta


def _ulps(a, b):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return np.abs(a - b) / np.maximum(np.spacing(np.abs(b)), np.float32(1e-45))


def test_load_reference_checkpoint(fx):
    z, gate, meta = fx
    assert meta == {"gate_layer": 1, "base_model": "synthetic"}
    assert gate.n_heads == 4 and gate.n_layers_bias == 3 and gate.d_model == 32
    assert gate.gate_branch.down_proj.weight.shape == (1, 256)
    assert all(p.dtype == torch.float32 for p in gate.gate_branch.parameters())
    raw = torch.from_numpy(z["raw"])[:, None]
    with torch.no_grad():
        b = gate(raw)
        agg = gate.aggregate(b)
    # the module mirror runs the same torch ops as the reference: identical on CPU
    assert torch.equal(b, torch.from_numpy(z["b"]))
    assert torch.equal(agg, torch.from_numpy(z["agg"]))


def test_save_gate_roundtrip_matches_reference_format(fx, tmp_path):
    z, gate, meta = fx
    ref = torch.load(os.path.join(GOLD, "e2e_gate_ckpt.pt"), map_location="cpu", weights_only=True)
    p = tmp_path / "g.pt"
    save_gate(gate, str(p), metadata=meta)
    mine = torch.load(str(p), map_location="cpu", weights_only=True)
    assert set(mine) == set(ref)
    for k in ref:
        if k != "state_dict":
            assert mine[k] == ref[k], k
    assert set(mine["state_dict"]) == set(ref["state_dict"])
    for k, v in ref["state_dict"].items():
        assert torch.equal(mine["state_dict"][k], v), k
    g2, m2 = load_gate(str(p))
    assert m2 == meta


def test_load_gate_rejects_variants(fx):
    ref = torch.load(os.path.join(GOLD, "e2e_gate_ckpt.pt"), map_location="cpu", weights_only=True)
    for key, bad in (("readout_residual", True), ("absorbed_readout", False), ("head_agg", "max"),
                     ("gate_branch_mode", "linear"), ("ste_factor", 0.5)):
        obj = dict(ref)
        obj[key] = bad
        with pytest.raises(ValueError):
            load_gate(obj)
    obj = dict(ref)
    obj["state_dict"] = {k: v for k, v in ref["state_dict"].items() if not k.startswith("gate_branch.")}
    with pytest.raises(ValueError):
        load_gate(obj)
    obj = dict(ref)
    obj["state_dict"] = dict(ref["state_dict"], **{"post_proj.weight": torch.zeros(1)})
    with pytest.raises(ValueError):
        load_gate(obj)
    with pytest.raises(ValueError):
        E2EGate(d_model=8, n_heads=2, n_layers_bias=0)


def test_oracle_e2e_transform_vs_reference(fx):
    z, gate, _ = fx
    gs = torch.nn.functional.softplus(gate.gate_scale).detach().numpy()
    assert _ulps(ge.softplus(gate.gate_scale.detach().numpy()), gs).max() <= 4
    b = ge.e2e_bias(z["raw"], gs)
    assert _ulps(b, z["b"]).max() <= 4
    agg = ge.aggregate(b)
    assert _ulps(agg, z["agg"]).max() <= 4
    assert _ulps(ge.ssmax_ratio(z["kept_positions"]), z["ssmax_ratio"]).max() <= 4


def test_oracle_selection_and_tables_vs_reference(fx):
    z, gate, _ = fx
    gs = torch.nn.functional.softplus(gate.gate_scale).detach().numpy()
    at = gate.attn_scale_eff().detach().numpy()
    cases = json.loads(bytes(z["cases_json"]).decode())
    agg = ge.aggregate(ge.e2e_bias(z["raw"], gs))
    for c in cases:
        K = c["K"]
        assert c["margin"] > 0      # no tie straddles the K boundary in these cases
        assert np.array_equal(ge.select(agg, K), z[f"K{K}_topk"])
        # the kernel's shortcut: top-K of the raw score itself, (raw desc, index asc)
        assert np.array_equal(ge.select(z["raw"], K), z[f"K{K}_topk"])
    raws = [z["raw"]] * len(cases)
    bias, s_eff = ge.phase2_tables(raws, [17] * len(cases), [c["n_kept"] for c in cases],
                                   z["kept_positions"], gs, at)
    for l in range(gate.n_layers_bias):
        assert np.array_equal(s_eff[l], ge.bf16_bits_to_f32(z[f"L{l}_s_eff"]))
        assert np.array_equal(bias[l], ge.bf16_bits_to_f32(z[f"L{l}_bias"]).transpose(0, 2, 1))


def test_raw_order_equals_aggregate_order_with_ties():
    """Selecting on the raw bf16 score gives the aggregate's (value desc, index asc)
    order: the aggregate is a positive scaling of the raw score, so ties and order
    coincide. Checked on heavily tied bf16 scores at every K."""
    rng = np.random.default_rng(4)
    raw = ge.bf16_round((rng.standard_normal(2000) * 3.0).astype(np.float32))
    raw[:7] = 0.0
    raw[7:11] = -0.0
    assert len(np.unique(raw)) < 1500      # about half the scores tie with another
    gs = ge.softplus(rng.standard_normal((5, 16)).astype(np.float32))
    agg = ge.aggregate(ge.e2e_bias(raw, gs))
    for K in list(range(1, 60)) + [100, 777, 1999, 2000]:
        assert np.array_equal(ge.select(raw, K), ge.select(agg, K)), K


def test_oracle_branch_score_vs_reference(fx):
    z, _, _ = fx
    got = ge.branch_score(z["gu"], z["readout_row"])
    assert np.array_equal(got, ge.bf16_bits_to_f32(z["branch_score"]))


def test_synthetic_gate_and_oracle_prefill_vs_reference():
    mg = _mg()
    d = np.load(os.path.join(GOLD, "prefill_e2e_tiny.npz"))
    meta = json.loads(bytes(d["meta_json"]).decode())
    model = mg.tiny_e2e_model()
    if mg.weights_digest(model) != meta["weights_sha256"]:
        pytest.skip("random init differs from the fixture's (version skew)")
    gate = synthetic_e2e_gate(model, meta["gate_layer"], seed=meta["e2e_seed"], device="cpu")
    assert mg.state_digest(gate.state_dict()) == meta["gate_sha256"]
    br = gate.gate_branch
    gp = dict(wg=br.gate_proj.weight.detach(), wu=br.up_proj.weight.detach(),
              w_row=br.down_proj.weight.detach()[0],
              gate_scale_eff=torch.nn.functional.softplus(gate.gate_scale).detach(),
              attn_scale_eff=gate.attn_scale_eff().detach(), eps=1e-6, gain=1.0)
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    out = opre.gated_prefill_e2e(model, gp, prompts, d["starts"].tolist(), d["ends"].tolist(),
                                 meta["gate_layer"], int(d["K"]))
    assert out["n_kepts"] == d["n_kepts"].tolist() and out["K_clampeds"] == d["K_clampeds"].tolist()
    for b in range(2):
        assert out["kept_positions"][b] == d["kept"][b, :d["n_kepts"][b]].tolist()
    assert out["first_tokens"].tolist() == d["first_tokens"].tolist()
    assert np.abs(out["logits"].numpy() - d["logits"]).max() <= 1e-4


def test_module_path_phase2_prologue_vs_reference(fx):
    """The patched attention module's Phase-2 prologue (used when the transformers
    layers run the B200 attention) forms s_eff and the scaled bias exactly as the
    reference's _phase2_q_bias does (bf16, bit for bit)."""
    from types import SimpleNamespace
    from tokengate_b200.model import _phase2_q_scale_and_bias
    z, gate, _ = fx
    eff = gate.attn_scale_eff().detach()
    r = torch.from_numpy(z["ssmax_ratio"])
    gb = torch.from_numpy(z["gate_bias_batched"].view(np.int16)).view(torch.bfloat16)
    B, n = r.shape
    for l in range(gate.n_layers_bias):
        mod = SimpleNamespace(attn_scale=eff[l], ssmax_ratio=r, gate_bias=gb[..., l, :], _gate_per_head=True)
        qs, bias = _phase2_q_scale_and_bias(mod, B, n, torch.bfloat16)
        assert np.array_equal(qs.numpy(), ge.bf16_bits_to_f32(z[f"L{l}_s_eff"]))
        assert bias.dtype == torch.bfloat16
        assert np.array_equal(bias.view(torch.int16).numpy().view(np.uint16), z[f"L{l}_bias"])
