"""The finalized gate (E2EGate) on the B200 kernels vs the CPU oracle and the reference fixtures.

  * branch_score: bit-exact against the oracle's restatement (same fixed order,
    IEEE-only silu), and against the reference's own bf16 branch output
    (e2e_gate.npz); within one bf16 ulp of torch's eager bf16 chain;
  * phase2_tables: against the reference's _phase2_q_bias outputs (bf16, bit for
    bit) and against the oracle on random cases: q_scale and bias equal to the
    oracle's bf16 values except where the fp32 log / rsqrt of the ssmax ratio and
    the sequence RMS round differently (at most one bf16 ulp, on <= 1% of entries);
  * the whole prefill with a finalized gate: stage parity (scores bit-exact,
    kept positions = oracle selection on the aggregate of those scores), and
    result parity with the fp32 reference run (same n_kept / K_clamped,
    kept overlap >= 0.9, first tokens, logits within bf16 tolerance);
  * batched == single-request; the gate checkpoint through load_model.
"""
import importlib.util
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle.prefill as opre
from oracle import gate_e2e as ge
from tokengate_b200 import ops
from tokengate_b200 import prefill as tgp
from tokengate_b200.gate import e2e_kernel_weights, load_gate, save_gate, synthetic_e2e_gate
from tokengate_b200.inference import load_model, with_state_span
from tokengate_b200.model import patch_model

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


def _bf16_close(got, ref, max_frac_diff):
    """Entries equal, except a fraction <= max_frac_diff that differ by <= 1 bf16 ulp."""
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    diff = got != ref
    frac = diff.mean()
    assert frac <= max_frac_diff, f"{frac:.4%} of entries differ"
    if diff.any():
        rel = np.abs(got[diff] - ref[diff]) / np.abs(ref[diff])
        assert rel.max() <= 2.0 ** -7, f"difference above one bf16 ulp: {rel.max()}"


@pytest.mark.parametrize("inter", [256, 1024, 6144])
def test_branch_score_bit_exact(cuda, inter):
    g = torch.Generator(device=cuda).manual_seed(inter)
    B, S = 3, 300
    gu = (torch.randn(B, S, 2 * inter + 16, device=cuda, generator=g) * 2).to(torch.bfloat16)
    gu[0, 5, :8] = torch.tensor([-200., -90., -20., 0., -0., 20., 90., 200.])
    w = (torch.randn(inter, device=cuda, generator=g) * inter ** -0.5).to(torch.bfloat16)
    begins, counts = [5, 0, 100], [290, 1, 0]
    out = ops.branch_score(gu, w, begins, counts)
    torch.cuda.synchronize()
    for b in range(B):
        rows = gu[b, begins[b]:begins[b] + counts[b]]
        if counts[b] == 0:
            continue
        ref = ge.branch_score(_bits(rows), _bits(w))
        assert np.array_equal(out[b, :counts[b]].cpu().numpy().view(np.uint32), ref.view(np.uint32))
        # torch's eager bf16 chain (the reference's ops): silu, mul, 1-row linear
        eager = F.linear(F.silu(rows[:, :inter]) * rows[:, inter:2 * inter], w.view(1, -1))[:, 0]
        _bf16_close(out[b, :counts[b]].cpu().numpy(), eager.float().cpu().numpy(), 0.05)
    assert not (out.cpu().numpy().view(np.uint32) == 0x80000000).any()     # no -0


def test_branch_score_every_gate_pattern(cuda):
    """Every bf16 gate pattern (inf and NaN included), one per row: row r holds
    pattern r at column r % 16 with u = 1 there and 0 elsewhere, w = 1 on the
    first 16 columns, so the score is the row's bf16(silu(g)) itself. Bit-exact
    against the oracle's IEEE SiLU (NaN patterns: NaN on both sides)."""
    inter = 256
    n = 1 << 16
    r = torch.arange(n, device=cuda)
    col = r % 16
    g_bits = torch.zeros(n, inter, dtype=torch.int32, device=cuda)
    g_bits[r, col] = torch.where(r >= 32768, r - 65536, r).to(torch.int32)   # int16 range
    g = g_bits.to(torch.int16).view(torch.bfloat16)
    u = torch.zeros(n, inter, dtype=torch.bfloat16, device=cuda)
    u[r, col] = 1.0
    gu = torch.cat([g, u], dim=1).unsqueeze(0).contiguous()
    w = torch.zeros(inter, dtype=torch.bfloat16, device=cuda)
    w[:16] = 1.0
    out = ops.branch_score(gu, w, [0], [n])[0].cpu().numpy()
    ref = ge.branch_score(_bits(gu[0]), _bits(w))
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(out), nan)
    assert np.array_equal(out[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert nan.sum() == 2 * 127 + 1             # the NaN patterns and silu(-inf) = -inf / inf


def test_branch_score_vs_reference_fixture(cuda):
    z = np.load(os.path.join(GOLD, "e2e_gate.npz"))
    gu = torch.from_numpy(z["gu"].view(np.int16)).view(torch.bfloat16).to(cuda).unsqueeze(0)
    w = torch.from_numpy(z["readout_row"].view(np.int16)).view(torch.bfloat16).to(cuda)
    n = gu.shape[1]
    out = ops.branch_score(gu, w, [0], [n])
    assert np.array_equal(out[0].cpu().numpy(), ge.bf16_bits_to_f32(z["branch_score"]))


def test_phase2_tables_vs_reference_fixture(cuda):
    z = np.load(os.path.join(GOLD, "e2e_gate.npz"))
    gate, _ = load_gate(os.path.join(GOLD, "e2e_gate_ckpt.pt"))
    ew = e2e_kernel_weights(gate.to(cuda), cuda)
    cases = json.loads(bytes(z["cases_json"]).decode())
    B = len(cases)
    raw = torch.from_numpy(z["raw"]).to(cuda).unsqueeze(0).expand(B, -1).contiguous()
    keep = torch.from_numpy(z["kept_positions"]).to(cuda)
    n_state = [raw.shape[1]] * B
    bias, qs = ops.phase2_tables(raw, [17] * B, n_state, keep, [c["n_kept"] for c in cases],
                                 ew.gate_scale, ew.attn_scale, ew.eps, ew.gain)
    for l in range(gate.n_layers_bias):
        _bf16_close(qs[l].cpu().numpy(), ge.bf16_bits_to_f32(z[f"L{l}_s_eff"]), 0.01)
        _bf16_close(bias[l].cpu().numpy(), ge.bf16_bits_to_f32(z[f"L{l}_bias"]).transpose(0, 2, 1), 0.01)


@pytest.mark.parametrize("H", [16, 1])
def test_phase2_tables_vs_oracle(cuda, H):
    rng = np.random.default_rng(H)
    Lp = 5
    lens, starts, ends, Ks = [900, 1500, 64], [30, 0, 3], [850, 1400, 60], [100, 1400, 1]
    B = 3
    n_state = [e - s for s, e in zip(starts, ends)]
    raws = [ge.bf16_round((rng.standard_normal(n) * 0.6).astype(np.float32)) for n in n_state]
    scores = torch.zeros(B, max(n_state), device=cuda)
    for b in range(B):
        scores[b, :n_state[b]] = torch.from_numpy(raws[b])
    n_kept = [starts[b] + Ks[b] + lens[b] - ends[b] for b in range(B)]
    n_alloc = max(n_kept) + 7
    keep, _, _ = ops.topk_select(scores, n_state, Ks, starts, lens, n_alloc, bias_dtype=None)
    gs = torch.from_numpy(ge.softplus(rng.standard_normal((Lp, H)).astype(np.float32))).to(cuda)
    at = torch.from_numpy(ge.softplus(rng.standard_normal((Lp, H)).astype(np.float32) * 0.5 + 0.55)).to(cuda)
    bias, qs = ops.phase2_tables(scores, starts, n_state, keep, n_kept, gs, at, 1e-6, 1.0)
    torch.cuda.synchronize()
    rb, rq = ge.phase2_tables(raws, starts, n_kept, keep.cpu().numpy(), gs.cpu().numpy(), at.cpu().numpy())
    _bf16_close(qs.cpu().numpy(), rq, 0.01)
    _bf16_close(bias.cpu().numpy(), rb, 0.01)
    # pads carry bf16(-1e9) * mean_h s_eff, exactly where n_kept ends
    for b in range(B):
        assert (bias[:, b, :, n_kept[b]:] < -1e8).all()
        assert (bias[:, b, :, :n_kept[b]] > -1e8).all()


@pytest.fixture(scope="module")
def tiny_e2e(cuda):
    mg = _mg()
    d = np.load(os.path.join(GOLD, "prefill_e2e_tiny.npz"))
    meta = json.loads(bytes(d["meta_json"]).decode())
    cpu_model = mg.tiny_e2e_model()
    if mg.weights_digest(cpu_model) != meta["weights_sha256"]:
        pytest.skip("random init differs from the fixture's (version skew)")
    cpu_gate = synthetic_e2e_gate(cpu_model, meta["gate_layer"], seed=meta["e2e_seed"], device="cpu")
    assert mg.state_digest(cpu_gate.state_dict()) == meta["gate_sha256"]
    weights = opre.weights_fp32(cpu_model)
    br = cpu_gate.gate_branch
    gp = dict(wg=br.gate_proj.weight.detach(), wu=br.up_proj.weight.detach(),
              w_row=br.down_proj.weight.detach()[0],
              gate_scale_eff=F.softplus(cpu_gate.gate_scale).detach(),
              attn_scale_eff=cpu_gate.attn_scale_eff().detach(), eps=1e-6, gain=1.0)
    model = mg.tiny_e2e_model().to(cuda).to(torch.bfloat16).eval()
    patch_model(model)
    gate = synthetic_e2e_gate(cpu_model, meta["gate_layer"], seed=meta["e2e_seed"], device="cpu").to(cuda)
    return dict(d=d, meta=meta, cpu_model=cpu_model, weights=weights, model=model, gate=gate, gp=gp)


def _record(monkeypatch):
    seen = {}
    orig_bs, orig_topk, orig_tab = ops.branch_score, ops.topk_select, ops.phase2_tables

    def bs(gu, w_row, begins, counts, out=None):
        r = orig_bs(gu, w_row, begins, counts, out)
        seen.setdefault("gu", []).append(gu.detach().clone())
        seen["w_row"] = w_row.detach().clone()
        return r

    def topk(*a, **k):
        r = orig_topk(*a, **k)
        seen["sel_scores"] = a[0].detach().clone()
        seen["keep"] = r[0].detach().clone()
        return r

    def tab(*a, **k):
        r = orig_tab(*a, **k)
        seen["tables"] = (r[0].detach().clone(), r[1].detach().clone())
        seen["gs"], seen["at"] = a[5].detach().clone(), a[6].detach().clone()
        return r

    monkeypatch.setattr(ops, "branch_score", bs)
    monkeypatch.setattr(ops, "topk_select", topk)
    monkeypatch.setattr(ops, "phase2_tables", tab)
    return seen


def _logit_check(got, ref, max_abs=0.15, min_cos=0.999):
    got = got.float().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    cos = (got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref))
    assert err <= max_abs and cos >= min_cos, f"logits max-abs {err} cos {cos}"


@pytest.mark.parametrize("fused", [False, True])
def test_e2e_prefill_vs_reference_fixture_and_stages(tiny_e2e, monkeypatch, fused):
    """fused=False: the [gate | up] GEMM + branch_score readout, whose scores
    are checked bit for bit against the oracle on the GPU's own projection;
    fused=True: the branch as one GEMM with the readout in its epilogue (no
    projection to check against), scores within a bf16 ulp of the unfused
    chain's. Both: the selection on the kernel's scores, tables, and result
    parity with the reference's own run."""
    d, model, gate = tiny_e2e["d"], tiny_e2e["model"], tiny_e2e["gate"]
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    starts, ends, K = d["starts"].tolist(), d["ends"].tolist(), int(d["K"])
    monkeypatch.setattr(tgp, "_BRANCH_FUSED", False)
    seen = _record(monkeypatch)
    if fused:
        tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, K)
        unfused_scores = [seen["sel_scores"][b, :ends[b] - starts[b]].clone() for b in range(2)]
        monkeypatch.setattr(tgp, "_BRANCH_FUSED", True)
        seen.clear()
    logits = []
    h = model.lm_head.register_forward_hook(lambda m, a, o: logits.append(o.detach()))
    try:
        first, cache, kept, n_kepts, K_cl = tgp.prefill_batch_for_decode(model, gate, prompts, starts,
                                                                          ends, 1, K)
    finally:
        h.remove()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert n_kepts == d["n_kepts"].tolist() and K_cl == d["K_clampeds"].tolist()
    # stage parity on the GPU's own intermediates: the branch score (bit-exact), the
    # selection on the aggregate of those scores (bit-exact), the tables (bf16 values)
    raws = []
    for b in range(2):
        got = seen["sel_scores"][b, :ends[b] - starts[b]].cpu().numpy()
        if fused:
            assert "gu" not in seen
            ref = got
            un = unfused_scores[b].cpu().numpy()
            # the GEMM's and the dot's own fp32 orders: about a bf16 ulp of the score
            # (or of the row's scale, under cancellation); most scores equal
            assert (np.abs(got - un) <= 2.0 ** -7 * np.abs(un) + 2.0 ** -9 * np.abs(un).max()).all()
            assert (got == un).mean() >= 0.8, f"{(got == un).mean():.3f} of the scores equal"
        else:
            gu = seen["gu"][b][0]
            ref = ge.branch_score(_bits(gu), _bits(seen["w_row"]))
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        raws.append(ref)
        agg = ge.aggregate(ge.e2e_bias(ref, seen["gs"].cpu().numpy()))
        top = ge.select(agg, K_cl[b])
        exp_keep = np.concatenate([np.arange(starts[b]), starts[b] + top, np.arange(ends[b], len(prompts[b]))])
        assert kept[b, :n_kepts[b]].cpu().numpy().tolist() == exp_keep.tolist()
    rb, rq = ge.phase2_tables(raws, starts, n_kepts, seen["keep"].cpu().numpy(), seen["gs"].cpu().numpy(),
                              seen["at"].cpu().numpy())
    _bf16_close(seen["tables"][1].cpu().numpy(), rq, 0.01)
    _bf16_close(seen["tables"][0].cpu().numpy(), rb, 0.01)
    # result parity vs the reference's own fp32 CPU run
    for b in range(2):
        n = n_kepts[b]
        overlap = len(set(d["kept"][b, :n].tolist()) & set(kept[b, :n].tolist())) / n
        assert overlap >= 0.9, f"kept overlap {overlap}"
    assert first[:, 0].tolist() == d["first_tokens"].tolist()
    _logit_check(logits[-1], d["logits"])


def test_e2e_prefill_vs_oracle(tiny_e2e):
    model, gate = tiny_e2e["model"], tiny_e2e["gate"]
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (520, 300, 129)]
    starts, ends = [10, 0, 5], [500, 290, 100]
    first, _, kept, n_kepts, K_cl = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 64)
    res = opre.gated_prefill_e2e(tiny_e2e["cpu_model"], tiny_e2e["gp"], prompts, starts, ends, 1, 64,
                                 weights=tiny_e2e["weights"])
    assert n_kepts == res["n_kepts"] and K_cl == res["K_clampeds"]
    for b in range(3):
        n = n_kepts[b]
        overlap = len(set(res["kept_positions"][b]) & set(kept[b, :n].tolist())) / n
        assert overlap >= 0.9, f"request {b}: kept overlap {overlap}"


def test_e2e_batched_equals_single(tiny_e2e):
    model, gate = tiny_e2e["model"], tiny_e2e["gate"]
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (400, 333)]
    starts, ends = [7, 40], [390, 300]
    fb, _, kb, nb, _ = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 50)
    for b in range(2):
        f1, _, k1, n1, _ = tgp.prefill_batch_for_decode(model, gate, [prompts[b]], [starts[b]], [ends[b]],
                                                        1, 50)
        assert n1[0] == nb[b]
        assert k1[0, :n1[0]].tolist() == kb[b, :nb[b]].tolist()
        assert f1[0, 0].item() == fb[b, 0].item()


def test_e2e_checkpoint_through_load_model(tiny_e2e, cuda, tmp_path):
    small = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=2,
                 num_key_value_heads=1, head_dim=128, vocab_size=500, rope_theta=1e6)
    tm = load_model(base_model=small, gate_layer=1, device=cuda, gate="e2e")
    p = tmp_path / "gate.pt"
    save_gate(tm.gate, str(p), metadata={"gate_layer": 1})
    tm2 = load_model(str(p), base_model=small, device=cuda)
    ids = with_state_span([1, 2, 3], list(range(10, 300)), [4, 5])
    a = tm.generate(ids, max_kept_prefill_tokens=16)
    b = tm2.generate(ids, max_kept_prefill_tokens=16)
    assert a.n_kept == b.n_kept == [3 + 16 + 2]
    assert a.kept_pos == b.kept_pos and a.token_ids == b.token_ids
    with pytest.raises(NotImplementedError):
        tgp.prefill_batch_for_decode(tm.model, tm.gate, [list(range(50))], [5], [40], 1, 8, fused=False)
