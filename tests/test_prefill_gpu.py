"""End-to-end gated prefill on the B200 kernels vs the CPU oracle and the reference fixture.

  * stage parity, bit-exact: scores from the GPU Phase-1 hidden states equal
    the oracle scorer's; kept positions / bias row equal the oracle selection
    on those scores; compacted hidden rows and below-gate K/V rows equal the
    oracle gather;
  * result parity vs the fp32 oracle / reference fixture: same n_kept and
    K_clamped, kept-position overlap >= 0.95 (the reference's batched/single
    bar, tests/inference/test_bench_batched_equivalence.py:50-54), same first
    token, last-row logits within a bf16 tolerance (max-abs <= 0.15 and
    cosine >= 0.999 against fp32);
  * batched == single-request results (kept positions, first tokens).
"""
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

import oracle.prefill as opre
import oracle.select as osel
from tokengate_b200 import ops
from tokengate_b200 import prefill as tgp
from tokengate_b200.gate import LinLogSigGate
from tokengate_b200.inference import TokenGateModel, load_model, with_state_span
from tokengate_b200.model import patch_model

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


@pytest.fixture(scope="module")
def tiny(cuda):
    mg = _mg()
    d = np.load(os.path.join(GOLD, "prefill_tiny.npz"))
    meta = json.loads(bytes(d["meta_json"]).decode())
    cpu_model = mg.tiny_model()
    if mg.weights_digest(cpu_model) != meta["weights_sha256"]:
        pytest.skip("random init differs from the fixture's (version skew)")
    weights = opre.weights_fp32(cpu_model)
    model = mg.tiny_model().to(cuda).to(torch.bfloat16).eval()
    patch_model(model)
    gate = LinLogSigGate(cpu_model.config.hidden_size)
    with torch.no_grad():
        gate.readout.weight.copy_(torch.from_numpy(d["gate_w"]).view(1, -1))
    return dict(mg=mg, d=d, meta=meta, cpu_model=cpu_model, weights=weights, model=model, gate=gate)


def _record(monkeypatch):
    seen = {}
    orig_score, orig_topk, orig_gather = ops.gate_score, ops.topk_select, ops.gather_rows

    def score(hidden, w, begins, counts, out=None):
        seen["hidden"] = hidden.detach().clone()
        seen["w"] = w.detach().clone()
        r = orig_score(hidden, w, begins, counts, out)
        seen["scores"] = r.detach().clone()
        return r

    def topk(*a, **k):
        r = orig_topk(*a, **k)
        seen["keep"] = r[0].detach().clone()
        seen["bias"] = r[1].detach().clone()
        return r

    monkeypatch.setattr(ops, "gate_score", score)
    monkeypatch.setattr(ops, "topk_select", topk)
    return seen


def _logit_check(got, ref):
    got = got.float().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    cos = (got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref))
    assert err <= 0.15 and cos >= 0.999, f"logits max-abs {err} cos {cos}"


def test_prefill_vs_reference_fixture_and_stages(tiny, monkeypatch):
    d, model, gate = tiny["d"], tiny["model"], tiny["gate"]
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    starts, ends, K = d["starts"].tolist(), d["ends"].tolist(), int(d["K"])
    seen = _record(monkeypatch)
    logits = []
    h = model.lm_head.register_forward_hook(lambda m, a, o: logits.append(o.detach()))
    try:
        first, cache, kept, n_kepts, K_cl = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, K)
    finally:
        h.remove()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert n_kepts == d["n_kepts"].tolist() and K_cl == d["K_clampeds"].tolist()
    # stage parity (bit-exact) on the GPU's own intermediates
    hid = seen["hidden"]
    for b in range(2):
        rows = hid[b, starts[b]:ends[b]].view(torch.int16).cpu().numpy().view(np.uint16)
        ref_sc = osel.gate_score(rows, seen["w"].cpu().numpy())
        got_sc = seen["scores"][b, :ends[b] - starts[b]].cpu().numpy()
        assert np.array_equal(got_sc.view(np.uint32), ref_sc.view(np.uint32))
        ek, eb, _, nk = osel.topk_select(ref_sc, K_cl[b], starts[b], len(prompts[b]), max(n_kepts))
        assert np.array_equal(seen["keep"][b].cpu().numpy(), ek)
        eb16 = torch.from_numpy(eb).to(torch.bfloat16).view(torch.int16).numpy()
        assert np.array_equal(seen["bias"][b].view(torch.int16).cpu().numpy(), eb16)
        assert kept[b, :nk].tolist() == ek[:nk].tolist()
    # result parity vs the reference fixture (fp32 CPU run of the reference)
    for b in range(2):
        n = n_kepts[b]
        ref_keep = set(d["kept"][b, :n].tolist())
        overlap = len(ref_keep & set(kept[b, :n].tolist())) / n
        assert overlap >= 0.95, f"kept overlap {overlap}"
    assert first[:, 0].tolist() == d["first_tokens"].tolist()
    _logit_check(logits[-1], d["logits"])


def test_prefill_vs_oracle_on_gpu_selection(tiny):
    """Oracle fp32 prefill given the same kept positions as the GPU: logits agree within bf16 noise."""
    d, model, gate = tiny["d"], tiny["model"], tiny["gate"]
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (520, 300, 129)]
    starts, ends = [10, 0, 5], [500, 290, 100]
    first, _, kept, n_kepts, K_cl = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 64)
    res = opre.gated_prefill(tiny["cpu_model"], gate.readout.weight, prompts, starts, ends, 1, 64,
                             weights=tiny["weights"], bias_bf16=True)
    assert n_kepts == res["n_kepts"] and K_cl == res["K_clampeds"]
    for b in range(3):
        n = n_kepts[b]
        overlap = len(set(res["kept_positions"][b]) & set(kept[b, :n].tolist())) / n
        assert overlap >= 0.95


def test_batched_equals_single(tiny):
    model, gate = tiny["model"], tiny["gate"]
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (400, 333)]
    starts, ends = [7, 40], [390, 300]
    fb, _, kb, nb, _ = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 50)
    for b in range(2):
        f1, _, k1, n1, _ = tgp.prefill_batch_for_decode(model, gate, [prompts[b]], [starts[b]], [ends[b]], 1, 50)
        assert n1[0] == nb[b]
        assert k1[0, :n1[0]].tolist() == kb[b, :nb[b]].tolist()
        assert f1[0, 0].item() == fb[b, 0].item()


def test_prune_below_gate_kv(tiny):
    model, gate = tiny["model"], tiny["gate"]
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (300, 280)]
    starts, ends = [10, 20], [290, 200]
    _, full_cache, kept0, n0, _ = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 30)
    full_k = [full_cache.layers[i].k_tok.clone() for i in range(2)]
    full_v = [full_cache.layers[i].v_tok.clone() for i in range(2)]
    _, cache, kept, n_kepts, _ = tgp.prefill_batch_for_decode(model, gate, prompts, starts, ends, 1, 30,
                                                              prune_below_gate=True)
    assert kept.tolist() == kept0.tolist()
    W = max(n_kepts)
    for li in range(2):
        for b in range(2):
            idx = kept[b].cpu().numpy()
            for full, got in ((full_k[li], cache.layers[li].k_tok), (full_v[li], cache.layers[li].v_tok)):
                ref = osel.gather_rows(full[b].view(torch.int16).cpu().numpy(), idx, n_kepts[b], W)
                assert np.array_equal(got[b].view(torch.int16).cpu().numpy(), ref)
        assert cache.layers[li].keys.shape[2] == W    # reference (B, H, S, D) view


def test_generate_api(tiny, cuda):
    model, gate = tiny["model"], tiny["gate"]
    tm = TokenGateModel(model, gate, 1, "tiny")
    ids = with_state_span(list(range(5)), list(range(100, 400)), list(range(7)))
    out = tm.generate(ids, None, max_kept_prefill_tokens=25, max_new_tokens=1)
    assert out.n_kept == [5 + 25 + 7] and out.n_state == [300]
    assert out.kept_pos[0][:5] == list(range(5)) and out.kept_pos[0][-7:] == list(range(305, 312))
    assert len(out.token_ids[0]) == 1 and out.prefill_s > 0
    all_keep = tm.generate(ids, None, max_new_tokens=1)   # K = all
    assert all_keep.n_kept == [312]
    # the reference's default budget: 20 new tokens, the first one the prefill's
    dflt = tm.generate(ids, None, max_kept_prefill_tokens=25)
    assert len(dflt.token_ids[0]) == 20 and dflt.decode_s > 0
    assert dflt.token_ids[0][0] == out.token_ids[0][0] and dflt.kept_pos == out.kept_pos
    with pytest.raises(ValueError):
        tm.generate(ids, None, max_new_tokens=0)
    with pytest.raises(ValueError):
        tm.generate(list(range(10)), None)


def test_generate_tensor_ids_match_list_ids(tiny, cuda):
    """generate on the ids as a Python list, a pinned host tensor (scanned
    through a zero-copy view, copied whole and cut on the device) and a CUDA
    tensor: the same kept positions and first tokens; a tensor without a
    valid state span is rejected as the list is."""
    model, gate = tiny["model"], tiny["gate"]
    tm = TokenGateModel(model, gate, 1, "tiny")
    g = torch.Generator().manual_seed(41)
    ids = with_state_span(torch.randint(0, 1000, (6,), generator=g).tolist(),
                          torch.randint(0, 1000, (290,), generator=g).tolist(),
                          torch.randint(0, 1000, (9,), generator=g).tolist())
    ref = tm.generate(ids, None, max_kept_prefill_tokens=30, max_new_tokens=1)
    pinned = torch.tensor(ids, dtype=torch.long).pin_memory()
    for t in (pinned, torch.tensor(ids, dtype=torch.int32), pinned.to(cuda)):
        got = tm.generate(t, None, max_kept_prefill_tokens=30, max_new_tokens=1)
        assert got.n_kept == ref.n_kept and got.n_state == ref.n_state
        assert got.kept_pos == ref.kept_pos and got.token_ids == ref.token_ids
    with pytest.raises(ValueError):
        tm.generate(torch.arange(10).pin_memory(), None)


def test_load_model_synthetic(cuda):
    small = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=3, num_attention_heads=2,
                 num_key_value_heads=1, head_dim=128, vocab_size=500, rope_theta=1e6)
    tm = load_model(base_model=small, gate_layer=1, gate_attn="fa2", device=cuda)
    ids = with_state_span([1, 2, 3], list(range(10, 200)), [4, 5])
    out = tm.generate(ids, max_kept_prefill_tokens=16)
    assert out.n_kept == [3 + 16 + 2]
    with pytest.raises(ValueError):
        load_model(base_model=small, gate_layer=1, gate_attn="flex", device=cuda)


def test_phase2_rotary_rows_gathered_from_phase1_table(cuda):
    """The fused prefill's Phase-2 cos / sin: rows of Phase 1's table of
    positions 0..S-1 gathered at the kept positions (pad slots at position 0)
    equal the rotary module evaluated at those positions, bit for bit."""
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    cfg = Qwen3Config(hidden_size=2048, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      rope_theta=1e6, max_position_embeddings=40960)
    rot = Qwen3RotaryEmbedding(cfg).to(cuda)
    S, n_alloc = 32768, 2768
    h = torch.zeros(2, S, 8, dtype=torch.bfloat16, device=cuda)
    cos_t, sin_t = tgp._phase1_rope(rot, h, S, 2)
    g = torch.Generator().manual_seed(0)
    kept = torch.zeros(2, n_alloc, dtype=torch.int64)
    kept[0, :2700] = torch.sort(torch.randperm(S, generator=g)[:2700]).values
    kept[1] = torch.sort(torch.randperm(S, generator=g)[:n_alloc]).values
    kept = kept.to(cuda)
    cos2 = torch.empty(2, n_alloc, 128, dtype=torch.bfloat16, device=cuda)
    sin2 = torch.empty_like(cos2)
    ops.gather_rows([ops.gather_spec_rows(cos_t, cos2, 1), ops.gather_spec_rows(sin_t, sin2, 1)],
                    kept, [n_alloc, n_alloc], n_alloc, cuda)
    ref_cos, ref_sin = rot(h[:, :n_alloc], kept)
    torch.cuda.synchronize()
    assert torch.equal(cos2, ref_cos) and torch.equal(sin2, ref_sin)
