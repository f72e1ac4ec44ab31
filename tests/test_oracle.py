"""Pin the CPU oracle to the reference (CPU only).

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py
running the reference's own functions; these tests check that the oracle's
restatement reproduces them, so the GPU parity tests that compare against
the oracle compare against the reference by transitivity.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle.attention as oatt
import oracle.prefill as opre
import oracle.select as osel

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def _bf16_bits_to_f32(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


def test_attention_matches_reference_sdpa_small():
    d = _load("attn_sdpa_small.npz")
    for kvh in (1, 2, 4):
        q = np.transpose(d[f"kv{kvh}_q"], (0, 2, 1, 3))   # (B, H, S, D) -> (B, S, H, D)
        k = np.transpose(d[f"kv{kvh}_k"], (0, 2, 1, 3))
        v = np.transpose(d[f"kv{kvh}_v"], (0, 2, 1, 3))
        B, S, H, D = q.shape
        for tag, per_head in (("none", False), ("s", False), ("bs", False), ("sh", True), ("bsh", True)):
            bias = None
            if tag != "none":
                bias = oatt.bias_bhs(d[f"kv{kvh}_{tag}_bias"], per_head, B, H, S)
            out, _ = oatt.keybias_attention(q, k, v, bias, causal=True)
            ref = np.transpose(d[f"kv{kvh}_{tag}_out"], (0, 2, 1, 3))
            np.testing.assert_allclose(out, ref, atol=1e-5, rtol=1e-5, err_msg=f"kv{kvh} {tag}")


def test_attention_matches_reference_flex_d128():
    d = _load("attn_d128.npz")
    q = np.transpose(_bf16_bits_to_f32(d["q_bf16"]), (0, 2, 1, 3))
    k = np.transpose(_bf16_bits_to_f32(d["k_bf16"]), (0, 2, 1, 3))
    v = np.transpose(_bf16_bits_to_f32(d["v_bf16"]), (0, 2, 1, 3))
    B, S, H, D = q.shape
    cases = (("flex_h", d["bias_h"], True), ("sdpa_h", d["bias_h"], True),
             ("flex_s", d["bias_s"], False), ("flex_causal", None, False))
    for key, bias, per_head in cases:
        bb = None if bias is None else oatt.bias_bhs(bias, per_head, B, H, S)
        out, _ = oatt.keybias_attention(q, k, v, bb, causal=True)
        ref = np.transpose(d[key], (0, 2, 1, 3))
        np.testing.assert_allclose(out, ref, atol=2e-5, rtol=1e-5, err_msg=key)


def test_selection_matches_reference():
    d = _load("select.npz")
    cases = json.loads(bytes(d["cases_json"]).decode())
    for c in cases:
        scores = d[f"c{c['case']}_scores"]
        assert c["margin"] > 0, "fixture has a tie at the K boundary"
        for use_c in (False, True):
            keep, bias, tl, nk = osel.topk_select(scores, c["K_clamped"], c["start"], c["seq_len"],
                                                  c["n_alloc"], use_c=use_c)
            assert nk == c["n_kept"]
            assert np.array_equal(tl, d[c["key"] + "_topk"]), c["key"]
            assert np.array_equal(keep[:nk], d[c["key"] + "_keep"]), c["key"]
            assert np.array_equal(bias.view(np.uint32), d[c["key"] + "_bias"].view(np.uint32)), c["key"]


def test_selection_tie_rule():
    s = np.array([1.0, 3.0, 3.0, 2.0, 3.0, 3.0, -0.0, 0.0], dtype=np.float32)
    assert osel.topk_indices(s, 3).tolist() == [1, 2, 4]
    assert osel.topk_indices(s, 6).tolist() == [0, 1, 2, 3, 4, 5]
    assert osel.topk_indices(s, 7).tolist() == [0, 1, 2, 3, 4, 5, 7]   # +0.0 ranks above -0.0
    keep, _, tl, nk = osel.topk_select(s, 3, 2, 12, 10, use_c=True)
    assert tl.tolist() == [1, 2, 4] and keep[:nk].tolist() == [0, 1, 3, 4, 6, 10, 11]


def test_oracle_logsigmoid_accuracy():
    z = np.concatenate([np.linspace(-120, 60, 20001), np.random.default_rng(0).normal(0, 3, 20000),
                        [0.0, -0.0, 1e-30, -1e-30, 87.0, 88.7, 103.9, 104.1]]).astype(np.float32)
    got = osel.logsigmoid(z).astype(np.float64)
    ref = torch.nn.functional.logsigmoid(torch.from_numpy(z.astype(np.float64))).numpy()
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    err_ulp = np.abs(got - ref) / np.maximum(ulp, np.finfo(np.float32).tiny)
    assert err_ulp.max() <= 4.0, f"max error {err_ulp.max()} ulp at z={z[err_ulp.argmax()]}"


def test_oracle_scorer_matches_float_readout():
    g = torch.Generator().manual_seed(0)
    h = torch.randn(257, 2048, generator=g).to(torch.bfloat16)
    w = torch.randn(2048, generator=g) / 2048 ** 0.5
    got = osel.gate_score(h.view(torch.int16).numpy().view(np.uint16), w.numpy())
    ref = torch.nn.functional.logsigmoid(h.double() @ w.double()).numpy()
    np.testing.assert_allclose(got, ref, rtol=3e-6, atol=1e-6)


def test_gather_oracle():
    src = np.arange(40, dtype=np.int32).reshape(10, 4)
    out = osel.gather_rows(src, np.array([9, 2, 5, 0]), 3, 5)
    assert out.tolist() == [[36, 37, 38, 39], [8, 9, 10, 11], [20, 21, 22, 23], [0] * 4, [0] * 4]


def _tiny_model_and_fixture():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    d = _load("prefill_tiny.npz")
    meta = json.loads(bytes(d["meta_json"]).decode())
    model = mg.tiny_model()
    if mg.weights_digest(model) != meta["weights_sha256"]:
        pytest.skip("random init differs from the fixture's (torch/transformers version skew)")
    return mg, model, d, meta


def test_prefill_oracle_matches_reference():
    mg, model, d, meta = _tiny_model_and_fixture()
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    res = opre.gated_prefill(model, torch.from_numpy(d["gate_w"]), prompts, d["starts"].tolist(),
                             d["ends"].tolist(), meta["gate_layer"], int(d["K"]))
    assert res["n_kepts"] == d["n_kepts"].tolist()
    assert res["K_clampeds"] == d["K_clampeds"].tolist()
    for b in range(2):
        n = res["n_kepts"][b]
        assert res["kept_positions"][b] == d["kept"][b, :n].tolist()
    assert res["first_tokens"].tolist() == d["first_tokens"].tolist()
    np.testing.assert_allclose(res["logits"].numpy(), d["logits"], atol=2e-4, rtol=1e-4)


def test_cpu_paths_match_reference_fixtures():
    """The CPU-baseline restatements (oracle/cpu_paths.py) reproduce the
    reference's own FlexAttention key-bias outputs and sdpa_causal outputs."""
    import oracle.cpu_paths as ocp
    d = _load("attn_d128.npz")
    q, k, v = (torch.from_numpy(_bf16_bits_to_f32(d[n])) for n in ("q_bf16", "k_bf16", "v_bf16"))
    for key, bias, per_head in (("flex_h", d["bias_h"], True), ("flex_s", d["bias_s"], False)):
        b = torch.from_numpy(np.ascontiguousarray(bias))
        out = ocp.flex_keybias_attention(q, k, v, b, per_head=per_head).numpy()
        np.testing.assert_allclose(out, d[key], atol=2e-5, rtol=1e-5, err_msg=key)
        out2 = ocp.sdpa_causal(q, k, v, b, per_head=per_head).numpy()
        np.testing.assert_allclose(out2, d[key], atol=2e-5, rtol=1e-5, err_msg=f"sdpa {key}")
    s = _load("attn_sdpa_small.npz")
    for kvh in (1, 2, 4):
        qq, kk, vv = (torch.from_numpy(s[f"kv{kvh}_{n}"]) for n in "qkv")
        for tag, per_head in (("s", False), ("bs", False), ("sh", True), ("bsh", True)):
            b = torch.from_numpy(s[f"kv{kvh}_{tag}_bias"])
            ref = s[f"kv{kvh}_{tag}_out"]
            np.testing.assert_allclose(ocp.sdpa_causal(qq, kk, vv, b, per_head=per_head, chunk_size=5).numpy(),
                                       ref, atol=1e-5, rtol=1e-5, err_msg=f"kv{kvh} {tag}")
            np.testing.assert_allclose(ocp.flex_keybias_attention(qq, kk, vv, b, per_head=per_head).numpy(),
                                       ref, atol=1e-5, rtol=1e-5, err_msg=f"flex kv{kvh} {tag}")


def test_cpu_gate_select_compact_matches_oracle_selection():
    """The reference-ops CPU leg keeps what the selection oracle keeps on untied scores."""
    import oracle.cpu_paths as ocp
    g = torch.Generator().manual_seed(5)
    S, H = 600, 256
    hidden = torch.randn(S, H, generator=g).to(torch.bfloat16)
    w = torch.randn(H, generator=g) / H ** 0.5
    kv = [torch.randn(2, S, 128, generator=g).to(torch.bfloat16) for _ in range(2)]
    r = ocp.gate_select_compact(hidden, w, 40, 560, 77, kv)
    sc = r["scores"].numpy()
    assert len(np.unique(sc)) == len(sc)
    keep, _, _, nk = osel.topk_select(sc, 77, 40, S, 40 + 77 + 40)
    assert r["keep"].tolist() == keep[:nk].tolist()
    assert torch.equal(r["hidden"], hidden[r["keep"]])
    assert torch.equal(r["kv"][1], kv[1][:, r["keep"]])
