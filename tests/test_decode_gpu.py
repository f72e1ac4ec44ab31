"""Decode side on the B200: the tg_decode_attn kernel through the C ABI
against a float32 torch reference of the same math, and the gated
generation (prefill + decode over the gated KV cache) against the CPU
decode oracle (oracle/decode.py).

Tolerances: decode attention (bf16 in, fp32 softmax / accumulation, bf16 out)
max-abs <= 1e-2 and cosine >= 0.9999 against float32; generation logits
per decode step (bf16 model vs float32 oracle, teacher-forced to the same
tokens) max-abs <= 0.15 as in the prefill parity tests and cosine >= 0.998:
the tiny random models' logits have a std of ~0.3, so the bf16 rounding of
a decode step (two caches, every layer) moves the cosine by ~1e-3."""
import importlib.util
import os

import numpy as np
import pytest
import torch

import oracle.decode as odec
import oracle.prefill as opre
from tokengate_b200 import ops
from tokengate_b200.decode import generate_batch
from tokengate_b200.gate import LinLogSigGate, synthetic_e2e_gate
from tokengate_b200.inference import TokenGateModel, with_state_span
from tokengate_b200.model import patch_model

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


def _decode_ref(q, k, v, n_valid, n_prefix, n_keys, bias, q_scale):
    """float32 restatement: q' = bf16(q * bf16(qs)); softmax(scale q'.k + m) V."""
    qf = q.float().cpu()
    if q_scale is not None:
        s = q_scale.cpu().to(torch.bfloat16).float()
        qf = (qf * s[..., None]).to(torch.bfloat16).float()
    B, Hq, D = qf.shape
    G = Hq // k.shape[2]
    kf = k[:, :n_keys].float().cpu().repeat_interleave(G, dim=2)      # (B, N, Hq, D)
    vf = v[:, :n_keys].float().cpu().repeat_interleave(G, dim=2)
    s = torch.einsum("bhd,bnhd->bhn", qf, kf) * D ** -0.5
    m = torch.zeros(B, Hq, n_keys)
    if bias is not None:
        m[:, :, :n_prefix] = torch.broadcast_to(bias.cpu()[..., :n_prefix], (B, Hq, n_prefix))
    for b in range(B):
        m[b, :, int(n_valid[b]):n_prefix] = float("-inf")
    p = torch.softmax(s + m, dim=-1)
    return torch.einsum("bhn,bnhd->bhd", p, vf)


@pytest.mark.parametrize("B,Hq,Hkv,n_prefix,n_keys,valid,bias_kind,qs", [
    (1, 16, 8, 2768, 2771, [2700], "head", True),
    (2, 4, 2, 100, 103, [100, 57], "row", False),
    (1, 32, 8, 33000, 33003, [32768], None, False),
    (3, 8, 8, 256, 256, [256, 1, 200], "head", False),
    (1, 16, 2, 300, 520, [300], "row", True),
    (2, 16, 8, 1, 1, [1, 1], None, True),
])
def test_decode_attention_kernel(cuda, B, Hq, Hkv, n_prefix, n_keys, valid, bias_kind, qs):
    g = torch.Generator().manual_seed(n_keys + B)
    cap = n_keys + 5
    q = torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(B, cap, Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(B, cap, Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)
    bias = None
    if bias_kind == "head":
        bias = (torch.randn(B, Hq, n_prefix, generator=g) * 2).to(cuda)
    elif bias_kind == "row":
        bias = (torch.randn(B, 1, n_prefix, generator=g) * 2).to(cuda)
    q_scale = (0.5 + torch.rand(B, Hq, generator=g)).to(cuda) if qs else None
    n_valid = torch.tensor(valid, dtype=torch.int32, device=cuda)
    out = ops.decode_attention(q, k, v, n_valid, n_prefix, n_keys, bias=bias, q_scale=q_scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = _decode_ref(q, k, v, valid, n_prefix, n_keys, bias, q_scale)
    got = out.float().cpu()
    err = (got - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.reshape(-1), ref.reshape(-1), dim=0).item()
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


def test_decode_attention_rejects(cuda):
    q = torch.zeros(1, 4, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(1, 10, 2, 128, dtype=torch.bfloat16, device=cuda)
    nv = torch.tensor([5], dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError):
        ops.decode_attention(q, k, k, nv, 5, 11)                 # beyond the capacity
    with pytest.raises(ValueError):
        ops.decode_attention(q, k, k, nv, 6, 5)                  # prefix past n_keys
    from tokengate_b200._lib import TokenGateUnsupportedError
    q3 = torch.zeros(1, 6, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(TokenGateUnsupportedError):
        ops.decode_attention(q3, k, k, nv, 5, 5)                 # 3 query heads per kv head


def _logit_check(got, ref):
    got = got.float().cpu().numpy()
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref).max()
    cos = (got * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref))
    assert err <= 0.15 and cos >= 0.998, f"logits max-abs {err} cos {cos}"


@pytest.fixture(scope="module")
def tiny(cuda):
    mg = _mg()
    cpu_model = mg.tiny_model()
    model = mg.tiny_model().to(cuda).to(torch.bfloat16).eval()
    patch_model(model)
    return dict(mg=mg, cpu=cpu_model, w=opre.weights_fp32(cpu_model), model=model)


@pytest.mark.parametrize("phase2_form", [True, False])
def test_generate_vs_oracle_linear_gate(tiny, cuda, phase2_form):
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (300, 233)]
    starts, ends, K, steps = [20, 10], [280, 200], 30, 6
    gw = torch.randn(512, generator=g) * 0.05
    gate = LinLogSigGate(512).to(cuda)
    with torch.no_grad():
        gate.readout.weight.copy_(gw.view(1, -1))
    forced = torch.randint(0, 1000, (2, steps - 1), generator=g)
    lg = []
    r = generate_batch(tiny["model"], gate, prompts, starts, ends, 1, K, steps, phase2_form=phase2_form,
                       forced_tokens=forced, logits_out=lg)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = odec.gated_generate(tiny["cpu"], gw, prompts, starts, ends, 1, K, steps, phase2_form=phase2_form,
                              weights=tiny["w"], forced_tokens=forced)
    assert r.n_kepts == ref["n_kepts"] and r.steps == steps - 1
    for s in range(steps - 1):
        _logit_check(lg[s], ref["logits"][s + 1])


def test_generate_vs_oracle_e2e_gate(cuda):
    mg = _mg()
    cpu_model = mg.tiny_e2e_model()
    model = mg.tiny_e2e_model().to(cuda).to(torch.bfloat16).eval()
    patch_model(model)
    gate_cpu = synthetic_e2e_gate(cpu_model, 1, device="cpu")
    gate = synthetic_e2e_gate(model, 1, device=cuda)
    br = gate_cpu.gate_branch
    gp = dict(wg=br.gate_proj.weight.detach(), wu=br.up_proj.weight.detach(),
              w_row=br.down_proj.weight.detach()[0],
              gate_scale_eff=torch.nn.functional.softplus(gate_cpu.gate_scale).detach(),
              attn_scale_eff=gate_cpu.attn_scale_eff().detach(), eps=1e-6, gain=1.0)
    g = torch.Generator().manual_seed(22)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (300, 257)]
    starts, ends, K, steps = [20, 33], [280, 200], 40, 5
    forced = torch.randint(0, 1000, (2, steps - 1), generator=g)
    lg = []
    r = generate_batch(model, gate, prompts, starts, ends, 1, K, steps, forced_tokens=forced, logits_out=lg)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = odec.gated_generate(cpu_model, gp, prompts, starts, ends, 1, K, steps, e2e=True,
                              weights=opre.weights_fp32(cpu_model), forced_tokens=forced)
    assert r.n_kepts == ref["n_kepts"]
    for s in range(steps - 1):
        _logit_check(lg[s], ref["logits"][s + 1])


def test_generate_api_decodes_and_stops_at_eos(tiny, cuda):
    gate = LinLogSigGate(512).to(cuda)
    tm = TokenGateModel(tiny["model"], gate, 1, "tiny")
    ids = with_state_span(list(range(5)), list(range(100, 400)), list(range(7)))
    out = tm.generate(ids, None, max_kept_prefill_tokens=25, max_new_tokens=6)
    assert len(out.token_ids[0]) == 6 and out.decode_s > 0
    first = tm.generate(ids, None, max_kept_prefill_tokens=25, max_new_tokens=1)
    assert out.token_ids[0][0] == first.token_ids[0][0]

    class Tok:
        eos_token_id = out.token_ids[0][2]

        def decode(self, toks, skip_special_tokens=True):
            return " ".join(map(str, toks))

    cut = tm.generate(ids, Tok(), max_kept_prefill_tokens=25, max_new_tokens=6)
    n_eos = out.token_ids[0].index(Tok.eos_token_id)
    assert cut.token_ids[0] == out.token_ids[0][:n_eos + 1]
    assert cut.answers[0] == " ".join(map(str, out.token_ids[0][:n_eos]))


def test_decode_graph_equals_eager(tiny, cuda):
    """The decode step replayed as one CUDA graph gives the eager step's logits bit for bit."""
    g = torch.Generator().manual_seed(23)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (280, 300)]
    gate = LinLogSigGate(512).to(cuda)
    forced = torch.randint(0, 1000, (2, 7), generator=g)
    outs = []
    for use_graph in (False, True):
        lg = []
        generate_batch(tiny["model"], gate, prompts, [10, 20], [250, 290], 1, 40, 8, forced_tokens=forced,
                       logits_out=lg, use_graph=use_graph)
        outs.append(torch.stack(lg))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("B,N,K", [(1, 4096, 2048), (3, 2048, 6144), (8, 1000, 512), (5, 151936, 2048)])
def test_gemv_vs_cublas(cuda, B, N, K):
    """tg_gemv against torch's bf16 GEMM (cuBLAS): both accumulate in fp32 and
    round once to bf16, in different orders, so outputs agree to one bf16
    ulp (relative 2^-7 here, with an absolute floor for cancellations) and
    nearly all bit for bit."""
    g = torch.Generator(device=cuda).manual_seed(B * 7 + K)
    x = torch.randn(B, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    got = ops.gemv(x, w).float()
    ref = torch.nn.functional.linear(x, w).float()
    assert ((got - ref).abs() <= 2 ** -7 * ref.abs() + 2e-3).all()
    assert (got == ref).float().mean().item() >= 0.95
    if N % 16 == 0:   # the silu_mul reference takes an intermediate size that is a multiple of 8
        act = ops.gemv(x, w, swiglu=True).float()
        ref_act = ops.silu_mul(torch.nn.functional.linear(x, w)).float()
        assert ((act - ref_act).abs() <= 2 ** -6 * ref_act.abs() + 2e-3).all()
        assert (act == ref_act).float().mean().item() >= 0.9


def test_rotary_table_equals_per_step(tiny, cuda):
    """The decode step gathers its rotary cos / sin from a table the model's
    rotary embedding makes for all decode positions at once; that table is
    bit-identical to making each position's row on its own step."""
    inner = tiny["model"].model
    like = torch.empty((2, 1, 1), dtype=inner.embed_tokens.weight.dtype, device=cuda)
    pos = torch.tensor([[301], [4093]], device=cuda) + torch.arange(9, device=cuda).view(1, 9)
    cos_t, sin_t = inner.rotary_emb(like, pos)
    for s in range(9):
        c, si = inner.rotary_emb(like, pos[:, s:s + 1])
        assert torch.equal(c, cos_t[:, s:s + 1]) and torch.equal(si, sin_t[:, s:s + 1])
