"""Fused decoder-layer glue vs the transformers Qwen3 ops it replaces, on the GPU.

The reference computes these with transformers' modules (Qwen3RMSNorm, the
decoder-layer residual adds, apply_rotary_pos_emb, Qwen3MLP), so those
modules, run on the same bf16 inputs, are the checker. Tolerances: the
residual add is bit-exact; normalised outputs may differ by one bf16 ulp
where the variance (a 2048- or 128-term fp32 sum) rounds differently in
torch's reduction order — checked as max relative difference <= 2^-7 and
>= 99% of elements bit-identical.
"""
import pytest
import torch
import torch.nn.functional as F
from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

from tokengate_b200 import ops
from tokengate_b200 import prefill as tgp

pytestmark = pytest.mark.gpu


def _close_bf16(got, ref, min_exact=0.99, atol=0.0):
    """|got - ref| <= 2^-7 |ref| + atol everywhere, and >= min_exact bit-identical.

    atol covers outputs formed by cancellation (RoPE: y*cos + rot(y)*sin), where
    one ulp of an O(1) intermediate is a large relative error on a small result.
    """
    g, r = got.float(), ref.float()
    excess = ((g - r).abs() - (2 ** -7 * r.abs() + atol)).max().item()
    exact = (got.view(torch.int16) == ref.view(torch.int16)).float().mean().item()
    assert excess <= 0.0, f"exceeds the bound by {excess}"
    assert exact >= min_exact, f"only {exact:.4f} bit-identical"


@pytest.mark.parametrize("H", [2048, 4096, 512])
def test_add_rmsnorm(cuda, H):
    g = torch.Generator(device=cuda).manual_seed(H)
    h = torch.randn(3, 257, H, device=cuda, generator=g).to(torch.bfloat16)
    d = torch.randn(3, 257, H, device=cuda, generator=g).to(torch.bfloat16)
    norm = Qwen3RMSNorm(H, eps=1e-6).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(H, device=cuda, generator=g))
        ref_h = h + d
        ref_x = norm(ref_h)
    h2 = h.clone()
    out_h, x = ops.add_rmsnorm(h2, d, norm.weight, 1e-6, h_out=h2)
    assert out_h.data_ptr() == h2.data_ptr()
    assert torch.equal(out_h, ref_h)
    _close_bf16(x, ref_x)
    # norm only, and add only
    _, x0 = ops.add_rmsnorm(h, None, norm.weight, 1e-6)
    _close_bf16(x0, norm(h))
    h3, none = ops.add_rmsnorm(h.clone(), d, None, 0.0, want_x=False)
    assert none is None and torch.equal(h3, ref_h)


@pytest.mark.parametrize("S", [300, 20])
def test_qk_norm_rope(cuda, S):
    # S = 20: 40 rows, the few-row launch that spreads a row's heads over warps
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    B, nq, nkv, D = 2, 16, 8, 128
    g = torch.Generator(device=cuda).manual_seed(1)
    qkv = torch.randn(B, S, nq + 2 * nkv, D, device=cuda, generator=g).to(torch.bfloat16)
    qn = Qwen3RMSNorm(D, eps=1e-6).to(cuda).to(torch.bfloat16)
    kn = Qwen3RMSNorm(D, eps=1e-6).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        qn.weight.copy_(1 + 0.2 * torch.randn(D, device=cuda, generator=g))
        kn.weight.copy_(1 + 0.2 * torch.randn(D, device=cuda, generator=g))
    cfg = Qwen3Config(hidden_size=2048, num_attention_heads=nq, num_key_value_heads=nkv, head_dim=D,
                      rope_theta=1e6)
    rope = Qwen3RotaryEmbedding(cfg).to(cuda)
    pos = torch.stack([torch.arange(S), torch.sort(torch.randperm(32768)[:S]).values]).to(cuda)
    cos, sin = rope(qkv, pos)
    with torch.no_grad():
        q_ref, k_ref = apply_rotary_pos_emb(qn(qkv[:, :, :nq]).transpose(1, 2),
                                            kn(qkv[:, :, nq:nq + nkv]).transpose(1, 2), cos, sin)
    got = qkv.clone()
    ops.qk_norm_rope(got[:, :, :nq], got[:, :, nq:nq + nkv], qn.weight, kn.weight, cos, sin, 1e-6)
    # one bf16 ulp of the O(1) normalised intermediate (2^-7) as the absolute term
    _close_bf16(got[:, :, :nq], q_ref.transpose(1, 2), atol=2 ** -7)
    _close_bf16(got[:, :, nq:nq + nkv], k_ref.transpose(1, 2), atol=2 ** -7)
    assert torch.equal(got[:, :, nq + nkv:], qkv[:, :, nq + nkv:])   # v untouched
    # separate q and k buffers
    q2, k2 = qkv[:, :, :nq].contiguous(), qkv[:, :, nq:nq + nkv].contiguous()
    ops.qk_norm_rope(q2, k2, qn.weight, kn.weight, cos, sin, 1e-6)
    assert torch.equal(q2, got[:, :, :nq]) and torch.equal(k2, got[:, :, nq:nq + nkv])


def test_qk_norm_rope_few_rows_bit_identical(cuda):
    """At most 64 rows the launch spreads each row's heads over several warps;
    those rows come out bit-identical to the same rows of a larger launch
    (one warp per row)."""
    nq, nkv, D = 16, 8, 128
    g = torch.Generator(device=cuda).manual_seed(5)
    big = torch.randn(1, 100, nq + nkv, D, device=cuda, generator=g).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    cos = torch.randn(1, 100, D, device=cuda, generator=g).to(torch.bfloat16)
    sin = torch.randn(1, 100, D, device=cuda, generator=g).to(torch.bfloat16)
    small = big[:, :40].contiguous()
    ops.qk_norm_rope(big[:, :, :nq], big[:, :, nq:], qw, kw, cos, sin, 1e-6)
    ops.qk_norm_rope(small[:, :, :nq], small[:, :, nq:], qw, kw, cos[:, :40].contiguous(), sin[:, :40].contiguous(),
                     1e-6)
    torch.cuda.synchronize()
    assert torch.equal(small, big[:, :40])


def test_qk_norm_rope_append(cuda):
    """The decode form: one token per row, q/k normalised and rotated as by
    qk_norm_rope, and the finished k plus the v rows written to the caches'
    slot (read from the device)."""
    B, nq, nkv, D, cap = 3, 32, 8, 128, 50
    g = torch.Generator(device=cuda).manual_seed(3)
    qkv = torch.randn(B, 1, nq + 2 * nkv, D, device=cuda, generator=g).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(D, device=cuda, generator=g)).to(torch.bfloat16)
    cos = torch.randn(B, 1, D, device=cuda, generator=g).to(torch.bfloat16)
    sin = torch.randn(B, 1, D, device=cuda, generator=g).to(torch.bfloat16)
    ref = qkv.clone()
    ops.qk_norm_rope(ref[:, :, :nq], ref[:, :, nq:nq + nkv], qw, kw, cos, sin, 1e-6)
    kc = torch.randn(B, cap, nkv, D, device=cuda, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, cap, nkv, D, device=cuda, generator=g).to(torch.bfloat16)
    kc0, vc0 = kc.clone(), vc.clone()
    slot = torch.tensor([37], dtype=torch.int64, device=cuda)
    got = qkv.clone()
    ops.qk_norm_rope_append(got[:, :, :nq], got[:, :, nq:nq + nkv], got[:, :, nq + nkv:], qw, kw, cos, sin,
                            1e-6, kc, vc, slot)
    assert torch.equal(got, ref)
    assert torch.equal(kc[:, 37], ref[:, 0, nq:nq + nkv]) and torch.equal(vc[:, 37], qkv[:, 0, nq + nkv:])
    others = [s for s in range(cap) if s != 37]
    assert torch.equal(kc[:, others], kc0[:, others]) and torch.equal(vc[:, others], vc0[:, others])


@pytest.mark.parametrize("inter", [6144, 2400, 8])
def test_silu_mul(cuda, inter):
    # 2400: 300 vectors per row, a partial second pass of the per-row loop
    g = torch.Generator(device=cuda).manual_seed(2)
    gu = (torch.randn(5, 77, 2 * inter, device=cuda, generator=g) * 3).to(torch.bfloat16)
    out = ops.silu_mul(gu)
    ref = F.silu(gu[..., :inter]) * gu[..., inter:]
    _close_bf16(out, ref, min_exact=0.98)


def test_fused_prefill_matches_module_path(cuda):
    from tokengate_b200.inference import load_model
    small = dict(hidden_size=1024, intermediate_size=2048, num_hidden_layers=4, num_attention_heads=8,
                 num_key_value_heads=4, head_dim=128, vocab_size=2000, rope_theta=1e6)
    tm = load_model(base_model=small, gate_layer=1, device=cuda, seed=5)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, 2000, (n,), generator=g).tolist() for n in (900, 611)]
    starts, ends = [30, 11], [870, 600]
    logits = {}
    for fused in (False, True):
        seen = []
        hk = tm.model.lm_head.register_forward_hook(lambda m, a, o: seen.append(o.detach().float()))
        try:
            out = tgp.prefill_batch_for_decode(tm.model, tm.gate, prompts, starts, ends, 1, 64, fused=fused)
        finally:
            hk.remove()
        logits[fused] = (out, seen[-1])
    (f0, _, k0, n0, _), l0 = logits[False]
    (f1, _, k1, n1, _), l1 = logits[True]
    assert n0 == n1
    for b in range(2):
        overlap = len(set(k0[b, :n0[b]].tolist()) & set(k1[b, :n1[b]].tolist())) / n0[b]
        assert overlap >= 0.95
    cos = (l0 * l1).sum() / (l0.norm() * l1.norm())
    assert cos.item() >= 0.999, cos.item()
    assert (l0 - l1).abs().max().item() <= 0.15
