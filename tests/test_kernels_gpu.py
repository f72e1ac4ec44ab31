"""GPU parity of the four kernels through the C ABI, against the CPU oracle.

Tolerances:
  * attention (bf16 in, fp32 softmax/accumulate, bf16 out) vs the float64
    oracle on the same bf16-rounded inputs: max-abs <= 2e-2 and cosine >=
    0.9999 (the reference's own bf16 bar is max 0.05 / mean 0.002,
    tests/attention/test_flex_attention.py:132-133); lse within 1e-3 abs.
  * gate scorer: bit-exact against oracle/tg_oracle.c.
  * top-K / keep list / bias row: bit-exact against the oracle.
  * gather: bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle.attention as oatt
import oracle.select as osel
from tokengate_b200 import ops
from tokengate_b200._lib import TokenGateArgumentError, TokenGateUnsupportedError

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.9999


def _rand_qkv(B, Sq, Sk, Hq, Hkv, seed, dev, std=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Sq, Hq, 128, generator=g) * std).to(torch.bfloat16)
    k = (torch.randn(B, Sk, Hkv, 128, generator=g) * std).to(torch.bfloat16)
    v = torch.randn(B, Sk, Hkv, 128, generator=g).to(torch.bfloat16)
    return q.to(dev), k.to(dev), v.to(dev)


def _cos(a, b):
    a = a.reshape(-1).astype(np.float64)
    b = b.reshape(-1).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def _check_attn(q, k, v, bias_bhs, causal, rows=None, qrs=None, scale=None):
    out, lse = ops.keybias_attention(q, k, v, bias=bias_bhs, causal=causal, return_lse=True,
                                     q_row_scale=qrs, softmax_scale=scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    B, Sq, Hq, _ = q.shape
    Sk = k.shape[1]
    rows = np.arange(Sq) if rows is None else np.asarray(rows)
    bb = None
    if bias_bhs is not None:
        bb = torch.broadcast_to(bias_bhs.detach().cpu(), (B, Hq, Sk)).numpy()
    qref = q.float().cpu()
    if qrs is not None:
        # the reference scales q by the row scale in bf16 before attention
        # (qwen3_flex_attention.py:447-451); the kernel does the same
        qs = torch.broadcast_to(qrs.detach().cpu(), (B, Hq, Sq)).permute(0, 2, 1).unsqueeze(-1)
        qref = (qref * qs).to(torch.bfloat16).float()
    ref, ref_lse = oatt.keybias_attention(qref.numpy(), k.float().cpu().numpy(),
                                          v.float().cpu().numpy(), bb, scale=scale, causal=causal,
                                          rows=rows)
    got = out.float().cpu().numpy()[:, rows]
    err = np.abs(got - ref).max()
    cos = _cos(got, ref)
    assert np.isfinite(got).all()
    assert err <= ATOL, f"max-abs {err}"
    assert cos >= COS, f"cosine {cos}"
    lerr = np.abs(lse.cpu().numpy()[:, :, rows] - ref_lse).max()
    assert lerr <= 1e-3, f"lse max-abs {lerr}"
    return err, cos


@pytest.mark.parametrize("B,S,Hq,Hkv", [
    (1, 1, 2, 1), (1, 7, 2, 1), (1, 128, 2, 1), (1, 129, 2, 1), (2, 300, 4, 2),
    (1, 520, 4, 4), (1, 384, 3, 1), (2, 257, 4, 1),
])
@pytest.mark.parametrize("bias_kind", ["none", "scalar", "per_head"])
def test_attention_shapes(cuda, B, S, Hq, Hkv, bias_kind):
    q, k, v = _rand_qkv(B, S, S, Hq, Hkv, seed=S * 7 + Hq, dev=cuda)
    g = torch.Generator().manual_seed(11)
    bias = None
    if bias_kind == "scalar":
        bias = torch.nn.functional.logsigmoid(torch.randn(B, 1, S, generator=g) * 2).to(cuda)
    elif bias_kind == "per_head":
        bias = (torch.randn(B, Hq, S, generator=g) * 2).to(cuda)
        bias[..., -min(S - 1, 5):] = -1e9 if S > 1 else 0.0
    _check_attn(q, k, v, bias, causal=True)


def test_attention_config1_rows(cuda):
    """The key-bias op workload: B=1, S=4096, 16/8 heads; bias logsigmoid(2N) on the state span."""
    g = torch.Generator().manual_seed(0)
    S = 4096
    q = torch.randn(1, S, 16, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    b = torch.zeros(S)
    b[256:3840] = torch.nn.functional.logsigmoid(2 * torch.randn(3584, generator=g))
    rows = np.r_[0:5, 127:130, 1000:1003, 2047, 3839:3842, 4090:4096]
    _check_attn(q, k, v, b.to(cuda).view(1, 1, S), causal=True, rows=rows)


def test_attention_ragged_4093_padded(cuda):
    """test_attention_backends_grad.py:21-30 shape: S=4093, 16/8 heads, 0.5 N inputs, 2N per-head bias, -1e9 pads."""
    S = 4093
    q, k, v = _rand_qkv(1, S, S, 16, 8, seed=5, dev=cuda, std=0.5)
    g = torch.Generator().manual_seed(6)
    bias = torch.randn(S, 16, generator=g) * 2.0
    bias[-64:] = -1e9
    bias_bhs = bias.t().contiguous().view(1, 16, S).to(cuda)
    rows = np.r_[0:3, 126:131, 2000:2004, 4020:4093]
    _check_attn(q, k, v, bias_bhs, causal=True, rows=rows)


def test_attention_noncausal_and_cross_lengths(cuda):
    q, k, v = _rand_qkv(2, 200, 333, 4, 2, seed=3, dev=cuda)
    g = torch.Generator().manual_seed(4)
    bias = torch.randn(2, 4, 333, generator=g).to(cuda)
    _check_attn(q, k, v, bias, causal=False)


def test_attention_strided_views_and_row_scale(cuda):
    """Q/K/V as slices of one fused projection (B, S, Hq+2Hkv, D), and a per-row query scale."""
    B, S, Hq, Hkv = 2, 333, 4, 2
    g = torch.Generator().manual_seed(9)
    fused = torch.randn(B, S, Hq + 2 * Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)
    q, k, v = fused[:, :, :Hq], fused[:, :, Hq:Hq + Hkv], fused[:, :, Hq + Hkv:]
    qrs = (0.5 + torch.rand(B, Hq, S, generator=g)).to(cuda)
    bias = torch.randn(B, 1, S, generator=g).to(cuda)
    _check_attn(q, k, v, bias, causal=True, qrs=qrs, scale=0.07)


def test_attention_large_bias_range(cuda):
    """Biases spanning +-30 exercise the lazy max (rescale) path."""
    q, k, v = _rand_qkv(1, 1024, 1024, 2, 1, seed=21, dev=cuda)
    bias = torch.linspace(-30, 30, 1024).view(1, 1, 1024).to(cuda)
    _check_attn(q, k, v, bias, causal=True)
    bias2 = torch.linspace(30, -30, 1024).view(1, 1, 1024).to(cuda)
    _check_attn(q, k, v, bias2, causal=True)


def test_attention_max_outgrows_running_max(cuda):
    """Key blocks whose logits exceed every earlier block's by far: a steep
    ramp (each 128-key block ~25 above the last, so p would pass 2^16 and the
    polynomial exp2's clamp) and one key 120 above the rest (2^173: inf on
    the MUFU), in both bias templates."""
    q, k, v = _rand_qkv(1, 1024, 1024, 2, 1, seed=23, dev=cuda)
    ramp = torch.linspace(-100, 100, 1024).view(1, 1, 1024).to(cuda)
    _check_attn(q, k, v, ramp, causal=True)
    spike = torch.zeros(1, 1, 1024)
    spike[..., 700] = 120.0
    _check_attn(q, k, v, spike.to(cuda), causal=True)
    # no-bias template: the same growth carried by the keys themselves
    k2 = k.clone()
    k2[:, 640:768] = (q[:, 640:768].float().mean(dim=2, keepdim=True) * 6).to(torch.bfloat16)
    _check_attn(q, k2, v, None, causal=True)


def test_attention_rejects(cuda):
    q, k, v = _rand_qkv(1, 64, 64, 2, 1, seed=1, dev=cuda)
    with pytest.raises(TokenGateUnsupportedError):
        ops.keybias_attention(q[..., :64].contiguous(), k[..., :64].contiguous(), v[..., :64].contiguous())
    with pytest.raises(TokenGateArgumentError):
        ops.keybias_attention(q, k[:, :32], v[:, :32], causal=True)
    with pytest.raises(ValueError):
        ops.keybias_attention(q.cpu(), k.cpu(), v.cpu())


# ----------------------------------------------------------------- gate scorer
def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("H", [512, 2048, 4096])
def test_gate_score_bit_exact(cuda, H):
    g = torch.Generator().manual_seed(H)
    B, S = 3, 700
    h = torch.randn(B, S, H, generator=g).to(torch.bfloat16)
    w = torch.randn(H, generator=g) / H ** 0.5
    begins, counts = [0, 100, 650], [700, 400, 50]
    out = ops.gate_score(h.to(cuda), w.to(cuda), begins, counts)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        rows = _bf16_bits(h[b, begins[b]:begins[b] + counts[b]])
        ref = osel.gate_score(rows, w.numpy())
        assert np.array_equal(got[b, :counts[b]].view(np.uint32), ref.view(np.uint32)), f"request {b}"
        # and the reference float path (torch logsigmoid of the fp32 readout) within fp32 rounding
        torch_ref = torch.nn.functional.logsigmoid(h[b, begins[b]:begins[b] + counts[b]].double()
                                                   @ w.double()).numpy()
        np.testing.assert_allclose(got[b, :counts[b]], torch_ref, rtol=2e-5, atol=2e-6)


def test_gate_score_config2(cuda):
    """The gate-scoring workload: (1, 32768, 2048) bf16 N(0,1), state 512..32511, w ~ N(0, 1/2048)."""
    g = torch.Generator().manual_seed(2)
    h = torch.randn(1, 32768, 2048, generator=g).to(torch.bfloat16)
    w = torch.randn(2048, generator=g) / 2048 ** 0.5
    out = ops.gate_score(h.to(cuda), w.to(cuda), [512], [32000])
    ref = osel.gate_score(_bf16_bits(h[0, 512:32512]), w.numpy())
    assert np.array_equal(out.cpu().numpy()[0].view(np.uint32), ref.view(np.uint32))


# ----------------------------------------------------------------- top-K
def _check_topk(scores_np, ks, begins, seq_lens, n_alloc, dev):
    B = len(ks)
    n_state = [len(s) for s in scores_np]
    width = max(n_state)
    sc = np.zeros((B, width), dtype=np.float32)
    for b in range(B):
        sc[b, :n_state[b]] = scores_np[b]
    keep, bias, tl = ops.topk_select(torch.from_numpy(sc).to(dev), n_state, ks, begins, seq_lens,
                                     n_alloc, bias_dtype=torch.float32, want_topk_local=True)
    torch.cuda.synchronize()
    for b in range(B):
        ek, eb, etl, nk = osel.topk_select(scores_np[b], ks[b], begins[b], seq_lens[b], n_alloc)
        ck, cb, ctl, cnk = osel.topk_select(scores_np[b], ks[b], begins[b], seq_lens[b], n_alloc, use_c=True)
        assert np.array_equal(ek, ck) and np.array_equal(eb.view(np.uint32), cb.view(np.uint32))
        assert np.array_equal(keep[b].cpu().numpy(), ek), f"keep mismatch request {b}"
        assert np.array_equal(bias[b].cpu().numpy().view(np.uint32), eb.view(np.uint32))
        assert np.array_equal(tl[b, :ks[b]].cpu().numpy(), etl)


@pytest.mark.parametrize("K", [1, 100, 500, 2000, 31999, 32000])
def test_topk_config2_ties(cuda, K):
    """32000 bf16-rounded scores: many ties at the K-th value; lower indices win."""
    g = torch.Generator().manual_seed(K)
    s = torch.nn.functional.logsigmoid(torch.randn(32000, generator=g) * 2).to(torch.bfloat16).float().numpy()
    _check_topk([s], [K], [512], [32768], 512 + K + 256 + 3, cuda)


def test_topk_batched_ragged(cuda):
    g = torch.Generator().manual_seed(7)
    scores = [torch.randn(n, generator=g).numpy().astype(np.float32) for n in (10, 3000, 1, 777)]
    scores[0][:] = 0.5                      # all tied
    scores[3][::2] = -0.0                   # signed zeros
    scores[3][1::2] = 0.0
    ks = [3, 1000, 1, 400]
    begins = [0, 5, 2, 100]
    seq_lens = [10, 3010, 4, 900]
    _check_topk(scores, ks, begins, seq_lens, 1100, cuda)


def test_topk_rejects(cuda):
    sc = torch.zeros(1, 10, device=cuda)
    with pytest.raises(TokenGateArgumentError):
        ops.topk_select(sc, [10], [11], [0], [10], 20)
    with pytest.raises(TokenGateArgumentError):
        ops.topk_select(sc, [10], [5], [0], [10], 4)


# ----------------------------------------------------------------- gather
def test_gather_hidden_and_kv(cuda):
    g = torch.Generator().manual_seed(3)
    B, S, H, Hkv = 2, 1000, 2048, 8
    hid = torch.randn(B, S, H, generator=g).to(torch.bfloat16).to(cuda)
    k_tok = torch.randn(B, S, Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)   # token-major
    v_head = torch.randn(B, Hkv, S, 128, generator=g).to(torch.bfloat16).to(cuda)  # head-major
    n_alloc = 300
    n_valid = [290, 300]
    idx = torch.zeros(B, n_alloc, dtype=torch.int64)
    for b in range(B):
        idx[b, :n_valid[b]] = torch.sort(torch.randperm(S, generator=g)[:n_valid[b]]).values
    idx = idx.to(cuda)
    d_hid = torch.full((B, n_alloc, H), 7.0, dtype=torch.bfloat16, device=cuda)
    d_k = torch.full((B, n_alloc, Hkv, 128), 7.0, dtype=torch.bfloat16, device=cuda)
    d_v = torch.full((B, Hkv, n_alloc, 128), 7.0, dtype=torch.bfloat16, device=cuda)
    specs = [ops.gather_spec_rows(hid, d_hid, 1), ops.gather_spec_rows(k_tok, d_k, 1),
             ops.gather_spec_rows(v_head, d_v, 2)]
    ops.gather_rows(specs, idx, n_valid, n_alloc, cuda)
    torch.cuda.synchronize()
    for b in range(B):
        ii = idx[b].cpu().numpy()
        for src, dst, ax in ((hid, d_hid, 0), (k_tok, d_k, 0), (v_head, d_v, 1)):
            ref = osel.gather_rows(src[b].view(torch.int16).cpu().numpy(), ii, n_valid[b], n_alloc, axis=ax)
            assert np.array_equal(dst[b].view(torch.int16).cpu().numpy(), ref)
