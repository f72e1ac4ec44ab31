"""tg_gemm_swiglu_readout: the finalized gate's scoring branch as one GEMM with
the SwiGLU and the one-row readout in its epilogue.

Checked against (1) an fp32 restatement that rounds where the branch rounds
(bf16 projections, bf16 silu, bf16 product, bf16 score) and (2) the unfused
chain the prefill runs otherwise: cuBLAS's bf16 GEMM into [G | U] followed by
branch_score (itself bit-exact against the oracle). The fused kernel's fp32
orders are its own (the projection's accumulation, the dot's summation), so a
score can move by about one bf16 ulp of the score or of its largest term; most
scores must be equal. Bound written in _close.
"""
import pytest
import torch
import torch.nn.functional as F

from tokengate_b200 import ops
from tokengate_b200._lib import TokenGateArgumentError, TokenGateUnsupportedError

pytestmark = pytest.mark.gpu


def _terms(x, w_gu, w_r):
    inter = w_r.shape[0]
    g = (x.float() @ w_gu[:inter].float().t()).to(torch.bfloat16).float()
    u = (x.float() @ w_gu[inter:].float().t()).to(torch.bfloat16).float()
    s = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16).float()
    a = (s * u).to(torch.bfloat16).float()
    return a * w_r.float()


def _close(got, ref, terms, min_exact):
    """|got - ref| <= 2^-7 |ref| + 2^-7 max_k |a_k w_k| per row; >= min_exact of the rows equal."""
    got, ref = got.float(), ref.float()
    bound = 2.0 ** -7 * ref.abs() + 2.0 ** -7 * terms.abs().amax(dim=1)
    err = (got - ref).abs()
    assert bool((err <= bound).all()), f"max excess {(err - bound).max().item()}"
    exact = (got == ref).float().mean().item()
    assert exact >= min_exact, f"only {exact:.4f} of the scores equal"


def _case(M, K, inter, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    wr = (torch.randn(inter, device="cuda", generator=g) * inter ** -0.5).to(torch.bfloat16)
    return x, w, wr


@pytest.mark.parametrize("M,K,inter", [(1, 64, 128), (255, 128, 256), (257, 256, 384), (1000, 512, 1024),
                                       (2768, 2048, 6144)])
def test_readout_shapes(cuda, M, K, inter):
    x, w, wr = _case(M, K, inter, M * 7 + K + inter)
    got = ops.gemm_swiglu_readout(x, w, wr)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    terms = _terms(x, w, wr)
    ref = terms.sum(dim=1).to(torch.bfloat16).float()
    _close(got, ref, terms, 0.6)
    # the unfused chain: cuBLAS [G | U], then the bit-exact branch_score readout
    # (which serves inter a multiple of 256)
    if inter % 256 == 0:
        chain = ops.branch_score(F.linear(x, w).unsqueeze(0), wr, [0], [M])[0, :M]
        _close(got, chain, terms, 0.6)
    assert not bool((got.view(torch.int32) == torch.iinfo(torch.int32).min).any())   # no -0


def test_readout_bench_shape(cuda):
    """The finalized gate at the 32k prefill: 32000 state rows, hidden 2048, inter 6144."""
    M, K, inter = 32000, 2048, 6144
    x, w, wr = _case(M, K, inter, 32000)
    got = ops.gemm_swiglu_readout(x, w, wr)
    chain = ops.branch_score(F.linear(x, w).unsqueeze(0), wr, [0], [M])[0, :M]
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    rows = torch.arange(0, M, 97, device="cuda")
    terms = _terms(x[rows], w, wr)
    _close(got[rows], chain[rows], terms, 0.6)
    # every row: within a bf16 ulp or two of the chain
    rel = ((got - chain).abs() / chain.abs().clamp_min(1e-3)).max().item()
    assert rel < 0.05, rel


def test_readout_strided_rows_and_determinism(cuda):
    """State rows of one request inside a (S, H) boundary tensor: row stride H, offset start."""
    K, inter = 256, 512
    _, w, wr = _case(1, K, inter, 5)
    xs = (torch.randn(600, 2 * K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
          * 0.5).to(torch.bfloat16)
    x = xs[37:37 + 500, K // 2:K // 2 + K]   # row stride 2K, offset 256 bytes
    a = ops.gemm_swiglu_readout(x, w, wr)
    b = ops.gemm_swiglu_readout(x.contiguous(), w, wr)
    out = torch.full((520,), 7.0, device="cuda")
    ops.gemm_swiglu_readout(x, w, wr, out=out)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, out[:500])
    assert bool((out[500:] == 7.0).all())


def test_readout_empty_and_rejects(cuda):
    x, w, wr = _case(4, 128, 256, 9)
    assert ops.gemm_swiglu_readout(x[:0], w, wr).numel() == 0
    with pytest.raises(TokenGateUnsupportedError):
        ops.gemm_swiglu_readout(x[:, :96].contiguous(), w[:, :96].contiguous(), wr)     # K % 64
    x2, w2, wr2 = _case(4, 128, 192, 9)
    with pytest.raises(TokenGateUnsupportedError):
        ops.gemm_swiglu_readout(x2, w2, wr2)                                             # inter % 128
    buf = torch.zeros(257, dtype=torch.bfloat16, device="cuda")
    buf[1:].copy_(wr)
    with pytest.raises(TokenGateArgumentError):
        ops.gemm_swiglu_readout(x, w, buf[1:])                                           # misaligned readout row
    with pytest.raises(ValueError):
        ops.gemm_swiglu_readout(x, w[:, :64], wr)                                        # shape
