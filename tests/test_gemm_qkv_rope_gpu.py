"""tg_gemm_qkv_rope: the attention input projection with the q/k RMSNorm and
RoPE in its epilogue, against the eager chain it replaces (cuBLAS bf16 GEMM
into [q | k | v], then qk_norm_rope in place) and an fp32 restatement that
rounds where the eager ops round. The kernel's projection accumulates in its
own order (a value can land one bf16 ulp from cuBLAS's) and sums the squares
in its own order; everything else rounds at the same points."""
import pytest
import torch
import torch.nn.functional as F

from tokengate_b200 import ops

pytestmark = pytest.mark.gpu


def _rotary(B, S, dev, g, theta=1e6):
    inv = 1.0 / theta ** (torch.arange(0, 128, 2, device=dev).float() / 128)
    pos = torch.randint(0, 40000, (B, S), device=dev, generator=g).float()
    f = pos[..., None] * inv
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def _ref_fp32(x, w, nq, nk, qw, kw, cos, sin, eps):
    B, S, K = x.shape
    y = (x.float().reshape(-1, K) @ w.float().t()).to(torch.bfloat16).float().view(B, S, -1, 128)
    out = y.clone()
    c, s = cos.float()[:, :, None], sin.float()[:, :, None]
    for lo, hi, wt in ((0, nq, qw), (nq, nq + nk, kw)):
        h = y[:, :, lo:hi]
        inv = torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
        h = (h * inv).to(torch.bfloat16).float()
        h = (h * wt.float()).to(torch.bfloat16).float()
        rot = torch.cat([-h[..., 64:], h[..., :64]], dim=-1)
        a = (h * c).to(torch.bfloat16).float()
        b = (rot * s).to(torch.bfloat16).float()
        out[:, :, lo:hi] = a + b
    return out.to(torch.bfloat16)


def _check(out, x, w, nq, nk, qw, kw, cos, sin, eps, min_exact=0.99):
    ref = _ref_fp32(x, w, nq, nk, qw, kw, cos, sin, eps)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
    B, S, K = x.shape
    qkv = F.linear(x, w).view(B, S, nq + 2 * nk, 128)
    ops.qk_norm_rope(qkv[:, :, :nq], qkv[:, :, nq:nq + nk], qw, kw, cos, sin, eps)
    exact = (out == qkv).float().mean().item()
    assert exact >= min_exact, f"only {exact:.4f} of the outputs equal the eager chain"


@pytest.mark.parametrize("B,S,K,nq,nk", [(1, 1, 64, 2, 1), (1, 300, 256, 2, 1), (2, 257, 512, 4, 2),
                                         (1, 129, 128, 3, 1), (1, 2768, 2048, 16, 8)])
def test_gemm_qkv_rope_shapes(cuda, B, S, K, nq, nk):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + S + K + nq)
    nh = nq + 2 * nk
    x = torch.randn(B, S, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(nh * 128, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = _rotary(B, S, "cuda", g)
    out = ops.gemm_qkv_rope(x, w, nq, nk, qw, kw, cos, sin, 1e-6)
    assert out.shape == (B, S, nh, 128)
    _check(out, x, w, nq, nk, qw, kw, cos, sin, 1e-6)


def test_gemm_qkv_rope_strided_rotary(cuda):
    """cos / sin as views of wider tables (row stride 256), x rows of stride K + 64."""
    g = torch.Generator(device="cuda").manual_seed(3)
    B, S, K, nq, nk = 2, 200, 256, 4, 2
    nh = nq + 2 * nk
    xb = torch.randn(B, S, K + 64, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(nh * 128, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    qw = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    c, s = _rotary(B, S, "cuda", g)
    cw = torch.zeros(B, S, 256, device="cuda", dtype=torch.bfloat16)
    sw = torch.zeros(B, S, 256, device="cuda", dtype=torch.bfloat16)
    cw[..., :128] = c
    sw[..., :128] = s
    x2 = xb.reshape(B * S, K + 64)[:, :K]
    out = ops.gemm_qkv_rope(x2.unsqueeze(0), w, nq, nk, qw, kw,
                            cw.reshape(1, B * S, 256)[..., :128], sw.reshape(1, B * S, 256)[..., :128], 1e-6)
    _check(out, x2.unsqueeze(0), w, nq, nk, qw, kw, cw.reshape(1, B * S, 256)[..., :128],
           sw.reshape(1, B * S, 256)[..., :128], 1e-6)


def test_gemm_qkv_rope_bench_shape_sampled(cuda):
    """Phase 1 of the benchmarked model: 32768 rows, hidden 2048, 16/8 heads;
    rows sampled from the first, middle and last row tiles."""
    g = torch.Generator(device="cuda").manual_seed(9)
    B, S, K, nq, nk = 1, 32768, 2048, 16, 8
    nh = nq + 2 * nk
    x = torch.randn(B, S, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(nh * 128, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = _rotary(B, S, "cuda", g)
    out = ops.gemm_qkv_rope(x, w, nq, nk, qw, kw, cos, sin, 1e-6)
    rows = torch.cat([torch.arange(0, 300), torch.arange(16256, 16520), torch.arange(S - 300, S)]).cuda()
    _check(out[:, rows], x[:, rows], w, nq, nk, qw, kw, cos[:, rows], sin[:, rows], 1e-6)
    assert ops.device_error() == 0


def test_gemm_qkv_rope_rejects(cuda):
    x = torch.zeros(1, 4, 100, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(512, 100, device="cuda", dtype=torch.bfloat16)
    one = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    cs = torch.zeros(1, 4, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Exception):
        ops.gemm_qkv_rope(x, w, 2, 1, one, one, cs, cs, 1e-6)   # K not a multiple of 64
