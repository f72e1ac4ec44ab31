"""tg_gemm_swiglu: the Qwen3 MLP up-projection with the SwiGLU epilogue.

Checked against (1) an fp32 restatement that rounds where the eager chain
rounds (bf16 projections, bf16 silu, bf16 product) and (2) the eager chain
itself, cuBLAS bf16 GEMM into [G | U] followed by silu_mul: the kernel's
fp32 accumulation order is its own, so a projection can land one bf16 ulp
from cuBLAS's; everything else must agree bit for bit.
"""
import pytest
import torch
import torch.nn.functional as F

from tokengate_b200 import ops

pytestmark = pytest.mark.gpu


def _ref_fp32(x, w_gu, inter):
    g = (x.float() @ w_gu[:inter].float().t()).to(torch.bfloat16).float()
    u = (x.float() @ w_gu[inter:].float().t()).to(torch.bfloat16).float()
    a = (g / (1.0 + torch.exp(-g))).to(torch.bfloat16).float()
    return (a * u).to(torch.bfloat16)


def _check(out, x, w_gu, inter, min_exact=0.99):
    ref = _ref_fp32(x, w_gu, inter)
    # one bf16 ulp of a projection moves the product by about one ulp
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
    eager = ops.silu_mul(F.linear(x, w_gu))
    exact = (out == eager).float().mean().item()
    assert exact >= min_exact, f"only {exact:.4f} of the outputs equal the eager chain"


@pytest.mark.parametrize("M,K,inter", [(1, 64, 128), (255, 128, 256), (257, 256, 384), (1000, 512, 1024),
                                       (2768, 2048, 6144)])
def test_gemm_swiglu_shapes(cuda, M, K, inter):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + K + inter)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    out = ops.gemm_swiglu(x, w, inter)
    assert out.shape == (M, inter)
    _check(out, x, w, inter)


def test_gemm_swiglu_strided_rows_and_batch_dims(cuda):
    g = torch.Generator(device="cuda").manual_seed(5)
    K, inter = 256, 256
    big = (torch.randn(600, K + 64, device="cuda", generator=g)).to(torch.bfloat16)
    x = big[:, :K]                      # row stride K + 64
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    _check(ops.gemm_swiglu(x, w, inter), x, w, inter)
    x3 = (torch.randn(2, 300, K, device="cuda", generator=g)).to(torch.bfloat16)
    out3 = ops.gemm_swiglu(x3, w, inter)
    assert out3.shape == (2, 300, inter)
    _check(out3.view(-1, inter), x3.view(-1, K), w, inter)


def test_gemm_swiglu_bench_shape_sampled(cuda):
    """The Phase-1 shape of the benchmarked model: 32768 rows, hidden 2048,
    intermediate 6144 (all tiles of the persistent grid, many per cluster);
    rows sampled from the first, middle and last row tiles."""
    g = torch.Generator(device="cuda").manual_seed(11)
    M, K, inter = 32768, 2048, 6144
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    out = ops.gemm_swiglu(x, w, inter)
    rows = torch.cat([torch.arange(0, 300), torch.arange(16256, 16520), torch.arange(M - 300, M)]).cuda()
    _check(out[rows], x[rows], w, inter)
    assert ops.device_error() == 0


def test_gemm_swiglu_rejects(cuda):
    x = torch.zeros(4, 100, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(256, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Exception):
        ops.gemm_swiglu(x, w, 128)          # K not a multiple of 64
    x = torch.zeros(4, 128, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(200, 128, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(Exception):
        ops.gemm_swiglu(x, w, 100)          # inter not a multiple of 128
    assert ops.gemm_swiglu(torch.zeros(0, 128, device="cuda", dtype=torch.bfloat16),
                           torch.zeros(256, 128, device="cuda", dtype=torch.bfloat16), 128).shape == (0, 128)
