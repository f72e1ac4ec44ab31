"""tg_decode_attn_noalloc: decode attention for callers that cannot allocate
device memory where they call it (a host runtime binding the library over
FFI that owns the GPU's memory pool, or a path where cudaMalloc is not
allowed). It uses the library's fixed 8 MiB per-device scratch instead of a
caller workspace; this checks it through the C ABI against tg_decode_attn
(same kernel, caller workspace) on two calls in a row — the second reusing
the scratch the first left behind — with the attention tests' tolerance
(max-abs <= 1e-2, cosine >= 0.9999), and that an oversized problem is
refused. Kept in a file of its own, collected last."""
import ctypes

import pytest
import torch

from tokengate_b200 import _lib, ops
from tokengate_b200._lib import TokenGateArgumentError

pytestmark = pytest.mark.gpu


def _case(cuda, B, Hq, Hkv, n_prefix, n_keys, seed):
    g = torch.Generator().manual_seed(seed)
    cap = n_keys + 3
    q = torch.randn(B, Hq, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(B, cap, Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(B, cap, Hkv, 128, generator=g).to(torch.bfloat16).to(cuda)
    bias = (torch.randn(B, Hq, n_prefix, generator=g) * 2).to(cuda)
    qs = (0.5 + torch.rand(B, Hq, generator=g)).to(cuda)
    n_valid = torch.tensor([max(1, n_prefix - 7 * b) for b in range(B)], dtype=torch.int32, device=cuda)
    return q, k, v, bias, qs, n_valid


def _noalloc(q, k, v, bias, qs, n_valid, n_prefix, n_keys):
    B, Hq, D = q.shape
    out = torch.empty_like(q)
    st = _lib.lib().tg_decode_attn_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), qs.data_ptr(), qs.stride(0),
        k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
        bias.data_ptr(), bias.stride(0), bias.stride(1), n_valid.data_ptr(), n_prefix, n_keys,
        out.data_ptr(), out.stride(0), out.stride(1),
        B, Hq, k.shape[2], D, ctypes.c_float(D ** -0.5), torch.cuda.current_stream().cuda_stream)
    _lib.check(st)
    return out


def test_noalloc_decode_matches_workspace_entry(cuda):
    for B, Hq, Hkv, n_prefix, n_keys, seed in ((2, 16, 8, 2768, 2772, 1), (1, 32, 8, 9000, 9001, 2)):
        q, k, v, bias, qs, n_valid = _case(cuda, B, Hq, Hkv, n_prefix, n_keys, seed)
        got = _noalloc(q, k, v, bias, qs, n_valid, n_prefix, n_keys)
        ref = ops.decode_attention(q, k, v, n_valid, n_prefix, n_keys, bias=bias, q_scale=qs)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        err = (got.float() - ref.float()).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(got.float().reshape(-1), ref.float().reshape(-1), dim=0)
        assert err <= 1e-2 and cos.item() >= 0.9999, (B, n_keys, err, cos.item())


def test_noalloc_decode_rejects_oversized(cuda):
    # 64 rows x 32 heads x 80 key chunks x 528 B = 86.5 MB of partials > 8 MiB:
    # refused from the sizes alone, before any operand is read (so small
    # stand-in tensors do)
    q = torch.zeros(64, 32, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(1, 1, 8, 128, dtype=torch.bfloat16, device=cuda)
    qs = torch.ones(64, 32, device=cuda)
    bias = torch.zeros(1, 32, 1, device=cuda)
    nv = torch.full((64,), 10240, dtype=torch.int32, device=cuda)
    with pytest.raises(TokenGateArgumentError, match="8388608-byte buffer"):
        _noalloc(q, k, k, bias, qs, nv, 10240, 10240)
