"""tg_decode_attn_noalloc: decode attention for callers that cannot allocate
device memory where they call it (a host runtime binding the library over
FFI that owns the GPU's memory pool, or a path where cudaMalloc is not
allowed). It uses the library's fixed 8 MiB per-device scratch instead of a
caller workspace; this checks it through the C ABI against tg_decode_attn
(same kernel, same key chunks, caller workspace) on two calls in a row — the
second reusing the scratch the first left behind — bit for bit, and both
against a float32 restatement of the decode math with the decode tests'
tolerance (max-abs <= 1e-2, cosine >= 0.9999). Also: a cache of at most one
key chunk (no partials, the scratch unused), a second device when there is
one (its own scratch address), that an oversized problem is refused, and
that a device's first call inside a stream capture is refused cleanly.
Kept in a file of its own, collected last."""
import ctypes
import os
import subprocess
import sys
import textwrap

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


def _fp32_ref(q, k, v, n_valid, n_prefix, n_keys, bias, q_scale):
    """float32 decode math: q' = bf16(q * bf16(qs)); softmax(scale q'.k + bias, pads -inf) V."""
    qf = (q.float().cpu() * q_scale.cpu().to(torch.bfloat16).float()[..., None]).to(torch.bfloat16).float()
    B, Hq, D = qf.shape
    G = Hq // k.shape[2]
    kf = k[:, :n_keys].float().cpu().repeat_interleave(G, dim=2)
    vf = v[:, :n_keys].float().cpu().repeat_interleave(G, dim=2)
    s = torch.einsum("bhd,bnhd->bhn", qf, kf) * D ** -0.5
    m = torch.zeros(B, Hq, n_keys)
    m[:, :, :n_prefix] = bias.cpu()[..., :n_prefix]
    for b in range(B):
        m[b, :, int(n_valid[b]):n_prefix] = float("-inf")
    return torch.einsum("bhn,bnhd->bhd", torch.softmax(s + m, dim=-1), vf)


def _check(got, ref32):
    err = (got.float().cpu() - ref32).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.float().cpu().reshape(-1), ref32.reshape(-1), dim=0).item()
    assert err <= 1e-2 and cos >= 0.9999, (err, cos)


@pytest.mark.parametrize("B,Hq,Hkv,n_prefix,n_keys", [
    (2, 16, 8, 2768, 2772),    # 22 key chunks: partials in the scratch
    (1, 32, 8, 9000, 9001),
    (3, 16, 8, 100, 120),      # one chunk: no partials, the scratch unused
])
def test_noalloc_decode_matches_workspace_entry(cuda, B, Hq, Hkv, n_prefix, n_keys):
    q, k, v, bias, qs, n_valid = _case(cuda, B, Hq, Hkv, n_prefix, n_keys, n_keys)
    ref = ops.decode_attention(q, k, v, n_valid, n_prefix, n_keys, bias=bias, q_scale=qs)
    ref32 = _fp32_ref(q, k, v, n_valid.cpu(), n_prefix, n_keys, bias, qs)
    for _ in range(2):   # the second call reuses what the first left in the scratch
        got = _noalloc(q, k, v, bias, qs, n_valid, n_prefix, n_keys)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        assert torch.equal(got, ref), "no-alloc and workspace entry points differ"
        _check(got, ref32)


def test_noalloc_decode_second_device():
    """The scratch address is looked up per device: a call on cuda:1 after calls on cuda:0."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    dev = torch.device("cuda", 1)
    with torch.cuda.device(dev):
        q, k, v, bias, qs, n_valid = _case(dev, 2, 16, 8, 2768, 2772, 5)
        for _ in range(2):
            got = _noalloc(q, k, v, bias, qs, n_valid, 2768, 2772)
            ref = ops.decode_attention(q, k, v, n_valid, 2768, 2772, bias=bias, q_scale=qs)
            torch.cuda.synchronize(dev)
            assert torch.equal(got, ref)
        _check(got, _fp32_ref(q, k, v, n_valid.cpu(), 2768, 2772, bias, qs))


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


def test_noalloc_first_call_inside_capture_is_refused(cuda):
    """A device's first call resolves the scratch address, which a stream
    capture cannot record: inside a capture it must return
    TG_ERR_INVALID_ARGUMENT without touching the capture; after one call
    outside, calls inside a capture work. Run in a fresh process, so this
    device has made no call yet."""
    code = textwrap.dedent("""
        import torch
        import tests.test_zz_no_alloc as t
        from tokengate_b200._lib import TokenGateArgumentError
        dev = torch.device("cuda", 0)
        q, k, v, bias, qs, n_valid = t._case(dev, 1, 16, 8, 300, 305, 9)
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        refused = False
        with torch.cuda.graph(g, stream=s):
            try:
                t._noalloc(q, k, v, bias, qs, n_valid, 300, 305)
            except TokenGateArgumentError as e:
                refused = "before any stream capture" in str(e)
        assert refused
        ref = t._noalloc(q, k, v, bias, qs, n_valid, 300, 305)
        torch.cuda.synchronize()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=s):
            out = t._noalloc(q, k, v, bias, qs, n_valid, 300, 305)
        g2.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        print("NOALLOC_CAPTURE_OK")
    """)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "NOALLOC_CAPTURE_OK" in res.stdout, res.stdout[-2000:] + res.stderr[-2000:]
