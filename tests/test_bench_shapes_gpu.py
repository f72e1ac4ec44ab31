"""Parity at the shapes the benchmark times, through the C ABI, against the CPU oracle.

  * Phase-1 attention: B=1, S=32768, 16 query / 8 KV heads (the 32k gated
    prefill's dense layers), with no bias, a per-key bias and a per-head bias,
    against the float64 oracle on sampled rows: the first and last rows of
    the first, middle and last row blocks, row 32767, every row of the last
    row block's first 32 (the heaviest CTAs, both of their tiles: all heads
    are checked) and 32 seeded random rows;
  * Phase-2 attention: S=2768 (512 prefix + K=2000 + 256 suffix), the bench's
    per-key bias row (bf16 values, -1e9 pads on a shorter second request),
    and the finalized gate's form: a per-head bias with a per-row query scale;
  * top-K past 32768 state scores (a cluster of CTAs per request, the
    global-memory kernel past 8 x 32768): 130304 bf16-rounded scores with ties
    at the K=4000 boundary, the cluster sizes' edges, and a batch that mixes it
    with a 32000-score request and a tiny one, bit-exact against both
    selection oracles;
  * attention at the long-context shape: S=131072, 32 query / 8 KV heads;
  * the whole gated prefill of the Qwen3-1.7B-shape model at 8192 tokens,
    state [512, 7936), K=464 (the CPU-sampled workload of bench.py), against
    oracle/prefill.py: gate scores bit-exact against the oracle scorer on
    the GPU's own layer-1 hidden states, kept positions bit-exact against the
    oracle selection on those scores, kept overlap >= 0.95 with the fp32
    oracle's own selection, the same first token, and last-row logits (Phase
    2 of the oracle run on the GPU's kept rows) within cosine 0.999 and
    max-abs 0.25 of the fp32 oracle with >= 8 of its top-10 tokens. The
    max-abs bar is wider than the tiny models' 0.15: bf16 rounding noise
    grows over 28 layers (about sqrt(layers) times one layer's), and the
    maximum is taken over 151936 logits.

Attention tolerances are those of test_kernels_gpu.py: max-abs <= 2e-2,
cosine >= 0.9999, lse within 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle.prefill as opre
import oracle.select as osel
from tokengate_b200 import ops

from test_kernels_gpu import _check_attn, _check_topk

pytestmark = pytest.mark.gpu


def _rows_32k(seed: int) -> np.ndarray:
    S, BM = 32768, 128
    mid = (S // BM // 2) * BM
    fixed = [0, 1, 2, 127, mid, mid + 1, mid + 127, S - BM, S - BM + 1, S - 2, S - 1]
    fixed += list(range(S - BM, S - BM + 32))
    rnd = np.random.default_rng(seed).integers(0, S, 32)
    return np.unique(np.r_[fixed, rnd])


@pytest.fixture(scope="module")
def qkv_32k(cuda):
    g = torch.Generator().manual_seed(32768)
    S = 32768
    q = torch.randn(1, S, 16, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    return q, k, v


@pytest.mark.parametrize("bias_kind", ["none", "per_key", "per_head"])
def test_phase1_attention_32k(cuda, qkv_32k, bias_kind):
    q, k, v = qkv_32k
    S = q.shape[1]
    g = torch.Generator().manual_seed(7)
    bias = None
    if bias_kind == "per_key":
        b = torch.zeros(S)
        b[512:32512] = torch.nn.functional.logsigmoid(2 * torch.randn(32000, generator=g))
        bias = b.view(1, 1, S).to(cuda)
    elif bias_kind == "per_head":
        bias = (torch.randn(1, 16, S, generator=g) * 2).to(cuda)
    _check_attn(q, k, v, bias, causal=True, rows=_rows_32k(11))


def _phase2_bias_row(n_kept: int, n_alloc: int, g) -> torch.Tensor:
    """The Phase-2 bias row of a 512 / K / 256 request: 0 on the prefix and
    suffix, a bf16 log-sigmoid score on the kept state tokens, -1e9 pads."""
    b = torch.full((n_alloc,), -1e9)
    b[:n_kept] = 0.0
    K = n_kept - 512 - 256
    b[512:512 + K] = torch.nn.functional.logsigmoid(torch.randn(K, generator=g) * 2)
    return b.to(torch.bfloat16).float()


# B=1 is the bench's Phase-2 launch: its three heaviest row blocks (rows 2432
# and up) run one head per CTA; at B=2 every CTA takes a head pair.
@pytest.mark.parametrize("B", [1, 2])
def test_phase2_attention_2768_per_key(cuda, B):
    """The linear gate's Phase 2: (B, 1, n_alloc) bias row; request 1 is 68 rows shorter (pads)."""
    S, Hq, Hkv = 2768, 16, 8
    g = torch.Generator().manual_seed(2768)
    q = torch.randn(2, S, Hq, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    k = torch.randn(2, S, Hkv, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    v = torch.randn(2, S, Hkv, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    bias = torch.stack([_phase2_bias_row(2768, S, g), _phase2_bias_row(2700, S, g)])[:B].view(B, 1, S)
    rows = np.unique(np.r_[0:4, 127:130, 511:514, 1400:1403, 2432:2560:7, 2511:2514, 2640:2768:3, 2699, 2700,
                           2767])
    _check_attn(q, k, v, bias.to(cuda), causal=True, rows=rows)


@pytest.mark.parametrize("B", [1, 2])
def test_phase2_attention_2768_per_head_qscale(cuda, B):
    """The finalized gate's Phase 2: per-head bias (B, Hq, n_alloc) with -1e9
    pads and the scaled-softmax query scale (B, Hq, n_alloc)."""
    S, Hq, Hkv = 2768, 16, 8
    g = torch.Generator().manual_seed(2769)
    q = torch.randn(2, S, Hq, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    k = torch.randn(2, S, Hkv, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    v = torch.randn(2, S, Hkv, 128, generator=g).to(torch.bfloat16)[:B].to(cuda)
    bias = (torch.randn(2, Hq, S, generator=g) * 2).to(torch.bfloat16).float()
    bias[1, :, 2700:] = -1e9
    qrs = (0.8 + 0.6 * torch.rand(2, Hq, S, generator=g))
    bias, qrs = bias[:B].contiguous(), qrs[:B].contiguous()
    rows = np.unique(np.r_[0:3, 127:130, 1000:1003, 2000:2768:5, 2767])
    _check_attn(q, k, v, bias.to(cuda), causal=True, rows=rows, qrs=qrs.to(cuda))


# ----------------------------------------------------------------- top-K, global path
def _bf16_scores(n: int, seed: int) -> np.ndarray:
    g = torch.Generator().manual_seed(seed)
    return torch.nn.functional.logsigmoid(torch.randn(n, generator=g) * 2).to(torch.bfloat16).float().numpy()


def test_topk_global_path_130k_ties(cuda):
    """130304 state scores (a 131072-token prompt with a 512 prefix / 256
    suffix), K=4000: the K-th value's bf16 tie group straddles the boundary."""
    s = _bf16_scores(130304, 4000)
    order = np.sort(s)[::-1]
    kth = order[3999]
    ties = int((s == kth).sum())
    above = int((s > kth).sum())
    assert ties > 1 and above < 4000 < above + ties, "the K-th value must be a tie straddling K"
    _check_topk([s], [4000], [512], [131072], 512 + 4000 + 256, cuda)


@pytest.mark.parametrize("n,K", [(32769, 32768), (70000, 3000), (130304, 1), (262144, 4000), (262145, 4000)])
def test_topk_cluster_and_global_sizes(cuda, n, K):
    """Past 32768 scores one request runs on a cluster of CTAs (2, 3, 4 and the
    maximum 8 here: 32769 leaves one score to the second CTA), past 8 x 32768
    on the global-memory kernel; bf16 ties at the K-th value."""
    s = _bf16_scores(n, n + K)
    _check_topk([s], [K], [512], [n + 768], 512 + K + 256, cuda)


def test_topk_global_path_mixed_batch(cuda):
    """One launch over requests of 130304, 32000 and 5 state scores (the batch
    takes the CTA-cluster kernel: the two short requests leave three of their
    four CTAs without scores), K = 4000 / 2000 / 2 and all-tied rows."""
    a = _bf16_scores(130304, 1)
    b = _bf16_scores(32000, 2)
    c = np.full(5, -0.5, dtype=np.float32)
    _check_topk([a, b, c], [4000, 2000, 2], [512, 512, 3], [131072, 32768, 9], 4768, cuda)
    # K = n on the global path: every state token kept
    _check_topk([a[:40000]], [40000], [0], [40000], 40000, cuda)


# ----------------------------------------------------------------- whole prefill at 8192 tokens
def test_prefill_qwen3_1p7b_8192(cuda, monkeypatch):
    from tokengate_b200 import prefill as tgp
    from tokengate_b200.inference import load_model

    seq, s0, s1, K = 8192, 512, 7936, 464
    tm = load_model(base_model="qwen3-1.7b", gate_layer=1, gate_attn="b200", device=cuda, seed=0)
    g = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, tm.model.config.vocab_size, (seq,), generator=g).tolist()
    seen = {}
    orig_score, orig_topk = ops.gate_score, ops.topk_select

    def score(hidden, w, begins, counts, out=None):
        seen["hidden"] = hidden.detach().clone()
        r = orig_score(hidden, w, begins, counts, out)
        seen["scores"] = r.detach().clone()
        return r

    def topk(*a, **kw):
        r = orig_topk(*a, **kw)
        seen["keep"] = r[0].detach().clone()
        return r

    monkeypatch.setattr(ops, "gate_score", score)
    monkeypatch.setattr(ops, "topk_select", topk)
    logits = []
    hook = tm.model.lm_head.register_forward_hook(lambda m, a, o: logits.append(o.detach().float()))
    try:
        first, _cache, kept, n_kepts, K_cl = tgp.prefill_batch_for_decode(
            tm.model, tm.gate, [ids], [s0], [s1], 1, K)
    finally:
        hook.remove()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    n = n_kepts[0]
    assert n == s0 + K + (seq - s1) and K_cl == [K]
    w = tm.gate.readout.weight.detach().float().cpu().reshape(-1)
    # scores bit-exact against the oracle scorer on the GPU's own hidden states
    rows = seen["hidden"][0, s0:s1].view(torch.int16).cpu().numpy().view(np.uint16)
    ref_sc = osel.gate_score(rows, w.numpy())
    got_sc = seen["scores"][0, :s1 - s0].cpu().numpy()
    assert np.array_equal(got_sc.view(np.uint32), ref_sc.view(np.uint32))
    # kept positions bit-exact against the oracle selection on those scores
    ek, _, _, nk = osel.topk_select(ref_sc, K, s0, seq, n)
    assert nk == n
    assert np.array_equal(seen["keep"][0].cpu().numpy(), ek)
    gpu_kept = kept[0, :n].cpu().tolist()
    assert gpu_kept == ek[:n].tolist()
    # the fp32 oracle: its own selection (overlap) and Phase 2 on the GPU's kept rows (logits)
    res = opre.gated_prefill(tm.model, w, [ids], [s0], [s1], 1, K, weights=opre.weights_fp32(tm.model),
                             bias_bf16=True, kept_override=[gpu_kept])
    overlap = len(set(res["selected_positions"][0]) & set(gpu_kept)) / n
    state_overlap = (overlap * n - (n - K)) / K
    ref_logits = res["logits"][0].numpy().astype(np.float64)
    got = logits[-1][0].cpu().numpy().astype(np.float64)
    err = np.abs(got - ref_logits).max()
    cos = float(got @ ref_logits / (np.linalg.norm(got) * np.linalg.norm(ref_logits)))
    top2 = np.sort(ref_logits)[-2:]
    top10 = len(set(np.argsort(got)[-10:].tolist()) & set(np.argsort(ref_logits)[-10:].tolist()))
    diag = (f"kept overlap {overlap:.4f} (state tokens {state_overlap:.4f}), logits max-abs {err:.4f} "
            f"cosine {cos:.6f}, first token {int(first[0, 0])} vs oracle {int(res['first_tokens'][0])} "
            f"(oracle top-2 margin {top2[1] - top2[0]:.4f}), top-10 shared {top10}, "
            f"max |logit| {np.abs(ref_logits).max():.3f}")
    print(diag)
    assert overlap >= 0.95, diag
    assert err <= 0.25 and cos >= 0.999 and top10 >= 8, diag
    assert int(first[0, 0]) == int(res["first_tokens"][0]), diag


def test_attention_131k_qwen3_8b_heads(cuda):
    """The long-context scale-up's dense layers: B=1, S=131072, 32 query / 8 KV
    heads (GQA group 4), no bias and a per-key bias, against the float64
    oracle on sampled rows (first, middle and last row blocks, row 131071)."""
    S = 131072
    g = torch.Generator().manual_seed(131072)
    q = torch.randn(1, S, 32, 128, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(1, S, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    mid = S // 2
    rows = np.array([0, 1, 127, 128, mid, mid + 1, mid + 127, S - 128, S - 127, S - 2, S - 1])
    _check_attn(q, k, v, None, causal=True, rows=rows)
    b = torch.zeros(S)
    b[512:S - 256] = torch.nn.functional.logsigmoid(2 * torch.randn(S - 768, generator=g))
    _check_attn(q, k, v, b.view(1, 1, S).to(cuda), causal=True, rows=rows[[0, 4, 10]])
