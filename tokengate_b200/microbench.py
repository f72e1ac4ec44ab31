"""Single-kernel runs of the four hot-path kernels at the benchmarked shapes (timing and ncu captures).

    python -m tokengate_b200.microbench attn   [--seq 32768] [--batch 1] [--hq 16] [--hkv 8] [--iters 20]
    python -m tokengate_b200.microbench score  [--seq 32768] [--batch 1] [--iters 20]
    python -m tokengate_b200.microbench topk   [--k 2000] [--batch 1] [--iters 20]
    python -m tokengate_b200.microbench gather [--k 2000] [--batch 1] [--iters 20]
    python -m tokengate_b200.microbench branch [--seq 32768] [--inter 6144] [--batch 1]
    python -m tokengate_b200.microbench readout [--seq 32768] [--hidden 2048] [--inter 6144]
    python -m tokengate_b200.microbench tables [--k 2000] [--layers 26] [--hq 16] [--batch 1]
    python -m tokengate_b200.microbench decode [--seq 2768] [--batch 1] [--hq 16] [--hkv 8] [--no-bias]
    python -m tokengate_b200.microbench gemv [--n 12288] [--hidden 2048] [--batch 1]
    python -m tokengate_b200.microbench gemvchain [--layers 26] [--hidden 2048] [--inter 6144] [--batch 1]
    python -m tokengate_b200.microbench generate [--seq 32768] [--k 2000] [--batch 1] [--new 64] [--gate linear|e2e] [--proj gemv|cublas]

Prints one JSON line per run with the CUDA-event time per launch and the
algorithmic FLOPs or bytes of one launch (attention: 4*B*Hq*D*S(S+1)/2, also
timed as 10 launches in one CUDA graph, `ms_graph`;
score: the bf16 state rows + w + fp32 scores; topk: scores read + keep/bias
written; gather: hidden rows + 4 below-gate K/V tensors read and written;
branch: the bf16 [gate | up] state rows + w + fp32 scores; tables: the raw
scores and kept positions read once + both fp32 (L', B, H, n_alloc) tables
written; decode: the K and V rows of the n_keys cached tokens + q, bias
row and output, timed as 20 launches in one CUDA graph so the host launch
path is not what is measured). generate: the gated generation of the
Qwen3-1.7B-shape model (random init) — prefill seconds
and decode milliseconds per token.
"""
import argparse
import json

import torch

from . import ops


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _graph_time(fn, n, reps, warmup=3):
    """ms per call of fn, with n calls captured in one CUDA graph and replayed reps times."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(n):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (reps * n)


class _L2Flush:
    """A 256 MB buffer (twice the L2) READ before each timed launch: the
    kernel then finds none of its inputs in L2 and no dirty lines to write
    back (a memset flush leaves ~126 MB of dirty lines that the timed kernel
    would pay to evict)."""

    def __init__(self, dev):
        self.buf = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        torch.sum(self.buf, dim=0, out=self.sink)


def _time_flushed(fn, flush, iters=10, warmup=3):
    """Median CUDA-event ms of one fn() launch, L2 flushed before each. A
    ~1 ms device spin after the flush keeps the GPU busy while the host
    issues the start event and the launch (the Python op path takes tens of
    microseconds), so the events bracket the kernel's own time and not the
    host's launch path."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush()
        torch.cuda._sleep(2_000_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    return ts[len(ts) // 2]


def ops_table(dev, tflops_peak: float, hbm_peak_gbs: float, iters: int = 10) -> dict:
    """Single-kernel figures of the hot-path kernels at the benchmarked shapes,
    timed with CUDA events (median of `iters` launches, L2 flushed before each).

    attention: B=1, 16/8 heads, causal, S = 4096 (per-key bias: log-sigmoid of
    N(0,2) logits on [256, 3840), 0 elsewhere), 2768 (a Phase-2 bias row:
    0 on a 512 prefix / 256 suffix, bf16 scores between), 8192 and 32768
    (Phase 1: no bias); TFLOP/s of 4*Hq*D*S(S+1)/2 and the fraction of
    `tflops_peak`. gate score / top-K / gather at 32768 tokens, state
    [512, 32512), K=2000, for 1 and 8 requests: GB/s of the algorithmic bytes
    (score: the bf16 state rows + w + fp32 scores; top-K: scores read +
    kept positions and bias row written; gather: the hidden rows and the K/V
    rows of two below-gate layers, read and written) and the fraction of
    `hbm_peak_gbs`. branch_score: the finalized gate's readout over the same
    state rows' bf16 [gate | up] projections (inter 6144), GB/s of those rows
    + the readout row + fp32 scores (the SiLU table build included in the
    time). branch_fused: the whole branch of one request's 32000 state rows
    as one GEMM with the SwiGLU and readout epilogue, TFLOP/s of
    2*M*2048*12288, beside cuBLAS's [gate | up] GEMM + branch_score. gemm_swiglu: the MLP up-projection with the SwiGLU
    epilogue at hidden 2048, intermediate 6144 and M = 2768 (Phase 2) and
    32768 (Phase 1) rows: TFLOP/s of 2*M*2048*12288, beside cuBLAS's bf16
    GEMM into [gate | up] alone and with the silu_mul kernel after it (the
    chain it replaces). gemm_qkv_rope: the attention input projection with
    the q/k RMSNorm + RoPE epilogue at hidden 2048, 16/8 heads, the same row
    counts, beside cuBLAS's GEMM into [q | k | v] with qk_norm_rope after it."""
    g = torch.Generator(device=dev).manual_seed(0)
    flush = _L2Flush(dev)
    out = {"timing": f"CUDA events, median of {iters} launches, L2 flushed (a 256 MB read) before each",
           "attention": [], "gate_score": [], "topk": [], "gather": [], "branch_score": [], "branch_fused": [],
           "gemm_swiglu": [], "gemm_qkv_rope": []}
    for S, kind in ((4096, "per-key bias"), (2768, "Phase-2 bias row"), (8192, "no bias"), (32768, "no bias")):
        q = torch.randn(1, S, 16, 128, device=dev, dtype=torch.bfloat16, generator=g)
        k = torch.randn(1, S, 8, 128, device=dev, dtype=torch.bfloat16, generator=g)
        v = torch.randn(1, S, 8, 128, device=dev, dtype=torch.bfloat16, generator=g)
        bias = None
        if S == 4096:
            bias = torch.zeros(1, 1, S, device=dev)
            bias[..., 256:3840] = torch.nn.functional.logsigmoid(
                2 * torch.randn(3584, device=dev, generator=g))
        elif S == 2768:
            bias = torch.zeros(1, 1, S, device=dev)
            bias[..., 512:2512] = torch.nn.functional.logsigmoid(
                2 * torch.randn(2000, device=dev, generator=g)).to(torch.bfloat16).float()
        o = torch.empty_like(q)
        ms = _time_flushed(lambda: ops.keybias_attention(q, k, v, bias=bias, out=o), flush, iters)
        flops = 4.0 * 16 * 128 * S * (S + 1) / 2
        tf = flops / ms / 1e9
        out["attention"].append(dict(seq=S, heads="16/8", bias=kind, us=ms * 1e3, tflops=tf,
                                     frac=tf / tflops_peak))
        del q, k, v, o
    S, st0, st1, K, H = 32768, 512, 32512, 2000, 2048
    n_art, n_kept = st1 - st0, st0 + K + (S - st1)
    for B in (1, 8):
        h = torch.randn(B, S, H, device=dev, dtype=torch.bfloat16, generator=g)
        w = torch.randn(H, device=dev, generator=g) / H ** 0.5
        sc = ops.gate_score(h, w, [st0] * B, [n_art] * B)
        ms = _time_flushed(lambda: ops.gate_score(h, w, [st0] * B, [n_art] * B, out=sc), flush, iters)
        byts = B * (n_art * H * 2 + n_art * 4) + H * 4
        out["gate_score"].append(dict(requests=B, us=ms * 1e3, gbs=byts / ms / 1e6,
                                      frac=byts / ms / 1e6 / hbm_peak_gbs))
        keep = torch.empty(B, n_kept, dtype=torch.int64, device=dev)
        brow = torch.empty(B, n_kept, dtype=torch.bfloat16, device=dev)
        ms = _time_flushed(lambda: ops.topk_select(sc, [n_art] * B, [K] * B, [st0] * B, [S] * B, n_kept,
                                                   keep_out=keep, bias_out=brow), flush, iters)
        byts = B * (n_art * 4 + n_kept * 10)
        out["topk"].append(dict(requests=B, k=K, us=ms * 1e3, gbs=byts / ms / 1e6,
                                frac=byts / ms / 1e6 / hbm_peak_gbs))
        kv = [torch.randn(B, S, 8, 128, device=dev, dtype=torch.bfloat16, generator=g) for _ in range(4)]
        dh = torch.empty(B, n_kept, H, device=dev, dtype=torch.bfloat16)
        dkv = [torch.empty(B, n_kept, 8, 128, device=dev, dtype=torch.bfloat16) for _ in range(4)]
        specs = [ops.gather_spec_rows(h, dh, 1)] + [ops.gather_spec_rows(a, d, 1) for a, d in zip(kv, dkv)]
        ms = _time_flushed(lambda: ops.gather_rows(specs, keep, [n_kept] * B, n_kept, dev), flush, iters)
        byts = B * 2 * n_kept * (H * 2 + 4 * 8 * 128 * 2) + B * n_kept * 8
        out["gather"].append(dict(requests=B, k=K, us=ms * 1e3, gbs=byts / ms / 1e6,
                                  frac=byts / ms / 1e6 / hbm_peak_gbs))
        del h, kv, dh, dkv
        gu = torch.randn(B, n_art, 2 * 6144, device=dev, dtype=torch.bfloat16, generator=g)
        wr = (torch.randn(6144, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        bs = ops.branch_score(gu, wr, [0] * B, [n_art] * B)
        ms = _time_flushed(lambda: ops.branch_score(gu, wr, [0] * B, [n_art] * B, out=bs), flush, iters)
        byts = B * n_art * (4 * 6144 + 4) + 2 * 6144
        out["branch_score"].append(dict(requests=B, inter=6144, us=ms * 1e3, gbs=byts / ms / 1e6,
                                        frac=byts / ms / 1e6 / hbm_peak_gbs))
        del gu, bs
    K, inter = 2048, 6144
    w = (torch.randn(2 * inter, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
    x = (torch.randn(n_art, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    wr = (torch.randn(inter, device=dev, generator=g) * inter ** -0.5).to(torch.bfloat16)
    sc = torch.empty(n_art, device=dev)
    ms = _time_flushed(lambda: ops.gemm_swiglu_readout(x, w, wr, out=sc), flush, iters)
    gu = torch.nn.functional.linear(x, w)
    ms_lin = _time_flushed(lambda: torch.nn.functional.linear(x, w), flush, iters)
    ms_rd = _time_flushed(lambda: ops.branch_score(gu.unsqueeze(0), wr, [0], [n_art]), flush, iters)
    flops = 2.0 * n_art * K * 2 * inter
    out["branch_fused"].append(dict(rows=n_art, K=K, inter=inter, us=ms * 1e3, tflops=flops / ms / 1e9,
                                    frac=flops / ms / 1e9 / tflops_peak, cublas_gemm_us=ms_lin * 1e3,
                                    cublas_plus_branch_score_us=(ms_lin + ms_rd) * 1e3))
    del x, gu
    for M in (2768, 32768):
        x = (torch.randn(M, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        flops = 2.0 * M * K * 2 * inter
        ms = _time_flushed(lambda: ops.gemm_swiglu(x, w, inter), flush, iters)
        ms_lin = _time_flushed(lambda: torch.nn.functional.linear(x, w), flush, iters)
        gu = torch.nn.functional.linear(x, w)
        ms_silu = _time_flushed(lambda: ops.silu_mul(gu), flush, iters)
        tf, tf_lin = flops / ms / 1e9, flops / ms_lin / 1e9
        out["gemm_swiglu"].append(dict(rows=M, K=K, inter=inter, us=ms * 1e3, tflops=tf, frac=tf / tflops_peak,
                                       cublas_gemm_us=ms_lin * 1e3, cublas_gemm_tflops=tf_lin,
                                       vs_cublas_gemm=tf / tf_lin, cublas_plus_silu_mul_us=(ms_lin + ms_silu) * 1e3))
        del x, gu
    nq, nk = 16, 8
    nh = nq + 2 * nk
    w = (torch.randn(nh * 128, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
    for M in (2768, 32768):
        x = torch.randn(1, M, K, device=dev, dtype=torch.bfloat16, generator=g)
        ang = torch.rand(1, M, 128, device=dev, generator=g) * 6
        cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
        flops = 2.0 * M * K * nh * 128
        ms = _time_flushed(lambda: ops.gemm_qkv_rope(x, w, nq, nk, qw, kw, cos, sin, 1e-6), flush, iters)
        ms_lin = _time_flushed(lambda: torch.nn.functional.linear(x, w), flush, iters)
        qkv = torch.nn.functional.linear(x, w).view(1, M, nh, 128)
        ms_rope = _time_flushed(lambda: ops.qk_norm_rope(qkv[:, :, :nq], qkv[:, :, nq:nq + nk], qw, kw, cos, sin,
                                                          1e-6), flush, iters)
        tf = flops / ms / 1e9
        out["gemm_qkv_rope"].append(dict(rows=M, K=K, heads="16/8", us=ms * 1e3, tflops=tf, frac=tf / tflops_peak,
                                         cublas_gemm_us=ms_lin * 1e3, cublas_plus_qk_norm_rope_us=(ms_lin + ms_rope) * 1e3))
        del x, qkv
    assert ops.device_error() == 0
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=("attn", "score", "topk", "gather", "branch", "tables", "decode",
                                       "generate", "gemv", "gemvchain", "gemm", "qkv", "readout"))
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--new", type=int, default=64)
    ap.add_argument("--gate", default="linear", choices=("linear", "e2e"))
    ap.add_argument("--proj", default="gemv", choices=("gemv", "cublas"))
    ap.add_argument("--inter", type=int, default=6144)
    ap.add_argument("--layers", type=int, default=26)
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--k", type=int, default=2000)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-bias", action="store_true")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    B, S = a.batch, a.seq
    res = dict(kernel=a.kernel, batch=B)
    if a.kernel == "decode":
        cap = S + 8
        q = torch.randn(B, a.hq, 128, device=dev, dtype=torch.bfloat16, generator=g)
        k = torch.randn(B, cap, a.hkv, 128, device=dev, dtype=torch.bfloat16, generator=g)
        v = torch.randn(B, cap, a.hkv, 128, device=dev, dtype=torch.bfloat16, generator=g)
        bias = None if a.no_bias else torch.randn(B, a.hq, S, device=dev, generator=g)
        qs = None if a.no_bias else torch.rand(B, a.hq, device=dev, generator=g) + 0.5
        nv = torch.full((B,), S, dtype=torch.int32, device=dev)
        out = torch.empty(B, a.hq, 128, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.decode_attention(q, k, v, nv, S, S + 1, bias=bias, q_scale=qs, out=out)
        ms = _graph_time(fn, 20, a.iters)
        byts = B * ((S + 1) * a.hkv * 128 * 2 * 2 + a.hq * 128 * 4 + (0 if a.no_bias else a.hq * S * 4))
        res.update(seq=S, hq=a.hq, hkv=a.hkv, bias=not a.no_bias, ms=ms, us=ms * 1e3, mbytes=byts / 1e6,
                   gbs=byts / ms / 1e6)
    elif a.kernel == "gemm":
        # the MLP up-projection with the SwiGLU epilogue: --seq rows, --hidden K,
        # --inter intermediate columns; cuBLAS's GEMM into [gate | up] beside it
        M, K, I = S, a.hidden, a.inter
        x = (torch.randn(M, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        w = (torch.randn(2 * I, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
        ms = _graph_time(lambda: ops.gemm_swiglu(x, w, I), 3, a.iters)
        ms_ref = _graph_time(lambda: torch.nn.functional.linear(x, w), 3, a.iters)
        flops = 2.0 * M * K * 2 * I
        res.update(rows=M, k=K, inter=I, ms=ms, us=ms * 1e3, tflops=flops / ms / 1e9,
                   cublas_us=ms_ref * 1e3, cublas_tflops=flops / ms_ref / 1e9)
    elif a.kernel == "readout":
        # the finalized gate's branch as one GEMM (SwiGLU + readout epilogue):
        # --seq - 768 state rows, --hidden K, --inter; cuBLAS's GEMM + branch_score beside it
        M, K, I = S - 768, a.hidden, a.inter
        x = (torch.randn(M, K, device=dev, generator=g) * 0.5).to(torch.bfloat16)
        w = (torch.randn(2 * I, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
        wr = (torch.randn(I, device=dev, generator=g) * I ** -0.5).to(torch.bfloat16)
        sc = torch.empty(M, device=dev)
        ms = _graph_time(lambda: ops.gemm_swiglu_readout(x, w, wr, out=sc), 3, a.iters)
        gu = torch.nn.functional.linear(x, w).unsqueeze(0)
        ms_ref = _graph_time(lambda: torch.nn.functional.linear(x, w), 3, a.iters)
        ms_rd = _graph_time(lambda: ops.branch_score(gu, wr, [0], [M]), 3, a.iters)
        flops = 2.0 * M * K * 2 * I
        res.update(rows=M, k=K, inter=I, ms=ms, us=ms * 1e3, tflops=flops / ms / 1e9,
                   cublas_plus_branch_score_us=(ms_ref + ms_rd) * 1e3)
    elif a.kernel == "qkv":
        # the attention input projection with the q/k RMSNorm + RoPE epilogue:
        # --seq rows, --hidden K, --hq / --hkv heads; cuBLAS + qk_norm_rope beside it
        M, K, nq, nk = S, a.hidden, a.hq, a.hkv
        nh = nq + 2 * nk
        x = torch.randn(1, M, K, device=dev, dtype=torch.bfloat16, generator=g)
        w = (torch.randn(nh * 128, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
        qw = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
        ang = torch.rand(1, M, 128, device=dev, generator=g) * 6
        cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
        ms = _graph_time(lambda: ops.gemm_qkv_rope(x, w, nq, nk, qw, qw, cos, sin, 1e-6), 3, a.iters)
        qkv = torch.nn.functional.linear(x, w).view(1, M, nh, 128)

        def eager():
            torch.nn.functional.linear(x, w, out=qkv.view(1, M, nh * 128))
            ops.qk_norm_rope(qkv[:, :, :nq], qkv[:, :, nq:nq + nk], qw, qw, cos, sin, 1e-6)
        ms_ref = _graph_time(eager, 3, a.iters)
        flops = 2.0 * M * K * nh * 128
        res.update(rows=M, k=K, heads=f"{nq}/{nk}", ms=ms, us=ms * 1e3, tflops=flops / ms / 1e9,
                   cublas_plus_qk_norm_rope_us=ms_ref * 1e3)
    elif a.kernel == "gemv":
        x = torch.randn(B, a.hidden, device=dev, dtype=torch.bfloat16, generator=g)
        w = (torch.randn(a.n, a.hidden, device=dev, generator=g) / a.hidden ** 0.5).to(torch.bfloat16)
        out = torch.empty(B, a.n, device=dev, dtype=torch.bfloat16)
        ms = _graph_time(lambda: ops.gemv(x, w, out=out), 20, a.iters)
        ms_ref = _graph_time(lambda: torch.nn.functional.linear(x, w), 20, a.iters)
        byts = a.n * a.hidden * 2 + B * (a.hidden + a.n) * 2
        res.update(n=a.n, k=a.hidden, ms=ms, us=ms * 1e3, mbytes=byts / 1e6, gbs=byts / ms / 1e6,
                   cublas_us=ms_ref * 1e3, cublas_gbs=byts / ms_ref / 1e6)
    elif a.kernel == "gemvchain":
        # the decode step's layer projections alone: per layer q/k/v, o,
        # gate/up (+SwiGLU) and down GEMVs chained through their outputs, over
        # --layers + 2 layers of distinct weights (not L2-resident), one
        # CUDA graph; then the four kernels on one layer's (L2-resident)
        # weights, the per-layer latency floor of the chain
        H, I, NQ, NL = a.hidden, a.inter, 2 * a.hidden, a.layers + 2
        mk = lambda n, k: (torch.randn(n, k, device=dev, generator=g) / k ** 0.5).to(torch.bfloat16)
        W = [(mk(NQ, H), mk(H, H), mk(2 * I, H), mk(H, I)) for _ in range(NL)]
        x = torch.randn(B, H, device=dev, dtype=torch.bfloat16, generator=g)
        yq = torch.empty(B, NQ, device=dev, dtype=torch.bfloat16)
        yo = torch.empty(B, H, device=dev, dtype=torch.bfloat16)
        act = torch.empty(B, I, device=dev, dtype=torch.bfloat16)

        def layer(w):
            ops.gemv(x, w[0], out=yq)
            ops.gemv(yq[:, :H], w[1], out=yo)
            ops.gemv(yo, w[2], swiglu=True, out=act)
            ops.gemv(act, w[3], out=x)

        def chain():
            for w in W:
                layer(w)
        ms = _graph_time(chain, 1, a.iters)
        ms_l2 = _graph_time(lambda: layer(W[0]), NL, a.iters)
        byts = NL * sum(t.numel() for t in W[0]) * 2
        res.update(layers=NL, hidden=H, inter=I, ms=ms, us_per_layer=ms * 1e3 / NL, mbytes=byts / 1e6,
                   gbs=byts / ms / 1e6, l2_resident_us_per_layer=ms_l2 * 1e3)
    elif a.kernel == "generate":
        from .decode import generate_batch
        from .inference import load_model
        tm = load_model(base_model="qwen3-1.7b", gate_layer=1, gate_attn="b200", device=dev, seed=0,
                        gate="e2e" if a.gate == "e2e" else None)
        vocab = tm.model.config.vocab_size
        gh = torch.Generator().manual_seed(1000)
        prompts = [torch.randint(0, vocab, (S,), generator=gh) for _ in range(B)]
        st0, st1 = 512, S - 256
        run = lambda n: generate_batch(tm.model, tm.gate, prompts, [st0] * B, [st1] * B, 1, a.k, n,
                                       use_gemv=a.proj == "gemv")
        run(4)
        run(a.new)
        r = run(a.new)
        res.update(seq=S, k=a.k, gate=a.gate, proj=a.proj, new=a.new, prefill_ms=r.prefill_s * 1e3,
                   decode_ms_per_token=r.decode_s * 1e3 / max(r.steps, 1),
                   decode_tokens_per_s=B * r.steps / r.decode_s if r.steps else None)
    elif a.kernel == "attn":
        q = torch.randn(B, S, a.hq, 128, device=dev, dtype=torch.bfloat16, generator=g)
        k = torch.randn(B, S, a.hkv, 128, device=dev, dtype=torch.bfloat16, generator=g)
        v = torch.randn(B, S, a.hkv, 128, device=dev, dtype=torch.bfloat16, generator=g)
        bias = None if a.no_bias else torch.randn(B, 1, S, device=dev, generator=g)
        o = torch.empty_like(q)
        ms = _time(lambda: ops.keybias_attention(q, k, v, bias=bias, out=o), a.iters)
        # 10 launches in one CUDA graph, as the Phase-2 layers replay them: the
        # host's launch path is not timed and consecutive launches overlap
        # their prologues (programmatic stream serialization)
        ms_graph = _graph_time(lambda: ops.keybias_attention(q, k, v, bias=bias, out=o), 10, a.iters)
        flops = 4.0 * B * a.hq * 128 * S * (S + 1) / 2
        res.update(seq=S, hq=a.hq, hkv=a.hkv, bias=not a.no_bias, ms=ms, tflop=flops / 1e12,
                   tflops=flops / ms / 1e9, ms_graph=ms_graph, tflops_graph=flops / ms_graph / 1e9)
    elif a.kernel == "branch":
        n_art = S - 768
        gu = torch.randn(B, n_art, 2 * a.inter, device=dev, dtype=torch.bfloat16, generator=g)
        w = (torch.randn(a.inter, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        sc = ops.branch_score(gu, w, [0] * B, [n_art] * B)
        ms = _time(lambda: ops.branch_score(gu, w, [0] * B, [n_art] * B, out=sc), a.iters)
        byts = B * n_art * (4 * a.inter + 4) + 2 * a.inter
        res.update(seq=S, inter=a.inter, ms=ms, us=ms * 1e3, mbytes=byts / 1e6, gbs=byts / ms / 1e6)
    elif a.kernel == "tables":
        st0, st1 = 512, S - 256
        n_art = st1 - st0
        sc = (torch.randn(B, n_art, device=dev, generator=g) * 0.5).to(torch.bfloat16).float()
        n_kept = st0 + a.k + (S - st1)
        keep, _, _ = ops.topk_select(sc, [n_art] * B, [a.k] * B, [st0] * B, [S] * B, n_kept, bias_dtype=None)
        gs = torch.rand(a.layers, a.hq, device=dev, generator=g) + 0.5
        at = torch.rand(a.layers, a.hq, device=dev, generator=g) + 0.5
        fn = lambda: ops.phase2_tables(sc, [st0] * B, [n_art] * B, keep, [n_kept] * B, gs, at, 1e-6)
        ms = _time(fn, a.iters)
        byts = B * (n_art * 4 + n_kept * 8 + 2 * a.layers * a.hq * n_kept * 4)
        res.update(seq=S, k=a.k, layers=a.layers, hq=a.hq, ms=ms, us=ms * 1e3, mbytes=byts / 1e6,
                   gbs=byts / ms / 1e6)
    else:
        st0, st1 = 512, S - 256
        n_art = st1 - st0
        h = torch.randn(B, S, a.hidden, device=dev, dtype=torch.bfloat16, generator=g)
        w = torch.randn(a.hidden, device=dev, generator=g) / a.hidden ** 0.5
        sc = ops.gate_score(h, w, [st0] * B, [n_art] * B)
        n_kept = st0 + a.k + (S - st1)
        if a.kernel == "score":
            ms = _time(lambda: ops.gate_score(h, w, [st0] * B, [n_art] * B, out=sc), a.iters)
            byts = B * (n_art * a.hidden * 2 + n_art * 4) + a.hidden * 4
        elif a.kernel == "topk":
            keep = torch.empty(B, n_kept, dtype=torch.int64, device=dev)
            bias = torch.empty(B, n_kept, dtype=torch.bfloat16, device=dev)
            ms = _time(lambda: ops.topk_select(sc, [n_art] * B, [a.k] * B, [st0] * B, [S] * B, n_kept,
                                               keep_out=keep, bias_out=bias), a.iters)
            byts = B * (n_art * 4 + n_kept * 10)
        else:
            keep, _, _ = ops.topk_select(sc, [n_art] * B, [a.k] * B, [st0] * B, [S] * B, n_kept)
            kv = [torch.randn(B, S, a.hkv, 128, device=dev, dtype=torch.bfloat16, generator=g) for _ in range(4)]
            dh = torch.empty(B, n_kept, a.hidden, device=dev, dtype=torch.bfloat16)
            dkv = [torch.empty(B, n_kept, a.hkv, 128, device=dev, dtype=torch.bfloat16) for _ in range(4)]
            specs = [ops.gather_spec_rows(h, dh, 1)] + [ops.gather_spec_rows(s, d, 1) for s, d in zip(kv, dkv)]
            ms = _time(lambda: ops.gather_rows(specs, keep, [n_kept] * B, n_kept, dev), a.iters)
            byts = B * 2 * n_kept * (a.hidden * 2 + 4 * a.hkv * 128 * 2) + B * n_kept * 8
        res.update(seq=S, k=a.k, ms=ms, us=ms * 1e3, mbytes=byts / 1e6, gbs=byts / ms / 1e6)
    assert ops.device_error() == 0
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
