"""Benchmark: gated-prefill TTFT and prefill tokens/s, Qwen3-1.7B shape, 32k context, K=2000.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: a random-init Qwen3-1.7B-architecture model in
bf16 (28 layers, hidden 2048, 16/8 heads, head_dim 128, SwiGLU 6144, RoPE
theta 1e6, vocab 151936), gate at layer 1 (linear 2048 -> 1 + log-sigmoid),
one 32768-token prompt of uniform random ids per GPU per step, state span
[512, 32512), K = 2000 kept state tokens. A step is one full gated prefill
(Phase 1 on 32768 tokens, score, select, compact, Phase 2 on 2768 tokens,
first token). Requests are independent: with N GPUs every rank runs its own
replica on its own prompt, no collective on the data path (weak scaling);
the timing barrier and the max over ranks use torch.distributed.

Reported (one JSON line from rank 0):
  value        prefill tokens/s over all ranks, prompt ids already on the GPU,
               device time (CUDA events) of K steps, max over ranks;
  e2e          the same metric through the public API
               (TokenGateModel.generate with the ids in pinned host memory:
               the H2D copy of the ids and the D2H read of the first token and
               kept positions inside the timed region), wall clock with
               syncs, max over ranks;
  roofline     the key-bias attention kernel (the dominant kernel), its Phase-1
               launches (32768 tokens, no bias): algorithmic FLOPs
               (4*B*Hq*D*S(S+1)/2 per causal launch) over its CUDA-event time
               on its launch stream during the timed steps, against the
               measured sustained bf16 peak (frac) and the burst peak
               (frac_burst);
  gpu_launches this library's kernels launched in the timed steps (eager C-ABI
               calls plus those replayed in the Phase-2 graphs);
  serving      (every N) 64 independent 32768-token requests split over the
               ranks, static batches of 8, K=2000: aggregate tokens/s, p50
               TTFT, per-GPU TTFT spread and the slowest GPU's makespan;
  gpu_ops      (N=1) single-kernel figures at the benchmarked shapes: attention
               TFLOP/s at S = 4096 / 2768 / 8192 / 32768, gate score, top-K,
               gather and finalized-gate readout GB/s for 1 and 8 requests,
               the fused projections beside cuBLAS (microbench.ops_table);
  cpu_baseline (N=1) the CPU oracle's gated prefill (float32 torch, all host
               threads) at the same config, timed by parts (one Phase-1 layer
               on 32768 tokens, the selection, one Phase-2 layer, the head)
               and summed with the layer counts;
  cpu_baseline_ops (N=1) the reference's CPU torch paths for the key-bias
               attention op (S=4096, FlexAttention uncompiled and the sdpa
               compatibility path) and the scoring / selection / compaction
               ops (32768 tokens, K = 100 / 500 / 2000), restated in
               oracle/cpu_paths.py.
  --impl reference times the CPU prefill sample alone (rank 0), the
  reference arm: the reference's path is Python and CUDA code that cannot be
  built or shipped to the GPU box, so its CPU restatement stands in for it.
  Phase 2 runs as one CUDA graph per shape (tokengate_b200.phase2_graph, the
  reference's Phase-2 graph mode; bit-identical to eager launches);
  --no-phase2-graphs launches it eagerly.
  --gate e2e runs the same workload with the finalized gate instead of the
  synthetic linear one (a seeded E2EGate: SwiGLU scoring branch cloned from
  layer 1, per-layer per-head bias, scaled-softmax query scale); the default
  is the synthetic linear gate.
"""
import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEQ_LEN = 32768
STATE_BEGIN, STATE_END = 512, 32512
K_KEEP = 2000
GATE_LAYER = 1
MODEL = "qwen3-1.7b"
METRIC = "gated-prefill tokens/s (Qwen3-1.7B shape, 32k ctx, K=2000)"
# DRAM traffic of one Phase-1 attention launch (B=1, S=32768, Hq=16, Hkv=8),
# dram__bytes_read.sum + dram__bytes_write.sum of the ncu capture summarised
# in profiles/keybias_attn_32k.md (0.996 GB read + 0.106 GB written;
# algorithmic 0.256 + 0.128 GB: K/V re-read by the row blocks that share them)
ATTN_TRAFFIC_BYTES = 1.102e9
ATTN_TRAFFIC_SOURCE = ("profiles/keybias_attn_32k.md: ncu --set full --clock-control none -k regex:keybias "
                       "-s 3 -c 1 python -m tokengate_b200.microbench attn --seq 32768 --iters 3 --no-bias")


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(tflops=p["bf16_tflops_sustained"], tflops_burst=p["bf16_tflops"],
                    hbm=p["hbm_gbs"], source="measured")
    return dict(tflops=1590.0, tflops_burst=1590.0, hbm=6650.0, source="fallback")


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"tg_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu_index)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s, r in zip(sm, rows) if float(r[3] or 0) > 200.0] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": int(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


class KernelMeter:
    """Times this library's attention launches with CUDA events on the stream
    they are launched on, and counts the library's kernel launches: every
    C-ABI call that launches a kernel (_lib.LAUNCH_CALLS) plus the library
    kernels replayed inside Phase-2 CUDA graphs (phase2_graph.REPLAYED_LAUNCHES)."""

    def __init__(self):
        from tokengate_b200 import ops
        self.ops = ops
        self.orig_attn = ops.keybias_attention
        self.active = False
        self.attn = []   # (flops, seq, start_event, end_event)
        self.n0 = None
        self.launches = 0

    def install(self):
        ops = self.ops
        meter = self

        def attn(q, k, v, *a, **kw):
            if not meter.active:
                return meter.orig_attn(q, k, v, *a, **kw)
            s = torch.cuda.current_stream(q.device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            r = meter.orig_attn(q, k, v, *a, **kw)
            e1.record(s)
            B, Sq, Hq, D = q.shape
            Sk = k.shape[1]
            causal = kw.get("causal", True)
            pairs = Sq * (Sq + 1) / 2 if causal else Sq * Sk
            meter.attn.append((4.0 * B * Hq * D * pairs, Sq, e0, e1))
            return r

        ops.keybias_attention = attn

    @staticmethod
    def _count():
        from tokengate_b200 import _lib, phase2_graph
        return _lib.LAUNCH_CALLS + phase2_graph.REPLAYED_LAUNCHES

    def start(self):
        self.active = True
        self.n0 = self._count()

    def stop(self):
        self.active = False
        self.launches = self._count() - self.n0

    def attention_summary(self):
        flops = sum(f for f, _, _, _ in self.attn)
        ms = sum(e0.elapsed_time(e1) for _, _, e0, e1 in self.attn)
        return flops, ms, len(self.attn)


def build_model(device, gate_kind="linear"):
    from tokengate_b200.inference import load_model
    return load_model(base_model=MODEL, gate_layer=GATE_LAYER, gate_attn="b200", device=device, seed=0,
                      gate="e2e" if gate_kind == "e2e" else None)


def make_prompt(seed: int, n: int, vocab: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g, dtype=torch.long)


def synthetic_weights_fp32(seed: int = 0):
    """Random float32 weights of the Qwen3-1.7B shape in the CPU oracle's
    layout (per-layer dicts, globals, config), drawn directly: a CPU timing
    needs the shapes, not the GPU replica's values (whose CPU init takes
    minutes)."""
    from tokengate_b200.inference import QWEN3_SHAPES
    c = QWEN3_SHAPES[MODEL]
    H, I, D = c["hidden_size"], c["intermediate_size"], c["head_dim"]
    Hq, Hkv, V = c["num_attention_heads"], c["num_key_value_heads"], c["vocab_size"]
    g = torch.Generator().manual_seed(seed)
    rnd = lambda *shape: torch.randn(*shape, generator=g) * 0.02
    layers = []
    for _ in range(c["num_hidden_layers"]):
        layers.append({"input_layernorm.weight": torch.ones(H), "post_attention_layernorm.weight": torch.ones(H),
                       "self_attn.q_proj.weight": rnd(Hq * D, H), "self_attn.k_proj.weight": rnd(Hkv * D, H),
                       "self_attn.v_proj.weight": rnd(Hkv * D, H), "self_attn.o_proj.weight": rnd(H, Hq * D),
                       "self_attn.q_norm.weight": torch.ones(D), "self_attn.k_norm.weight": torch.ones(D),
                       "mlp.gate_proj.weight": rnd(I, H), "mlp.up_proj.weight": rnd(I, H),
                       "mlp.down_proj.weight": rnd(H, I)})
    emb = rnd(V, H)
    glob = dict(embed=emb, norm=torch.ones(H), lm_head=emb)
    cfg = dict(head_dim=D, rms_norm_eps=1e-6, rope_theta=c["rope_theta"], n_layers=c["num_hidden_layers"])
    return layers, glob, cfg


def cpu_prefill_sample(steps: int, warmup: int, weights=None):
    """The CPU oracle's gated prefill at the benchmarked config (32768-token
    prompt, state [512, 32512), K=2000, gate layer 1), timed by parts
    (oracle.prefill.prefill_by_parts: one Phase-1 layer on the 32768 tokens,
    the selection, one Phase-2 layer on the 2768 kept tokens, the head; the
    whole prefill's time is those parts times the layer counts). Returns
    (tokens/s, seconds per prefill, threads, parts)."""
    import oracle.prefill as opre
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if weights is None:
        weights = synthetic_weights_fp32()
    ids = make_prompt(1234, SEQ_LEN, weights[1]["embed"].shape[0]).tolist()
    w_gate = torch.randn(weights[1]["embed"].shape[1], generator=torch.Generator().manual_seed(1)) / 2048 ** 0.5
    runs = []
    for i in range(warmup + steps):
        r = opre.prefill_by_parts(weights, ids, STATE_BEGIN, STATE_END, GATE_LAYER, K_KEEP, w_gate)
        if i >= warmup:
            runs.append(r)
    runs.sort(key=lambda r: r["total_s"])
    med = runs[len(runs) // 2]
    return SEQ_LEN / med["total_s"], med["total_s"], threads, med["parts_s"]


def sample_desc():
    return (f"CPU oracle (oracle/prefill.py, float32 torch, all host threads) gated prefill of a "
            f"Qwen3-1.7B-shape model at the benchmarked config: {SEQ_LEN}-token prompt, state "
            f"[{STATE_BEGIN}, {STATE_END}), K={K_KEEP}, gate layer {GATE_LAYER}; timed by parts (the "
            f"embedding, one Phase-1 layer on {SEQ_LEN} tokens, the scoring/selection/compaction, one "
            f"Phase-2 layer on the kept tokens with the key bias, the head) and summed with the layer "
            f"counts (2 Phase-1 and 26 Phase-2 layers); tokens/s = {SEQ_LEN} / that prefill time")


def cpu_ops_baseline() -> dict:
    """The reference's CPU paths for the two op-level workloads, restated in
    oracle/cpu_paths.py (the reference checkout is not on the GPU box):
    the key-bias attention op (B=1, S=4096, 16/8 heads, head_dim 128, fp32
    N(0,1) Q/K/V, per-key bias log-sigmoid(N(0,2)) on [256, 3840) and 0 on
    the 256 prefix / suffix tokens) through FlexAttention uncompiled and
    through sdpa_compat's chunked path; and the scoring / selection /
    compaction torch ops of one 32768-token request (bf16 N(0,1) hidden,
    state [512, 32512), w ~ N(0, 1/2048), K in {100, 500, 2000}, the
    below-gate K/V of layers 0-1). Median of 2 runs after a warm-up."""
    import oracle.cpu_paths as ocp
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)

    def med(fn, n=2):
        fn()
        ts = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return sorted(ts)[len(ts) // 2]

    S = 4096
    Q = torch.randn(1, 16, S, 128, generator=g)
    K = torch.randn(1, 8, S, 128, generator=g)
    V = torch.randn(1, 8, S, 128, generator=g)
    b = torch.zeros(S)
    b[256:3840] = torch.nn.functional.logsigmoid(2 * torch.randn(3584, generator=g))
    flops = 4.0 * 16 * 128 * S * (S + 1) / 2
    t_flex = med(lambda: ocp.flex_keybias_attention(Q, K, V, b))
    t_sdpa = med(lambda: ocp.sdpa_causal(Q, K, V, b))
    attn = {"workload": "key-bias causal GQA attention, B=1, S=4096, 16/8 heads, head_dim 128, fp32",
            "flex_uncompiled_s": t_flex, "flex_uncompiled_gflops": flops / t_flex / 1e9,
            "sdpa_compat_s": t_sdpa, "sdpa_compat_gflops": flops / t_sdpa / 1e9,
            "note": "compiled FlexAttention on the CPU fails in this torch build; the reference's CPU "
                    "flex path therefore runs unfused"}
    del Q, K, V
    S, s0, s1 = 32768, 512, 32512
    hid = torch.randn(S, 2048, generator=g).to(torch.bfloat16)
    w = torch.randn(2048, generator=g) / 2048 ** 0.5
    kv = [torch.randn(8, S, 128, generator=g).to(torch.bfloat16) for _ in range(4)]
    gate = {"workload": "gate score + top-K + keep list + hidden / below-gate K/V gathers, one "
                        "32768-token request, hidden 2048, state [512, 32512)", "K": {}}
    for kk in (100, 500, 2000):
        gate["K"][str(kk)] = {"seconds": med(lambda: ocp.gate_select_compact(hid, w, s0, s1, kk, kv))}
    return {"threads": threads, "cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(),
            "kind": "port (oracle/cpu_paths.py restating the reference's torch calls)",
            "attention": attn, "gate_select_compact": gate}


def serving_sweep(tm, dev, world: int, rank: int, pg, n_requests: int = 64, batch: int = 8) -> dict:
    """The serving workload at this N: n_requests independent 32768-token
    requests (distinct seeds) split round-robin over the ranks, each rank
    serving its share in static batches of `batch` (a batch is submitted when
    the previous one returned), K=2000. TTFT = a batch's submission to its
    first tokens on the host; aggregate tokens/s = all requests' prompt
    tokens / the slowest rank's wall time (makespan)."""
    from tokengate_b200.serving import make_requests, serve_static, shard_requests
    reqs = make_requests(n_requests, SEQ_LEN, tm.model.config.vocab_size, STATE_BEGIN, STATE_END, seed=5000)
    mine = shard_requests(n_requests, world, rank)

    def prefill(ids, starts, ends, K):
        first, _c, _kp, n_kepts, _kc = tm.prefill([x.to(dev, non_blocking=True) for x in ids], starts, ends, K)
        return first, n_kepts

    def sync():
        torch.cuda.synchronize(dev)

    serve_static(prefill, reqs, mine[:batch], batch, K_KEEP, sync)   # warm-up (graphs, allocator)
    if pg is not None:
        pg.barrier()
    sync()
    t0 = time.perf_counter()
    recs = serve_static(prefill, reqs, mine, batch, K_KEEP, sync)
    wall = time.perf_counter() - t0
    mine_summary = (rank, wall, statistics.median(r["ttft_s"] for r in recs), [r["ttft_s"] for r in recs],
                    sum(r["n_tokens"] for r in recs))
    allr = [mine_summary]
    if pg is not None:
        allr = [None] * world
        pg.all_gather_object(allr, mine_summary)
    makespan = max(a[1] for a in allr)
    ttfts = sorted(t for a in allr for t in a[3])
    per_gpu = [a[2] * 1e3 for a in sorted(allr)]
    tokens = sum(a[4] for a in allr)
    return {"requests": n_requests, "batch": batch, "K": K_KEEP, "seq_len": SEQ_LEN, "n_gpus": world,
            "tokens_per_s": tokens / makespan, "p50_ttft_ms": statistics.median(ttfts) * 1e3,
            "per_gpu_p50_ttft_ms": per_gpu, "ttft_spread_ms": max(per_gpu) - min(per_gpu),
            "makespan_s": makespan, "per_gpu_wall_s": [a[1] for a in sorted(allr)],
            "timing": "host wall clock with device syncs around each batch; requests' ids in pageable host memory"}


def run_reference(args):
    world, rank, local = _dist()
    if rank != 0:
        return 0
    # the reference arm runs on the host only
    tps, sec, threads, parts = cpu_prefill_sample(args.steps, args.warmup)
    line = {"metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform random ids, random-init weights)",
            "impl": "reference",
            "config": {"workload": "Qwen3-1.7B-shape gated prefill, 32768-token prompt, state [512, 32512), "
                                   "K=2000, gate layer 1; CPU, timed by parts",
                       "model": MODEL, "global_batch": 1, "seq_len": SEQ_LEN, "K": K_KEEP,
                       "gate_layer": GATE_LAYER, "parallelism": "host cores"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample_desc(), "parts_s": parts},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.gpus > 1:
        line["note"] = ("one host process on all cores: the value is the host's, it does not grow with the "
                        "number of GPUs of the other arm")
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-serving", action="store_true", help="skip the 64-request serving sweep")
    ap.add_argument("--no-phase2-graphs", action="store_true",
                    help="launch the Phase-2 layers eagerly instead of replaying a CUDA graph")
    ap.add_argument("--gate", default="linear", choices=("linear", "e2e"),
                    help="linear: the synthetic linear gate; e2e: a seeded finalized gate (E2EGate)")
    ap.add_argument("--profile-step", action="store_true",
                    help="after the warm-up, run ONE step between cudaProfilerStart/Stop and exit "
                         "(for ncu --profile-from-start off); prints no bench line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)

    world, rank, local = _dist()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            ap.error("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        pg = dist

    tm = build_model(dev, args.gate)
    from tokengate_b200.prefill import set_phase2_graphs
    set_phase2_graphs(not args.no_phase2_graphs)
    vocab = tm.model.config.vocab_size
    prompt = make_prompt(1000 + rank, SEQ_LEN, vocab)
    ids_dev = prompt.to(dev)
    starts, ends = [STATE_BEGIN], [STATE_END]

    def step_device():
        return tm.prefill([ids_dev], starts, ends, K_KEEP)[0]

    from tokengate_b200.inference import with_state_span
    # one request's ids (state-span sentinels included) in pinned host
    # memory, as a serving front end hands them over; copied every step
    host_ids = torch.tensor(with_state_span(prompt[:STATE_BEGIN].tolist(), prompt[STATE_BEGIN:STATE_END].tolist(),
                                            prompt[STATE_END:].tolist()), dtype=torch.long).pin_memory()

    def step_e2e():
        return tm.generate(host_ids, None, max_new_tokens=1, max_kept_prefill_tokens=K_KEEP)

    meter = KernelMeter()
    meter.install()

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)

    def sum_over_ranks(x: float) -> float:
        if pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.SUM)
        return float(t.item())

    def max_over_ranks(x: float) -> float:
        if pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing
    for _ in range(args.warmup):
        step_device()
    barrier()
    if args.profile_step:
        torch.cuda.profiler.start()
        step_device()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if pg is not None:
            pg.destroy_process_group()
        return 0
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    meter.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Python's cyclic garbage collector stays off inside the timed loops (as
    # timeit runs it): a full collection pass landing in a 10-step window
    # would be timed as the GPU path's
    gc.collect()
    gc.disable()
    barrier()
    e0.record()
    for _ in range(args.steps):
        step_device()
    e1.record()
    barrier()
    gc.enable()
    meter.stop()
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1))
    ms_step = ms / args.steps
    value = world * SEQ_LEN * args.steps / (ms / 1e3)
    a_flops, a_ms, a_n = meter.attention_summary()
    launches = int(sum_over_ranks(meter.launches))

    # ---- end to end through the public API (host ids in, first token out)
    for _ in range(args.warmup):
        step_e2e()
    gc.collect()
    gc.disable()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = step_e2e()
    barrier()
    e2e_elapsed = time.perf_counter() - t0
    gc.enable()
    e2e_s = max_over_ranks(e2e_elapsed)
    e2e_value = world * SEQ_LEN * args.steps / e2e_s
    h2d = host_ids.numel() * 8
    d2h = 8 + out.n_kept[0] * 8

    peaks = _peaks()
    achieved = a_flops / (a_ms / 1e3) / 1e12 if a_ms > 0 else None
    metric = METRIC if args.gate == "linear" else METRIC[:-1] + ", finalized gate)"
    line = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "ttft_ms": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform random ids, random-init weights)",
        "config": {"workload": "Qwen3-1.7B-shape gated prefill, 32768-token prompt, "
                               "state [512, 32512), K=2000, gate layer 1",
                   "model": MODEL, "global_batch": world, "seq_len": SEQ_LEN, "K": K_KEEP,
                   "gate_layer": GATE_LAYER, "gate": args.gate,
                   "phase2": "eager" if args.no_phase2_graphs else "cuda graph per shape",
                   "parallelism": f"request replicas x{world}",
                   "l2": "working set > L2 (3.4 GB weights, ~1 GB activations per step); no flush"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s / args.steps * 1e3,
                "timing": "host wall clock around the steps, device synchronised at both ends; "
                          "Python's cyclic GC off inside the loop (as timeit)"},
        "gpu_launches": launches,
        "roofline": {"kernel": "keybias_attn_fwd_kernel (Phase 1: 32768 tokens, 16/8 heads, causal)",
                     "bound": "tensor", "achieved": achieved,
                     "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": (achieved / peaks["tflops"]) if achieved else None,
                     "peak_source": f"{peaks['source']} bf16 sustained (the kernel runs inside a long step)",
                     "peak_burst": peaks["tflops_burst"],
                     "frac_burst": (achieved / peaks["tflops_burst"]) if achieved else None,
                     "launches": a_n, "algorithmic_tflop": a_flops / 1e12, "kernel_ms": a_ms,
                     "traffic": ATTN_TRAFFIC_BYTES, "traffic_unit": "bytes per launch",
                     "traffic_source": ATTN_TRAFFIC_SOURCE},
        "clocks": clk,
    }
    if world == 1 and rank == 0:
        from tokengate_b200.microbench import ops_table
        oclk = ClockSampler(local)
        oclk.start()
        line["gpu_ops"] = ops_table(dev, peaks["tflops_burst"], peaks["hbm"])
        line["gpu_ops"]["clocks"] = oclk.stop()
        line["gpu_ops"]["peaks"] = (f"{peaks['source']}: bf16 burst {peaks['tflops_burst']} TFLOP/s, "
                                    f"HBM copy {peaks['hbm']} GB/s (each kernel timed alone)")
    # ---- the serving workload at this N (every rank takes part)
    if not args.no_serving:
        line["serving"] = serving_sweep(tm, dev, world, rank, pg)
    if world == 1 and rank == 0:
        if not args.no_cpu_baseline:
            del tm
            torch.cuda.empty_cache()
            tps, sec, threads, parts = cpu_prefill_sample(steps=1, warmup=0)
            line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                                    "sample": sample_desc(), "seconds": sec, "parts_s": parts}
            line["cpu_baseline_ops"] = cpu_ops_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
