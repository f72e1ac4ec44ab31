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
  roofline     the key-bias attention kernel (the dominant kernel): its
               algorithmic FLOPs (4*B*Hq*D*S(S+1)/2 per causal launch) over its
               CUDA-event time on its launch stream during the timed steps,
               against the measured sustained bf16 peak;
  cpu_baseline the CPU oracle's gated prefill (float32 torch, all host
               threads) on a bounded sample: the same model with an 8192-token
               prompt, state [512, 7936), K = 464 (the same K / state ratio).
  --impl reference times that CPU implementation alone (rank 0), the
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
CPU_SAMPLE = dict(seq_len=8192, state_begin=512, state_end=7936, K=464)
METRIC = "gated-prefill tokens/s (Qwen3-1.7B shape, 32k ctx, K=2000)"
# DRAM traffic of one Phase-1 attention launch (B=1, S=32768, Hq=16, Hkv=8),
# dram__bytes_read.sum + dram__bytes_write.sum from one ncu capture of the
# same launch shape (1.008 GB read + 0.112 GB written; algorithmic 0.256 +
# 0.128 GB: K/V re-read by the row blocks that share them)
ATTN_TRAFFIC_BYTES = 1.120e9
ATTN_TRAFFIC_SOURCE = ("ncu --set full --clock-control none -k regex:keybias -s 3 -c 1 "
                       "python -m tokengate_b200.microbench attn --seq 32768 --iters 3")


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
    """Counts this library's kernel launches and times the attention launches
    with CUDA events on the stream they are launched on."""

    def __init__(self):
        from tokengate_b200 import ops
        self.ops = ops
        self.orig = {n: getattr(ops, n) for n in ("keybias_attention", "gate_score", "topk_select",
                                                  "gather_rows", "add_rmsnorm", "qk_norm_rope",
                                                  "silu_mul", "branch_score", "phase2_tables")}
        self.active = False
        self.launches = 0
        self.attn = []   # (flops, start_event, end_event)

    def install(self):
        ops = self.ops
        meter = self

        def attn(q, k, v, *a, **kw):
            if not meter.active:
                return meter.orig["keybias_attention"](q, k, v, *a, **kw)
            s = torch.cuda.current_stream(q.device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            r = meter.orig["keybias_attention"](q, k, v, *a, **kw)
            e1.record(s)
            B, Sq, Hq, D = q.shape
            Sk = k.shape[1]
            causal = kw.get("causal", True)
            pairs = Sq * (Sq + 1) / 2 if causal else Sq * Sk
            meter.attn.append((4.0 * B * Hq * D * pairs, e0, e1))
            meter.launches += 1
            return r

        def counted(name, per_call):
            f = meter.orig[name]

            def g(*a, **kw):
                if meter.active:
                    meter.launches += per_call(a, kw)
                return f(*a, **kw)
            return g

        ops.keybias_attention = attn
        ops.gate_score = counted("gate_score", lambda a, kw: (len(a[2]) + 127) // 128)
        ops.topk_select = counted("topk_select", lambda a, kw: (a[0].shape[0] + 63) // 64)
        ops.gather_rows = counted("gather_rows", lambda a, kw: (a[1].shape[0] + 63) // 64)
        ops.add_rmsnorm = counted("add_rmsnorm", lambda a, kw: 1)
        ops.qk_norm_rope = counted("qk_norm_rope", lambda a, kw: 1)
        ops.silu_mul = counted("silu_mul", lambda a, kw: 1)
        ops.branch_score = counted("branch_score", lambda a, kw: (a[0].shape[0] + 127) // 128)
        ops.phase2_tables = counted("phase2_tables", lambda a, kw: (a[3].shape[0] + 127) // 128)

    def attention_summary(self):
        flops = sum(f for f, _, _ in self.attn)
        ms = sum(e0.elapsed_time(e1) for _, e0, e1 in self.attn)
        return flops, ms, len(self.attn)


def build_model(device, gate_kind="linear"):
    from tokengate_b200.inference import load_model
    return load_model(base_model=MODEL, gate_layer=GATE_LAYER, gate_attn="b200", device=device, seed=0,
                      gate="e2e" if gate_kind == "e2e" else None)


def make_prompt(seed: int, n: int, vocab: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n,), generator=g, dtype=torch.long)


def cpu_oracle_sample(tm, steps: int, warmup: int):
    """Time the CPU oracle's gated prefill on the bounded sample; returns (tokens/s, seconds/step, threads)."""
    import oracle.prefill as opre
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu_model = tm.model
    weights = opre.weights_fp32(cpu_model)
    c = CPU_SAMPLE
    ids = make_prompt(1234, c["seq_len"], tm.model.config.vocab_size).tolist()
    if getattr(tm.gate, "gate_branch", None) is not None:
        br, gt = tm.gate.gate_branch, tm.gate
        gp = dict(wg=br.gate_proj.weight.detach().cpu(), wu=br.up_proj.weight.detach().cpu(),
                  w_row=br.down_proj.weight.detach().cpu()[0],
                  gate_scale_eff=torch.nn.functional.softplus(gt.gate_scale.detach().cpu()),
                  attn_scale_eff=torch.nn.functional.softplus(gt.attn_scale.detach().cpu()),
                  eps=float(gt.b_norm.variance_epsilon), gain=float(gt.b_norm.weight.detach().cpu()[0]))

        def run():
            opre.gated_prefill_e2e(cpu_model, gp, [ids], [c["state_begin"]], [c["state_end"]], GATE_LAYER,
                                   c["K"], weights=weights)
    else:
        w = tm.gate.readout.weight.detach().cpu()

        def run():
            opre.gated_prefill(cpu_model, w, [ids], [c["state_begin"]], [c["state_end"]], GATE_LAYER, c["K"],
                               weights=weights, bias_bf16=True)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        run()
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    sec = statistics.median(times)
    return c["seq_len"] / sec, sec, threads


def sample_desc():
    c = CPU_SAMPLE
    return (f"CPU oracle (oracle/prefill.py, float32 torch) gated prefill of the same Qwen3-1.7B-shape "
            f"model: one {c['seq_len']}-token prompt, state [{c['state_begin']}, {c['state_end']}), "
            f"K={c['K']}, gate layer {GATE_LAYER}; tokens/s = {c['seq_len']} / median step time")


def run_reference(args):
    world, rank, local = _dist()
    if rank != 0:
        return 0
    # the reference arm runs on the host only: build the same random-init model on the CPU
    from tokengate_b200.inference import synthetic_qwen3
    from tokengate_b200.gate import LinLogSigGate
    model = synthetic_qwen3(MODEL, seed=0, device="cpu", dtype=torch.bfloat16)

    class _TM:
        pass
    tm = _TM()
    tm.model = model
    tm.gate = LinLogSigGate(model.config.hidden_size, generator=torch.Generator().manual_seed(1))
    tps, sec, threads = cpu_oracle_sample(tm, args.steps, args.warmup)
    line = {"metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform random ids, random-init weights)",
            "impl": "reference",
            "config": {"workload": "Qwen3-1.7B-shape gated prefill, bounded CPU sample",
                       "model": MODEL, "global_batch": 1, "seq_len": CPU_SAMPLE["seq_len"],
                       "K": CPU_SAMPLE["K"], "gate_layer": GATE_LAYER, "parallelism": "host cores"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample_desc()},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    meter.active = True
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(args.steps):
        step_device()
    e1.record()
    barrier()
    meter.active = False
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1))
    ms_step = ms / args.steps
    value = world * SEQ_LEN * args.steps / (ms / 1e3)
    a_flops, a_ms, a_n = meter.attention_summary()
    launches = int(sum_over_ranks(meter.launches))

    # ---- end to end through the public API (host ids in, first token out)
    for _ in range(args.warmup):
        step_e2e()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = step_e2e()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
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
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s / args.steps * 1e3},
        "gpu_launches": launches,
        "roofline": {"kernel": "keybias_attn_fwd_kernel", "bound": "tensor", "achieved": achieved,
                     "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": (achieved / peaks["tflops"]) if achieved else None,
                     "peak_source": f"{peaks['source']} bf16 sustained",
                     "launches": a_n, "algorithmic_tflop": a_flops / 1e12, "kernel_ms": a_ms,
                     "traffic": ATTN_TRAFFIC_BYTES, "traffic_unit": "bytes per launch",
                     "traffic_source": ATTN_TRAFFIC_SOURCE},
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:   # rank 0 at N=1 only
        tps, sec, threads = cpu_oracle_sample(tm, steps=1, warmup=0)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": sample_desc(), "seconds": sec}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
