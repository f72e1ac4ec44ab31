"""Request-sharded batched serving of gated prefills on the GPUs of one node.

The serving sweep: N independent long-context requests, sharded across the
GPUs (one process per GPU, one model replica each; requests are independent,
so no collective touches the data path), each GPU serving its share in
static batches. Mirrors:
  * round-robin request split across replicas (tokengate/generators.py:269-296);
  * static batching: a batch is submitted when the previous one returned, the
    last batch may be smaller (benchmarks/batching.py:54-60);
and reports aggregate prefill tokens/s (all requests' prompt tokens / the
slowest rank's wall time) and the median TTFT (a batch's submission to its
first tokens on the host).

    python -m torch.distributed.run --nproc-per-node N -m tokengate_b200.serving \
        --requests 64 --seq 32768 --k 100,500,2000,all --batch 8
"""
import argparse
import json
import math
import os
import statistics
import time
from typing import Callable, Dict, List, Sequence

import torch

ALL_K = 10_000_000


def shard_requests(n_requests: int, world: int, rank: int) -> List[int]:
    """Request indices served by `rank`: i with i % world == rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    return list(range(rank, n_requests, world))


def static_batches(indices: Sequence[int], size: int) -> List[List[int]]:
    """Consecutive batches of `size` requests, the last one possibly smaller."""
    if size < 1:
        raise ValueError("batch size must be positive")
    return [list(indices[i:i + size]) for i in range(0, len(indices), size)]


def serve_static(prefill: Callable, requests: Dict[int, dict], indices: Sequence[int], batch: int,
                 K: int, sync: Callable[[], None] = lambda: None) -> List[dict]:
    """Serve `indices` in static batches. prefill(ids_list, starts, ends, K) ->
    (first_tokens (B,1), n_kepts). Returns one record per request."""
    records = []
    for bidx in static_batches(indices, batch):
        reqs = [requests[i] for i in bidx]
        sync()
        t0 = time.perf_counter()
        first, n_kepts = prefill([r["ids"] for r in reqs], [r["start"] for r in reqs],
                                 [r["end"] for r in reqs], K)
        first_host = first.cpu() if torch.is_tensor(first) else torch.as_tensor(first)
        sync()
        dt = time.perf_counter() - t0
        for j, i in enumerate(bidx):
            records.append(dict(idx=i, ttft_s=dt, n_kept=int(n_kepts[j]),
                                first_token=int(first_host.reshape(-1)[j]),
                                n_tokens=len(requests[i]["ids"]) if not torch.is_tensor(requests[i]["ids"])
                                else int(requests[i]["ids"].numel())))
    return records


def summarize(records: List[dict], wall_s: float) -> dict:
    """Aggregate prefill tokens/s over `wall_s` and the TTFT distribution."""
    if not records:
        raise ValueError("no records")
    ttft = sorted(r["ttft_s"] for r in records)
    tokens = sum(r["n_tokens"] for r in records)
    return dict(requests=len(records), tokens=tokens, wall_s=wall_s, tokens_per_s=tokens / wall_s,
                p50_ttft_ms=statistics.median(ttft) * 1e3,
                p90_ttft_ms=ttft[min(len(ttft) - 1, max(0, math.ceil(0.9 * len(ttft)) - 1))] * 1e3,
                max_ttft_ms=ttft[-1] * 1e3)


def gather_records(records: List[dict], wall_s: float):
    """All ranks' records and the slowest rank's wall time (every rank gets them)."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return records, wall_s
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, (records, wall_s))
    merged = sorted((r for recs, _ in out for r in recs), key=lambda r: r["idx"])
    return merged, max(w for _, w in out)


def make_requests(n: int, seq: int, vocab: int, state_begin: int, state_end: int, seed: int = 0) -> Dict[int, dict]:
    """Synthetic requests: uniform random ids (distinct seed per request)."""
    reqs = {}
    for i in range(n):
        g = torch.Generator().manual_seed(seed + i)
        reqs[i] = dict(ids=torch.randint(0, vocab, (seq,), generator=g, dtype=torch.long),
                       start=state_begin, end=state_end)
    return reqs


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="qwen3-1.7b")
    ap.add_argument("--gate-layer", type=int, default=1)
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--seq", type=int, default=32768)
    ap.add_argument("--state", default="512,32512", help="state span begin,end")
    ap.add_argument("--k", default="100,500,2000,all")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=1, help="warm-up batches per K (not timed)")
    ap.add_argument("--gate", default="linear", choices=("linear", "e2e"),
                    help="linear: the synthetic log-sigmoid gate; e2e: a seeded finalized gate")
    ap.add_argument("--no-phase2-graphs", action="store_true",
                    help="launch the Phase-2 layers eagerly instead of replaying a CUDA graph per shape")
    a = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=dev)

    from .inference import load_model
    tm = load_model(base_model=a.model, gate_layer=a.gate_layer, device=dev, seed=0,
                    gate="e2e" if a.gate == "e2e" else None)
    from .prefill import set_phase2_graphs
    set_phase2_graphs(not a.no_phase2_graphs)
    s0, s1 = (int(x) for x in a.state.split(","))
    reqs = make_requests(a.requests, a.seq, tm.model.config.vocab_size, s0, s1)
    mine = shard_requests(a.requests, world, rank)

    def prefill(ids, starts, ends, K):
        first, _c, _kp, n_kepts, _kc = tm.prefill([x.to(dev, non_blocking=True) for x in ids], starts, ends, K)
        return first, n_kepts

    def sync():
        torch.cuda.synchronize(dev)

    results = []
    for ks in a.k.split(","):
        K = ALL_K if ks == "all" else int(ks)
        for _ in range(a.warmup):
            serve_static(prefill, reqs, mine[:a.batch], a.batch, K, sync)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        sync()
        t0 = time.perf_counter()
        recs = serve_static(prefill, reqs, mine, a.batch, K, sync)
        wall = time.perf_counter() - t0
        recs, wall = gather_records(recs, wall)
        summ = summarize(recs, wall)
        summ.update(K=ks, n_gpus=world, batch=a.batch, seq=a.seq, model=a.model, gate=a.gate,
                    phase2="eager" if a.no_phase2_graphs else "cuda graph per shape")
        results.append(summ)
        if rank == 0:
            print(json.dumps(summ), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return results


if __name__ == "__main__":
    main()
