"""Headline benchmark: Llama-3-8B-shaped serving on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|library|reference]

``--impl library`` is the measured baseline: the same engine, scheduler and
workload on cuBLAS GEMMs, vLLM's paged flash-attention, torch elementwise ops
and NCCL collectives, with the same CUDA-graph decode buckets.

Workload: 256 concurrent requests, 1024-token prompts
drawn uniformly from the vocabulary (seeded), 256 greedy output tokens each,
paged KV with 16-token pages, CUDA-graph decode at batch 1..256, random-init
weights N(0, 0.02) of the Llama-3-8B shape (32 layers, hidden 4096, 32 heads,
8 KV heads, FFN 14336, vocab 128256), bf16.  With N > 1 the model is tensor
parallel over N GPUs of one node (launched by torchrun, one rank per GPU), so
the total work is fixed ("strong" scaling).

One benchmark *step* is one complete pass of that workload (all 256 requests
admitted at t = 0 and run to completion).  Metrics:

* ``value``: output tokens / device time.  Device time is the sum over engine
  iterations of CUDA-event time from the step's first kernel to its sampled
  ids, max over ranks.
* ``e2e.value``: output tokens / wall time of ``LLMEngine.generate`` (the
  public API) including host scheduling, the per-iteration upload of the
  packed step block from pinned host memory and the int32 readback.
* ``ttft_p50_ms`` / ``tpot_p50_ms`` from the timed passes.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_VALUE = None  # the reference publishes no throughput number
METRIC = "output tok/s/box at 1/2/4/8 B200 (max over ranks); p50 TTFT; p50 TPOT"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "library", "torch", "reference"],
                    help="torch is an alias of library")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--layers", type=int, default=0, help="0 = the full model")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--step-token-budget", type=int, default=8192)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="row-parallel all-reduce: fused into the GEMM kernel, or NCCL after it")
    ap.add_argument("--sp", action="store_true",
                    help="sequence parallelism (residual stream sharded by tokens; reduce-scatter inside the "
                         "GEMM with the fused comm where the shape allows, library all-gather)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="synchronous steps (default: overlapped, step n+1 planned and launched before step n's "
                         "tokens reach the host)")
    ap.add_argument("--opt", default="",
                    help="comma-separated opt-in paths to enable: " + ",".join(sorted(OPT_IN)))
    ap.add_argument("--json-out", default="")
    ap.add_argument("--profile", default="", help="write a per-kernel time table of one extra pass here")
    return ap.parse_args()


def pct(xs, q, nd):
    """The q-th percentile (nearest rank) of xs, rounded; None when empty."""
    if not xs:
        return None
    ys = sorted(xs)
    k = min(len(ys) - 1, max(0, int(round(q / 100.0 * len(ys) + 0.5)) - 1))
    return round(ys[k], nd)


def reference_unavailable(args):
    line = {"impl": "reference", "unavailable": (
        "vectie/lunaflux is a MoonBit project with no Python package (pip: neither setup.py nor "
        "pyproject.toml), no moon toolchain on this image and no CUDA kernels to run")}
    print(json.dumps(line))


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        load = [r for r in rows if (num(r[4]) or 0) >= 50] or rows
        sm = [num(r[1]) for r in load if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i in range(4) if r[6 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": max((num(r[3]) or 0) for r in rows)}


# Opt-in kernel paths (off by default until measured), as environment switches
# read by the extension and the operator set at first use.
OPT_IN = {
    "pdl": "LUNAFLUX_PDL",
    "qkv_rope": "LUNAFLUX_FUSE_QKV_ROPE",
    "ll_gemm": "LUNAFLUX_FUSED_LL_GEMM",
    "gemm_2sm": "LUNAFLUX_GEMM_2SM",
    "cluster_mb2": "LUNAFLUX_GEMM_CLUSTER_MB2",
}


def main():
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return 0
    if args.impl == "torch":
        args.impl = "library"
    opts_on = [o for o in args.opt.split(",") if o]
    for o in opts_on:
        if o not in OPT_IN:
            raise SystemExit(f"unknown --opt {o!r} (known: {', '.join(sorted(OPT_IN))})")
        os.environ[OPT_IN[o]] = "1"
    import numpy as np
    import torch
    import torch.distributed as dist

    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.contracts import SamplingParameters
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models import spec as specs
    from lunaflux_b200.models.weights import build_runtime, random_source
    from lunaflux_b200.parallel.comm import TPComm, env_rank_world, init_distributed
    from lunaflux_b200.parallel.tp import TPShard

    rank, world, local = env_rank_world()
    if world != args.gpus:
        args.gpus = world if world > 1 else args.gpus
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        init_distributed("nccl", device_id=local)
    spec = specs.PRESETS[args.model]()
    if world > 1:
        if args.impl == "ours" and args.comm == "fused":
            from lunaflux_b200.parallel.fused import FusedTPComm
            comm = FusedTPComm(args.step_token_budget + args.requests, spec.hidden, dev)
        else:
            comm = TPComm()
    if args.layers:
        spec = spec.with_layers(args.layers)
    shard = TPShard(rank, world, spec)
    t0 = time.time()
    weights = build_runtime(spec, random_source(spec, args.seed, dev, torch.bfloat16), shard, dev)
    torch.cuda.synchronize()
    t_load = time.time() - t0
    if args.impl == "ours":
        from lunaflux_b200.ops import KernelOps
        ops = KernelOps()
    else:
        from lunaflux_b200.ops import LibraryOps
        ops = LibraryOps(dev)
    max_ctx = args.prompt_len + args.output_len + 16
    sched = SchedulerConfig(step_token_budget=args.step_token_budget, max_active_requests=args.requests,
                            prefill_chunk_tokens=args.step_token_budget, emergency_decode_page_reserve=args.requests,
                            max_waiting_requests=max(4096, args.requests))
    pages = args.requests * (-(-max_ctx // 16)) + 2 * args.requests + 64
    opts = EngineOptions(max_context=max_ctx, num_pages=pages,
                         graph_sizes=() if args.no_graphs else EngineOptions().graph_sizes,
                         sequence_parallel=args.sp, overlap_steps=args.overlap)
    engine = LLMEngine(weights, ops, dev, sched, CacheConfig(prefix_enabled=False), opts, comm=comm)
    if not args.no_graphs:
        engine.runner.capture_all(False)
    torch.cuda.synchronize()
    # as a server does once it is up: the start-up objects leave the cyclic
    # collector's generations, so a full collection does not stall a step
    gc.collect()
    gc.freeze()

    # synthetic seeded prompts, uniform over the vocabulary, held in pinned host memory
    g = torch.Generator().manual_seed(args.seed)
    prompts = torch.randint(0, spec.vocab, (args.requests, args.prompt_len), generator=g, dtype=torch.int32)
    prompts = prompts.pin_memory()
    greedy = SamplingParameters()

    def one_pass():
        engine.results.clear()
        toks = engine.generate(prompts, args.output_len, greedy)
        return sum(len(t) for t in toks)

    for _ in range(args.warmup):
        one_pass()
    # ---- timed region
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    r = engine.runner
    dev_ms0, h2d0, d2h0, launches0, steps0 = r.device_ms, r.h2d_bytes, r.d2h_bytes, getattr(ops, "launches", 0), r.steps
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ttfts, tpots = [], []
    emits = []     # wall time of every engine iteration that emitted tokens (inter-token latency)

    def on_outputs(outs):
        if outs:
            emits.append(time.perf_counter())

    engine.listeners.append(on_outputs)
    tokens = 0
    wall0 = time.perf_counter()
    ev0.record()
    for _ in range(args.steps):
        engine.results.clear()
        rids = []
        for i in range(args.requests):
            rids.append(engine.add_request(prompts[i].numpy(), args.output_len, greedy))
        engine.run_until_done()
        for rid in rids:
            res = engine.results.pop(rid)
            tokens += len(res.tokens)
            if res.ttft is not None:
                ttfts.append(res.ttft * 1e3)
            if res.tpot is not None:
                tpots.append(res.tpot * 1e3)
    ev1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    engine.listeners.remove(on_outputs)
    itls = [(b - a) * 1e3 for a, b in zip(emits, emits[1:])]
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    span_ms = ev0.elapsed_time(ev1)
    dev_ms = r.device_ms - dev_ms0
    if world > 1:
        t = torch.tensor([dev_ms, span_ms, wall], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, span_ms, wall = t.tolist()
    steps_run = r.steps - steps0
    value = tokens / (dev_ms / 1e3)
    e2e = tokens / wall
    h2d = (r.h2d_bytes - h2d0) / args.steps
    d2h = (r.d2h_bytes - d2h0) / args.steps
    launches = getattr(ops, "launches", 0) - launches0
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "output tokens/s (device-timed, whole box)",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded uniform prompts, random-init N(0,0.02) weights)",
        "impl": args.impl,
        "config": {"model": f"{args.model} ({spec.layers} layers)", "global_batch": args.requests,
                   "seq_len": args.prompt_len, "output_len": args.output_len, "parallelism": f"tp{world}", "comm": (args.comm if world > 1 else "none"),
                   "overlap_steps": bool(args.overlap), "opt_in": opts_on,
                   "l2": "weights (16 GB) and KV (>10 GB) exceed L2 every step; no flush needed",
                   "engine_iterations_per_step": steps_run / args.steps},
        "ttft_p50_ms": pct(ttfts, 50, 2), "ttft_p95_ms": pct(ttfts, 95, 2), "ttft_p99_ms": pct(ttfts, 99, 2),
        "tpot_p50_ms": pct(tpots, 50, 3), "tpot_p95_ms": pct(tpots, 95, 3), "tpot_p99_ms": pct(tpots, 99, 3),
        "itl_p50_ms": pct(itls, 50, 3), "itl_p95_ms": pct(itls, 95, 3), "itl_p99_ms": pct(itls, 99, 3),
        "goodput_req_s": round(args.requests * args.steps / wall, 2),
        "serving": serving_summary(engine.metrics),
        "e2e": {"value": round(e2e, 1), "unit": "output tokens/s through LLMEngine.generate (wall clock)",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "event_span_ms_per_step": round(span_ms / args.steps, 3),
        "clocks": clk,
        "load_s": round(t_load, 1),
    }
    if rank == 0:
        print(json.dumps(line))
        if args.json_out:
            with open(args.json_out, "w") as f:
                json.dump(line, f, indent=1)
    if args.profile:
        # One extra, untimed pass under the CUDA activity profiler: kernel time shares only.
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            one_pass()
            torch.cuda.synchronize()
        if rank == 0:
            table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=25, max_name_column_width=90)
            with open(args.profile, "w") as f:
                f.write(table)
            print(table)
    if world > 1:
        # Captured CUDA graphs still reference the NCCL communicator, and tearing
        # it down under them can block; every rank is past its last collective
        # here, so synchronise once more and leave the process directly.
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)
    return 0


def serving_summary(m):
    """The engine's serving metrics over the warm-up and timed passes (the
    reference's benchmark set: queue time, tokens per step, prefix hit rate,
    graph-capture time, failure and cancellation counts).  Queue quantiles are
    histogram bucket upper bounds."""
    def hist(h):
        return h.snapshot().get("", {"count": 0, "sum": 0.0, "p50": None, "p99": None})

    q, tok, rows, cap = hist(m.queue), hist(m.step_tokens), hist(m.step_rows), hist(m.graph_capture)
    steps = sum(m.graph.values.values())
    hit = m.prefix_hit_rate()
    return {
        "queue_p50_ms_le": None if q["p50"] is None else round(q["p50"] * 1e3, 3),
        "queue_p99_ms_le": None if q["p99"] is None else round(q["p99"] * 1e3, 3),
        "tokens_per_step_mean": round(tok["sum"] / tok["count"], 2) if tok["count"] else None,
        "rows_per_step_mean": round(rows["sum"] / rows["count"], 2) if rows["count"] else None,
        "graph_captures": cap["count"], "graph_capture_s": round(cap["sum"], 3),
        "graph_step_share": round(m.graph.get(mode="captured") / steps, 4) if steps else None,
        "prefix_hit_rate": None if hit is None else round(hit, 4),
        "finished": {k or "none": int(v) for k, v in m.finished.snapshot().items()},
        "failed": {k: int(v) for k, v in m.failed.snapshot().items()},
    }


if __name__ == "__main__":
    sys.exit(main())
