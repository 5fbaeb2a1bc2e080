"""Benchmarks of configurations 2-5 (one JSON line per run, rank 0).

    python -m lunaflux_b200.bench.configs --workload config3 [--layers N] [--scale F]
    torchrun --nproc-per-node 8 -m lunaflux_b200.bench.configs --workload config5

Same engine and kernels as ``bench.py``; ``--scale`` shrinks the request
count (and ``--layers`` the depth) for quick checks, and the JSON line says
so.  Tensor parallel over all ranks; Mixtral additionally places its experts
expert-parallel (one expert per rank at 8 GPUs).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch
import torch.distributed as dist

from ..config import CacheConfig, SchedulerConfig
from ..engine.engine import EngineOptions, LLMEngine
from ..models import spec as specs
from ..models.weights import build_runtime, random_source
from ..ops import KernelOps
from ..parallel.comm import TPComm, env_rank_world, init_distributed
from ..parallel.tp import TPShard
from . import workloads as W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="config2", choices=sorted(W.WORKLOADS))
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--scale", type=float, default=1.0, help="fraction of the requests to run")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--no-realtime", action="store_true", help="ignore arrival times (all at t = 0)")
    ap.add_argument("--step-token-budget", type=int, default=8192)
    ap.add_argument("--no-overlap", action="store_true", help="synchronous steps")
    ap.add_argument("--json-out", default="")
    a = ap.parse_args()
    rank, world, local = env_rank_world()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        init_distributed("nccl", device_id=local)
    wl = W.WORKLOADS[a.workload]()
    if a.scale < 1.0:
        wl.items = wl.items[: max(1, int(len(wl.items) * a.scale))]
    spec = specs.PRESETS[wl.model]()
    if a.layers:
        spec = spec.with_layers(a.layers)
    rows = len(wl.items) if a.workload != "config5" else 256
    if world > 1:
        if a.comm == "fused" and not spec.is_moe:
            from ..parallel.fused import FusedTPComm
            comm = FusedTPComm(a.step_token_budget + rows, spec.hidden, dev)
        else:
            comm = TPComm()
    ep = world if spec.is_moe else 1
    t0 = time.time()
    weights = build_runtime(spec, random_source(spec, 0, dev, torch.bfloat16), TPShard(rank, world, spec), dev,
                            ep_rank=rank if ep > 1 else 0, ep_size=ep)
    torch.cuda.synchronize()
    load_s = time.time() - t0
    max_ctx = max(len(it.prompt) + it.max_new for it in wl.items) + 16
    sched = SchedulerConfig(step_token_budget=a.step_token_budget, max_active_requests=rows,
                            prefill_chunk_tokens=a.step_token_budget, emergency_decode_page_reserve=min(rows, 256),
                            max_waiting_requests=max(4096, len(wl.items)))
    pages = rows * (-(-max_ctx // 16)) + 2 * rows + 64
    if wl.prefix_cache:
        pages += 8 * 2048 // 16
    eng = LLMEngine(weights, KernelOps(), dev, sched, CacheConfig(prefix_enabled=wl.prefix_cache),
                    EngineOptions(max_context=max_ctx, num_pages=pages, overlap_steps=not a.no_overlap), comm=comm)
    if spec.is_moe and wl.router_zipf:
        eng.runner.router_bias = W.zipf_router_bias(spec.experts, wl.router_zipf, dev)
    for _ in range(a.warmup):
        warm = W.Workload(wl.name, wl.model, wl.items[: min(len(wl.items), 16)], wl.prefix_cache)
        W.run(eng, warm, comm, realtime=False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    dev_ms0 = eng.runner.device_ms
    st = W.run(eng, wl, comm, realtime=not a.no_realtime)
    torch.cuda.synchronize()
    dev_ms = eng.runner.device_ms - dev_ms0
    # every request has ended (finished or cancelled): once the prefix cache
    # gives its pages back, no page may still be allocated
    sched_ = eng.scheduler
    if getattr(sched_, "prefix", None) is not None:
        sched_.prefix.evict(1 << 30)
    leaked = sched_.allocator.allocated_page_count()
    if world > 1:
        t = torch.tensor([dev_ms, st.wall_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, st.wall_s = t.tolist()
    line = {"workload": a.workload, "model": f"{wl.model} ({spec.layers} layers)", "n_gpus": world,
            "parallelism": f"tp{world}" + (f"+ep{ep}" if ep > 1 else ""), "comm": a.comm if world > 1 else "none",
            "requests": len(wl.items), "scaled": a.scale < 1.0 or bool(a.layers),
            "output_tok_per_s_device": round(st.tokens / (dev_ms / 1e3), 1) if dev_ms else None,
            "output_tok_per_s_wall": round(st.tokens / st.wall_s, 1), **st.summary(), "load_s": round(load_s, 1), "leaked_pages": leaked,
            "data": "synthetic (seeded), random-init weights"}
    if rank == 0:
        print(json.dumps(line), flush=True)
        if a.json_out:
            with open(a.json_out, "w") as f:
                json.dump(line, f, indent=1)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
