"""Row-parallel GEMM + all-reduce micro-benchmark (fused kernel vs GEMM -> NCCL).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m lunaflux_b200.bench.comm [--json out.json]

For each shape (the o_proj and down projections of Llama-3-8B at decode and
prefill row counts, K divided by the tensor-parallel degree) it times, with
CUDA events on the launching stream and as the max over ranks (decode row
counts replayed from a CUDA graph, as the engine runs them):

* ``gemm``   the local tcgen05 GEMM alone (no communication),
* ``nccl``   the same GEMM followed by the NCCL all-reduce of its output,
* ``fused``  one fused GEMM + all-reduce (``FusedTPComm.gemm_allreduce``),

and reports the roofline of the fused operation: the slower of the GEMM at
the measured bf16 peak and the bytes this rank must move over NVLink
(2 x (world-1)/world x output bytes for a bandwidth-optimal all-reduce) at
770 GB/s per direction.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from lunaflux_b200.bench.kernels import peaks
from lunaflux_b200.parallel.comm import init_distributed
from lunaflux_b200.parallel.fused import FusedTPComm
from lunaflux_b200.ops import _ext

NVLINK_GBS = 770.0


def _time(fn, iters: int, warmup: int, graph: bool) -> float:
    """Mean time per call, max over ranks.  With ``graph`` the calls are
    replayed from one CUDA graph (the decode path runs captured, so host
    launch overhead is not part of its cost)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        run = g.replay
    dist.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    if graph:
        run()
    else:
        for _ in range(iters):
            run()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default="")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="")
    ap.add_argument("--single-kernel-decode", action="store_true",
                    help="decode rows: the cluster split-K GEMM runs the low-latency all-reduce in its epilogue")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_distributed("nccl", device_id=local)
    world, rank = dist.get_world_size(), dist.get_rank()
    C = _ext.load()
    if args.single_kernel_decode:
        C.gemm_set_ll_fused(True)
    hidden = 4096
    shapes = []
    for M in (256, 8192):
        for name, K in (("o", 4096), ("down", 14336)):
            shapes.append((f"M{M} {name}", M, K // world))
    max_rows = max(M for _, M, _ in shapes)
    comm = FusedTPComm(max_rows, hidden, torch.device("cuda", local), tile_min_k=0)  # the fused kernels themselves
    ws = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    _, tflops, src = peaks()
    rows = []
    for name, M, K in shapes:
        if args.only and args.only not in name:
            continue
        g = torch.Generator(device="cuda").manual_seed(1234 + rank)
        A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g) * 0.1
        B = torch.randn(hidden, K, device="cuda", dtype=torch.bfloat16, generator=g) * 0.1
        D = torch.empty(M, hidden, device="cuda", dtype=torch.bfloat16)

        def gemm():
            C.gemm(A, B, D, 0, 0, ws)

        def nccl():
            C.gemm(A, B, D, 0, 0, ws)
            dist.all_reduce(D)

        def fused():
            return comm.gemm_allreduce(A, B, ws)

        graph = M <= 512
        t_gemm = _time(gemm, args.iters, 3, graph)
        t_nccl = _time(nccl, args.iters, 3, graph)
        t_fused = _time(fused, args.iters, 3, graph)
        # numerics: fused vs NCCL sum
        nccl()
        D2 = fused()
        torch.cuda.synchronize()
        err = float((D.float() - D2.float()).abs().max())
        flops = 2.0 * M * hidden * K
        comm_bytes = 2.0 * (world - 1) / world * M * hidden * 2
        roof_ms = max(flops / (tflops * 1e12), comm_bytes / (NVLINK_GBS * 1e9)) * 1e3
        row = dict(case=name, world=world, M=M, N=hidden, K=K, gemm_ms=round(t_gemm, 4), nccl_ms=round(t_nccl, 4),
                   fused_ms=round(t_fused, 4), cuda_graph=graph, fused_vs_nccl=round(t_nccl / t_fused, 3),
                   roofline_ms=round(roof_ms, 4), fused_frac_of_roofline=round(roof_ms / t_fused, 3),
                   max_abs_diff=err, peaks=src)
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    if rank == 0 and args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)
    dist.barrier()
    os._exit(0)


if __name__ == "__main__":
    main()
