"""Fused GEMM + all-reduce on 2+ GPUs (one process per GPU, NCCL bootstrap).

Every rank multiplies its own A_r by its own B_r; the fused kernels must return
sum_r A_r . B_r^T on every rank: the low-latency protocol (decode rows), the
flag protocol's tile path and split-K finalize path, and the partial-sum
reduction of each, over many calls in a row (exercising the epochs, both
ping-pong slots and the counter re-arming).
Reference: the fp32 products all-reduced with NCCL.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _leave(q):
    """A rank process leaves once its result has reached the queue, without the
    process-group teardown (which can block on exit and hold the parent)."""
    q.close()
    q.join_thread()
    os._exit(0)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


SHAPES = [(256, 4096, 512), (1, 4096, 1792), (8192, 4096, 512), (300, 4096, 1024), (37, 4096, 14336 // 8)]


def _worker(rank, world, port, q, fused_ll=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    try:
        from lunaflux_b200.parallel.comm import init_distributed
        from lunaflux_b200.parallel.fused import FusedTPComm
        init_distributed("nccl", timeout_s=120, device_id=rank)
        # default routing (low-latency protocol up to 1024 rows, tile path above)
        # and the flag protocol everywhere (split-K finalize kernel, tile path)
        comms = [FusedTPComm(8192, 4096, dev), FusedTPComm(8192, 4096, dev, ll_rows=0, tile_min_k=0)]
        C = comms[0].C
        if fused_ll:
            # decode rows: the cluster split-K GEMM runs the low-latency protocol in its epilogue
            C.gemm_set_ll_fused(True)
            comms = comms[:1]
        ws = torch.zeros(512 * 32768, device=dev)
        errs = []
        for it in range(3):
            for ci, comm in enumerate(comms):
                for (M, N, K) in SHAPES:
                    g = torch.Generator(device=dev).manual_seed(1000 * rank + 7 * it + M)
                    A = torch.randn(M, K, device=dev, generator=g).bfloat16()
                    B = (torch.randn(N, K, device=dev, generator=g) * 0.05).bfloat16()
                    part = A.float() @ B.float().t()
                    ref = part.clone()
                    dist.all_reduce(ref)
                    # The library baseline on the same data: bf16 partials, bf16 all-reduce.
                    lib = part.bfloat16()
                    dist.all_reduce(lib)
                    lib_err = float((lib.float() - ref).abs().max().item())
                    outs = [comm.gemm_allreduce(A, B, ws).clone()]
                    if M <= 1024:
                        ws[: M * N].copy_(part.flatten())
                        outs.append(comm.reduce_partials(ws[: M * N].view(M, N)).clone())
                    torch.cuda.synchronize(dev)
                    code = C.read_error(True)[0]
                    for out in outs:
                        err = (out.float() - ref).abs()
                        # bf16 partials are summed over `world` ranks: allow the rounding of
                        # every partial, and never more than twice the library's own error.
                        tol = (3e-2 + 3e-2 * ref.abs()) * max(1.0, world / 2)
                        bad = int((err > tol).sum().item())
                        mx = float(err.max().item())
                        if mx > max(2 * lib_err, 0.05):
                            bad = max(bad, 1)
                        errs.append((ci, M, N, K, code, bad, mx))
        comm = comms[0]
        q.put((rank, errs, comm.multicast))
        dist.barrier()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))
    _leave(q)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_gemm_allreduce_matches_nccl():
    _run(fused_ll=False)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_single_kernel_decode_gemm_allreduce_matches_nccl():
    _run(fused_ll=True)


def _run(fused_ll):
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fused_ll)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, errs, mc = q.get(timeout=300)
        res[r] = (errs, mc)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():    # a rank stuck in its library teardown: the results are in
            p.kill()
            p.join(timeout=10)
    for r, (errs, mc) in res.items():
        assert not isinstance(errs, str), errs
        for (ci, M, N, K, code, bad, mx) in errs:
            assert code == 0, f"rank {r} comm {ci} {M}x{N}x{K}: device error {code}"
            assert bad == 0, f"rank {r} comm {ci} {M}x{N}x{K}: {bad} elements off (max {mx}); multicast={mc}"


def _rs_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    try:
        from lunaflux_b200.parallel.comm import init_distributed
        from lunaflux_b200.parallel.fused import FusedTPComm
        init_distributed("nccl", timeout_s=120, device_id=rank)
        comm = FusedTPComm(8192, 4096, dev)
        errs = []
        for it in range(3):
            for rows, K in ((128, 512), (1024, 1792), (256, 4096 // world)):
                M, N = rows * world, 4096
                g = torch.Generator(device=dev).manual_seed(100 * rank + it + rows)
                A = torch.randn(M, K, device=dev, generator=g).bfloat16()
                B = (torch.randn(N, K, device=dev, generator=g) * 0.05).bfloat16()
                part = A.float() @ B.float().t()
                ref = torch.empty(rows, N, device=dev)
                dist.reduce_scatter_tensor(ref, part)
                # the kernel sums bf16-rounded partials: each is off by at most
                # half a bf16 ulp (2^-8 of its magnitude), which matters where
                # large partials of opposite sign cancel
                part_abs = torch.empty(rows, N, device=dev)
                dist.reduce_scatter_tensor(part_abs, part.abs())
                out = torch.empty(rows, N, device=dev, dtype=torch.bfloat16)
                ok = comm.gemm_reduce_scatter(A, B, out)
                torch.cuda.synchronize(dev)
                code = comm.C.read_error(True)[0]
                err = (out.float() - ref).abs()
                tol = (3e-2 + 3e-2 * ref.abs()) * max(1.0, world / 2) + part_abs * 2.0 ** -7
                errs.append((rows, K, ok, code, int((err > tol).sum().item()), float(err.max().item())))
        q.put((rank, errs))
        dist.barrier()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
    _leave(q)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_reduce_scatter_matches_nccl():
    """The row-parallel GEMM with the reduce-scatter in the kernel (tiles
    dealt to their rows' owner) against the fp32 partials reduce-scattered by
    NCCL, over repeated calls (both ping-pong slots)."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rs_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():    # a rank stuck in its library teardown: the results are in
            p.kill()
            p.join(timeout=10)
    for r, errs in res.items():
        assert not isinstance(errs, str), errs
        for (rows, K, ok, code, bad, mx) in errs:
            assert ok and code == 0 and bad == 0, (r, rows, K, ok, code, bad, mx)
