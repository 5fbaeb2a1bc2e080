"""Mixtral-style MoE on the CPU path: single rank and expert parallel (gloo)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.spec import LlamaSpec
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps
from lunaflux_b200.oracle.reference import ReferenceModel


def moe_spec():
    return LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=256, max_position=512,
                     dtype="fp32", experts=4, experts_per_token=2)


def prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]


def make(spec, ck, comm=None, rank=0, world=1, a2a=False):
    from lunaflux_b200.parallel.tp import TPShard
    w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec), ep_rank=rank, ep_size=world)
    return LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=64, max_active_requests=4,
                                                           prefill_chunk_tokens=64, emergency_decode_page_reserve=1),
                     CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=(),
                                                  sequence_parallel=a2a, moe_all_to_all=a2a, overlap_steps=a2a),
                     comm=comm)


def test_moe_single_rank_matches_oracle():
    spec = moe_spec()
    ck = random_checkpoint(spec, 0)
    ref = ReferenceModel(spec, ck)
    outs = make(spec, ck).generate(prompts(), 8)
    for p, o in zip(prompts(), outs):
        assert o == ref.generate_greedy(p, 8)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, a2a=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lunaflux_b200.parallel.comm import TPComm
        spec = moe_spec()
        ck = random_checkpoint(spec, 0)
        eng = make(spec, ck, TPComm(), rank, world, a2a)
        assert (eng.runner.moe_a2a is not None) == a2a
        out = eng.generate(prompts(), 8)
        if a2a:
            assert eng.runner.moe_a2a.calls > 0
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,a2a", [(2, False), (2, True), (4, True)])
def test_moe_expert_parallel_matches_oracle(world, a2a):
    """Experts sharded over the ranks: on the replicated rows (summed by the
    all-reduce), or on token-sharded rows with the dispatch / combine
    all-to-all (sequence parallelism, overlapped steps)."""
    spec = moe_spec()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, a2a)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    ref = ReferenceModel(spec, random_checkpoint(spec, 0))
    expect = [ref.generate_greedy(p, 8) for p in prompts()]
    for r in range(world):
        assert res[r] == expect, r
