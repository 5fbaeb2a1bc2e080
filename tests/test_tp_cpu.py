"""Tensor parallelism on CPU ranks (gloo, world size 2 and 4).

Each rank holds its column/row shards of the tiny Llama, runs the same
deterministic scheduler, all-reduces the row-parallel outputs and exchanges
per-shard argmax keys; the tokens must equal the single-rank oracle's.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, sp=False, overlap=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lunaflux_b200.config import CacheConfig, SchedulerConfig
        from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
        from lunaflux_b200.models.spec import LlamaSpec
        from lunaflux_b200.models.weights import build_runtime, random_checkpoint
        from lunaflux_b200.ops.torch_ops import TorchOps
        from lunaflux_b200.parallel.comm import TPComm
        from lunaflux_b200.parallel.tp import TPShard
        spec = LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256,
                         max_position=512, dtype="fp32")
        ck = random_checkpoint(spec, 0)
        w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec))
        eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=64, max_active_requests=4,
                                                              prefill_chunk_tokens=64, emergency_decode_page_reserve=1),
                        CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=(), sequence_parallel=sp,
                                                    overlap_steps=overlap),
                        comm=TPComm())
        assert eng.runner.sp == sp
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]
        outs = eng.generate(prompts, 12)
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,sp,overlap", [(2, False, False), (4, False, False), (2, True, False),
                                               (4, True, False), (2, False, True), (4, True, True)])
def test_tp_matches_oracle(world, sp, overlap):
    """TP alone, TP with sequence parallelism (the residual stream sharded
    by tokens between a reduce-scatter and an all-gather, odd token counts
    padded to a multiple of the world size), and TP with overlapped steps."""
    from lunaflux_b200.models.spec import LlamaSpec
    from lunaflux_b200.models.weights import random_checkpoint
    from lunaflux_b200.oracle.reference import ReferenceModel
    spec = LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256, max_position=512,
                     dtype="fp32")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, sp, overlap)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = ReferenceModel(spec, random_checkpoint(spec, 0))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]
    expect = [ref.generate_greedy(p, 12) for p in prompts]
    for r in range(world):
        assert results[r] == expect, f"rank {r}"


def _stochastic_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lunaflux_b200.config import CacheConfig, SchedulerConfig
        from lunaflux_b200.contracts import SamplingParameters
        from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
        from lunaflux_b200.models.spec import LlamaSpec
        from lunaflux_b200.models.weights import build_runtime, random_checkpoint
        from lunaflux_b200.ops.torch_ops import TorchOps
        from lunaflux_b200.parallel.comm import TPComm
        from lunaflux_b200.parallel.tp import TPShard
        spec = LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256,
                         max_position=512, dtype="fp32")
        ck = random_checkpoint(spec, 0)
        w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec))
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]
        outs = []
        for cand in (False, True):
            eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=64, max_active_requests=4,
                                                                  prefill_chunk_tokens=64,
                                                                  emergency_decode_page_reserve=1),
                            CacheConfig(), EngineOptions(max_context=256, num_pages=64, graph_sizes=(),
                                                         tp_sample_candidates=cand), comm=TPComm())
            assert eng.runner.sample_candidates == cand
            sp = SamplingParameters.sample(1.3, top_k=40, top_p=0.95, seed=5)
            outs.append(eng.generate(prompts, 12, sp, seeds=[11, 12, 13, 14]))
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_stochastic_candidates_equal_full_gather(world):
    """Vocabulary-parallel stochastic sampling from each shard's 64 largest
    keys draws exactly the tokens of the full-logit gather (top_k <= 64)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stochastic_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full, cand = results[0]
    assert full == cand
    assert any(len(set(o)) > 1 for o in full)
    for r in range(world):
        assert results[r] == results[0]
