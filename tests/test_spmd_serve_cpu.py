"""Tensor-parallel serving on gloo ranks (CPU): rank 0 serves the framed TCP
protocol on an engine shard wrapped by ``SpmdLeader``, rank 1 follows in lock
step; concurrent clients (one cancelled mid-stream by disconnecting) get the
oracle's tokens, and both ranks end with no work and no pages held."""
import asyncio
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spec():
    from lunaflux_b200.models.spec import LlamaSpec
    return LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=172, vocab=256, max_position=512,
                     dtype="fp32")


PROMPTS = [[5, 6, 7], [9, 10, 11, 12, 13], [1, 2, 3, 4], [200, 100]]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lunaflux_b200.config import CacheConfig, SchedulerConfig
        from lunaflux_b200.contracts.inference import (CompletedEvent, FailedEvent, GenerateRequest, TokenEvent,
                                                       default_limits)
        from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
        from lunaflux_b200.models.weights import build_runtime, random_checkpoint
        from lunaflux_b200.ops.torch_ops import TorchOps
        from lunaflux_b200.parallel.comm import TPComm
        from lunaflux_b200.parallel.tp import TPShard
        from lunaflux_b200.service.framed_wire import (EVENT_HEADER, EVENT_MAGIC, FrameReader, decode_event,
                                                       encode_request)
        from lunaflux_b200.service.server import EngineService, TCPServer
        from lunaflux_b200.service.spmd import SharedClock, SpmdLeader, follower_loop
        from lunaflux_b200.tokenizer.bpe import synthetic_byte_tokenizer
        spec = _spec()
        ck = random_checkpoint(spec, 0)
        w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec))
        clock = SharedClock()
        eng = LLMEngine(w, TorchOps(), "cpu", SchedulerConfig(step_token_budget=32, max_active_requests=3,
                                                              prefill_chunk_tokens=32, emergency_decode_page_reserve=1),
                        CacheConfig(), EngineOptions(max_context=256, num_pages=48, graph_sizes=(), overlap_steps=True),
                        comm=TPComm(), clock=clock)
        if rank != 0:
            follower_loop(eng, clock)
            q.put((rank, (eng.has_work(), eng.scheduler.allocator.allocated_page_count()
                          - eng.scheduler.prefix.page_count())))
            return
        leader = SpmdLeader(eng, clock)
        svc = EngineService(leader, synthetic_byte_tokenizer(), default_limits(256, 512))
        svc.start()

        async def client(port, rid, prompt, n, drop):
            r, wr = await asyncio.open_connection("127.0.0.1", port)
            wr.write(encode_request(GenerateRequest(rid, input_tokens=tuple(prompt), max_new_tokens=n)))
            await wr.drain()
            fr = FrameReader(EVENT_MAGIC, header=EVENT_HEADER)
            toks = []
            while True:
                data = await r.read(65536)
                if not data:
                    break
                evs = [decode_event(f, rid) for f in fr.feed(data)]
                toks += [e.token_id for e in evs if isinstance(e, TokenEvent)]
                if drop and toks:
                    break
                if evs and isinstance(evs[-1], (CompletedEvent, FailedEvent)):
                    break
            wr.close()
            return toks

        async def main():
            srv = TCPServer(svc)
            port = await srv.start()
            outs = await asyncio.gather(*(client(port, 10 + i, p, 8 if i != 1 else 40, i == 1)
                                          for i, p in enumerate(PROMPTS)))
            for _ in range(200):
                if not eng.has_work() and not eng.live:
                    break
                await asyncio.sleep(0.05)
            srv.close()
            return outs

        try:
            outs = asyncio.run(main())
        finally:
            svc.stop()
            leader.shutdown()
        q.put((0, (outs, eng.has_work(), eng.scheduler.allocator.allocated_page_count()
                   - eng.scheduler.prefix.page_count())))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_serving_lock_step():
    from lunaflux_b200.models.weights import random_checkpoint
    from lunaflux_b200.oracle.reference import ReferenceModel
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    outs, busy0, held0 = res[0]
    busy1, held1 = res[1]
    assert not busy0 and not busy1 and held0 == 0 and held1 == 0
    ref = ReferenceModel(_spec(), random_checkpoint(_spec(), 0))
    for i, (p, o) in enumerate(zip(PROMPTS, outs)):
        want = ref.generate_greedy(p, 8 if i != 1 else 40)
        assert o == want[:len(o)] and (i == 1 or len(o) == 8)
