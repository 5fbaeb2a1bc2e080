"""Rank loss on real GPUs: two supervised tensor-parallel ranks (one per GPU,
NCCL with NVLS off, no symmetric or multicast memory), rank 1 leaves between
steps: it finishes its step's device work and exits instead of reporting, so
neither rank has a kernel or a collective in flight, and the supervisor sees
the dead process before it issues another step.  The generation is restarted:
requests that had produced tokens fail with the retryable worker_unavailable
code, the waiting ones complete in the new generation with the tokens a
fault-free run produces."""
import os

import pytest
import torch

from lunaflux_b200.contracts import PublicErrorCode
from lunaflux_b200.engine.supervisor import Supervisor

pytestmark = pytest.mark.gpu

PROMPTS = [[5, 6, 7], [9, 10, 11, 12, 13], [1, 2, 3, 4], [200, 100]]


def _spec():
    from lunaflux_b200.models.spec import LlamaSpec
    return LlamaSpec(hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, ffn=2816, vocab=4096,
                     rope_theta=500000.0, max_position=2048, dtype="bf16")


class _LeavesBetweenSteps:
    """Rank 1 of generation 1: completes its second step, then exits before reporting it."""

    def __init__(self, eng, rank):
        self.eng, self.rank, self.steps = eng, rank, 0
        self.gen = int(os.environ.get("LUNAFLUX_GENERATION", "1"))
        self.leave = os.environ.get("LF_TEST_LEAVE") == "1"

    def __getattr__(self, k):
        return getattr(self.eng, k)

    def step(self):
        out = self.eng.step()          # synchronous steps: the device work is done when this returns
        self.steps += 1
        if self.leave and self.rank == 1 and self.gen == 1 and self.steps == 2:
            torch.cuda.synchronize()
            os._exit(3)
        return out


def gpu_factory(rank, world):
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops import KernelOps
    from lunaflux_b200.parallel.comm import TPComm, init_distributed
    from lunaflux_b200.parallel.tp import TPShard
    torch.cuda.set_device(rank)
    init_distributed("nccl", timeout_s=60, device_id=rank)
    spec = _spec()
    ck = {k: v.bfloat16().float() for k, v in random_checkpoint(spec, 11).items()}
    w = build_runtime(spec, lambda n: ck[n], TPShard(rank, world, spec), device=torch.device("cuda", rank),
                      dtype=torch.bfloat16)
    eng = LLMEngine(w, KernelOps(), torch.device("cuda", rank),
                    SchedulerConfig(step_token_budget=256, max_active_requests=8, prefill_chunk_tokens=256,
                                    emergency_decode_page_reserve=4),
                    CacheConfig(prefix_enabled=False),
                    EngineOptions(max_context=512, num_pages=128, graph_sizes=(), overlap_steps=False), comm=TPComm())
    return _LeavesBetweenSteps(eng, rank)


def _run(leave, monkeypatch):
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    monkeypatch.setenv("LUNAFLUX_FUSED_MULTICAST", "0")
    monkeypatch.setenv("LF_TEST_LEAVE", "1" if leave else "0")
    sup = Supervisor(2, gpu_factory, heartbeat_s=0.2, dead_after_s=30.0, step_timeout_s=300.0)
    sup.start()
    try:
        sup.submit(1, PROMPTS[0], 6)
        sup.submit(2, PROMPTS[1], 6)
        sup.step()                      # prefill of 1 and 2: they produce their first tokens
        sup.submit(3, PROMPTS[2], 6)
        sup.submit(4, PROMPTS[3], 6)
        sup.run_until_done()
    finally:
        sup.close()
    return sup


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_rank_leaving_between_steps_restarts_the_generation(monkeypatch):
    clean = _run(False, monkeypatch)
    assert clean.failures == 0
    sup = _run(True, monkeypatch)
    assert sup.failures == 1 and sup.generation == 2
    for rid in (1, 2):
        assert sup.reqs[rid].error is PublicErrorCode.WORKER_UNAVAILABLE
    for rid in (3, 4):
        assert sup.reqs[rid].error is None
        assert sup.reqs[rid].tokens == clean.reqs[rid].tokens
