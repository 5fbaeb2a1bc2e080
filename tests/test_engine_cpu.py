"""Configuration #1 (CPU plumbing) and scheduler behaviour on the CPU path.

Tiny Llama: 2 layers, hidden 64, 4 heads, 2 KV heads, head_dim 16, SwiGLU FFN
172, vocab 256, fp32, weights N(0, 0.02) from seed 0, saved as safetensors
and loaded back.  Four requests with prompt lengths 5/9/13/17 uniform over
the vocab, greedy decode of 16 tokens, paged KV (page 16), continuous
batching with at most 4 rows: output must equal the unpaged full-recompute
oracle token for token.
"""
import os

import pytest
import torch

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import FinishReason, PublicErrorCode, SamplingParameters
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.safetensors import SafetensorsFile, save_file
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps
from lunaflux_b200.oracle.reference import ReferenceModel


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    spec = tiny_llama()
    path = str(tmp_path_factory.mktemp("ck") / "model.safetensors")
    save_file(random_checkpoint(spec, 0), path)
    f = SafetensorsFile(path)
    ck = {k: f.tensor(k).clone() for k in f.keys()}
    return spec, ck


def engine(spec, ck, rows=4, budget=64, pages=64, prefix=True, clock=None):
    w = build_runtime(spec, lambda n: ck[n])
    sched = SchedulerConfig(step_token_budget=budget, max_active_requests=rows, prefill_chunk_tokens=budget,
                            emergency_decode_page_reserve=1, waiting_age_threshold_steps=8)
    kw = {"clock": clock} if clock else {}
    return LLMEngine(w, TorchOps(), "cpu", sched, CacheConfig(prefix_enabled=prefix),
                     EngineOptions(max_context=256, num_pages=pages, graph_sizes=()), **kw)


def prompts_1():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]


def test_config1_token_for_token(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck)
    prompts = prompts_1()
    outs = eng.generate(prompts, 16)
    for p, o in zip(prompts, outs):
        assert o == ref.generate_greedy(p, 16)
    eng.scheduler.debug_check_invariants()
    # every page is back in the free queue or held by the prefix cache
    s = eng.scheduler
    assert s.allocator.allocated_page_count() == (s.prefix.page_count() if s.prefix else 0)


def test_chunked_prefill_small_budget_same_tokens(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck, rows=2, budget=6)
    prompts = prompts_1()
    outs = eng.generate(prompts, 8)
    for p, o in zip(prompts, outs):
        assert o == ref.generate_greedy(p, 8)


def test_preemption_under_page_pressure(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck, rows=4, budget=64, pages=6, prefix=False)
    prompts = prompts_1()
    outs = eng.generate(prompts, 20)
    for p, o in zip(prompts, outs):
        assert o == ref.generate_greedy(p, 20)
    assert eng.scheduler.preemptions > 0
    eng.scheduler.debug_check_invariants()


def test_prefix_cache_hit_same_tokens(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck)
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, 256, (40,), generator=g).tolist()
    a = shared + [1, 2, 3]
    b = shared + [7, 8]
    eng.generate([a], 4)
    out_b = eng.generate([b], 4)[0]
    assert eng.scheduler.prefix_hit_tokens >= 32
    assert out_b == ref.generate_greedy(b, 4)


def test_stop_token_and_limits(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    p = prompts_1()[0]
    full = ref.generate_greedy(p, 10)
    eng = engine(spec, ck)
    rid = eng.add_request(p, 10, stop_ids=[full[3]])
    eng.run_until_done()
    res = eng.results[rid]
    assert res.tokens == full[:full.index(full[3]) + 1]
    assert res.reason is FinishReason.STOP_SEQUENCE
    rid = eng.add_request(p, 3)
    eng.run_until_done()
    assert eng.results[rid].reason is FinishReason.TOKEN_LIMIT and len(eng.results[rid].tokens) == 3


def test_cancel_releases_pages(tiny):
    spec, ck = tiny
    eng = engine(spec, ck, prefix=False)
    rids = [eng.add_request(p, 50) for p in prompts_1()]
    for _ in range(3):
        eng.step()
    assert eng.cancel(rids[1])
    eng.run_until_done()
    assert eng.results[rids[1]].reason is FinishReason.CANCELLED
    assert all(len(eng.results[r].tokens) == 50 for r in rids if r != rids[1])
    assert eng.scheduler.allocator.allocated_page_count() == 0
    eng.scheduler.debug_check_invariants()


def test_deadline_expiry(tiny):
    spec, ck = tiny
    now = [0.0]
    eng = engine(spec, ck, prefix=False, clock=lambda: now[0])
    rid = eng.add_request(prompts_1()[0], 100, deadline_s=1.0)
    eng.step()
    now[0] = 5.0
    eng.run_until_done()
    assert eng.results[rid].error is PublicErrorCode.DEADLINE_EXCEEDED


def test_stochastic_replay_matches_host_sampler(tiny):
    """Sampling through the engine equals the fp64 host sampler applied to the
    oracle's logits with the counter-addressed draw."""
    from lunaflux_b200.sampling.host import counter_unit, stochastic_sample
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck)
    p = prompts_1()[2]
    sp = SamplingParameters.sample(0.75, top_k=40, top_p=0.5, seed=99)
    out = eng.generate([p], 6, sp)[0]
    seq = list(p)
    for i, tok in enumerate(out):
        logits = ref.forward(seq)[-1].double().numpy()
        exp = stochastic_sample(logits, 0.75, 40, 0.5, counter_unit(99, i))
        assert tok == exp
        seq.append(tok)


def test_worker_failure_fails_active_keeps_waiting(tiny):
    spec, ck = tiny
    eng = engine(spec, ck, rows=1, prefix=False)
    r1 = eng.add_request(prompts_1()[0], 5)
    r2 = eng.add_request(prompts_1()[1], 5)
    eng.step()
    eng.scheduler.fail_active(PublicErrorCode.WORKER_UNAVAILABLE)
    eng._drain_terminals()
    assert eng.results[r1].error is PublicErrorCode.WORKER_UNAVAILABLE
    eng.run_until_done()
    assert len(eng.results[r2].tokens) == 5


def test_page_starvation_never_stalls(tiny):
    """Every running request blocked on KV pages mid-prefill: the scheduler
    recomputes the youngest instead of stalling, and a request that cannot fit
    the cache on its own fails with context_overflow."""
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck, rows=4, budget=16, pages=6, prefix=False)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 256, (n,), generator=g).tolist() for n in (30, 31, 29, 33)]
    rids = [eng.add_request(p, 6) for p in prompts]
    steps = eng.run_until_done(max_steps=2000)
    assert not eng.has_work() and steps < 2000
    for p, r in zip(prompts, rids):
        assert eng.results[r].tokens == ref.generate_greedy(p, 6)
    assert eng.scheduler.preemptions > 0
    from lunaflux_b200.scheduler.scheduler import AdmissionRejected
    with pytest.raises(AdmissionRejected):
        eng.add_request(torch.randint(0, 256, (100,), generator=g).tolist(), 4)      # 7 pages > 6
    big = eng.add_request(torch.randint(0, 256, (60,), generator=g).tolist(), 40)    # grows past the arena
    eng.run_until_done(max_steps=200)
    assert eng.results[big].error is PublicErrorCode.CONTEXT_OVERFLOW
    assert 0 < len(eng.results[big].tokens) < 40
    assert eng.scheduler.allocator.allocated_page_count() == 0


def test_admission_rejects_token_ids_outside_the_vocabulary(tiny):
    """Reference: scheduler/core 'admission rejects token IDs outside the
    loaded worker vocabulary'; nothing is queued and the engine keeps serving."""
    from lunaflux_b200.scheduler.scheduler import AdmissionRejected
    spec, ck = tiny
    eng = engine(spec, ck)
    for bad in ([1, 2, spec.vocab], [-1, 3]):
        with pytest.raises(AdmissionRejected) as e:
            eng.add_request(bad, 4)
        assert e.value.code is PublicErrorCode.INVALID_REQUEST
    assert not eng.has_work()
    assert len(eng.generate([[1, 2, 3]], 3)[0]) == 3
