"""Overlapped steps (``EngineOptions.overlap_steps``): step n+1 is planned and
launched before step n's tokens reach the host; its decode rows take those
tokens on the device.  Outputs must equal the synchronous engine and the
full-recompute oracle token for token, through chunked prefill, preemption,
prefix hits, stop tokens, cancellation and stochastic sampling."""
import pytest
import torch

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import FinishReason, SamplingParameters
from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
from lunaflux_b200.models.spec import tiny_llama
from lunaflux_b200.models.weights import build_runtime, random_checkpoint
from lunaflux_b200.ops.torch_ops import TorchOps
from lunaflux_b200.oracle.reference import ReferenceModel


@pytest.fixture(scope="module")
def tiny():
    spec = tiny_llama()
    return spec, random_checkpoint(spec, 0)


def engine(spec, ck, overlap=True, rows=4, budget=64, pages=64, prefix=True):
    w = build_runtime(spec, lambda n: ck[n])
    sched = SchedulerConfig(step_token_budget=budget, max_active_requests=rows, prefill_chunk_tokens=budget,
                            emergency_decode_page_reserve=1, waiting_age_threshold_steps=8)
    return LLMEngine(w, TorchOps(), "cpu", sched, CacheConfig(prefix_enabled=prefix),
                     EngineOptions(max_context=256, num_pages=pages, graph_sizes=(), overlap_steps=overlap))


def prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 256, (n,), generator=g).tolist() for n in (5, 9, 13, 17)]


@pytest.mark.parametrize("rows,budget,pages", [(4, 64, 64), (2, 6, 64), (4, 64, 6)])
def test_overlap_matches_oracle(tiny, rows, budget, pages):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck, rows=rows, budget=budget, pages=pages, prefix=pages > 6)
    ps = prompts()
    outs = eng.generate(ps, 12)
    for p, o in zip(ps, outs):
        assert o == ref.generate_greedy(p, 12)
    s = eng.scheduler
    if pages == 6:
        assert s.preemptions > 0
    assert not s.inflight and not eng._launched
    s.debug_check_invariants()
    assert s.allocator.allocated_page_count() == (s.prefix.page_count() if s.prefix else 0)


def test_overlap_keeps_two_steps_in_flight(tiny):
    spec, ck = tiny
    eng = engine(spec, ck)
    for p in prompts():
        eng.add_request(p, 8)
    seen = 0
    while eng.has_work():
        eng.step()
        seen = max(seen, len(eng.scheduler.inflight))
        # a decode row whose input is still pending reads it on the device
    assert seen == 1        # after each step one plan stays queued behind the commit
    assert eng.runner.steps > 0


def test_overlap_forwards_tokens_on_device(tiny):
    spec, ck = tiny
    eng = engine(spec, ck)
    eng.add_request(prompts()[0], 6)
    fwd_rows = []
    orig = eng.runner.launch

    def spy(plan, table):
        fwd_rows.extend(r.fwd for r in plan.rows if r.decode)
        return orig(plan, table)

    eng.runner.launch = spy
    eng.run_until_done()
    assert fwd_rows and all(f == 0 for f in fwd_rows)


def test_overlap_stochastic_equals_sync(tiny):
    spec, ck = tiny
    sp = SamplingParameters.sample(0.9, top_k=50, top_p=0.9, seed=7)
    ps = prompts()
    a = engine(spec, ck, overlap=False).generate(ps, 10, sp, seeds=[1, 2, 3, 4])
    b = engine(spec, ck, overlap=True).generate(ps, 10, sp, seeds=[1, 2, 3, 4])
    assert a == b


def test_overlap_stop_token_and_prefix(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    p = prompts()[0]
    full = ref.generate_greedy(p, 10)
    eng = engine(spec, ck)
    rid = eng.add_request(p, 10, stop_ids=[full[3]])
    eng.run_until_done()
    res = eng.results[rid]
    assert res.tokens == full[:full.index(full[3]) + 1]
    assert res.reason is FinishReason.STOP_SEQUENCE
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, 256, (40,), generator=g).tolist()
    eng.generate([shared + [1, 2, 3]], 4)
    b = shared + [7, 8]
    assert eng.generate([b], 4)[0] == ref.generate_greedy(b, 4)
    assert eng.scheduler.prefix_hit_tokens >= 32


def test_overlap_cancel_in_flight(tiny):
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    eng = engine(spec, ck, prefix=False)
    ps = prompts()
    rids = [eng.add_request(p, 20) for p in ps]
    for _ in range(4):
        eng.step()
    assert eng.scheduler.inflight            # the cancelled request has a row on the device
    assert eng.cancel(rids[1])
    eng.run_until_done()
    assert eng.results[rids[1]].reason is FinishReason.CANCELLED
    for i in (0, 2, 3):
        assert eng.results[rids[i]].tokens == ref.generate_greedy(ps[i], 20)
    assert eng.scheduler.allocator.allocated_page_count() == 0
    eng.scheduler.debug_check_invariants()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_overlap_randomized_workload_equals_sync(tiny, seed):
    """Random arrivals, prompt and output lengths, stop tokens, cancellations
    and page pressure (preemption): the overlapped engine finishes every
    request with the synchronous engine's tokens and reasons."""
    import random
    spec, ck = tiny
    rnd = random.Random(seed)
    events = []          # (step, kind, payload)
    for i in range(14):
        n = rnd.randint(1, 40)
        prompt = [rnd.randrange(256) for _ in range(n)]
        events.append((rnd.randint(0, 20), "add", (i, prompt, rnd.randint(8, 48), [rnd.randrange(256)])))
    for i in rnd.sample(range(14), 3):
        events.append((rnd.randint(2, 30), "cancel", i))

    def run(overlap):
        eng = engine(spec, ck, overlap=overlap, rows=4, budget=32, pages=9, prefix=False)
        rid_of = {}
        step = 0
        while step < 400:
            for (at, kind, payload) in events:
                if at != step:
                    continue
                if kind == "add":
                    i, prompt, max_new, stops = payload
                    rid_of[i] = eng.add_request(prompt, max_new, stop_ids=stops)
                elif payload in rid_of:
                    eng.cancel(rid_of[payload])
            eng.step()
            step += 1
            if step > 31 and not eng.has_work():
                break
        assert not eng.has_work()
        eng.scheduler.debug_check_invariants()
        assert eng.scheduler.allocator.allocated_page_count() == 0
        stats["preemptions"] += eng.scheduler.preemptions
        return {i: (eng.results[r].tokens, eng.results[r].reason, eng.results[r].error) for i, r in rid_of.items()}

    stats = {"preemptions": 0}

    a, b = run(False), run(True)
    assert stats["preemptions"] > 0          # the page budget forces preemption
    # a cancellation lands on a different step boundary relative to the
    # in-flight token, so cancelled requests may differ in length; every
    # other request must be identical
    for i in a:
        if a[i][1] is FinishReason.CANCELLED or b[i][1] is FinishReason.CANCELLED:
            assert a[i][1] is b[i][1]
            n = min(len(a[i][0]), len(b[i][0]))
            assert a[i][0][:n] == b[i][0][:n]
        else:
            assert a[i] == b[i], i


@pytest.mark.parametrize("seed,overlap", [(3, False), (3, True), (4, True)])
def test_randomized_prefix_sharing_matches_oracle(tiny, seed, overlap):
    """Shared prompt prefixes (radix cache hits, publication on finish),
    staggered arrivals, stop tokens and page pressure: every request's greedy
    tokens equal the unpaged oracle's, truncated at its stop token."""
    import random
    spec, ck = tiny
    ref = ReferenceModel(spec, ck)
    rnd = random.Random(seed)
    prefixes = [[rnd.randrange(256) for _ in range(rnd.choice((16, 32)))] for _ in range(2)]
    reqs = []
    for i in range(10):
        p = rnd.choice(prefixes) + [rnd.randrange(256) for _ in range(rnd.randint(1, 12))]
        reqs.append((rnd.randint(0, 12), p, rnd.randint(2, 10), rnd.randrange(256)))
    eng = engine(spec, ck, overlap=overlap, rows=3, budget=24, pages=14, prefix=True)
    rid_of = {}
    step = 0
    while step < 500 and (step <= 12 or eng.has_work()):
        for i, (at, p, n, stop) in enumerate(reqs):
            if at == step:
                rid_of[i] = eng.add_request(p, n, stop_ids=[stop])
        eng.step()
        step += 1
    assert not eng.has_work()
    for i, (at, p, n, stop) in enumerate(reqs):
        want = ref.generate_greedy(p, n)
        if stop in want:
            want = want[:want.index(stop) + 1]
        assert eng.results[rid_of[i]].tokens == want, i
    s = eng.scheduler
    assert s.prefix_hit_tokens > 0
    s.debug_check_invariants()
    assert s.allocator.allocated_page_count() == s.prefix.page_count()
