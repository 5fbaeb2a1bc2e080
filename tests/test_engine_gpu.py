"""End-to-end engine on the GPU: the sm_100a path against the fp32 oracle."""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


def small_spec(layers=2):
    from lunaflux_b200.models.spec import LlamaSpec
    return LlamaSpec(hidden=1024, layers=layers, heads=8, kv_heads=2, head_dim=128, ffn=2816, vocab=4096,
                     rope_theta=500000.0, max_position=2048, dtype="bf16")


def bf16_checkpoint(spec, seed=0):
    from lunaflux_b200.models.weights import random_checkpoint
    ck = random_checkpoint(spec, seed)
    return {k: v.bfloat16().float() for k, v in ck.items()}


def make_engine(spec, ck, graphs=True, budget=256, rows=8, prefix=False, overlap=False):
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.weights import build_runtime
    from lunaflux_b200.ops import KernelOps
    w = build_runtime(spec, lambda n: ck[n], device="cuda", dtype=torch.bfloat16)
    sched = SchedulerConfig(step_token_budget=budget, max_active_requests=rows, prefill_chunk_tokens=budget,
                            emergency_decode_page_reserve=4)
    opts = EngineOptions(max_context=1024, num_pages=512, graph_sizes=(1, 2, 4, 8) if graphs else (),
                         overlap_steps=overlap)
    return LLMEngine(w, KernelOps(), "cuda", sched, CacheConfig(prefix_enabled=prefix), opts)


def check_near_argmax(ref, prompt, out, slack=0.05):
    """Each generated token must be (near-)argmax of the fp32 oracle's logits
    given the same prefix; bf16 activations allow near-ties to flip."""
    seq = list(prompt) + list(out)
    logits = ref.forward(seq)
    n = len(prompt)
    for i, tok in enumerate(out):
        row = logits[n - 1 + i]
        gap = (row.max() - row[tok]).item()
        assert gap <= slack * row.std().item() + 1e-4, f"token {i}: gap {gap:.4g} (std {row.std().item():.4g})"


def test_engine_matches_oracle_greedy():
    from lunaflux_b200.oracle.reference import ReferenceModel
    spec = small_spec()
    ck = bf16_checkpoint(spec)
    ref = ReferenceModel(spec, ck)
    eng = make_engine(spec, ck)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (5, 70, 300, 17, 129)]
    outs = eng.generate(prompts, 12)
    assert eng.runner.ops.read_error(True)[0] == 0
    for p, o in zip(prompts, outs):
        assert len(o) == 12
        check_near_argmax(ref, p, o)
    eng.scheduler.debug_check_invariants()


def test_graph_replay_equals_eager_forward_bitwise():
    """A captured decode bucket replays exactly what the eager forward computes
    on the same packed inputs: logits and sampled ids are bitwise equal, for
    every bucket the steps use (the same kernels run with the same split plan;
    the eager rerun rewrites the step's K / V pages with identical values)."""
    from lunaflux_b200.engine.step_inputs import device_views, make_layout
    spec = small_spec()
    ck = bf16_checkpoint(spec, seed=3)
    eng = make_engine(spec, ck, graphs=True)
    r = eng.runner
    g = torch.Generator().manual_seed(2)
    for n in (33, 64, 100):
        eng.add_request(torch.randint(0, spec.vocab, (n,), generator=g).tolist(), 24)
    checked = set()
    while eng.has_work():
        eng.step()
        b = r.last_bucket
        if b is None or b in checked:
            continue
        torch.cuda.synchronize()
        logits_graph = r.logits[:b].clone()
        tok_graph = r.out_tok[:b].clone()
        L = make_layout(b, 0, b, b, r.W)
        splits = min(r.ops.decode_splits(b, r.Hkv, r.max_context), r.max_splits)
        r.forward(device_views(r.in_dev, L), b, 0, 0, b, b, 0, splits, False, gather=False)
        torch.cuda.synchronize()
        assert torch.equal(r.logits[:b], logits_graph), f"bucket {b}: logits differ"
        assert torch.equal(r.out_tok[:b], tok_graph), f"bucket {b}: sampled ids differ"
        checked.add(b)
    assert checked, "no step replayed a graph"
    assert r.ops.read_error(True)[0] == 0


def test_decode_steps_allocate_nothing():
    """Steady state: once every request decodes, a step (packed upload, graph
    replay, on-device sampling, token readback) makes no device allocation.
    Reference behaviour: tests/hot_path_alloc (zero allocations after warm-up)."""
    spec = small_spec()
    ck = bf16_checkpoint(spec, seed=4)
    eng = make_engine(spec, ck, graphs=True)
    g = torch.Generator().manual_seed(5)
    for n in (20, 31, 45, 60):
        eng.add_request(torch.randint(0, spec.vocab, (n,), generator=g).tolist(), 48)
    for _ in range(8):                      # prefill, then warm-up decode steps (graph capture)
        eng.step()
    assert all(r.num_computed >= len(r.prompt) for r in eng.live.values())
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    for _ in range(16):
        assert eng.step()
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == before
    assert eng.runner.last_bucket is not None      # the steps replayed a captured graph
    assert eng.runner.ops.read_error(True)[0] == 0


def test_overlapped_steps_equal_synchronous():
    """Overlapped steps (decode inputs forwarded on the device, inside the
    captured graphs) give the synchronous engine's tokens exactly."""
    from lunaflux_b200.contracts import SamplingParameters
    spec = small_spec()
    ck = bf16_checkpoint(spec, seed=8)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (7, 50, 130, 260, 19)]
    for sp in (None, SamplingParameters.sample(0.8, top_k=40, top_p=0.95, seed=5)):
        a = make_engine(spec, ck).generate(prompts, 16, sp)
        eng = make_engine(spec, ck, overlap=True)
        b = eng.generate(prompts, 16, sp)
        assert a == b
        assert eng.runner.ops.read_error(True)[0] == 0


def test_stochastic_is_reproducible():
    from lunaflux_b200.contracts import SamplingParameters
    spec = small_spec(1)
    ck = bf16_checkpoint(spec, seed=4)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (9, 40)]
    sp = SamplingParameters.sample(0.7, top_p=0.9, seed=1234)
    a = make_engine(spec, ck).generate(prompts, 8, sp)
    b = make_engine(spec, ck).generate(prompts, 8, sp)
    assert a == b


def test_prefix_cache_reuse_gives_same_tokens():
    spec = small_spec()
    ck = bf16_checkpoint(spec, seed=6)
    g = torch.Generator().manual_seed(7)
    shared = torch.randint(0, spec.vocab, (64,), generator=g).tolist()
    p1 = shared + torch.randint(0, spec.vocab, (10,), generator=g).tolist()
    eng = make_engine(spec, ck, prefix=True)
    first = eng.generate([p1], 6)[0]
    again = eng.generate([p1], 6)[0]
    assert eng.scheduler.prefix_hit_tokens >= 64
    assert first == again


def min_router_margin(ref, prompt):
    """Smallest gap between the k-th and (k+1)-th router score over the
    prompt's tokens and the model's layers (fp32 oracle)."""
    import lunaflux_b200.oracle.reference as R
    margins = []
    orig = R.moe_mlp

    def spy(x, router, experts, top_k):
        s = (x @ router.t()).sort(-1, descending=True).values
        margins.append(float((s[:, top_k - 1] - s[:, top_k]).min()))
        return orig(x, router, experts, top_k)
    R.moe_mlp = spy
    try:
        ref.forward(prompt)
    finally:
        R.moe_mlp = orig
    return min(margins)


def test_moe_engine_matches_oracle():
    from lunaflux_b200.models.spec import LlamaSpec
    from lunaflux_b200.oracle.reference import ReferenceModel
    spec = LlamaSpec(hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, ffn=1024, vocab=4096,
                     rope_theta=1e6, max_position=2048, dtype="bf16", experts=8, experts_per_token=2)
    ck = bf16_checkpoint(spec, seed=9)
    ref = ReferenceModel(spec, ck)
    eng = make_engine(spec, ck)
    # Top-k routing is discontinuous: a prompt whose router scores for the
    # k-th and (k+1)-th expert nearly tie in fp32 can route differently under
    # bf16 activations, which no kernel tolerance covers.  Use prompts whose
    # routing margins are clear of bf16 rounding.
    g = torch.Generator().manual_seed(3)
    prompts = []
    for n in (7, 64, 200):
        while True:
            p = torch.randint(0, spec.vocab, (n,), generator=g).tolist()
            if min_router_margin(ref, p) > 5e-3:
                prompts.append(p)
                break
    outs = eng.generate(prompts, 8)
    assert eng.runner.ops.read_error(True)[0] == 0
    for p, o in zip(prompts, outs):
        check_near_argmax(ref, p, o, slack=0.1)


def test_every_launch_admitted_by_its_contract(monkeypatch):
    """With LUNAFLUX_CHECK_LAUNCHES=1 every KernelOps call of a mixed prefill /
    decode / prefix-hit workload (graphs on) passes its operand contract, and
    every packed step passes paged admission against the KV arena."""
    monkeypatch.setenv("LUNAFLUX_CHECK_LAUNCHES", "1")
    spec = small_spec()
    ck = bf16_checkpoint(spec, seed=4)
    eng = make_engine(spec, ck, graphs=True, prefix=True)
    ops = eng.runner.ops
    assert eng.runner.check_steps and ops.admitted == 0
    g = torch.Generator().manual_seed(5)
    shared = torch.randint(0, spec.vocab, (48,), generator=g).tolist()
    prompts = [shared + torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (3, 90, 200)]
    outs = eng.generate(prompts, 10)
    assert all(len(o) == 10 for o in outs)
    assert ops.admitted > 0 and ops.read_error(True)[0] == 0
