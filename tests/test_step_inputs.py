"""The packed step block against a scalar restatement of its layout (CPU).

Reference behaviour: engine/device_step (mixed rows produce exact CSR / SoA
values without page generations; randomized staging matches a scalar
reference; repeated packing reuses fixed storage; page-boundary sequence
lengths).  Plans come from the real scheduler driving random requests,
including preemption, prefix hits, chunked prefill and overlapped planning
(forwarded decode tokens), and every packed block also passes paged
admission against the KV arena."""
import random

import numpy as np
import pytest

from lunaflux_b200.config import CacheConfig, SchedulerConfig
from lunaflux_b200.contracts import SamplingParameters
from lunaflux_b200.engine.step_inputs import PARAM_INTS, build_host_step, make_layout
from lunaflux_b200.ops.launch_contract import check_paged_step
from lunaflux_b200.prefix.radix import PrefixIdentity
from lunaflux_b200.sampling.host import PARAM_DTYPE
from lunaflux_b200.scheduler.scheduler import Request, Scheduler

P = 16


def scalar_pack(plan, table, W, bucket=None):
    """The block as a dict of field -> list, built row by row."""
    pr = [r for r in plan.rows if not r.decode]
    dr = [r for r in plan.rows if r.decode]
    Rd = len(dr) if bucket is None else bucket
    srows = [r for r in plan.rows if r.sample]
    Rs = len(srows) if bucket is None else bucket
    f = {k: [] for k in ("tokens", "positions", "slots", "p_qstart", "p_seqlen", "p_bt", "d_tok", "d_seqlen",
                         "d_bt", "d_fwd", "s_idx")}
    params = []

    def tok_at(req, i):
        return req.prompt[i] if i < len(req.prompt) else req.output[i - len(req.prompt)]

    def slot(req, pos):
        return int(table[req.table.index, pos // P]) * P + pos % P

    q = 0
    f["p_qstart"] = [0]
    last = {}
    for r in pr:
        for pos in range(r.start, r.start + r.n):
            f["tokens"].append(tok_at(r.req, pos))
            f["positions"].append(pos)
            f["slots"].append(slot(r.req, pos))
        q += r.n
        f["p_qstart"].append(q)
        f["p_seqlen"].append(r.start + r.n)
        f["p_bt"] += [int(x) for x in table[r.req.table.index, :W]]
        last[id(r)] = q - 1
    Tp = q
    for i in range(Rd):
        f["d_tok"].append(Tp + i)
        if i < len(dr):
            r = dr[i]
            req = r.req
            f["tokens"].append(req.output[-1] if req.output else req.prompt[-1])
            f["positions"].append(r.start)
            f["slots"].append(slot(req, r.start))
            f["d_seqlen"].append(r.start + 1)
            f["d_bt"] += [int(x) for x in table[req.table.index, :W]]
            f["d_fwd"].append(r.fwd)
            last[id(r)] = Tp + i
        else:
            f["tokens"].append(0)
            f["positions"].append(0)
            f["slots"].append(-1)
            f["d_seqlen"].append(1)
            f["d_bt"] += [0] * W
            f["d_fwd"].append(-1)
    for r in plan.rows:
        if r.sample:
            sp = r.req.sampling
            f["s_idx"].append(last[id(r)])
            stoch = sp.mode.value == 1
            params.append((1 if stoch else 0, (sp.top_k or 0) if stoch else 0, sp.temperature if stoch else 1.0,
                           (sp.top_p if sp.top_p is not None else 1.0) if stoch else 1.0, sp.seed, r.sample_index))
    T = Tp + Rd
    for i in range(len(params), Rs):
        f["s_idx"].append(Tp + i)
        params.append((0, 0, 1.0, 1.0, 0, 0))
    return f, params, T


def drive(seed, overlap):
    """Yields (scheduler, plan) for every step of a random workload."""
    rng = random.Random(seed)
    cfg = SchedulerConfig(step_token_budget=96, max_active_requests=6, prefill_chunk_tokens=40,
                          emergency_decode_page_reserve=2, waiting_age_threshold_steps=5)
    s = Scheduler(cfg, CacheConfig(tokens_per_page=P, prefix_enabled=True), 40,
                  PrefixIdentity("m" * 64, "t", b"", P, 2), max_context=256)
    if overlap:
        s.max_inflight = 2
    shared = [rng.randrange(1, 90) for _ in range(2 * P)]
    for i in range(14):
        prompt = (shared if rng.random() < 0.5 else []) + [rng.randrange(1, 90) for _ in range(rng.randint(1, 60))]
        sp = (SamplingParameters.sample(0.7, top_k=rng.choice([None, 5]), top_p=rng.choice([None, 0.9]),
                                        seed=rng.randrange(1 << 40))
              if rng.random() < 0.5 else SamplingParameters())
        s.add_request(Request(rid=i + 1, prompt=prompt, max_new=rng.randint(1, 24), sampling=sp))
    pending = []
    steps = 0
    while s.has_work() and steps < 400:
        plan = s.schedule()
        if plan is not None:
            yield s, plan
            pending.append(plan)
        if pending and (plan is None or len(pending) >= s.max_inflight):
            done = pending.pop(0)
            s.complete(done, [rng.randrange(1, 90) for _ in done.sample_rows])
        steps += 1
        if rng.random() < 0.05 and s.running:
            s.cancel(rng.choice(s.running).rid)


@pytest.mark.parametrize("seed,overlap", [(0, False), (1, False), (2, True), (3, True), (4, False)])
def test_packed_block_matches_scalar_layout(seed, overlap):
    W = 16
    buf = np.full(1 << 14, 0x5A5A5A5A, dtype=np.int32)   # reused across steps: stale words must not leak
    n = 0
    for s, plan in drive(seed, overlap):
        table = s.tables.matrix
        hs = build_host_step(plan, table, P, W, buf)
        L = hs.layout
        want, params, T = scalar_pack(plan, table, W)
        assert L.T == T
        for name, vals in want.items():
            o, ln = L.field(name)
            assert ln == len(vals), name
            assert hs.buf[o:o + ln].tolist() == vals, (name, plan.seq)
            assert o % 4 == 0                                  # 16-byte aligned fields
        o, ln = L.field("s_params")
        got = hs.buf[o:o + ln].view(PARAM_DTYPE)
        exp = np.array(params, dtype=PARAM_DTYPE)
        assert np.array_equal(got, exp)
        check_paged_step(L, hs.buf, 41, P, vocab=100)
        assert hs.max_q_len == max([r.n for r in plan.rows if not r.decode], default=0)
        assert hs.any_forwarded == any(r.fwd >= 0 for r in plan.rows if r.decode)
        n += 1
    assert n > 20


def test_decode_bucket_padding():
    """A decode-only plan padded to a graph bucket: padded rows write the
    reserved zero page (slot -1), read length 1, sample the token after the
    real ones; the layout depends only on the bucket."""
    W = 16
    buf = np.zeros(1 << 14, dtype=np.int32)
    for s, plan in drive(7, False):
        if plan.prefill_rows or not plan.rows:
            continue
        bucket = len(plan.rows) + 3
        hs = build_host_step(plan, s.tables.matrix, P, W, buf, bucket=bucket)
        want, params, T = scalar_pack(plan, s.tables.matrix, W, bucket=bucket)
        assert hs.layout == make_layout(bucket, 0, bucket, bucket, W)
        for name, vals in want.items():
            o, ln = hs.layout.field(name)
            assert hs.buf[o:o + ln].tolist() == vals, name
        check_paged_step(hs.layout, hs.buf, 41, P)
        with pytest.raises(ValueError):
            build_host_step(type(plan)(plan.seq, plan.rows + [plan.rows[0].__class__(
                plan.rows[0].req, 0, 2, False, False, 0)]), s.tables.matrix, P, W, buf, bucket=bucket)
        return
    pytest.fail("no decode-only plan")


@pytest.mark.parametrize("length", [P - 1, P, P + 1, 2 * P, 2 * P + 1])
def test_page_boundary_lengths_need_exactly_ceil_pages(length):
    """A row of `length` tokens is packed with ceil(length / P) pages in its
    block table and admitted; with its last table entry cleared (a table one
    page short) the step is rejected."""
    from lunaflux_b200.ops.launch_contract import PagedIssue, PagedStepError
    cfg = SchedulerConfig(step_token_budget=64, max_active_requests=2, prefill_chunk_tokens=64)
    s = Scheduler(cfg, CacheConfig(tokens_per_page=P, prefix_enabled=False), 16, None, max_context=64)
    req = Request(rid=1, prompt=list(range(1, length + 1)), max_new=1, sampling=SamplingParameters())
    s.add_request(req)
    plan = s.schedule()
    assert len(req.pages) == -(-length // P)
    W = s.pages_per_request
    hs = build_host_step(plan, s.tables.matrix, P, W, np.zeros(4096, dtype=np.int32))
    check_paged_step(hs.layout, hs.buf, 17, P)
    o, _ = hs.layout.field("p_bt")
    hs.buf[o + len(req.pages) - 1] = 0
    with pytest.raises(PagedStepError) as e:
        check_paged_step(hs.layout, hs.buf, 17, P)
    assert e.value.issue is PagedIssue.SLOT
    assert PARAM_INTS == 8
