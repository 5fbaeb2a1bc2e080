"""Page allocator failure contract, run on the Python reference and the C++
core alike: every rejected operation leaves the allocator exactly as it was
(free FIFO order, counts, reference counts).  Reference:
kv/page_allocator/allocator_test.mbt ('exact run failure leaves allocator
and reusable output unchanged', 'reference underflow overflow and double
release do not mutate ownership', 'checkpoint authentication rejects wrong
stale duplicate and nested use', 'allocation rollback restores several runs
atomically', 'limits reject unbounded and inconsistent construction')."""
import pytest

from lunaflux_b200.kv.page_allocator import (NativePageAllocator, OutOfPages, PageAllocatorError, PageId,
                                             PyPageAllocator, native_available)

IMPLS = [PyPageAllocator] + ([NativePageAllocator] if native_available() else [])


def snapshot(a, ids):
    return (list(a._free), a.free_page_count(), a.allocated_page_count(), a.retired_page_count(),
            [(a.active_reference_count(p) if a.validate_active(p) else -1) for p in ids])


def rejected(a, ids, fn, *args, exc=PageAllocatorError):
    before = snapshot(a, ids)
    with pytest.raises(exc):
        fn(*args)
    assert snapshot(a, ids) == before
    a.debug_check_invariants()


@pytest.fixture(params=IMPLS, ids=lambda c: c.__name__)
def impl(request):
    return request.param


def test_run_failure_is_transactional(impl):
    a = impl(6)
    held = a.allocate_run(4)
    a.release_active(held[1])
    rejected(a, held, a.allocate_run, 4, exc=OutOfPages)      # 3 free
    rejected(a, held, a.allocate_run, -1)
    assert a.allocate_run(0) == []
    got = a.allocate_run(3)                                   # exactly what is free
    assert len(got) == 3 and a.free_page_count() == 0
    rejected(a, held + got, a.allocate_one, exc=OutOfPages)


def test_reference_underflow_overflow_and_double_release(impl):
    a = impl(4, max_active_refs=2, max_cached_refs=1)
    p = a.allocate_one()
    q = a.allocate_one()
    a.retain_active(p)                                        # 2 active: the limit
    rejected(a, [p, q], a.retain_active, p)
    a.retain_cached(p)
    rejected(a, [p, q], a.retain_cached, p)
    rejected(a, [p, q], a.release_cached, q)                  # no cached reference
    a.release_active(q)
    rejected(a, [p, q], a.release_active, q)                  # double release: stale now
    a.release_active(p)
    a.release_active(p)
    assert a.active_reference_count(p) == 0 and a.cached_reference_count(p) == 1
    rejected(a, [p], a.release_active, p)                     # underflow while still cached
    a.release_cached(p)
    assert a.free_page_count() == 4


def test_stale_and_foreign_ids(impl):
    a = impl(3)
    p = a.allocate_one()
    a.release_active(p)
    p2 = a.allocate_one() if a._free[0] == p.index - a.first_index else None
    ids = [p] + ([p2] if p2 else [])
    for bad in (p, PageId(0, 0), PageId(a.first_index + 3, 0), PageId(-1, 0), PageId(p.index, p.generation + 7)):
        if p2 is not None and bad == p2:
            continue
        rejected(a, ids, a.retain_active, bad)
        rejected(a, ids, a.release_active, bad)
        rejected(a, ids, a.retain_cached, bad)
        assert not a.validate_active(bad)


def test_checkpoint_authentication(impl):
    a = impl(6)
    base = a.allocate_run(2)
    t = a.checkpoint()
    rejected(a, base, a.checkpoint)                           # nested
    rejected(a, base, a.commit_checkpoint, t + 1)             # wrong token
    rejected(a, base, a.rollback_to, t - 1)
    rejected(a, base, a.retain_active, base[0])               # counts frozen while open
    rejected(a, base, a.release_active, base[0])
    a.commit_checkpoint(t)
    rejected(a, base, a.commit_checkpoint, t)                 # consumed
    rejected(a, base, a.rollback_to, t)
    t2 = a.checkpoint()
    assert t2 != t                                            # a token is never reused
    a.rollback_to(t2)


def test_rollback_restores_several_runs_atomically(impl):
    a = impl(8)
    keep = a.allocate_run(3)
    a.release_active(keep[0])
    a.release_active(keep[2])
    before = snapshot(a, keep)
    gens = {}
    t = a.checkpoint()
    runs = [a.allocate_run(2), [a.allocate_one()], a.allocate_run(3)]
    for r in runs:
        for pid in r:
            gens[pid.index] = pid.generation
    assert a.free_page_count() == 1                           # 8 - 1 held - 6 provisional
    a.rollback_to(t)
    assert snapshot(a, keep) == before
    for r in runs:
        for pid in r:
            assert not a.validate_active(pid)
    # the same slots come back in the same order, at the same generations
    again = a.allocate_run(6)
    assert [(p.index, p.generation) for p in again] == [(p.index, p.generation) for r in runs for p in r]
    a.debug_check_invariants()


@pytest.mark.parametrize("cap", [0, -4])
def test_construction_limits(impl, cap):
    with pytest.raises((PageAllocatorError, ValueError)):
        impl(cap)


# ----------------------------------------------------------------- block tables
# Reference: kv/block_table/arena_test.mbt ('append failures are
# transactional', 'truncate preflight preserves table and reusable output',
# 'dense mapping resolves exact logical pages and token offsets').

from lunaflux_b200.kv.block_table import BlockTableError, NativeBlockTableArena, PyBlockTableArena  # noqa: E402

TABLES = [PyBlockTableArena] + ([NativeBlockTableArena] if native_available() else [])


@pytest.fixture(params=[(t, a) for t in TABLES for a in IMPLS], ids=lambda p: f"{p[0].__name__}-{p[1].__name__}")
def arena_alloc(request):
    t, a = request.param
    return t(4, 4, tokens_per_page=16), a(16)


def table_state(bt, tid):
    return bt.pages(tid), bt.matrix[tid.index].tolist()


def test_table_bounds_checks(arena_alloc):
    bt, a = arena_alloc
    tid = bt.allocate()
    pages = a.allocate_run(3)
    bt.append_pages(tid, pages)
    assert bt.page_at(tid, 2) == pages[2]
    assert bt.resolve_token_position(tid, 47) == (pages[2].index, 15)
    for bad in (-1, 3):
        with pytest.raises(BlockTableError):
            bt.page_at(tid, bad)
    for bad in (-1, -16, 48):
        with pytest.raises(BlockTableError):
            bt.resolve_token_position(tid, bad)
    before = table_state(bt, tid)
    with pytest.raises(BlockTableError):
        bt.append_pages(tid, a.allocate_run(2))          # 3 + 2 > 4
    with pytest.raises(BlockTableError):
        bt.truncate(tid, -1, a)
    assert table_state(bt, tid) == before
    assert bt.truncate(tid, 5, a) == [] and table_state(bt, tid) == before


def test_truncate_preflight_keeps_table_and_allocator(arena_alloc):
    bt, a = arena_alloc
    tid = bt.allocate()
    pages = a.allocate_run(3)
    bt.append_pages(tid, pages)
    ids = list(pages)
    # the last page lost its active reference elsewhere: releasing it would fail
    a.retain_cached(pages[2])
    a.release_active(pages[2])
    before = (table_state(bt, tid), snapshot(a, ids[:2]), a.cached_reference_count(pages[2]))
    with pytest.raises(PageAllocatorError):
        bt.truncate(tid, 1, a)
    assert (table_state(bt, tid), snapshot(a, ids[:2]), a.cached_reference_count(pages[2])) == before
    # counts frozen by an open allocator checkpoint: also refused up front
    a.retain_active(pages[2])
    t = a.checkpoint()
    with pytest.raises(PageAllocatorError):
        bt.truncate(tid, 0, a)
    a.rollback_to(t)
    assert bt.pages(tid) == pages
    # a valid truncate releases exactly the dropped pages
    assert bt.truncate(tid, 1, a) == pages[1:]
    assert a.validate_active(pages[0]) and not a.validate_active(pages[1])
    assert bt.matrix[tid.index].tolist() == [pages[0].index, 0, 0, 0]
    bt.reset_and_release(tid, a)
    a.release_cached(pages[2])
    assert a.free_page_count() == 16 and bt.free_table_count() == 4
