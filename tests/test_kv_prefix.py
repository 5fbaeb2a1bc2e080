"""Page allocator, block tables and the radix prefix index (CPU).

Randomised ownership model checking in the style of the reference's
kv/page_allocator/randomized_test.mbt: every operation is mirrored in a
plain model and ``debug_check_invariants`` runs after each one.
"""
import random

import pytest

from lunaflux_b200.kv.block_table import BlockTableArena, BlockTableError
from lunaflux_b200.kv.layout import KVLayout
from lunaflux_b200.kv.page_allocator import OutOfPages, PageAllocator, PageAllocatorError
from lunaflux_b200.prefix.radix import PrefixIdentity, PrefixIndex


def test_allocate_release_generations():
    a = PageAllocator(4)
    p = a.allocate_one()
    assert p.index == 1 and p.generation == 0
    a.release_active(p)
    with pytest.raises(PageAllocatorError):
        a.release_active(p)  # stale generation
    q = a.allocate_run(4)
    assert sorted(x.index for x in q) == [1, 2, 3, 4]
    assert [x for x in q if x.index == 1][0].generation == 1
    with pytest.raises(OutOfPages):
        a.allocate_one()
    a.debug_check_invariants()


def test_active_and_cached_refs():
    a = PageAllocator(2)
    p = a.allocate_one()
    a.retain_cached(p)
    a.release_active(p)
    assert a.free_page_count() == 1  # still cached
    a.retain_active(p)  # a prefix hit
    a.release_active(p)
    a.release_cached(p)
    assert a.free_page_count() == 2
    a.debug_check_invariants()


def test_terminal_generation_retires():
    a = PageAllocator(1, max_generation=2)
    for _ in range(3):
        a.release_active(a.allocate_one())
    assert a.retired_page_count() == 1 and a.free_page_count() == 0
    a.debug_check_invariants()


def test_checkpoint_rollback_restores_fifo():
    a = PageAllocator(5)
    first = a.allocate_run(2)
    a.release_active(first[0])
    order_before = list(a._free)
    tok = a.checkpoint()
    a.allocate_run(3)
    with pytest.raises(PageAllocatorError):
        a.release_active(first[1])  # refcounts frozen during a checkpoint
    a.rollback_to(tok)
    assert list(a._free) == order_before
    a.debug_check_invariants()
    tok = a.checkpoint()
    got = a.allocate_run(2)
    a.commit_checkpoint(tok)
    assert all(a.validate_active(p) for p in got)


def test_randomized_ownership():
    rng = random.Random(0)
    a = PageAllocator(32, max_generation=50)
    live = []  # (pid, active, cached)
    for _ in range(3000):
        op = rng.random()
        if op < 0.35 and a.free_page_count():
            n = rng.randint(1, min(4, a.free_page_count()))
            for p in a.allocate_run(n):
                live.append([p, 1, 0])
        elif op < 0.55 and live:
            e = rng.choice(live)
            a.retain_active(e[0])
            e[1] += 1
        elif op < 0.7 and live:
            e = rng.choice(live)
            a.retain_cached(e[0])
            e[2] += 1
        elif live:
            e = rng.choice(live)
            if e[1] and (not e[2] or rng.random() < 0.5):
                a.release_active(e[0])
                e[1] -= 1
            elif e[2]:
                a.release_cached(e[0])
                e[2] -= 1
            if e[1] == 0 and e[2] == 0:
                live.remove(e)
                assert not a.validate_active(e[0])
        a.debug_check_invariants()
        assert a.allocated_page_count() == len(live)


def test_block_table_matrix_and_truncate():
    a = PageAllocator(10)
    t = BlockTableArena(2, 4, 16)
    tid = t.allocate()
    pids = a.allocate_run(3)
    t.append_pages(tid, pids)
    assert list(t.matrix[tid.index, :3]) == [p.index for p in pids]
    assert t.resolve_token_position(tid, 17) == (pids[1].index, 1)
    with pytest.raises(BlockTableError):
        t.append_pages(tid, a.allocate_run(2))
    t.truncate(tid, 1, a)
    assert t.page_count(tid) == 1 and t.matrix[tid.index, 1] == 0
    t.reset_and_release(tid, a)
    with pytest.raises(BlockTableError):
        t.page_count(tid)


def test_block_table_checkpoint_rollback():
    a = PageAllocator(10)
    t = BlockTableArena(1, 8, 16)
    tid = t.allocate()
    t.append_pages(tid, a.allocate_run(2))
    t.checkpoint()
    t.note(tid)
    t.append_pages(tid, a.allocate_run(3))
    t.rollback()
    assert t.page_count(tid) == 2 and t.matrix[tid.index, 2] == 0


def ident(scope=b"", P=4):
    return PrefixIdentity("m" * 64, "t", scope, P, 2)


def test_radix_lookup_insert_full_pages_only():
    a = PageAllocator(16)
    idx = PrefixIndex(a, 4)
    toks = list(range(10))
    pids = a.allocate_run(3)
    assert idx.insert(ident(), toks, pids) == 2  # only 2 full pages of 4
    assert idx.page_count() == 2
    hit = idx.lookup(ident(), list(range(8)) + [99])
    assert idx.pages_of(hit) == pids[:2]
    assert idx.lookup(ident(b"other"), toks) == []  # identity salting
    assert idx.lookup(ident(), [1] + toks) == []
    idx.debug_check_invariants()


def test_radix_lru_eviction_skips_referenced():
    a = PageAllocator(8)
    idx = PrefixIndex(a, 2)
    p1 = a.allocate_run(2)
    p2 = a.allocate_run(2)
    idx.insert(ident(P=2), [1, 2, 3, 4], p1)
    idx.insert(ident(P=2), [9, 9, 8, 8], p2)
    for p in p1 + p2:
        a.release_active(p)  # only the cache owns them now
    nodes = idx.lookup(ident(P=2), [1, 2, 3, 4])
    idx.retain(nodes)
    freed = idx.evict(10)
    assert freed == 2  # only the unreferenced chain [9,9],[8,8]
    assert a.free_page_count() == 6
    idx.release(nodes)
    assert idx.evict(10) == 2
    assert a.free_page_count() == 8
    idx.debug_check_invariants()


def test_kv_layout_offsets():
    L = KVLayout(layers=2, kv_heads=8, tokens_per_page=16, head_dim=128)
    assert L.bytes_per_page == 2 * 2 * 8 * 16 * 128 * 2
    assert L.element_offset(10, 0, 0, 0, 0, 0, 1) == 1
    assert L.element_offset(10, 0, 0, 1, 0, 0, 0) == 8 * 16 * 128
    with pytest.raises(IndexError):
        L.element_offset(10, 0, 2, 0, 0, 0, 0)


def _prefix_classes():
    from lunaflux_b200.prefix import radix
    out = [radix.PyPrefixIndex]
    try:
        from lunaflux_b200 import _host  # noqa: F401
        out.append(radix.NativePrefixIndex)
    except ImportError:
        pass
    return out


@pytest.mark.parametrize("cls", _prefix_classes(), ids=lambda c: c.__name__)
@pytest.mark.parametrize("seed", range(4))
def test_radix_matches_a_path_model_with_lru_eviction(cls, seed):
    """Model check of the prefix index (reference: prefix/radix/index.mbt and
    eviction.mbt): the cached set is a prefix-closed set of page paths;
    lookup returns the longest cached path (its pages are the ones first
    inserted for it); evicting one page removes the least recently used
    unreferenced leaf; every cached page holds exactly one cached reference
    and is freed when evicted."""
    rng = random.Random(seed)
    P = 2
    a = PageAllocator(4096)
    idx = cls(a, P)
    idn = ident(P=P)
    model = {}       # path (tuple of page keys) -> page
    recency = {}     # path -> last touch
    refs = {}        # path -> retain count
    held = []        # (nodes, paths) retained by "requests"
    clock = 0

    def paths_of(tokens, n):
        return [tuple(tuple(tokens[j * P:(j + 1) * P]) for j in range(i + 1)) for i in range(n)]

    for _ in range(400):
        op = rng.random()
        toks = [rng.randrange(3) for _ in range(rng.randrange(1, 11))]
        full = len(toks) // P
        if op < 0.4:
            pages = a.allocate_run(full) if full else []
            clock += 1
            added = idx.insert(idn, toks, pages)
            new = 0
            for p, pid in zip(paths_of(toks, full), pages):
                if p not in model:
                    model[p] = pid
                    new += 1
                recency[p] = clock
            assert added == new
            for pid in pages:
                a.release_active(pid)        # the cache (if it took the page) is the only owner now
        elif op < 0.7:
            clock += 1
            nodes = idx.lookup(idn, toks)
            want = 0
            for p in paths_of(toks, full):
                if p not in model:
                    break
                want += 1
                recency[p] = clock
            assert len(nodes) == want
            ps = paths_of(toks, want)
            assert idx.pages_of(nodes) == [model[p] for p in ps]
            if nodes and rng.random() < 0.5:
                idx.retain(nodes)
                for p in ps:
                    refs[p] = refs.get(p, 0) + 1
                held.append((nodes, ps))
        elif op < 0.85 and held:
            nodes, ps = held.pop(rng.randrange(len(held)))
            idx.release(nodes)
            for p in ps:
                refs[p] -= 1
        else:
            leaves = [p for p in model if refs.get(p, 0) == 0
                      and not any(q[:len(p)] == p and len(q) > len(p) for q in model)]
            freed = idx.evict(1)
            if not leaves:
                assert freed == 0
                continue
            assert freed == 1
            oldest = min(leaves, key=lambda p: recency[p])
            del model[oldest]
            recency.pop(oldest)
            # every other leaf is still there (each probe is a lookup: it touches the path)
            for p in leaves:
                clock += 1
                got = len(idx.lookup(idn, [t for k in p for t in k]))
                assert got == (len(p) - 1 if p == oldest else len(p)), (p, oldest)
                for i in range(1, got + 1):
                    recency[p[:i]] = clock
        idx.debug_check_invariants()
        a.debug_check_invariants()
        assert idx.page_count() == len(model)
        assert a.free_page_count() == a.capacity - len(model)
