"""The C++ block-table and radix prefix cores against their Python reference
implementations: the same random operation sequences on both, every result,
error and counter compared (reference semantics: kv/block_table/arena.mbt,
prefix/radix/index.mbt and eviction.mbt)."""
import random

import numpy as np
import pytest

from lunaflux_b200.kv.block_table import (BlockTableError, NativeBlockTableArena, PyBlockTableArena)
from lunaflux_b200.kv.page_allocator import (NativePageAllocator, OutOfPages, PageAllocatorError, PageId,
                                             PyPageAllocator, native_available)
from lunaflux_b200.prefix.radix import NativePrefixIndex, PrefixIdentity, PrefixIndex, PyPrefixIndex

pytestmark = pytest.mark.skipif(not native_available(), reason="host extension not built")


def _both(fn_py, fn_nat):
    """Runs both; returns (result_py, result_nat) or the pair of exception types."""
    out = []
    for fn in (fn_py, fn_nat):
        try:
            out.append(("ok", fn()))
        except (BlockTableError, PageAllocatorError, OutOfPages, RuntimeError, ValueError) as e:
            out.append(("err", type(e).__name__))
    return out


@pytest.mark.parametrize("seed", range(6))
def test_block_tables_differential_random(seed):
    rng = random.Random(seed)
    ap, an = PyPageAllocator(64), NativePageAllocator(64)
    tp, tn = PyBlockTableArena(5, 9, 4), NativeBlockTableArena(5, 9, 4)
    live = []                                       # (tid_py, tid_nat)
    ckpt = False
    for step in range(600):
        op = rng.choice(["alloc", "alloc", "append", "append", "append", "truncate", "reset", "release", "query",
                         "ckpt", "rollback", "commit"])
        if op == "alloc":
            rp, rn = _both(tp.allocate, tn.allocate)
            assert rp[0] == rn[0]
            if rp[0] == "ok":
                assert tuple(rp[1]) == tuple(rn[1])
                live.append((rp[1], rn[1]))
        elif op in ("append", "truncate", "reset", "release", "query") and live:
            i = rng.randrange(len(live))
            a, b = live[i]
            if op == "append":
                n = rng.randint(0, 4)
                if ckpt:
                    tp.note(a)
                    tn.note(b)
                if ap.free_page_count() < n:
                    continue
                pp, pn = ap.allocate_run(n), an.allocate_run(n)
                assert pp == pn
                rp, rn = _both(lambda: tp.append_pages(a, pp), lambda: tn.append_pages(b, pn))
                assert rp[0] == rn[0]
                if rp[0] == "err":
                    for p in pp:
                        ap.release_active(p)
                    for p in pn:
                        an.release_active(p)
            elif op == "truncate" and not ckpt:
                keep = rng.randint(0, 9)
                rp, rn = _both(lambda: tp.truncate(a, keep, ap), lambda: tn.truncate(b, keep, an))
                assert rp == rn
            elif op == "reset" and not ckpt:
                rp, rn = _both(lambda: tp.reset_and_release(a, ap), lambda: tn.reset_and_release(b, an))
                assert rp == rn
                live.pop(i)
            elif op == "release":
                rp, rn = _both(lambda: tp.release(a), lambda: tn.release(b))
                assert rp[0] == rn[0]
                if rp[0] == "ok":
                    live.pop(i)
            elif op == "query":
                assert tp.page_count(a) == tn.page_count(b)
                assert tp.pages(a) == tn.pages(b)
                pos = rng.randint(0, 40)
                rp, rn = _both(lambda: tuple(tp.resolve_token_position(a, pos)),
                               lambda: tuple(tn.resolve_token_position(b, pos)))
                assert rp == rn
        elif op == "ckpt" and not ckpt:
            tp.checkpoint()
            tn.checkpoint()
            ckpt = True
        elif op == "rollback" and ckpt:
            tp.rollback()
            tn.rollback()
            ckpt = False
        elif op == "commit" and ckpt:
            tp.commit_checkpoint()
            tn.commit_checkpoint()
            ckpt = False
        assert np.array_equal(tp.matrix, tn.matrix)
        assert tp.free_table_count() == tn.free_table_count()
        assert ap.free_page_count() == an.free_page_count()
    tn.debug_check_invariants()


def test_block_table_stale_ids_and_matrix_view():
    a = NativePageAllocator(8)
    t = NativeBlockTableArena(2, 4, 16)
    tid = t.allocate()
    t.append_pages(tid, a.allocate_run(3))
    assert list(t.matrix[tid.index, :4]) == [p.index for p in t.pages(tid)] + [0]
    with pytest.raises(BlockTableError):
        t.append_pages(tid, a.allocate_run(2))           # 5 pages > 4
    with pytest.raises(BlockTableError):
        t.release(tid)                                     # still owns pages
    t.reset_and_release(tid, a)
    with pytest.raises(BlockTableError):
        t.page_count(tid)                                  # stale generation
    assert tuple(t.allocate()) == (0, 1)                   # the slot comes back one generation on
    m = t.matrix
    del t
    assert m.sum() == 0                                    # the view keeps the core alive


def _ident(scope=b"", P=4):
    return PrefixIdentity("m" * 64, "t", scope, P, 2)


@pytest.mark.parametrize("seed", range(8))
def test_prefix_index_differential_random(seed):
    """Inserts / lookups / retains / releases / evictions over a small token
    alphabet (so sequences share prefixes and keys collide in content), on
    the Python index over the Python allocator and the C++ index over the C++
    allocator: the matched pages, eviction counts (hence LRU order), page
    counts, statistics and the allocators' free queues agree at every step."""
    rng = random.Random(seed)
    P = 2
    ap, an = PyPageAllocator(200), NativePageAllocator(200)
    ip, inn = PyPrefixIndex(ap, P, max_pages=60), NativePrefixIndex(an, P, max_pages=60)
    held = []   # (nodes_py, nodes_nat)
    scopes = [b"", b"s"]
    for step in range(800):
        op = rng.choice(["insert", "insert", "lookup", "lookup", "release", "evict"])
        ident = _ident(rng.choice(scopes), P)
        if op == "insert":
            L = rng.randint(0, 12)
            toks = [rng.randint(0, 2) for _ in range(L)]
            n = min(rng.randint(0, L // P + 1), an.free_page_count())
            pp, pn = ap.allocate_run(n), an.allocate_run(n)
            assert pp == pn
            assert ip.insert(ident, toks, pp) == inn.insert(ident, toks, pn)
            for p in pp:
                ap.release_active(p)       # the cache (if it took them) is now the only owner
            for p in pn:
                an.release_active(p)
        elif op == "lookup":
            L = rng.randint(0, 12)
            toks = [rng.randint(0, 2) for _ in range(L)]
            mp = rng.choice([None, 0, 1, 3])
            a, b = ip.lookup(ident, toks, mp), inn.lookup(ident, np.asarray(toks, dtype=np.int32), mp)
            assert ip.pages_of(a) == inn.pages_of(b)
            if a and rng.random() < 0.5:
                ip.retain(a)
                inn.retain(b)
                held.append((a, b))
        elif op == "release" and held:
            a, b = held.pop(rng.randrange(len(held)))
            ip.release(a)
            inn.release(b)
        elif op == "evict":
            k = rng.randint(0, 6)
            assert ip.evict(k) == inn.evict(k)
        assert ip.page_count() == inn.page_count()
        assert (ip.hits, ip.lookups, ip.hit_tokens, ip.evicted_pages) == \
            (inn.hits, inn.lookups, inn.hit_tokens, inn.evicted_pages)
        assert list(ap._free) == list(an._free)
        if step % 50 == 0:
            ip.debug_check_invariants()
            inn.debug_check_invariants()
            assert ip.evictable_pages() == inn.evictable_pages()
    for a, b in held:
        ip.release(a)
        inn.release(b)
    assert ip.evict(1 << 20) == inn.evict(1 << 20)
    assert ip.page_count() == inn.page_count() == 0
    assert ap.free_page_count() == an.free_page_count() == 200


def test_prefix_index_errors_and_selection():
    an = NativePageAllocator(16)
    idx = PrefixIndex(an, 4)
    assert isinstance(idx, NativePrefixIndex)
    assert isinstance(PrefixIndex(PyPageAllocator(16), 4), PyPrefixIndex)
    pids = an.allocate_run(2)
    idx.insert(_ident(), list(range(8)), pids)
    nodes = idx.lookup(_ident(), list(range(8)))
    assert idx.pages_of(nodes) == pids
    with pytest.raises(RuntimeError):
        idx.release(nodes)                  # never retained
    with pytest.raises(ValueError):
        idx.lookup(_ident(P=8), list(range(8)))
    for p in pids:
        an.release_active(p)
    assert idx.evict(5) == 2
    with pytest.raises(RuntimeError):
        idx.pages_of(nodes)                 # evicted handles are stale
    assert an.free_page_count() == 16
