"""The C++ host cores against their Python reference implementations."""
import random

import pytest

from lunaflux_b200.kv.page_allocator import (NativePageAllocator, OutOfPages, PageAllocatorError, PyPageAllocator,
                                             native_available)

pytestmark = pytest.mark.skipif(not native_available(), reason="host extension not built")


def test_allocator_differential_random():
    rng = random.Random(7)
    a = PyPageAllocator(24, max_generation=40)
    b = NativePageAllocator(24, max_generation=40)
    live = []
    for step in range(4000):
        op = rng.random()
        if op < 0.05 and a._ckpt is None:
            ta, tb = a.checkpoint(), b.checkpoint()
            n = rng.randint(0, min(3, a.free_page_count()))
            got = a.allocate_run(n)
            assert got == b.allocate_run(n)
            if rng.random() < 0.5:
                a.rollback_to(ta)
                b.rollback_to(tb)
            else:
                a.commit_checkpoint(ta)
                b.commit_checkpoint(tb)
                live.extend([p, 1, 0] for p in got)  # committed pages are owned now
        elif op < 0.35:
            n = rng.randint(1, 4)
            ea = eb = None
            try:
                ra = a.allocate_run(n)
            except OutOfPages:
                ea = True
            try:
                rb = b.allocate_run(n)
            except OutOfPages:
                eb = True
            assert ea == eb
            if not ea:
                assert ra == rb
                live.extend([p, 1, 0] for p in ra)
        elif live:
            e = rng.choice(live)
            kind = rng.choice(["ra", "rc", "xa", "xc"])
            try:
                if kind == "ra":
                    a.retain_active(e[0])
                    b.retain_active(e[0])
                    e[1] += 1
                elif kind == "rc":
                    a.retain_cached(e[0])
                    b.retain_cached(e[0])
                    e[2] += 1
                elif kind == "xa" and e[1]:
                    a.release_active(e[0])
                    b.release_active(e[0])
                    e[1] -= 1
                elif kind == "xc" and e[2]:
                    a.release_cached(e[0])
                    b.release_cached(e[0])
                    e[2] -= 1
            except PageAllocatorError:
                pytest.fail("unexpected allocator error")
            if e[1] == 0 and e[2] == 0:
                live.remove(e)
                assert not a.validate_active(e[0]) and not b.validate_active(e[0])
        assert (a.free_page_count(), a.allocated_page_count(), a.retired_page_count()) == \
            (b.free_page_count(), b.allocated_page_count(), b.retired_page_count())
        assert list(a._free) == list(b._free)
        b.debug_check_invariants()
    from lunaflux_b200.kv.page_allocator import PageId
    with pytest.raises(PageAllocatorError):
        b.release_active(PageId(10_000, 0))


def test_bpe_native_equals_reference():
    from lunaflux_b200.tokenizer.bpe import Tokenizer
    from .test_tokenizer import MERGES, make_json
    text, _ = make_json(MERGES + [("a", "a"), ("aa", "a"), ("e", "l")])
    tok = Tokenizer.from_json(text)
    assert tok._native is not None
    rng = random.Random(0)
    alphabet = b"unrelated aaaa el\x00\xc3\xa9"
    for _ in range(300):
        data = bytes(rng.choice(alphabet) for _ in range(rng.randint(0, 60)))
        assert tok._bpe(data) == tok._bpe_reference(data)
