"""Radix prefix cache over full KV pages.

Reference: prefix/radix/index.mbt:11-406 and eviction.mbt:2.  Kept from the
reference: identity-rooted trees (model + plan digest, tokenizer digest,
cache scope, page layout) so entries never cross identities; only *full*
pages are stored or returned; per-entry active references; deterministic
least-recently-used eviction of entries with no active reference; the cache
holds a *cached* reference on every page it stores (page_allocator semantics).

Changed for throughput: the reference scans an uncompressed token trie
linearly (O(tokens x nodes)); here each edge is one page of tokens, children
are found by a dict keyed on that page's token tuple, so a lookup is O(pages)
and eviction pops leaves from a recency heap.  Unlike the reference, this
index is wired into the scheduler's admission path.

``PrefixIndex(allocator, ...)`` builds the C++ core (``_host.PrefixTree``,
which takes and drops its cached page references in the native allocator
directly) when the allocator is the native one, else ``PyPrefixIndex``, the
reference implementation the core is tested against.  Both return opaque
node handles from ``lookup``; ``pages_of`` maps them to their PageIds.
"""
from __future__ import annotations

import heapq
import itertools
from dataclasses import dataclass, field
from typing import Dict, Hashable, List, Optional, Sequence, Tuple

from ..kv.page_allocator import PageAllocator, PageId


@dataclass(frozen=True)
class PrefixIdentity:
    model_digest: str
    tokenizer_digest: str
    scope: bytes
    tokens_per_page: int
    layout_version: int


@dataclass(eq=False)
class _Node:
    key: Tuple[int, ...]
    page: Optional[PageId]
    parent: Optional["_Node"]
    children: Dict[Tuple[int, ...], "_Node"] = field(default_factory=dict)
    refs: int = 0
    recency: int = 0
    depth: int = 0


class PyPrefixIndex:
    def __init__(self, allocator: PageAllocator, tokens_per_page: int, max_pages: int = 1 << 30):
        self.allocator = allocator
        self.P = tokens_per_page
        self.max_pages = max_pages
        self._roots: Dict[PrefixIdentity, _Node] = {}
        self._clock = itertools.count(1)
        self._pages = 0
        self._heap: List[Tuple[int, int, _Node]] = []  # (recency, tiebreak, leaf) candidates
        self._tie = itertools.count()
        self.hits = 0
        self.lookups = 0
        self.hit_tokens = 0
        self.evicted_pages = 0

    def page_count(self) -> int:
        return self._pages

    def _root(self, ident: PrefixIdentity) -> _Node:
        if ident.tokens_per_page != self.P:
            raise ValueError("identity layout does not match this index")
        r = self._roots.get(ident)
        if r is None:
            r = self._roots[ident] = _Node((), None, None)
        return r

    def lookup(self, ident: PrefixIdentity, tokens: Sequence[int], max_pages: Optional[int] = None) -> List[_Node]:
        """Longest chain of cached full pages that prefixes ``tokens``.

        Returns the matched nodes (root excluded).  Callers that use them must
        call ``retain`` (and retain active references on the pages)."""
        self.lookups += 1
        node = self._root(ident)
        out = []
        n_full = len(tokens) // self.P
        if max_pages is not None:
            n_full = min(n_full, max_pages)
        now = next(self._clock)
        for i in range(n_full):
            key = tuple(tokens[i * self.P:(i + 1) * self.P])
            child = node.children.get(key)
            if child is None:
                break
            child.recency = now
            out.append(child)
            node = child
        if out:
            self.hits += 1
            self.hit_tokens += len(out) * self.P
            self._push_leaf(out[-1])
        return out

    def pages_of(self, nodes: Sequence[_Node]) -> List[PageId]:
        return [n.page for n in nodes]

    def retain(self, nodes: Sequence[_Node]):
        for n in nodes:
            n.refs += 1

    def release(self, nodes: Sequence[_Node]):
        for n in nodes:
            if n.refs <= 0:
                raise RuntimeError("prefix node released more often than retained")
            n.refs -= 1
            if n.refs == 0 and not n.children:
                self._push_leaf(n)

    def insert(self, ident: PrefixIdentity, tokens: Sequence[int], pages: Sequence[PageId]) -> int:
        """Publishes the full pages of a sequence.  Returns pages newly cached."""
        node = self._root(ident)
        n_full = min(len(tokens) // self.P, len(pages))
        added = 0
        now = next(self._clock)
        for i in range(n_full):
            key = tuple(tokens[i * self.P:(i + 1) * self.P])
            child = node.children.get(key)
            if child is None:
                if self._pages >= self.max_pages:
                    break
                self.allocator.retain_cached(pages[i])
                child = _Node(key, pages[i], node, depth=node.depth + 1)
                node.children[key] = child
                self._pages += 1
                added += 1
            child.recency = now
            node = child
        if node.parent is not None and not node.children:
            self._push_leaf(node)
        return added

    def _push_leaf(self, n: _Node):
        heapq.heappush(self._heap, (n.recency, next(self._tie), n))

    def evict(self, pages_needed: int) -> int:
        """Evicts least-recently-used unreferenced leaves until ``pages_needed``
        pages were released (or nothing evictable remains)."""
        freed = 0
        while freed < pages_needed and self._heap:
            rec, _, n = heapq.heappop(self._heap)
            if n.parent is None or n.children or n.refs > 0 or rec != n.recency:
                if n.parent is not None and not n.children and n.refs == 0 and rec != n.recency:
                    self._push_leaf(n)  # stale heap entry; re-queue with its current recency
                continue
            parent = n.parent
            del parent.children[n.key]
            n.parent = None
            self.allocator.release_cached(n.page)
            self._pages -= 1
            self.evicted_pages += 1
            freed += 1
            if parent.parent is not None and not parent.children and parent.refs == 0:
                self._push_leaf(parent)
        return freed

    def evictable_pages(self) -> int:
        cnt = 0
        stack = list(self._roots.values())
        while stack:
            n = stack.pop()
            stack.extend(n.children.values())
            if n.parent is not None and n.refs == 0:
                cnt += 1
        return cnt

    def debug_check_invariants(self):
        total = 0
        stack = [(r, 0) for r in self._roots.values()]
        while stack:
            n, d = stack.pop()
            if n.parent is not None:
                total += 1
                assert n.depth == d and len(n.key) == self.P
                assert self.allocator.cached_reference_count(n.page) >= 1
            for c in n.children.values():
                assert c.parent is n
                stack.append((c, d + 1))
        assert total == self._pages


class NativePrefixIndex:
    """The same index backed by the C++ core; node handles are ints."""

    def __init__(self, allocator, tokens_per_page: int, max_pages: int = 1 << 30):
        from .. import _host
        self._h = _host
        self.allocator = allocator
        self.P = tokens_per_page
        self.max_pages = max_pages
        self._c = _host.PrefixTree(allocator._c, tokens_per_page, max_pages)
        self._roots: Dict[PrefixIdentity, int] = {}

    def _call(self, fn, *a):
        try:
            return fn(*a)
        except self._h.PrefixError as e:
            raise RuntimeError(str(e)) from None
        except self._h.PageError as e:
            from ..kv.page_allocator import PageAllocatorError
            raise PageAllocatorError(str(e)) from None

    def _root(self, ident: PrefixIdentity) -> int:
        if ident.tokens_per_page != self.P:
            raise ValueError("identity layout does not match this index")
        r = self._roots.get(ident)
        if r is None:
            r = self._roots[ident] = self._c.new_root()
        return r

    @property
    def hits(self) -> int:
        return self._c.stats()[0]

    @property
    def lookups(self) -> int:
        return self._c.stats()[1]

    @property
    def hit_tokens(self) -> int:
        return self._c.stats()[2]

    @property
    def evicted_pages(self) -> int:
        return self._c.stats()[3]

    def page_count(self) -> int:
        return self._c.page_count()

    def lookup(self, ident: PrefixIdentity, tokens: Sequence[int], max_pages: Optional[int] = None) -> List[int]:
        return self._call(self._c.lookup, self._root(ident), tokens, -1 if max_pages is None else max(0, max_pages))

    def pages_of(self, nodes: Sequence[int]) -> List[PageId]:
        return [PageId(i, g) for i, g in self._call(self._c.pages_of, list(nodes))]

    def retain(self, nodes: Sequence[int]):
        self._call(self._c.retain, list(nodes))

    def release(self, nodes: Sequence[int]):
        self._call(self._c.release, list(nodes))

    def insert(self, ident: PrefixIdentity, tokens: Sequence[int], pages: Sequence[PageId]) -> int:
        return self._call(self._c.insert, self._root(ident), tokens, list(pages))

    def evict(self, pages_needed: int) -> int:
        return self._call(self._c.evict, pages_needed)

    def evictable_pages(self) -> int:
        return self._c.evictable_pages()

    def debug_check_invariants(self):
        self._call(self._c.debug_check_invariants)


def PrefixIndex(allocator, tokens_per_page: int, max_pages: int = 1 << 30):
    """The prefix index for `allocator`: the C++ core over the native page
    allocator (unless LUNAFLUX_HOST_CORE=python), else the Python class."""
    import os
    if hasattr(allocator, "_c") and hasattr(allocator, "_h") and os.environ.get("LUNAFLUX_HOST_CORE", "native") == "native":
        return NativePrefixIndex(allocator, tokens_per_page, max_pages)
    return PyPrefixIndex(allocator, tokens_per_page, max_pages)
