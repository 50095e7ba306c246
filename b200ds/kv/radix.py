"""Radix prefix cache over whole KV pages.

Keys are token ids in page-sized chunks; each tree node owns one page.  A
new request matches the longest cached page-aligned prefix, retains those
pages and prefills only the rest.  Finished requests insert their full pages;
unreferenced leaves are evicted LRU when the pool runs short.

With a host tier (kv/host_cache.py) eviction moves a page to host memory
and keeps its node (page -1, host_page set); matching such a node copies it
back into a new device page.  Device-resident nodes stay prefix-closed: a
node is moved out only when none of its children is on the device, and
matching restores nodes root first.  When the host tier is full its LRU
host-only leaves are dropped.

Reference parity: radix caching lives in SGLang (absent from the
reference); this is the engine's own.
"""
from __future__ import annotations

import itertools
from typing import Dict, List, Optional, Tuple

from .pool import PagePool


class _Node:
    __slots__ = ("key", "page", "host_page", "children", "parent", "last_use", "locks")

    def __init__(self, key: Tuple[int, ...], page: int, parent: Optional["_Node"]):
        self.key = key
        self.page = page            # device page, -1 while the page lives in the host tier
        self.host_page = -1
        self.children: Dict[Tuple[int, ...], _Node] = {}
        self.parent = parent
        self.last_use = 0
        self.locks = 0


class RadixCache:
    def __init__(self, pool: PagePool, host=None):
        self.pool = pool
        self.ps = pool.page_size
        self.host = host            # HostKVPool or None
        self.root = _Node((), -1, None)
        self._clock = itertools.count(1)
        self.num_nodes = 0
        self.offloads = 0           # pages moved to the host tier
        self.restores = 0           # pages copied back for a match

    def _chunks(self, tokens: List[int]):
        n = len(tokens) // self.ps
        return [tuple(tokens[i * self.ps:(i + 1) * self.ps]) for i in range(n)]

    def match(self, tokens: List[int]) -> Tuple[List[int], List[_Node]]:
        """Longest cached page-aligned prefix: (pages, nodes).  The pages are
        retained for the caller; release with :meth:`unlock`."""
        node = self.root
        pages, nodes = [], []
        t = next(self._clock)
        for ch in self._chunks(tokens):
            nxt = node.children.get(ch)
            if nxt is None or (nxt.page < 0 and not self._restore(nxt)):
                break
            nxt.last_use = t
            nxt.locks += 1
            pages.append(nxt.page)
            nodes.append(nxt)
            node = nxt
        self.pool.retain(pages)
        return pages, nodes

    def _restore(self, n: _Node) -> bool:
        """Bring a host-tier node back into a device page (False when none
        can be had).  Its ancestors are on the device and locked by the
        caller's match, so eviction here cannot take them."""
        if self.host is None or n.host_page < 0:
            return False
        if self.pool.num_free == 0 and self.evict(1) == 0:
            return False
        gp = self.pool.alloc(1)[0]          # the tree's reference
        self.host.restore(n.host_page, gp)
        self.host.free(n.host_page)
        n.page, n.host_page = gp, -1
        self.restores += 1
        return True

    def match_len(self, tokens: List[int]) -> int:
        """Pages of the longest cached prefix, without retaining them or
        touching their recency (for scheduling decisions)."""
        node, n = self.root, 0
        for ch in self._chunks(tokens):
            node = node.children.get(ch)
            if node is None:
                break
            n += 1
        return n

    def unlock(self, nodes: List[_Node]) -> None:
        for n in nodes:
            n.locks -= 1
        self.pool.release([n.page for n in nodes])

    def insert(self, tokens: List[int], pages: List[int]) -> None:
        """Insert the full pages of a finished sequence (tokens covering
        len(pages)*page_size at least).  The tree takes its own reference."""
        node = self.root
        t = next(self._clock)
        for ch, pg in zip(self._chunks(tokens), pages):
            nxt = node.children.get(ch)
            if nxt is None:
                nxt = _Node(ch, pg, node)
                node.children[ch] = nxt
                self.pool.retain([pg])
                self.num_nodes += 1
            elif nxt.page < 0:              # the host copy is superseded by this device page
                nxt.page = pg
                self.pool.retain([pg])
                self.host.free(nxt.host_page)
                nxt.host_page = -1
            nxt.last_use = t
            node = nxt

    def evict(self, need_pages: int) -> int:
        """Free up to need_pages device pages from unlocked nodes none of
        whose children is on the device (LRU): moved to the host tier when
        there is one (dropping LRU host-only leaves to make room), else
        dropped with their host-only descendants."""
        freed = 0
        while freed < need_pages:
            cands = [n for n in self._iter() if n is not self.root and n.page >= 0 and n.locks == 0
                     and all(c.page < 0 for c in n.children.values())]
            if not cands:
                break
            cands.sort(key=lambda n: n.last_use)
            for n in cands:
                if freed >= need_pages:
                    break
                if self.host is not None and self._host_room():
                    n.host_page = self.host.offload(n.page)
                    self.offloads += 1
                    self.pool.release([n.page])
                    n.page = -1
                else:
                    self._drop(n)
                freed += 1
        return freed

    def _host_room(self) -> bool:
        """A free host page, dropping the LRU host-only leaf if needed."""
        if self.host.num_free > 0:
            return True
        leaves = [n for n in self._iter() if n is not self.root and n.page < 0 and not n.children]
        if not leaves:
            return False
        self._drop(min(leaves, key=lambda n: n.last_use))
        return True

    def _drop(self, n: _Node) -> None:
        """Remove n and its (host-only) subtree from the tree."""
        stack = [n]
        while stack:
            m = stack.pop()
            stack.extend(m.children.values())
            if m.page >= 0:
                self.pool.release([m.page])
            elif m.host_page >= 0:
                self.host.free(m.host_page)
            self.num_nodes -= 1
        del n.parent.children[n.key]

    def clear(self) -> int:
        """Drop every node (none may be locked); returns the device pages
        released."""
        freed = 0
        for n in list(self._iter()):
            if n is self.root:
                continue
            assert n.locks == 0, "clear() with a locked prefix"
            if n.page >= 0:
                self.pool.release([n.page])
                freed += 1
            elif n.host_page >= 0:
                self.host.free(n.host_page)
        self.root.children = {}
        self.num_nodes = 0
        return freed

    def _iter(self):
        stack = [self.root]
        while stack:
            n = stack.pop()
            yield n
            stack.extend(n.children.values())
