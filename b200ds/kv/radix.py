"""Radix prefix cache over whole KV pages.

Keys are token ids in page-sized chunks; each tree node owns one page.  A
new request matches the longest cached page-aligned prefix, retains those
pages and prefills only the rest.  Finished requests insert their full pages;
unreferenced leaves are evicted LRU when the pool runs short.

Reference parity: radix caching lives in SGLang (absent from the
reference); this is the engine's own.
"""
from __future__ import annotations

import itertools
from typing import Dict, List, Optional, Tuple

from .pool import PagePool


class _Node:
    __slots__ = ("key", "page", "children", "parent", "last_use", "locks")

    def __init__(self, key: Tuple[int, ...], page: int, parent: Optional["_Node"]):
        self.key = key
        self.page = page
        self.children: Dict[Tuple[int, ...], _Node] = {}
        self.parent = parent
        self.last_use = 0
        self.locks = 0


class RadixCache:
    def __init__(self, pool: PagePool):
        self.pool = pool
        self.ps = pool.page_size
        self.root = _Node((), -1, None)
        self._clock = itertools.count(1)
        self.num_nodes = 0

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
            if nxt is None:
                break
            nxt.last_use = t
            nxt.locks += 1
            pages.append(nxt.page)
            nodes.append(nxt)
            node = nxt
        self.pool.retain(pages)
        return pages, nodes

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
            nxt.last_use = t
            node = nxt

    def evict(self, need_pages: int) -> int:
        """Free up to need_pages pages from unlocked leaves (LRU)."""
        freed = 0
        while freed < need_pages:
            leaves = [n for n in self._iter() if not n.children and n.locks == 0 and n is not self.root]
            if not leaves:
                break
            leaves.sort(key=lambda n: n.last_use)
            for lf in leaves:
                if freed >= need_pages:
                    break
                del lf.parent.children[lf.key]
                self.pool.release([lf.page])
                self.num_nodes -= 1
                freed += 1
        return freed

    def _iter(self):
        stack = [self.root]
        while stack:
            n = stack.pop()
            yield n
            stack.extend(n.children.values())
