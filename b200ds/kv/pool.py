"""Paged KV-cache page allocator with reference counts.

Pages hold `page_size` consecutive token slots of every layer's latent cache
(the tensors themselves live in the model: [num_pages * page_size, 576] e4m3
per layer).  Pages are reference-counted so a radix-cached prefix can be
shared by several running requests.

Reference parity: the reference's KV pools belong to SGLang (absent); its
"uniform FP8" pool layout is fork_attn.py:174-185.
"""
from __future__ import annotations

from typing import List


class OutOfPages(RuntimeError):
    pass


class PagePool:
    def __init__(self, num_pages: int, page_size: int):
        self.num_pages = num_pages
        self.page_size = page_size
        # page 0 is reserved as a scratch page for padded (CUDA-graph) rows
        self.free: List[int] = list(range(num_pages - 1, 0, -1))
        self.ref = [0] * num_pages

    @property
    def num_free(self) -> int:
        return len(self.free)

    def alloc(self, n: int) -> List[int]:
        if n > len(self.free):
            raise OutOfPages(f"need {n} pages, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        for p in out:
            self.ref[p] = 1
        return out

    def retain(self, pages: List[int]) -> None:
        for p in pages:
            assert self.ref[p] > 0, p
            self.ref[p] += 1

    def release(self, pages: List[int]) -> None:
        for p in pages:
            assert self.ref[p] > 0, p
            self.ref[p] -= 1
            if self.ref[p] == 0:
                self.free.append(p)

    def pages_for(self, tokens: int) -> int:
        return (tokens + self.page_size - 1) // self.page_size
