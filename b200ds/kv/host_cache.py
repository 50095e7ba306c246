"""Host-memory tier of the prefix cache.

A KV page holds `page_size` token slots of every per-slot cache tensor of the
model (the latent rows of every layer, and where present the indexer keys and
scales and the Engram token ids), and page_size / r rows of a tensor with one
row per r slots (the compressed rows of a compressed-attention layer, paged
with the same page ids).  When the radix cache must free device
pages it moves unlocked pages here instead of dropping them; a later prefix
match copies them back into freshly allocated device pages.  All copies are
issued on the current stream, in order with the kernels that read or
overwrite those slots, so no extra synchronisation is needed (the host
buffers are pinned on GPU runs).

Reference parity: the reference's KV pools belong to SGLang (absent); this
tier is the engine's own.
"""
from __future__ import annotations

from typing import List

import torch


class HostKVPool:
    def __init__(self, tensors: List[torch.Tensor], num_pages: int, page_size: int):
        self.tensors = tensors
        self.page_size = page_size
        self.num_pages = num_pages
        pin = any(t.is_cuda for t in tensors)
        slots = max(int(t.shape[0]) for t in tensors)
        # rows of each tensor that belong to one page (page_size for per-slot tensors)
        self.rows = [page_size * int(t.shape[0]) // slots for t in tensors]
        self.host = [torch.empty((num_pages, n) + tuple(t.shape[1:]), dtype=t.dtype, pin_memory=pin)
                     for t, n in zip(tensors, self.rows)]
        self.free_pages: List[int] = list(range(num_pages - 1, -1, -1))

    @property
    def num_free(self) -> int:
        return len(self.free_pages)

    def offload(self, gpu_page: int) -> int:
        """Copy device page gpu_page into a free host page; returns it."""
        hp = self.free_pages.pop()
        for t, h, n in zip(self.tensors, self.host, self.rows):
            h[hp].copy_(t[gpu_page * n: (gpu_page + 1) * n], non_blocking=True)
        return hp

    def restore(self, host_page: int, gpu_page: int) -> None:
        """Copy host page host_page into device page gpu_page."""
        for t, h, n in zip(self.tensors, self.host, self.rows):
            t[gpu_page * n: (gpu_page + 1) * n].copy_(h[host_page], non_blocking=True)

    def free(self, host_page: int) -> None:
        self.free_pages.append(host_page)
