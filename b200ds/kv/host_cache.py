"""Host-memory tier of the prefix cache.

A KV page holds `page_size` token slots of every per-slot cache tensor of the
model (the latent rows of every layer, and where present the indexer keys and
scales and the Engram token ids).  When the radix cache must free device
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
        self.host = [torch.empty((num_pages, page_size) + tuple(t.shape[1:]), dtype=t.dtype, pin_memory=pin)
                     for t in tensors]
        self.free_pages: List[int] = list(range(num_pages - 1, -1, -1))

    @property
    def num_free(self) -> int:
        return len(self.free_pages)

    def offload(self, gpu_page: int) -> int:
        """Copy device page gpu_page into a free host page; returns it."""
        hp = self.free_pages.pop()
        s = gpu_page * self.page_size
        for t, h in zip(self.tensors, self.host):
            h[hp].copy_(t[s: s + self.page_size], non_blocking=True)
        return hp

    def restore(self, host_page: int, gpu_page: int) -> None:
        """Copy host page host_page into device page gpu_page."""
        s = gpu_page * self.page_size
        for t, h in zip(self.tensors, self.host):
            t[s: s + self.page_size].copy_(h[host_page], non_blocking=True)

    def free(self, host_page: int) -> None:
        self.free_pages.append(host_page)
