"""Context parallelism for long prompts under DP attention.

Under data-parallel attention every rank holds the full attention weights, so
one long prompt can prefill on all ranks at once: each chunk's tokens are
split round-robin over the ranks (position p goes to rank (p - start) % W,
which evens out the causal attention work), every rank runs the layer stack
on its own rows, and after each layer's cache stores the ranks all-gather the
new cache rows (the fp8 latent + rope row, and for sparse models the indexer
key and its scale), so every rank's paged cache holds the whole chunk before
its queries attend.  The MoE exchange runs as in any DP step (each rank's
rows routed to the expert owners).  After the last chunk the rank holding the
prompt's last position broadcasts that row's final hidden state; the owner
rank computes the logits and samples with its own request state, and keeps
the cache for decoding while the other ranks free (or prefix-cache) theirs.

Reference parity: the reference runs stock SGLang context parallelism for
extend batches (`is_cp_active`, tokens strided by `attn_cp_rank ::
attn_cp_size`, fork_loop.py:242-258) and materialises the gathered fp8 KV
before its prefill attention (`_materialize_cp_unified_fp8_kv`,
fork_attn.py:101,303-307).
"""
from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace
from typing import List, Optional, Sequence

import torch

from ..models.batch import ForwardBatch


def rank_positions(start: int, n: int, world: int, rank: int) -> List[int]:
    """Absolute positions of chunk [start, start + n) that `rank` computes."""
    return list(range(start + rank, start + n, world))


def holder_of_last(n: int, world: int) -> int:
    """The rank holding the chunk's last position."""
    return (n - 1) % world


@dataclass
class CPLayout:
    """How one chunk's cache rows travel: every rank contributes `counts[q]`
    rows padded to `tmax`; row j of rank q belongs to position start + q +
    j * W.  `src_rows` index the gathered [W * tmax] rows in chunk-position
    order and `dst_slots` are this rank's cache slots of those positions;
    `ids` are the chunk's token ids in position order."""
    counts: List[int]
    tmax: int
    start: int
    src_rows: torch.Tensor       # [n] int64
    dst_slots: torch.Tensor      # [n] int64
    ids: torch.Tensor            # [n] int32
    _dev: dict = None

    def on(self, device):
        """The index tensors on `device` (moved once per chunk)."""
        if self._dev is None:
            self._dev = {}
        key = str(device)
        if key not in self._dev:
            self._dev[key] = (self.src_rows.to(device, non_blocking=True),
                              self.dst_slots.to(device, non_blocking=True))
        return self._dev[key]

    def whole(self, fb: ForwardBatch) -> SimpleNamespace:
        """The whole chunk as one sequence (positions, slots, ids, q_seq,
        block table on fb's device): what a step that runs on every row of
        the chunk at once reads (the compressor's block means, the token
        cache of the n-gram hashes)."""
        dev = fb.out_slots.device
        key = "whole:" + str(dev)
        if self._dev is None:
            self._dev = {}
        if key not in self._dev:
            n = int(self.ids.shape[0])
            self._dev[key] = SimpleNamespace(
                positions=torch.arange(self.start, self.start + n, dtype=torch.int32).to(dev),
                out_slots=self.on(dev)[1], input_ids=self.ids.to(dev), q_seq=torch.zeros(n, dtype=torch.int32,
                                                                                          device=dev),
                block_table=fb.block_table)
        return self._dev[key]


def layout(start: int, n: int, world: int, pages: Sequence[int], page_size: int,
           tokens: Sequence[int] = ()) -> CPLayout:
    """Chunk position start + k sits on rank k % W as that rank's row k // W,
    so in position order the gathered rows are (k % W) * tmax + k // W."""
    counts = [len(range(q, n, world)) for q in range(world)]
    tmax = max(max(counts), 1)
    k = torch.arange(n, dtype=torch.int64)
    src = (k % world) * tmax + k // world
    pos = start + k
    pg = torch.as_tensor(list(pages), dtype=torch.int64)
    slots = pg[pos // page_size] * page_size + pos % page_size
    ids = (torch.as_tensor(list(tokens[start:start + n]), dtype=torch.int32) if len(tokens)
           else torch.zeros(n, dtype=torch.int32))
    return CPLayout(counts, tmax, start, src, slots, ids)


def build_cp_batch(prompt: Sequence[int], start: int, n: int, world: int, rank: int, pages: Sequence[int],
                   page_size: int) -> ForwardBatch:
    """This rank's rows of chunk [start, start + n) as one sequence whose
    query positions are strided (the attention kernels mask by each query's
    own position, so the rows need not be contiguous).  A rank with no rows
    this chunk runs one dummy token on the scratch page 0 (its rows are not
    gathered: counts say zero)."""
    pos = rank_positions(start, n, world, rank)
    if pos:
        ids = [prompt[p] for p in pos]
        slots = [pages[p // page_size] * page_size + p % page_size for p in pos]
        bt_pages = list(pages)
        seq_len = start + n
    else:
        ids, pos, slots, bt_pages, seq_len = [0], [0], [0], [0], 1
    T = len(ids)
    bt = torch.tensor([bt_pages], dtype=torch.int32)
    fb = ForwardBatch(
        input_ids=torch.tensor(ids, dtype=torch.int32),
        positions=torch.tensor(pos, dtype=torch.int32),
        q_seq=torch.zeros(T, dtype=torch.int32),
        out_slots=torch.tensor(slots, dtype=torch.int64),
        seq_lens=torch.tensor([seq_len], dtype=torch.int32),
        block_table=bt,
        last_idx=torch.tensor([T - 1], dtype=torch.int64),
        is_decode=False,
        max_q_len=T,
        max_seq_len=seq_len,
    )
    fb.cp = layout(start, n, world, pages, page_size, prompt)
    fb.dp_tmax = fb.cp.tmax
    return fb


def _rows_u8(buf: torch.Tensor) -> torch.Tensor:
    """A per-slot cache tensor as [slots, bytes] uint8."""
    return buf.view(torch.uint8).reshape(buf.shape[0], -1)


def gather_rows(bufs: Sequence[torch.Tensor], fb: ForwardBatch, ps,
                extra: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """All-gather this chunk's freshly stored cache rows of every buffer in
    `bufs` (one collective for all of them) and write them into this rank's
    slots, so each rank's cache holds the whole chunk.  `extra` (one fp32
    value per row of this rank) travels along; returned for the whole chunk
    in position order."""
    cp: CPLayout = fb.cp
    views = [_rows_u8(b) for b in bufs]
    widths = [v.shape[1] for v in views]
    own = fb.out_slots
    cols = [v[own] for v in views]
    if extra is not None:
        e = torch.empty(extra.shape[0], dtype=torch.float32, device=extra.device)
        e.copy_(extra)          # fresh stride-1 storage (a strided column of one row counts as contiguous)
        cols.append(e.view(torch.uint8).reshape(-1, 4))
    pack = torch.cat(cols, 1)
    if pack.shape[0] < cp.tmax:
        pack = torch.cat([pack, pack.new_zeros(cp.tmax - pack.shape[0], pack.shape[1])], 0)
    elif pack.shape[0] > cp.tmax:        # a dummy row on a rank with no rows: tmax >= 1 already
        pack = pack[: cp.tmax]
    g = ps.ep_all_gather(pack.contiguous())
    src, dst = cp.on(g.device)
    rows = g[src]
    off = 0
    for v, w in zip(views, widths):
        v[dst] = rows[:, off:off + w]
        off += w
    if extra is None:
        return None
    return rows[:, off:off + 4].contiguous().view(torch.float32).reshape(-1)
