"""Per-step batch metadata shared by the model, the KV pool and the kernels."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class ForwardBatch:
    """A flat ("ragged") batch: tokens of all sequences concatenated.

    input_ids [T], positions [T] (absolute), q_seq [T] (row of block_table
    each token belongs to), out_slots [T] (KV-cache slot the token's latent is
    written to), seq_lens [B] (cached length after this step), block_table
    [B, max_pages], last_idx [B] (token index whose logits are returned)."""
    input_ids: torch.Tensor
    positions: torch.Tensor
    q_seq: torch.Tensor
    out_slots: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    last_idx: torch.Tensor
    is_decode: bool = False
    max_q_len: int = 1
    max_seq_len: int = 0
    # DP attention: token rows per rank this step (the max over ranks), which
    # sizes the expert-parallel exchange; 0 = this batch's own token count.
    dp_tmax: int = 0
    # Optional per-request sampling parameters (engine fills them)
    temperature: Optional[torch.Tensor] = None
    top_p: Optional[torch.Tensor] = None
    top_k: Optional[torch.Tensor] = None
    # Prefill tail [B]: window-only late layers compute only the rows at
    # positions >= tail_from[sequence] (and each sequence's last row)
    tail_from: Optional[torch.Tensor] = None
    # Context-parallel prefill chunk (parallel.cp.CPLayout): the layer stack
    # all-gathers each layer's new cache rows over the ranks before attention
    cp: Optional[object] = None

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.shape[0])

    @property
    def batch_size(self) -> int:
        return int(self.seq_lens.shape[0])

    def tail_rows(self) -> torch.Tensor:
        """Indices of the rows the window-only late layers compute."""
        keep = self.positions.long() >= self.tail_from.to(self.positions.device).long()[self.q_seq.long()]
        keep[self.last_idx.long()] = True
        return keep.nonzero().flatten()

    def take_rows(self, rows: torch.Tensor) -> "ForwardBatch":
        """The same sequences with only token rows `rows` (ascending, each
        sequence's last row included): per-sequence metadata is unchanged,
        last_idx points into the kept rows."""
        last = torch.searchsorted(rows, self.last_idx.to(rows.device).long())
        kw = dict(self.__dict__)
        kw.update(input_ids=self.input_ids[rows], positions=self.positions[rows], q_seq=self.q_seq[rows],
                  out_slots=self.out_slots[rows], last_idx=last.to(self.last_idx.dtype), tail_from=None)
        return ForwardBatch(**kw)

    def to(self, device) -> "ForwardBatch":
        kw = {}
        for k, v in self.__dict__.items():
            kw[k] = v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v
        return ForwardBatch(**kw)


def build_batch(seqs: List[dict], page_size: int, device="cpu", pad_pages: int = 0) -> ForwardBatch:
    """seqs: list of {"tokens": new token ids, "start": cached length before
    this step, "pages": page ids}.  Builds the flat metadata on the host."""
    ids, pos, qs, slots, lens, last = [], [], [], [], [], []
    max_pages = max(max(len(s["pages"]) for s in seqs), pad_pages)
    bt = torch.zeros(len(seqs), max(max_pages, 1), dtype=torch.int32)
    t = 0
    max_q = 1
    for b, s in enumerate(seqs):
        toks = s["tokens"]
        st = s["start"]
        n = len(toks)
        max_q = max(max_q, n)
        ids.extend(toks)
        for j in range(n):
            p = st + j
            pos.append(p)
            qs.append(b)
            slots.append(s["pages"][p // page_size] * page_size + p % page_size)
        lens.append(st + n)
        t += n
        last.append(t - 1)
        if s["pages"]:
            bt[b, : len(s["pages"])] = torch.tensor(s["pages"], dtype=torch.int32)
    fb = ForwardBatch(
        input_ids=torch.tensor(ids, dtype=torch.int32),
        positions=torch.tensor(pos, dtype=torch.int32),
        q_seq=torch.tensor(qs, dtype=torch.int32),
        out_slots=torch.tensor(slots, dtype=torch.int64),
        seq_lens=torch.tensor(lens, dtype=torch.int32),
        block_table=bt,
        last_idx=torch.tensor(last, dtype=torch.int64),
        is_decode=(max_q == 1),
        max_q_len=max_q,
        max_seq_len=max(lens),
    )
    return fb.to(device) if str(device) != "cpu" else fb
