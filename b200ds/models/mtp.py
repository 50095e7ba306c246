"""Multi-token-prediction (MTP) draft for speculative decoding.

DeepSeek-V3's MTP module predicts token x_{j+1} from the main model's final
(pre-norm) hidden state h_{j-1} and the embedding of x_j:
    z = eh_proj [ RMSNorm(Emb(x_j)) ; RMSNorm(h_{j-1}) ]  (enorm / hnorm)
    u = one decoder layer (MLA + MoE) over z          -> MTP hidden
    logits = LM head (shared) of RMSNorm(u)           (shared_head.norm)
Its sequence is shifted by one: the row for token position j sits at MTP
position j - 1, attends to MTP positions <= j - 1 and writes its latent KV
to the request's slot of position j - 1, in an MTP cache of its own (same
pages as the main model).  Deeper drafts chain the module on its own hidden
state.

Reference parity: the reference drafts with a separate DSPARK model fed by
aux hidden states of the target (fork_loop.py:102, 182-189, 359-364; its
verify mode is `target_verify`); this MTP draft follows DeepSeek-V3's own
MTP design (HF checkpoint layer `num_hidden_layers`: enorm, hnorm, eh_proj,
shared_head).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from .. import ops
from .batch import ForwardBatch, build_batch


class MTPDraft:
    def __init__(self, block, enorm: torch.Tensor, hnorm: torch.Tensor, eh_proj):
        self.block = block          # a one-layer DeepseekModel sharing the main model's embedding / LM head
        self.enorm = enorm
        self.hnorm = hnorm
        self.eh_proj = eh_proj

    def allocate_kv(self, num_pages: int) -> None:
        self.block.allocate_kv(num_pages)

    def kv_bytes_per_token(self) -> int:
        return self.block.kv_bytes_per_token()

    @torch.no_grad()
    def forward(self, fb: ForwardBatch, prev_h: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """fb: MTP rows (tokens x_j at MTP positions j - 1); prev_h [T, D]:
        the hidden state that produced each row's token.  Returns (logits of
        each sequence's last row [B, V], MTP hidden of those rows [B, D])."""
        c = self.block.cfg
        cuda = prev_h.is_cuda
        dt = torch.bfloat16 if cuda else torch.float32
        e = ops.rmsnorm(self.block.embed[fb.input_ids.long()].to(dt), self.enorm, c.rms_norm_eps)
        hh = ops.rmsnorm(prev_h.to(dt), self.hnorm, c.rms_norm_eps)
        z = self.eh_proj(torch.cat([e.to(dt), hh.to(dt)], -1), out_dtype=dt)
        logits = self.block.forward(fb, x0=z)
        return logits, self.block.last_residual[fb.last_idx]


def mtp_batch(rows: List[dict], page_size: int, device) -> Optional[ForwardBatch]:
    """rows: per request {"tokens": [x_j ...] (consecutive token positions
    j0..), "j0": first token position (>= 1), "pages"} -> the MTP batch (MTP
    positions j - 1)."""
    seqs = [{"tokens": r["tokens"], "start": r["j0"] - 1, "pages": r["pages"]} for r in rows if r["tokens"]]
    if not seqs:
        return None
    return build_batch(seqs, page_size, device=device)
