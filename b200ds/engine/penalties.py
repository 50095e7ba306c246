"""Logit adjustments requested per sampling request, applied to the
full-vocabulary logits of the eager path before sampling:

  * logit_bias {token: b} (OpenAI form): b is added to that token's logit;
  * repetition_penalty r (CTRL / HF form): every token already in the prompt
    or the output has its logit divided by r when positive, multiplied by r
    when negative;
  * presence_penalty a and frequency_penalty f (OpenAI form): a token that
    occurs c > 0 times in the output loses a + f * c;
  * min_tokens n: the end-of-sequence id and the request's stop ids are
    masked (logit -1e30) until the output holds n tokens;
  * min_p m: with temperature T > 0, tokens whose probability under
    softmax(logits / T) is below m times the largest are masked (greedy rows
    are unaffected);
  * guided_regex / guided_choice: tokens that cannot extend the output to a
    match are masked (engine/guided.py).

Steps with such requests run the forward that returns logits instead of the
token-only decode graph (the graph's on-device sampler has no per-request
history).  Log-probabilities stay those of the raw logits.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

# masked logit: finite (a sampler's max / exp / division by the temperature
# stay well defined) and below any real logit
MASKED = -1e30


def needs_adjust(p) -> bool:
    return (p.presence_penalty != 0.0 or p.frequency_penalty != 0.0 or p.repetition_penalty != 1.0
            or p.min_p > 0.0 or p.min_tokens > 0 or p.guided_regex is not None or bool(p.guided_choice)
            or p.guided_json is not None or bool(p.logit_bias))


def adjust_logits(logits: torch.Tensor, reqs: Sequence, sample: Optional[Sequence[bool]] = None,
                  eos: Optional[int] = None, tokenizer=None) -> torch.Tensor:
    """A copy of logits [B, V] with row i adjusted for reqs[i] (rows whose
    request needs nothing, or that do not sample this step, are unchanged).
    Guided requests (engine/guided.py) are masked last; one that cannot
    continue gets `guide_done` set."""
    out = logits.float().clone()
    V = out.shape[1]
    dev = out.device
    for i, r in enumerate(reqs):
        p = r.params
        if not needs_adjust(p) or (sample is not None and not sample[i]):
            continue
        row = out[i]
        if p.logit_bias:
            ids = torch.tensor([int(t) for t in p.logit_bias], dtype=torch.long, device=dev)
            row[ids] += torch.tensor([float(v) for v in p.logit_bias.values()], dtype=row.dtype, device=dev)
        if p.repetition_penalty != 1.0:
            seen = torch.tensor(sorted(set(r.prompt) | set(r.output)), dtype=torch.long, device=dev)
            if seen.numel():
                v = row[seen]
                row[seen] = torch.where(v > 0, v / p.repetition_penalty, v * p.repetition_penalty)
        if (p.presence_penalty != 0.0 or p.frequency_penalty != 0.0) and r.output:
            cnt = torch.bincount(torch.tensor(r.output, dtype=torch.long, device=dev), minlength=V)[:V].float()
            row -= p.presence_penalty * (cnt > 0).float() + p.frequency_penalty * cnt
        if p.min_tokens > 0 and len(r.output) < p.min_tokens:
            ids = list(p.stop_token_ids) + ([eos] if eos is not None and not p.ignore_eos else [])
            ids = [t for t in ids if 0 <= t < V]
            if ids:
                row[torch.tensor(ids, dtype=torch.long, device=dev)] = MASKED
        if p.min_p > 0.0 and p.temperature > 0:
            pr = (row / p.temperature).softmax(-1)
            row.masked_fill_(pr < p.min_p * pr.max(), MASKED)
    if any(r.params.guided_regex is not None or r.params.guided_choice or r.params.guided_json is not None
           for r in reqs):
        from .guided import apply_guides
        for i in apply_guides(out, reqs, sample, tokenizer, eos, MASKED):
            reqs[i].guide_done = True
    return out
