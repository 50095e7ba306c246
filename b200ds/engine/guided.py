"""Guided decoding: the output text must match a regular expression (or be
one of a list of choices, compiled to an alternation).

Each sampled row keeps only the tokens whose text extends the output so far
(tokens that add no text, such as special ids, are excluded) to a prefix of
some match (partial full-match of the `regex` package).  The
candidates are checked in logit order, a block of them at a time, until one
block yields allowed tokens, so the usual cost is one block per step; the
end-of-sequence id is allowed once the text is a complete match.  When no
token can extend the text the request ends ("stop").

Steps with guided requests run the full-logits path (like the penalties);
log-probabilities stay those of the raw logits.
"""
from __future__ import annotations

import re
from typing import List, Optional

import torch

BLOCK = 64


def guide_pattern(p) -> Optional[str]:
    if p.guided_regex is not None:
        return p.guided_regex
    if p.guided_choice:
        return "(?:" + "|".join(re.escape(c) for c in p.guided_choice) + ")"
    return None


class Guide:
    def __init__(self, pattern: str, choices: Optional[List[str]] = None):
        import regex
        self.rx = regex.compile(pattern)
        self.choices = choices

    def may_grow(self, text: str) -> bool:
        """False when no longer text can match (known for choice lists; a
        regular expression is assumed extendable)."""
        if self.choices is None:
            return True
        return any(len(c) > len(text) and c.startswith(text) for c in self.choices)

    def can_extend(self, text: str) -> bool:
        return self.rx.fullmatch(text, partial=True) is not None

    def complete(self, text: str) -> bool:
        return self.rx.fullmatch(text) is not None


def guide_of(r) -> Guide:
    g = getattr(r, "guide", None)
    if g is None:
        g = r.guide = Guide(guide_pattern(r.params), r.params.guided_choice or None
                            if r.params.guided_regex is None else None)
    return g


def allowed_mask(row: torch.Tensor, r, tokenizer, eos: Optional[int]) -> Optional[torch.Tensor]:
    """Bool mask [V] of the tokens guided request r may emit next given the
    logits row, or None when none may (the request is done)."""
    g = guide_of(r)
    out = list(r.output)
    V = row.shape[0]
    mask = torch.zeros(V, dtype=torch.bool)
    cur = tokenizer.decode(out)
    done_ok = g.complete(cur)
    order = torch.argsort(row.float().cpu(), descending=True).tolist() if g.may_grow(cur) else []
    for b in range(0, len(order), BLOCK):
        for t in order[b: b + BLOCK]:
            if t == eos:
                continue
            txt = tokenizer.decode(out + [t])
            if len(txt) > len(cur) and g.can_extend(txt):      # adds text (special ids add none)
                mask[t] = True
        if bool(mask.any()):
            break
    if done_ok and eos is not None and 0 <= eos < V:
        mask[eos] = True
    return mask if bool(mask.any()) else None


def apply_guides(logits: torch.Tensor, reqs, sample, tokenizer, eos: Optional[int], masked: float) -> List[int]:
    """Mask logits rows of guided requests in place; returns the indices of
    rows whose request cannot continue."""
    ended = []
    for i, r in enumerate(reqs):
        if guide_pattern(r.params) is None or (sample is not None and not sample[i]):
            continue
        m = allowed_mask(logits[i], r, tokenizer, eos)
        if m is None:
            ended.append(i)
            continue
        logits[i].masked_fill_(~m.to(logits.device), masked)
    return ended
