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
    if p.guided_json is not None:
        return JSON_OBJECT if p.guided_json == "object" else schema_to_regex(p.guided_json)
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


# ---------------------------------------------------------------------------
# JSON schema -> regular expression (a practical subset)
# ---------------------------------------------------------------------------

_WS = "[ ]?"
_STR_CH = r'(?:[^"\\\x00-\x1f]|\\["\\/bfnrt])'
_INT = r"-?(?:0|[1-9][0-9]{0,17})"
_NUM = _INT + r"(?:\.[0-9]{1,17})?(?:[eE][+-]?[0-9]{1,3})?"


def schema_to_regex(schema: dict) -> str:
    """Regular expression of the compact JSON texts a schema accepts, for
    this subset: type string (maxLength / minLength, enum, const), integer,
    number, boolean, null; object with properties (emitted in declaration
    order, all present); array with items (minItems / maxItems); enum,
    const, anyOf / oneOf.  Numbers are bounded to 18 digits so a guided
    output always reaches its end.  Anything else raises ValueError."""
    import json
    if not isinstance(schema, dict):
        raise ValueError("schema must be an object")
    for k in ("enum", "const"):
        if k in schema:
            vals = schema[k] if k == "enum" else [schema[k]]
            return "(?:" + "|".join(re.escape(json.dumps(v, separators=(",", ":"))) for v in vals) + ")"
    for k in ("anyOf", "oneOf"):
        if k in schema:
            return "(?:" + "|".join(schema_to_regex(s) for s in schema[k]) + ")"
    t = schema.get("type")
    if isinstance(t, list):
        return "(?:" + "|".join(schema_to_regex(dict(schema, type=x)) for x in t) + ")"
    if t == "string":
        lo, hi = int(schema.get("minLength", 0)), schema.get("maxLength")
        return '"' + _STR_CH + ("{%d,%d}" % (lo, int(hi)) if hi is not None else ("{%d,}" % lo if lo else "*")) + '"'
    if t == "integer":
        return _INT
    if t == "number":
        return _NUM
    if t == "boolean":
        return "(?:true|false)"
    if t == "null":
        return "null"
    if t == "object":
        props = schema.get("properties") or {}
        if not props:
            return r"\{" + _WS + r"\}"
        parts = [re.escape(json.dumps(k)) + _WS + ":" + _WS + schema_to_regex(v) for k, v in props.items()]
        return r"\{" + _WS + ("," + _WS).join(parts) + _WS + r"\}"
    if t == "array":
        item = schema_to_regex(schema.get("items") or {"type": "string", "maxLength": 64})
        lo, hi = int(schema.get("minItems", 0)), schema.get("maxItems")
        more = "(?:," + _WS + item + ")"
        if hi is not None:
            hi = int(hi)
            body = "" if hi == 0 else item + more + "{%d,%d}" % (max(lo - 1, 0), hi - 1)
            opt = lo == 0 and hi > 0
        else:
            body = item + more + ("{%d,}" % (lo - 1) if lo > 1 else "*")
            opt = lo == 0
        inner = ("(?:" + body + ")?") if opt else body
        return r"\[" + _WS + inner + _WS + r"\]"
    raise ValueError(f"unsupported schema: {json.dumps(schema)[:80]}")


# response_format {"type": "json_object"}: a flat JSON object (string keys of
# up to 64 characters, primitive values)
_KEY = '"' + _STR_CH + '{1,64}"'
_PRIM = "(?:" + '"' + _STR_CH + '{0,256}"' + "|" + _NUM + "|true|false|null)"
_PAIR = _KEY + _WS + ":" + _WS + _PRIM
JSON_OBJECT = r"\{" + _WS + "(?:" + _PAIR + "(?:," + _WS + _PAIR + "){0,63})?" + _WS + r"\}"
