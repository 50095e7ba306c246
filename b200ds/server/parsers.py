"""Chat output parsers for the DeepSeek formats.

* Reasoning (DeepSeek-R1 style): text up to the first "</think>" (an
  opening "<think>" is optional, the chat template may have written it) is
  the reasoning; the rest is the answer.
* Tool calls (DeepSeek-V3 style): a block

      <｜tool▁calls▁begin｜><｜tool▁call▁begin｜>function<｜tool▁sep｜>NAME
      ```json
      {ARGUMENTS}
      ```<｜tool▁call▁end｜>...<｜tool▁calls▁end｜>

  becomes OpenAI `tool_calls` entries; text before the block is the content.

These are the formats of the published DeepSeek chat templates; the parsers
only read text, so they work with any tokenizer that keeps the markers.
"""
from __future__ import annotations

import json
import re
import uuid
from typing import List, Optional, Tuple

THINK_OPEN, THINK_CLOSE = "<think>", "</think>"
CALLS_BEGIN, CALLS_END = "<｜tool▁calls▁begin｜>", "<｜tool▁calls▁end｜>"
CALL_BEGIN, CALL_END, SEP = "<｜tool▁call▁begin｜>", "<｜tool▁call▁end｜>", "<｜tool▁sep｜>"
_CALL = re.compile(re.escape(CALL_BEGIN) + r"(?P<type>\w+)" + re.escape(SEP) + r"(?P<name>[^\n]+)\n"
                   r"```(?:json)?\n(?P<args>.*?)\n```" + re.escape(CALL_END), re.S)


def split_reasoning(text: str) -> Tuple[Optional[str], str]:
    """(reasoning or None, answer)."""
    i = text.find(THINK_CLOSE)
    if i < 0:
        if text.lstrip().startswith(THINK_OPEN):        # still thinking (cut by max_tokens)
            return text.lstrip()[len(THINK_OPEN):].strip(), ""
        return None, text
    r = text[:i]
    j = r.find(THINK_OPEN)
    if j >= 0:
        r = r[j + len(THINK_OPEN):]
    return r.strip(), text[i + len(THINK_CLOSE):].lstrip()


def parse_tool_calls(text: str) -> Tuple[str, List[dict]]:
    """(content before the tool-call block, OpenAI tool_calls).  Calls whose
    arguments are not JSON keep them as the raw string."""
    i = text.find(CALLS_BEGIN)
    if i < 0:
        return text, []
    content = text[:i].rstrip()
    calls = []
    for m in _CALL.finditer(text, i):
        args = m.group("args").strip()
        try:
            args = json.dumps(json.loads(args), ensure_ascii=False)
        except ValueError:
            pass
        calls.append({"id": "call_" + uuid.uuid4().hex[:24], "type": m.group("type"),
                      "function": {"name": m.group("name").strip(), "arguments": args}})
    return content, calls


def stream_reasoning(text: str) -> Tuple[str, str]:
    """(reasoning, answer) of a partial output for streaming: text that might
    still become a "<think>" / "</think>" marker is held back."""
    t = text
    if THINK_OPEN.startswith(t.lstrip()) and len(t.lstrip()) < len(THINK_OPEN):
        return "", ""                                       # maybe the opening marker
    if t.lstrip().startswith(THINK_OPEN):
        t = t.lstrip()[len(THINK_OPEN):]
    i = t.find(THINK_CLOSE)
    if i >= 0:
        return t[:i], t[i + len(THINK_CLOSE):]
    hold = next((k for k in range(min(len(THINK_CLOSE) - 1, len(t)), 0, -1) if THINK_CLOSE.startswith(t[-k:])), 0)
    return t[: len(t) - hold], ""
