"""Tokenizers: the checkpoint's Hugging Face tokenizer when a directory with
tokenizer files is given, else a byte-level tokenizer (random-init models
have no vocabulary; ids are bytes offset past the special tokens)."""
from __future__ import annotations

import json
import os
from typing import List, Optional


class ByteTokenizer:
    """Text <-> ids as UTF-8 bytes + 3 (0 = bos, 1 = eos, 2 = pad)."""

    bos_token_id = 0
    eos_token_id = 1
    pad_token_id = 2

    def __init__(self, vocab_size: int = 259):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> List[int]:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids: List[int], keep_special: bool = False) -> str:
        return bytes([(i - 3) % 256 for i in ids if i >= 3]).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, add_generation_prompt: bool = True) -> str:
        parts = [f"<|{m.get('role', 'user')}|>{m.get('content', '')}" for m in messages]
        if add_generation_prompt:
            parts.append("<|assistant|>")
        return "".join(parts)

    def encode_chat(self, messages, tools=None) -> List[int]:
        head = f"<|tools|>{json.dumps(tools)}" if tools else ""
        return self.encode(head + self.apply_chat_template(messages))


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, trust_remote_code=False)
        self.eos_token_id = self.tok.eos_token_id

    def encode(self, text: str) -> List[int]:
        return self.tok.encode(text, add_special_tokens=True)

    def decode(self, ids: List[int], keep_special: bool = False) -> str:
        return self.tok.decode(ids, skip_special_tokens=not keep_special)

    def apply_chat_template(self, messages, add_generation_prompt: bool = True) -> str:
        return self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=add_generation_prompt)

    def encode_chat(self, messages, tools=None) -> List[int]:
        """Token ids of the chat template (with the request's tools, when the
        template renders them): the template writes its own BOS, so the text
        is not encoded again with special tokens added."""
        kw = {"tools": tools} if tools else {}
        text = self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True, **kw)
        return self.tok.encode(text, add_special_tokens=False)


def load_tokenizer(path: Optional[str]):
    if path and os.path.isdir(path) and any(os.path.exists(os.path.join(path, f))
                                             for f in ("tokenizer.json", "tokenizer_config.json")):
        return HFTokenizer(path)
    return ByteTokenizer()
