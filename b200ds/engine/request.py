"""Request and sampling-parameter records."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0        # <= 0: greedy
    top_p: float = 1.0
    top_k: int = 0                  # <= 0: disabled
    seed: Optional[int] = None
    ignore_eos: bool = False
    stop_token_ids: List[int] = field(default_factory=list)
    stop: List[str] = field(default_factory=list)    # stop strings (engine API; needs a tokenizer)
    logprobs: Optional[int] = None  # record each output token's log-probability and this many top alternatives
    presence_penalty: float = 0.0   # output tokens seen at least once lose this much logit
    frequency_penalty: float = 0.0  # ... and this much per occurrence
    repetition_penalty: float = 1.0  # prompt / output tokens: positive logits / r, negative * r
    min_p: float = 0.0              # drop tokens below min_p x the top probability (temperature > 0)
    min_tokens: int = 0             # no end-of-sequence / stop token before this many output tokens
    priority: int = 0               # schedule_policy "priority": lower is admitted first
    logit_bias: Optional[dict] = None  # token id -> value added to its logit (OpenAI logit_bias)
    guided_regex: Optional[str] = None        # the output text must match this regular expression
    guided_choice: Optional[List[str]] = None  # ... or be one of these strings
    guided_json: Optional[object] = None       # ... or be JSON matching this schema ("object": any flat object)
    prompt_logprobs: Optional[int] = None  # log-probability of every prompt token (+ top-n); computes the
                                           # whole prompt (no prefix-cache reuse)


@dataclass
class Request:
    rid: int
    prompt: List[int]
    params: SamplingParams
    output: List[int] = field(default_factory=list)
    pages: List[int] = field(default_factory=list)
    cached: int = 0                  # tokens whose KV is in the cache
    prefix_nodes: list = field(default_factory=list)
    prefix_pages: int = 0            # leading pages shared with the radix cache
    finished: bool = False
    finish_reason: Optional[str] = None
    t_arrive: float = field(default_factory=time.perf_counter)
    t_first: Optional[float] = None
    t_done: Optional[float] = None
    token_times: List[float] = field(default_factory=list)
    # per output token (SamplingParams.logprobs set): (token, logprob, [(alt token, logprob), ...])
    logprobs: List[tuple] = field(default_factory=list)
    # per prompt position (prompt_logprobs set): None for the first token, then (token, logprob, top-n)
    prompt_lp: List[Optional[tuple]] = field(default_factory=list)
    gen: Optional[torch.Generator] = None
    # context-parallel prefill (DP attention): the rank that decodes the
    # request (None = an ordinary request), its place in the ranks' shared
    # context-parallel queue, and an abort waiting for the ranks to agree
    cp_owner: Optional[int] = None
    cp_seq: int = -1
    cp_abort: bool = False

    @property
    def all_tokens(self) -> List[int]:
        return self.prompt + self.output

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.output)

    def uniform(self) -> float:
        if self.gen is None:
            self.gen = torch.Generator().manual_seed(self.params.seed if self.params.seed is not None else self.rid)
        return float(torch.rand((), generator=self.gen))
