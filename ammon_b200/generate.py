"""Greedy decode over an AutoregressiveModel (src/generate.rs, src/model.rs).

``generate_tokens`` keeps the reference loop's exact semantics: prompt tokens after
the first are forced and emitted, the loop runs ``max_new_tokens - 1`` positions
(``max_new_tokens`` clamped to the model's ``max_seq_len``), ``stop_on`` ends the
loop without emitting, and the timer starts after the first step.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Optional, Protocol, Sequence

from .tokenizer import Tokenizer, sample_argmax


class AutoregressiveModel(Protocol):
    """src/model.rs:7-11."""

    def vocab_size(self) -> int: ...

    def max_seq_len(self) -> int: ...

    def step(self, token: int, pos: int): ...


@dataclass
class GenerateOptions:
    """src/generate.rs:8-26."""
    max_new_tokens: int = 50
    bos: bool = True
    eos: bool = False
    stop_on: Optional[int] = None


@dataclass
class GenerateTokenOutput:
    tokens: List[int] = field(default_factory=list)
    prompt_tokens: int = 0
    tokens_per_second: float = 0.0


@dataclass
class GenerateOutput:
    text: str = ""
    tokens: List[int] = field(default_factory=list)
    prompt_tokens: int = 0
    tokens_per_second: float = 0.0


def generate_tokens(model: AutoregressiveModel, prompt_tokens: Sequence[int],
                    max_new_tokens: int, stop_on: Optional[int] = None) -> GenerateTokenOutput:
    """src/generate.rs:43-91."""
    if len(prompt_tokens) == 0:
        raise ValueError("expected at least one prompt token")
    max_new_tokens = min(int(max_new_tokens), int(model.max_seq_len()))
    tokens: List[int] = []
    token = int(prompt_tokens[0])
    pos = 0
    start = None
    while pos < max(max_new_tokens - 1, 0):
        logits = model.step(token, pos)
        if pos < len(prompt_tokens) - 1:
            nxt = int(prompt_tokens[pos + 1])
        else:
            nxt = sample_argmax(logits)
        pos += 1
        if stop_on is not None and stop_on == nxt:
            break
        tokens.append(nxt)
        token = nxt
        if start is None:
            start = time.perf_counter()
    elapsed = time.perf_counter() - start if start is not None else 0.0
    gen = max(pos - 1, 0)
    return GenerateTokenOutput(tokens=tokens, prompt_tokens=len(prompt_tokens),
                               tokens_per_second=gen / elapsed if elapsed > 0 else 0.0)


def generate(model: AutoregressiveModel, tokenizer: Tokenizer, prompt: str,
             options: GenerateOptions = GenerateOptions()) -> GenerateOutput:
    """src/generate.rs:93-118. A model with a batched-prefill loop of its own (the library's
    batch-1 Llama model: ``generate(prompt, max_new_tokens, stop_on)``) runs the prompt through
    it; the ids are those of generate_tokens."""
    prompt_tokens = tokenizer.encode(prompt, options.bos, options.eos)
    own = getattr(model, "generate", None)
    if callable(own) and getattr(getattr(model, "cfg", None), "batch", 0) == 1:
        out = own(prompt_tokens, options.max_new_tokens, options.stop_on)
    else:
        out = generate_tokens(model, prompt_tokens, options.max_new_tokens, options.stop_on)
    text = []
    prev = prompt_tokens[0]
    for tok in out.tokens:
        text.append(tokenizer.decode(prev, tok))
        prev = tok
    return GenerateOutput(text="".join(text), tokens=out.tokens,
                          prompt_tokens=out.prompt_tokens,
                          tokens_per_second=out.tokens_per_second)
