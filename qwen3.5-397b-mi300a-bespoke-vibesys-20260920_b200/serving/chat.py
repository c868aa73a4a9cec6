"""Chat-template rendering at the token-id level, and the text-side tokenizer adapter.

Qwen3.5's template renders a conversation as::

    <|im_start|>user\\n{content}<|im_end|>\\n<|im_start|>assistant\\n{reply}<|im_end|>\\n ...

and, when generation is requested with thinking disabled, appends
``<|im_start|>assistant\\n<think>\\n\\n</think>\\n\\n``. The history rendering of that same turn in
the next request has no ``<think>`` block, so the reusable prefix of a prompt ends *before*
``<think>\\n\\n</think>\\n\\n``: that span is the prompt's ``suffix_len`` (reference
``server.py:631-663``, ``scheduler.py:33-41``). ``TokenTemplate`` builds prompts directly from
token ids, which is what the id-level workloads and the tiny parity model use; with a real
tokenizer the ids come from its special tokens.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class TokenTemplate:
    im_start: int
    im_end: int
    user: int
    assistant: int
    system: int
    nl: int
    think: int
    think_end: int

    @classmethod
    def for_vocab(cls, vocab: int) -> TokenTemplate:
        """Reserved ids at the top of a synthetic vocabulary (the tiny model's eos is vocab-1)."""
        top = vocab - 2
        return cls(im_start=top, im_end=top - 1, user=top - 2, assistant=top - 3, system=top - 4, nl=top - 5,
                   think=top - 6, think_end=top - 7)

    @property
    def reserved(self) -> set[int]:
        return {self.im_start, self.im_end, self.user, self.assistant, self.system, self.nl, self.think,
                self.think_end}

    def turn(self, role: str, ids: list[int]) -> list[int]:
        r = {"user": self.user, "assistant": self.assistant, "system": self.system}[role]
        return [self.im_start, r, self.nl] + list(ids) + [self.im_end, self.nl]

    def generation_suffix(self, enable_thinking: bool = False) -> list[int]:
        head = [self.im_start, self.assistant, self.nl]
        return head if enable_thinking else head + [self.think, self.nl, self.nl, self.think_end, self.nl, self.nl]

    def render(self, messages: list[tuple[str, list[int]]], add_generation_prompt: bool = True,
               enable_thinking: bool = False) -> tuple[list[int], int]:
        """Prompt ids and ``suffix_len`` (the trailing think block, excluded from caching)."""
        out: list[int] = []
        for role, ids in messages:
            out += self.turn(role, ids)
        if not add_generation_prompt:
            return out, 0
        suf = self.generation_suffix(enable_thinking)
        return out + suf, (0 if enable_thinking else len(suf) - 3)
