"""Tokenizer adapters and incremental detokenization.

``load_tokenizer(model_dir)`` returns the checkpoint's HuggingFace tokenizer when the directory
has one, and otherwise ``ByteTokenizer``: UTF-8 bytes map to ids 0..255 and the chat-template
specials sit at the top of the vocabulary (``chat.TokenTemplate.for_vocab``), which is what the
random-init models use. ``Detokenizer`` turns a growing id list into text deltas whose
concatenation equals decoding the whole list at once (it holds back text that ends in an
incomplete UTF-8 sequence); reference behaviour ``server.py:325-349``. ``PromptCache`` reuses the
ids of the longest previously tokenized prefix that ends at a special token (reference
``prompt_cache.py:21-80``).
"""

from __future__ import annotations

import os
from collections import OrderedDict

from .chat import TokenTemplate


class ByteTokenizer:
    """Bytes as token ids plus the template specials; ``eos`` is the model's eos id."""

    def __init__(self, vocab: int, eos: int):
        self.vocab = vocab
        self.eos_token_id = eos
        self.template = TokenTemplate.for_vocab(vocab)
        self._special = self.template.reserved | {eos}

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def render_chat(self, messages: list[dict], enable_thinking: bool = False) -> tuple[list[int], int]:
        msgs = [(m["role"], self.encode(str(m.get("content") or ""))) for m in messages]
        return self.template.render(msgs, True, enable_thinking)

    def render_tail(self, messages: list[dict], enable_thinking: bool = False) -> tuple[list[int], int]:
        """Ids after the content of the assistant message ``messages[-2]`` (its closing tokens,
        the later turns, the generation prompt) and the prompt's ``suffix_len``."""
        t = self.template
        rest = [(m["role"], self.encode(str(m.get("content") or ""))) for m in messages[-1:]]
        ids, suffix = t.render(rest, True, enable_thinking)
        return [t.im_end, t.nl] + ids, suffix


class HFTokenizer:
    """A HuggingFace tokenizer with Qwen's chat template."""

    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path)
        self.eos_token_id = self.tok.eos_token_id
        self.enable_prompt_cache()

    PROBES = ([{"role": "user", "content": "Hello! How are you today?"}],
              [{"role": "system", "content": "Be brief."}, {"role": "user", "content": "2+2?"},
               {"role": "assistant", "content": "4"}, {"role": "user", "content": "And 3+3, explained?"}])

    def enable_prompt_cache(self, capacity: int = 256) -> bool:
        """Tokenize chat prompts incrementally (``PromptCache``) if, on a few probe
        conversations, that gives exactly the ids of full tokenization; else encode in full."""
        self.prompts = PromptCache(self, capacity)
        try:
            samples = [self.tok.apply_chat_template(list(m), tokenize=False, add_generation_prompt=True)
                       for m in self.PROBES]
            samples += [s2 for s in samples for s2 in (s, s + "<|im_start|>user\nmore<|im_end|>\n")]
            ok = self.prompts.selfcheck(samples)
        except Exception:  # noqa: BLE001 - a template the probes do not fit: full encoding
            ok = False
        if not ok:
            self.prompts = None
        return ok

    def encode_prompt(self, text: str) -> list[int]:
        return self.prompts.encode(text) if getattr(self, "prompts", None) is not None else self.encode(text)

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    PLACEHOLDER = "\u2063qb-reply-placeholder\u2063"

    def render_tail(self, messages: list[dict], enable_thinking: bool = False) -> tuple[list[int], int] | None:
        """Ids after the content of the assistant message ``messages[-2]`` and the prompt's
        ``suffix_len``: the template is rendered with a placeholder reply and split there. None
        when the template changes the reply text or the tail does not open with a special token
        (the ids could not be joined at that point)."""
        reply = messages[-2].get("content")
        if not isinstance(reply, str) or any(self.PLACEHOLDER in str(m.get("content")) for m in messages):
            return None
        marked = [*messages[:-2], {**messages[-2], "content": self.PLACEHOLDER}, messages[-1]]
        try:
            text = self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                                enable_thinking=enable_thinking)
            mtext = self.tok.apply_chat_template(marked, tokenize=False, add_generation_prompt=True,
                                                 enable_thinking=enable_thinking)
        except Exception:  # noqa: BLE001 - an unfamiliar template: ordinary prompt
            return None
        if mtext.count(self.PLACEHOLDER) != 1:
            return None
        head, tail = mtext.split(self.PLACEHOLDER)
        if text != head + reply.strip() + tail:
            return None
        if not tail or not any(tail.startswith(s) for s in self.tok.all_special_tokens):
            return None
        _, suffix = self.render_chat(messages, enable_thinking)
        return self.encode(tail), suffix

    def render_chat(self, messages: list[dict], enable_thinking: bool = False) -> tuple[list[int], int]:
        text = self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                            enable_thinking=enable_thinking)
        ids = self.encode_prompt(text)
        suffix = 0
        if not enable_thinking:
            bare = self.tok.apply_chat_template(messages, tokenize=False, add_generation_prompt=True,
                                                enable_thinking=True)
            common = os.path.commonprefix([text, bare])
            suffix = max(0, len(ids) - len(self.encode(common)))
        return ids, suffix


def load_tokenizer(model_dir: str | None, vocab: int, eos: int):
    if model_dir and any(os.path.exists(os.path.join(model_dir, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        try:
            return HFTokenizer(model_dir)
        except Exception:
            pass
    return ByteTokenizer(vocab, eos)


class Detokenizer:
    """Incremental decode: ``push(id)`` returns the new text a full decode would add."""

    def __init__(self, tokenizer, window: int = 8):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.prefix = 0  # start of the decode window
        self.read = 0  # ids already reflected in emitted text
        self.window = window

    def push(self, tid: int) -> str:
        self.ids.append(tid)
        prev = self.tok.decode(self.ids[self.prefix:self.read])
        cur = self.tok.decode(self.ids[self.prefix:])
        if cur.endswith("�"):
            return ""  # incomplete multi-byte character: wait for more ids
        delta = cur[len(prev):]
        self.read = len(self.ids)
        if self.read - self.prefix > self.window:
            self.prefix = self.read - self.window
        return delta

    def flush(self) -> str:
        prev = self.tok.decode(self.ids[self.prefix:self.read])
        cur = self.tok.decode(self.ids[self.prefix:])
        self.read = len(self.ids)
        return cur[len(prev):]


class PromptCache:
    """Incremental tokenization of chat prompts that share a prefix with an earlier prompt."""

    def __init__(self, tokenizer, capacity: int = 256, boundary: str = "<|im_end|>"):
        self.tok = tokenizer
        self.capacity = capacity
        self.boundary = boundary
        self.entries: OrderedDict[str, list[int]] = OrderedDict()

    def encode(self, text: str) -> list[int]:
        """Ids of ``text``: the cached ids of its longest cached prefix that ends at a turn
        boundary, plus the encoding of the rest. The prefix up to ``text``'s own last boundary
        is cached for the next turn, built from the same pieces, so each call encodes only the
        characters after the longest cached prefix."""
        best = ""
        for k in self.entries:
            if len(k) > len(best) and text.startswith(k):
                best = k
        head = list(self.entries[best]) if best else []
        if best:
            self.entries.move_to_end(best)
        cut = text.rfind(self.boundary)
        end = cut + len(self.boundary) if cut >= 0 else 0
        if end > len(best):  # a new boundary past the cached prefix: extend and cache it
            head = head + self.tok.encode(text[len(best):end])
            key = text[:end]
            self.entries[key] = head
            self.entries.move_to_end(key)
            if len(self.entries) > self.capacity:
                self.entries.popitem(last=False)
            best = key
        return list(head) + (self.tok.encode(text[len(best):]) if len(text) > len(best) else [])

    def selfcheck(self, samples: list[str]) -> bool:
        """Incremental ids equal full tokenization for every sample (run at boot)."""
        return all(self.encode(s) == self.tok.encode(s) for s in samples)
