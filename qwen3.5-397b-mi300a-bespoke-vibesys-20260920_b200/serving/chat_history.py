"""Exact token ids for chat history the model itself wrote.

A chat client sends the previous assistant reply back as text. Encoding that text again need
not give the ids the model generated (a detokenised-then-retokenised reply can split
differently), and the template renders a finished assistant turn differently from the one being
generated (the think block of the generation prompt is dropped from history). Either way the
new prompt stops matching the session cache at the start of the reply, and the whole reply is
prefilled again: a longer time to first token on every later turn.

``ChatHistory`` records, for every finished chat completion, the prompt ids and the generated
ids under a key of (the request's messages, the reply text, the template options). When a new
request ends in [..., assistant reply, user message] and its history and reply match a record,
the prompt becomes the recorded prompt + the generated ids (without their closing stop id) +
the template's tail after the reply, which the tokenizer renders (``render_tail``). A template
whose rendering of the reply cannot be located falls back to the ordinary prompt.

Reference behaviour: ``server.py:519-580`` (``_history_registry_prompt``); the tail is found the
same way for HuggingFace templates (a placeholder reply, rendered and split).
"""

from __future__ import annotations

import hashlib
import json
from collections import Counter, OrderedDict


class ChatHistory:
    def __init__(self, capacity: int = 4096):
        self.capacity = capacity
        self._recs: OrderedDict[str, tuple[list[int], list[int]]] = OrderedDict()
        self.stats: Counter = Counter()

    def clear(self) -> None:
        self._recs.clear()

    @staticmethod
    def key(history: list[dict], reply_text: str, options: dict) -> str:
        raw = json.dumps([history, reply_text.strip(), options], sort_keys=True, ensure_ascii=False, default=str)
        return hashlib.sha256(raw.encode()).hexdigest()

    def record(self, messages: list[dict], options: dict, reply_text: str, prompt_ids, out_ids) -> None:
        k = self.key(list(messages), reply_text, options)
        self._recs[k] = (list(prompt_ids), list(out_ids))
        self._recs.move_to_end(k)
        while len(self._recs) > self.capacity:
            self._recs.popitem(last=False)

    def splice(self, tok, messages: list[dict], options: dict, stop_ids=()) -> tuple[list[int], int] | None:
        """(prompt ids, suffix_len) built from the recorded ids, or None (ordinary prompt)."""
        if len(messages) < 2 or messages[-2].get("role") != "assistant" or messages[-1].get("role") != "user":
            return None
        reply = messages[-2].get("content")
        if not isinstance(reply, str):
            return None
        rec = self._recs.get(self.key(list(messages[:-2]), reply, options))
        if rec is None:
            self.stats["miss"] += 1
            return None
        got = tok.render_tail(messages, bool(options.get("enable_thinking", False)))
        if got is None:
            self.stats["tail_unavailable"] += 1
            return None
        tail, suffix = got
        prompt, out = rec
        if out and (out[-1] in stop_ids or (tail and out[-1] == tail[0])):
            out = out[:-1]  # the tail opens with the template's own closing token
        self._recs.move_to_end(self.key(list(messages[:-2]), reply, options))
        self.stats["spliced"] += 1
        return prompt + out + tail, suffix
