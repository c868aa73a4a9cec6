"""Chat history with the exact generated ids (CPU): a recorded reply sent back as history is
spliced in as the generated ids, so the next prompt extends the cached sequence."""

from qwen35_b200.serving.chat_history import ChatHistory
from qwen35_b200.serving.tokenizer import ByteTokenizer, HFTokenizer


def test_splice_with_the_token_template():
    tok = ByteTokenizer(4096, 4095)
    t = tok.template
    h = ChatHistory()
    first = [{"role": "user", "content": "hi"}]
    prompt, _ = tok.render_chat(first)
    out = tok.encode("hello there") + [tok.eos_token_id]
    h.record(first, {}, tok.decode(out), prompt, out)
    nxt = first + [{"role": "assistant", "content": "hello there"}, {"role": "user", "content": "more"}]
    ids, suffix = h.splice(tok, nxt, {}, {tok.eos_token_id, t.im_end})
    tail = [t.im_end, t.nl] + t.turn("user", tok.encode("more")) + t.generation_suffix(False)
    assert ids == prompt + out[:-1] + tail
    assert suffix == tok.render_chat(nxt)[1]
    assert ids[:len(prompt) + len(out) - 1] == prompt + out[:-1]  # the cached sequence, token for token
    # another reply text, other history or other template options: ordinary prompt
    assert h.splice(tok, first + [{"role": "assistant", "content": "hello"}, nxt[-1]], {}) is None
    assert h.splice(tok, [{"role": "user", "content": "yo"}] + nxt[1:], {}) is None
    assert h.splice(tok, nxt, {"enable_thinking": True}) is None
    assert h.splice(tok, nxt[:2], {}) is None  # does not end with a user message
    assert h.stats["spliced"] == 1
    # a reply that ended on the template's closing token itself: that token is not doubled
    out2 = tok.encode("ok") + [t.im_end]
    h.record(first, {"x": 1}, tok.decode(out2), prompt, out2)
    ids2, _ = h.splice(tok, first + [{"role": "assistant", "content": "ok"}, nxt[-1]], {"x": 1})
    assert ids2 == prompt + out2[:-1] + tail


def test_lru_capacity():
    h = ChatHistory(capacity=2)
    for i in range(3):
        h.record([{"role": "user", "content": str(i)}], {}, "r", [i], [i])
    assert len(h._recs) == 2


class _FakeHF:
    """A Qwen-like text template over a character-level encoding."""

    all_special_tokens = ["<|im_start|>", "<|im_end|>"]

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True, enable_thinking=False):
        out = ""
        for m in messages:
            out += f"<|im_start|>{m['role']}\n{str(m['content']).strip()}<|im_end|>\n"
        if add_generation_prompt:
            out += "<|im_start|>assistant\n" + ("" if enable_thinking else "<think>\n\n</think>\n\n")
        return out

    def encode(self, text, add_special_tokens=False):
        return [ord(c) for c in text]


def test_hf_tail_found_by_placeholder():
    tok = object.__new__(HFTokenizer)
    tok.tok = _FakeHF()
    tok.eos_token_id = None
    msgs = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": " hello "},
            {"role": "user", "content": "more"}]
    tail, suffix = tok.render_tail(msgs)
    assert "".join(map(chr, tail)) == "<|im_end|>\n<|im_start|>user\nmore<|im_end|>\n<|im_start|>assistant\n" \
                                      "<think>\n\n</think>\n\n"
    assert suffix == tok.render_chat(msgs)[1] > 0
    # a template that rewrites the reply cannot be split: ordinary prompt
    tok.tok.apply_chat_template = lambda m, **k: _FakeHF.apply_chat_template(
        tok.tok, [{**x, "content": str(x["content"]).upper()} for x in m], **k)
    assert tok.render_tail(msgs) is None


def test_stop_ids_from_config_generation_config_and_tokenizer(tmp_path):
    import json

    from qwen35_b200.serving.server import stop_ids

    tok = ByteTokenizer(4096, 4095)
    assert stop_ids(None, 7, tok) == {7, 4095}
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [11, 12]}))
    assert stop_ids(str(tmp_path), 7, tok) == {7, 11, 12, 4095}


def test_hf_prompts_tokenized_incrementally_after_selfcheck():
    tok = object.__new__(HFTokenizer)
    tok.tok = _FakeHF()
    tok.eos_token_id = None
    assert tok.enable_prompt_cache()
    msgs = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "hello"},
            {"role": "user", "content": "more"}]
    ids, _ = tok.render_chat(msgs)
    full = tok.encode(tok.tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True))
    assert ids == full and tok.prompts.entries  # the prefix up to the last turn end is cached

    class _Merging(_FakeHF):  # an encoder whose ids depend on text before the boundary
        def encode(self, text, add_special_tokens=False):
            return [len(text)] + [ord(c) for c in text]

    tok.tok = _Merging()
    assert not tok.enable_prompt_cache() and tok.prompts is None
    assert tok.render_chat(msgs)[0] == tok.encode(tok.tok.apply_chat_template(msgs, tokenize=False,
                                                                               add_generation_prompt=True))


class _CountingTok:
    """Whitespace-free byte tokenizer stand-in that records every ``encode`` input length."""

    def __init__(self):
        self.lengths = []

    def encode(self, text):
        self.lengths.append(len(text))
        return [ord(c) for c in text]


def test_prompt_cache_encodes_each_turn_incrementally():
    from qwen35_b200.serving.tokenizer import PromptCache

    tok = _CountingTok()
    pc = PromptCache(tok, capacity=8)
    conv = "<|im_start|>system\nbe brief<|im_end|>\n"
    cached = 0  # length of the longest cached boundary prefix
    for turn in range(6):
        conv += f"<|im_start|>user\nquestion number {turn}<|im_end|>\n<|im_start|>assistant\n"
        tok.lengths.clear()
        ids = pc.encode(conv)
        assert ids == [ord(c) for c in conv]
        # only the characters after the previous turn's cached boundary are encoded, once
        assert sum(tok.lengths) == len(conv) - cached, (turn, tok.lengths)
        cached = conv.rfind("<|im_end|>") + len("<|im_end|>")
        conv += f"answer {turn}<|im_end|>\n"
    assert len(pc.entries) <= 8
