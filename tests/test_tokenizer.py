"""Streaming detokenization and the token-level chat template (no GPU): the deltas the
detokenizer emits add up to exactly the full decode, never split a multi-byte character, skip
special ids, and do not depend on the decode window; the template's turns, generation prompt and
the thinking-suffix length the session cache splits on."""

import pytest

from qwen35_b200.serving.chat import TokenTemplate
from qwen35_b200.serving.tokenizer import ByteTokenizer, Detokenizer

TEXT = "plain ascii, é (2 bytes), 中文 (3 bytes), 😀 (4 bytes) and back to ascii."


@pytest.mark.parametrize("window", [1, 2, 8, 64])
def test_deltas_add_up_to_the_full_decode(window):
    tok = ByteTokenizer(4096, 4095)
    ids = tok.encode(TEXT)
    d = Detokenizer(tok, window=window)
    out = []
    for t in ids:
        piece = d.push(t)
        assert "�" not in piece  # an incomplete character waits for its next bytes
        out.append(piece)
    out.append(d.flush())
    assert "".join(out) == TEXT == tok.decode(ids)


def test_special_ids_add_no_text_and_a_cut_character_flushes_as_a_full_decode_would():
    tok = ByteTokenizer(4096, 4095)
    t = tok.template
    d = Detokenizer(tok)
    ids = tok.encode("ab") + [t.im_end, t.nl] + tok.encode("c")
    text = "".join(d.push(i) for i in ids) + d.flush()
    assert text == "abc"
    d2 = Detokenizer(tok)
    cut = tok.encode("x😀")[:-1]  # the emoji's last byte never arrives
    streamed = "".join(d2.push(i) for i in cut)
    assert streamed == "x"
    assert streamed + d2.flush() == tok.decode(cut)  # the replacement character, as a full decode gives


def test_template_turns_and_generation_suffix():
    t = TokenTemplate.for_vocab(4096)
    assert len(t.reserved) == 8 and max(t.reserved) == 4094  # below the tiny model's eos (4095)
    ids, suffix = t.render([("system", [1, 2]), ("user", [3])])
    turn_sys = [t.im_start, t.system, t.nl, 1, 2, t.im_end, t.nl]
    turn_user = [t.im_start, t.user, t.nl, 3, t.im_end, t.nl]
    gen = [t.im_start, t.assistant, t.nl]
    think = [t.think, t.nl, t.nl, t.think_end, t.nl, t.nl]
    assert ids == turn_sys + turn_user + gen + think
    assert suffix == len(think)  # the empty think block is not part of the cached history
    ids2, suffix2 = t.render([("user", [3])], enable_thinking=True)
    assert ids2 == turn_user + gen and suffix2 == 0
    ids3, suffix3 = t.render([("user", [3])], add_generation_prompt=False)
    assert ids3 == turn_user and suffix3 == 0


def test_byte_tokenizer_chat_tail_continues_a_recorded_reply():
    """The ids after an assistant reply's content (its closing tokens, the next user turn, the
    generation prompt) extend the prompt that produced the reply to the full rendering."""
    tok = ByteTokenizer(4096, 4095)
    msgs = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"},
            {"role": "user", "content": "more"}]
    full, suffix = tok.render_chat(msgs)
    first, _ = tok.render_chat(msgs[:1])
    reply = tok.encode("yo")
    tail, tail_suffix = tok.render_tail(msgs)
    head = first[: len(first) - 9]  # drop the first prompt's generation prompt + think block
    gen_head = first[len(head): len(head) + 3]
    assert head + gen_head + reply + tail == full and tail_suffix == suffix
