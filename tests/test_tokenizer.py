"""The host-side byte-level BPE tokenizer (tokenizer.py, restating h2-own-inference-engine/engine/tokenizer.js).

Pinned three ways (the real Qwen2.5 vocabulary is not available here):
  - the reference's own cases (tests/golden/tokenizer_cases.json, extracted from m1-llm/reference.json): every case
    has at least as many ids as pre-tokenizer pieces, and where the counts are equal each single-byte piece carries
    the id the reference gives it (Qwen2's first 256 ids are the bytes in GPT-2's byte-table order);
  - an independent byte-level BPE (Hugging Face `tokenizers`, the library that produced the reference's ids) trained
    here on a synthetic corpus, with Qwen2's pre-tokenizer: identical ids on many strings;
  - decode(encode(text)) == NFC(text), special tokens, the streaming decoder and the ChatML prompt.
"""
import json
import os
import random
import unicodedata

import pytest

from e2e_browser_voice_agent_b200 import tokenizer as T

import bpe_vocab

HERE = os.path.dirname(os.path.abspath(__file__))
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def fixture():
    with open(os.path.join(HERE, "golden", "tokenizer_cases.json")) as f:
        return json.load(f)


def byte_rank():
    """byte -> its position in GPT-2's table order (printable bytes first): the byte's id in Qwen2's vocabulary"""
    table = T.byte_table()
    order = sorted(range(256), key=lambda b: ord(table[b]))
    return {b: i for i, b in enumerate(order)}


def pieces_with_special(tok, text):
    out = []
    for part in T.regex.split("(" + "|".join(T.regex.escape(s) for s in SPECIAL) + ")", unicodedata.normalize("NFC", text)):
        if part:
            out.extend([part] if part in SPECIAL else tok.pieces(part))
    return out


def test_byte_table_is_a_printable_bijection():
    t = T.byte_table()
    assert len(set(t)) == 256
    assert all(len(c) == 1 and not c.isspace() and c.isprintable() for c in t)
    assert t[ord("A")] == "A" and t[0x20] == chr(256 + 32) and t[0] == chr(256)


def test_pre_tokenizer_against_the_reference_cases():
    d = fixture()
    tok = T.Tokenizer({"tokenizer.ggml.tokens": ["x"], "tokenizer.ggml.merges": []})
    rank = byte_rank()
    equal = 0
    for c in d["cases"]:
        p = pieces_with_special(tok, c["text"])
        assert len(p) <= c["n_ids"], c["text"]
        if len(p) == c["n_ids"]:
            equal += 1
            for piece, i in zip(p, c["ids"]):
                b = piece.encode("utf-8")
                if len(b) == 1:
                    assert i == rank[b[0]], (c["text"], piece, i)
    assert equal >= 5
    for c in d["chat_prompts"]:
        assert len(pieces_with_special(tok, c["prompt"])) <= c["n_ids"]


@pytest.fixture(scope="module")
def trained():
    pytest.importorskip("tokenizers")
    import bpe_vocab
    hf, (tokens, merges, types) = bpe_vocab.train()
    ours = T.Tokenizer({"tokenizer.ggml.tokens": tokens, "tokenizer.ggml.merges": merges,
                        "tokenizer.ggml.token_type": types})
    return hf, ours, random.Random(11)


def test_bpe_matches_an_independent_byte_level_bpe(trained):
    hf, ours, rng = trained
    texts = bpe_vocab.corpus(rng, 400) + ["Hello, world!", "  two  spaces and\ttab", "emoji 🙂👍 and 日本語", "line\r\nbreaks\n\n",
                                 "trailing spaces   ", "it's 12345 or 3.14159...", ""]
    for s in texts:
        assert ours.encode(s) == hf.encode(s).ids, repr(s)


def test_round_trip_special_tokens_and_streaming(trained):
    _, tok, rng = trained
    for s in bpe_vocab.corpus(rng, 200):
        s = unicodedata.normalize("NFC", s)
        assert tok.decode(tok.encode(s)) == s
    chat = T.chat_prompt([{"role": "user", "content": "hi there"}])
    assert chat.startswith("<|im_start|>system\n") and chat.endswith("<|im_start|>assistant\n")
    ids = tok.encode(chat)
    assert ids[0] == tok.ids["<|im_start|>"] and tok.ids["<|im_end|>"] in ids
    assert tok.decode(ids) == chat
    s = "naïve 🙂👍 日本語 done"
    dec = tok.stream_decoder()
    assert "".join(dec(i) for i in tok.encode(s)) == s


def test_from_gguf_without_merges_is_none():
    assert T.Tokenizer.from_gguf({"tokenizer.ggml.tokens": ["a", "b"]}) is None
