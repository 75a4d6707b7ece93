"""Byte-level BPE tokenizer of the engine's Qwen2 models, from the vocabulary and merge list stored in the GGUF file
(the host-side text front end of h2-own-inference-engine/engine/tokenizer.js:1-110; no tokenizer library).

  text -> NFC -> split around the special tokens -> pre-split with Qwen2's pattern (words, single digits, punctuation
  runs, newlines, spaces) -> each piece's UTF-8 bytes as printable characters (GPT-2's byte table) -> pairs merged by
  rank until none is in the merge list -> token ids

Same observable behaviour as tokenizer.js: ties between equal-rank pairs go to the leftmost; every occurrence of the
chosen pair is merged left to right in one pass; control and user-defined tokens (GGUF token types 3 and 4) are
matched literally, longest first; a symbol without a token raises. Token ids only feed the CUDA engine, so this
module runs on the host.
"""
from __future__ import annotations

import unicodedata
from typing import Callable, Dict, List, Optional, Sequence

import regex

# JavaScript's \s (the reference's pattern runs in JavaScript): ECMAScript white space and line terminators. Python's
# own \s differs on U+001C..U+001F (space there) and U+FEFF (not).
_WS = "\\t\\n\\v\\f\\r \\u00a0\\u1680\\u2000-\\u200a\\u2028\\u2029\\u202f\\u205f\\u3000\\ufeff"
# Qwen2's pre-tokenizer pattern (tokenizer.js:24): contractions, a word with one optional leading non-letter,
# single digits, punctuation runs with trailing newlines, newline runs, trailing spaces, other spaces.
PRE = regex.compile(r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}"
                    r"| ?[^" + _WS + r"\p{L}\p{N}]+[\r\n]*|[" + _WS + r"]*[\r\n]+|[" + _WS + r"]+(?![^" + _WS + r"])"
                    r"|[" + _WS + r"]+")


def byte_table() -> List[str]:
    """GPT-2's byte -> character table (tokenizer.js:9-19): printable Latin-1 bytes map to themselves, the other 68
    bytes to code points 256, 257, ... in byte order, so every byte is one visible character."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    table = [""] * 256
    for b in keep:
        table[b] = chr(b)
    extra = 256
    for b in range(256):
        if not table[b]:
            table[b] = chr(extra)
            extra += 1
    return table


class Tokenizer:
    def __init__(self, meta: Dict):
        self.tokens: List[str] = list(meta["tokenizer.ggml.tokens"])
        types = meta.get("tokenizer.ggml.token_type")
        # (a repeated string keeps its last index, as a JavaScript Map built from the list does)
        self.ids: Dict[str, int] = {t: i for i, t in enumerate(self.tokens)}
        self.ranks: Dict[str, int] = {m: i for i, m in enumerate(meta.get("tokenizer.ggml.merges") or [])}
        self.b2u = byte_table()
        self.u2b = {c: b for b, c in enumerate(self.b2u)}
        self.special = [t for i, t in enumerate(self.tokens) if types is not None and types[i] in (3, 4)]
        self._special_set = set(self.special)
        self.special_re = (regex.compile("(" + "|".join(regex.escape(s) for s in sorted(self.special, key=len, reverse=True)) + ")")
                           if self.special else None)
        self.cache: Dict[str, List[int]] = {}

    @classmethod
    def from_gguf(cls, meta: Dict) -> Optional["Tokenizer"]:
        """The tokenizer of a GGUF file's metadata, or None when it carries no merge list (the seeded benchmark
        models have synthetic token strings only)."""
        return cls(meta) if meta.get("tokenizer.ggml.merges") else None

    def bpe(self, piece: str) -> List[int]:
        hit = self.cache.get(piece)
        if hit is not None:
            return hit
        syms = [self.b2u[b] for b in piece.encode("utf-8")]
        while len(syms) > 1:
            best, best_rank = -1, None
            for i in range(len(syms) - 1):
                r = self.ranks.get(syms[i] + " " + syms[i + 1])
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best < 0:
                break
            a, b = syms[best], syms[best + 1]
            merged, i = [], 0
            while i < len(syms):
                if i < len(syms) - 1 and syms[i] == a and syms[i + 1] == b:
                    merged.append(a + b)
                    i += 2
                else:
                    merged.append(syms[i])
                    i += 1
            syms = merged
        out = []
        for s in syms:
            t = self.ids.get(s)
            if t is None:
                raise ValueError(f"no token for {s!r}")
            out.append(t)
        if len(self.cache) < 50000:
            self.cache[piece] = out
        return out

    def pieces(self, text: str) -> List[str]:
        """The pre-tokenizer's pieces of a text without special tokens (the matches of PRE)."""
        return [m.group(0) for m in PRE.finditer(text)]

    def encode(self, text: str) -> List[int]:
        out: List[int] = []
        text = unicodedata.normalize("NFC", text)
        parts = self.special_re.split(text) if self.special_re else [text]
        for part in parts:
            if not part:
                continue
            if part in self._special_set:
                out.append(self.ids[part])
                continue
            for p in self.pieces(part):
                out.extend(self.bpe(p))
        return out

    def token_bytes(self, i: int) -> bytes:
        """The bytes of one token (special tokens as their literal UTF-8 text)."""
        t = self.tokens[i]
        if t in self._special_set:
            return t.encode("utf-8")
        return bytes(self.u2b[c] for c in t)

    def decode(self, ids: Sequence[int]) -> str:
        return b"".join(self.token_bytes(int(i)) for i in ids).decode("utf-8", errors="replace")

    def stream_decoder(self) -> Callable[[int], str]:
        """A decoder fed one token at a time that holds back the bytes of a character split across tokens."""
        import codecs
        dec = codecs.getincrementaldecoder("utf-8")(errors="replace")
        return lambda i: dec.decode(self.token_bytes(int(i)))


def chat_prompt(messages: Sequence[Dict[str, str]], add_generation_prompt: bool = True) -> str:
    """Qwen2.5's ChatML prompt for plain text messages (tokenizer.js:104-110)."""
    s = ""
    if not messages or messages[0].get("role") != "system":
        s += "<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n"
    for m in messages:
        s += f"<|im_start|>{m['role']}\n{m['content']}<|im_end|>\n"
    if add_generation_prompt:
        s += "<|im_start|>assistant\n"
    return s
