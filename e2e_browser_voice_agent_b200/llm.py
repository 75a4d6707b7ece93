"""The engine's public face over token ids: h2-own-inference-engine/engine/llm.js restated for the cuda backend.

  llm = LLM.load(path_to_gguf, ctx=2048)        # llm.js:13-33 (backend "cuda"; the file is read from disk)
  nxt = llm.feed(ids)                           # llm.js:45-54: reuses the longest common prefix of the cache
  for piece in llm.chat(messages, max_tokens=128): ...   # llm.js:56-82: text in, streamed text out
  out = llm.generate_ids(ids, steps)            # llm.js:86-97: greedy continuation for correctness checks

The text front end (tokenizer.py: byte-level BPE from the GGUF's vocabulary and merges, ChatML prompts) runs on the
host; chat needs a GGUF that carries a merge list (the seeded benchmark models carry synthetic token strings only).
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Sequence

from . import gguf as G
from .backend import CudaBackend
from .tokenizer import Tokenizer, chat_prompt


class LLM:
    @staticmethod
    def load(path: str, backend: str = "cuda", ctx: int = 2048, **opts) -> "LLM":
        if backend != "cuda":
            raise ValueError(f"backend {backend!r}: this engine provides the 'cuda' backend only")
        t0 = time.perf_counter()
        parsed, data = G.load_file(path)
        cfg = G.qwen2_config(parsed["meta"])
        if cfg["arch"] != "qwen2":
            raise ValueError(f"unsupported architecture {cfg['arch']}")  # llm.js:19
        tok = Tokenizer.from_gguf(parsed["meta"])
        t1 = time.perf_counter()
        be = CudaBackend(parsed, data, cfg, ctx=ctx, **opts)
        llm = LLM(be, cfg, tok)
        llm.load_times = {"read": (t1 - t0) * 1e3, "prepare": (time.perf_counter() - t1) * 1e3}
        return llm

    def __init__(self, backend: CudaBackend, cfg: Dict, tokenizer: Optional[Tokenizer] = None):
        self.be = backend
        self.cfg = cfg
        self.tok = tokenizer
        self.seen: List[int] = []   # tokens whose K/V are in the cache, in order (llm.js:37)
        self.stats: Optional[Dict] = None
        # generation stops at the end-of-sequence token and at <|endoftext|> (llm.js:40)
        self.stop_ids = {cfg.get("eos")}
        if tokenizer is not None and "<|endoftext|>" in tokenizer.ids:
            self.stop_ids.add(tokenizer.ids["<|endoftext|>"])

    @property
    def backend(self) -> str:
        return self.be.name

    def feed(self, ids: Sequence[int], temperature: float = 0.0, seed: int = 1) -> Dict:
        """Process ids as a continuation of the cache, reusing the longest common prefix (llm.js:45-54)."""
        ids = [int(t) for t in ids]
        common = 0
        while common < len(ids) and common < len(self.seen) and ids[common] == self.seen[common]:
            common += 1
        if common == len(ids):
            common -= 1  # always run at least one token to get fresh logits
        self.seen = ids[:common]
        fresh = ids[common:]
        nxt = self.be.forward(fresh, common, temperature=temperature, seed=seed)
        self.seen.extend(fresh)
        return {"next": nxt, "prefilled": len(fresh), "reused": common}

    def chat(self, messages: Sequence[Dict[str, str]], max_tokens: int = 256, temperature: float = 0.0,
             seed: int = 1, stop=None):
        """Stream the assistant's reply as text pieces (llm.js:56-82): the ChatML prompt, oldest exchanges dropped
        (never the system prompt) until prompt + reply fit the context, the cached prefix reused, tokens decoded as
        they come (characters split across tokens held back), the end-of-turn token kept in the history so the next
        turn's prompt matches the cache. stop (optional): a callable returning True to end the reply early."""
        if self.tok is None:
            raise RuntimeError("this model's GGUF carries no merge list: chat needs its tokenizer")
        msgs = list(messages)
        ids = self.tok.encode(chat_prompt(msgs))
        while len(ids) + max_tokens > self.be.ctx - 8 and len(msgs) > 2:
            msgs = [msgs[0]] + msgs[3:] if msgs[0].get("role") == "system" else msgs[2:]
            ids = self.tok.encode(chat_prompt(msgs))
        dec = self.tok.stream_decoder()
        t0 = time.perf_counter()
        r = self.feed(ids, temperature=temperature, seed=seed)
        nxt, t_first = r["next"], time.perf_counter() - t0
        out: List[int] = []
        while nxt not in self.stop_ids and len(out) < max_tokens and not (stop and stop()):
            out.append(nxt)
            piece = dec(nxt)
            if piece:
                yield piece
            nxt = self.be.forward([nxt], len(self.seen), temperature=temperature, seed=seed)
            self.seen.append(out[-1])
        if nxt in self.stop_ids:
            self.be.forward([nxt], len(self.seen), temperature=temperature, seed=seed)
            self.seen.append(nxt)
        total = time.perf_counter() - t0
        n = len(out)
        self.stats = {"prompt_tokens": len(ids), "prefilled": r["prefilled"], "reused": r["reused"],
                      "first_token_ms": t_first * 1e3, "tokens": n,
                      "decode_tok_per_s": (n - 1) / (total - t_first) if n > 1 and total > t_first else 0.0,
                      "total_ms": total * 1e3, "ids": out}

    def generate_ids(self, ids: Sequence[int], steps: int) -> List[int]:
        """Greedy continuation of raw token ids; resets the cache (llm.js:86-97)."""
        self.seen = []
        out: List[int] = []
        nxt = self.feed(ids)["next"]
        for i in range(steps):
            out.append(nxt)
            if i == steps - 1:
                break
            nxt = self.be.forward([nxt], len(self.seen), temperature=0)
            self.seen.append(out[-1])
        return out

    def reset(self) -> None:
        self.seen = []
