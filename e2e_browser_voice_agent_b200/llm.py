"""The engine's public face over token ids: h2-own-inference-engine/engine/llm.js restated for the cuda backend.

  llm = LLM.load(path_to_gguf, ctx=2048)        # llm.js:13-33 (backend "cuda"; the file is read from disk)
  nxt = llm.feed(ids)                           # llm.js:45-54: reuses the longest common prefix of the cache
  out = llm.generate_ids(ids, steps)            # llm.js:86-97: greedy continuation for correctness checks

Text in / text out (the tokenizer, llm.js chat) is outside this engine's scope: it runs on token ids.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional, Sequence

from . import gguf as G
from .backend import CudaBackend


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
        t1 = time.perf_counter()
        be = CudaBackend(parsed, data, cfg, ctx=ctx, **opts)
        llm = LLM(be, cfg)
        llm.load_times = {"read": (t1 - t0) * 1e3, "prepare": (time.perf_counter() - t1) * 1e3}
        return llm

    def __init__(self, backend: CudaBackend, cfg: Dict):
        self.be = backend
        self.cfg = cfg
        self.seen: List[int] = []   # tokens whose K/V are in the cache, in order (llm.js:37)
        self.stats: Optional[Dict] = None

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
