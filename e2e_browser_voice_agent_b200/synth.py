"""Seeded synthetic Qwen2 models in GGUF, the inputs of the benchmark configurations.

The reference publishes no numbers on public data; its benchmark configurations specify seeded models instead:
linear and embedding weights ~ N(0, 0.02) quantized to Q4_0, norm weights 1.0 (f32), q/k/v biases ~ N(0, 0.02)
(f32), RoPE theta 1e6, RMSNorm eps 1e-6, and uniform-random prompt ids. Tensor names and shapes follow the
Qwen2 GGUF layout the reference loader reads (cpu-worker.js:57-128). The vocabulary strings are synthetic: the
token loop only needs their count (gguf.js:84).

lm_head modes:
  "tied"  no output.weight; logits use token_embd (Q4_0), as the 0.5B benchmark configuration specifies;
  "q8"    output.weight = Q8_0 quantization of the same float embedding matrix (the layout of the real file the
          reference ships against, which its CPU path requires: cpu-worker.js:126);
  "q4"    output.weight = an independently seeded Q4_0 matrix (untied, the 7B configuration).
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Dict

import numpy as np

from . import gguf as G

# The benchmark configurations (architecture hyper-parameters).
CONFIGS: Dict[str, Dict] = {
    "qwen2-0.5b": dict(layers=24, dim=896, heads=14, kv_heads=2, ffn=4864, vocab=151936, rope_theta=1e6,
                       eps=1e-6, lm_head="tied"),
    "qwen2-7b": dict(layers=28, dim=3584, heads=28, kv_heads=4, ffn=18944, vocab=152064, rope_theta=1e6,
                     eps=1e-6, lm_head="q4"),
    # small models with the same structure, for fast parity tests
    "tiny": dict(layers=2, dim=128, heads=2, kv_heads=1, ffn=256, vocab=512, rope_theta=1e6, eps=1e-6,
                 lm_head="tied"),
    "small": dict(layers=3, dim=256, heads=4, kv_heads=2, ffn=640, vocab=2048, rope_theta=1e6, eps=1e-6,
                  lm_head="tied"),
    "small-q8": dict(layers=3, dim=256, heads=4, kv_heads=2, ffn=640, vocab=2048, rope_theta=1e6, eps=1e-6,
                     lm_head="q8"),
    "gqa7": dict(layers=2, dim=448, heads=7, kv_heads=1, ffn=1024, vocab=4096, rope_theta=1e6, eps=1e-6,
                 lm_head="tied"),
    "hd128": dict(layers=2, dim=512, heads=4, kv_heads=2, ffn=1024, vocab=2048, rope_theta=1e6, eps=1e-6,
                  lm_head="q4"),
    # lm_heads of 16384 rows of 64 blocks (the tensor-core one-token matvec, as the 7B output matrix takes it)
    "q8-wide": dict(layers=1, dim=2048, heads=16, kv_heads=4, ffn=2048, vocab=16384, rope_theta=1e6, eps=1e-6,
                    lm_head="q8"),
    "q4-wide": dict(layers=1, dim=2048, heads=16, kv_heads=4, ffn=2048, vocab=16384, rope_theta=1e6, eps=1e-6,
                    lm_head="q4"),
    # the 7B layer shapes (hidden 3584, 28 / 4 heads of 128, FFN 18944, untied lm_head) with 2 layers and a smaller
    # vocabulary, for parity tests against the oracle at the 7B matrix sizes
    "qwen2-7b-2l": dict(layers=2, dim=3584, heads=28, kv_heads=4, ffn=18944, vocab=8192, rope_theta=1e6, eps=1e-6,
                        lm_head="q4"),
}


def _normal(rng: np.random.Generator, n: int, std: float = 0.02) -> np.ndarray:
    return (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float32)


def build(path: str, cfg: Dict, seed: int = 0, tokenizer=None) -> None:
    """Write the seeded model described by cfg to path (GGUF v3). tokenizer (optional): (tokens, merges, token
    types) written as the GGUF tokenizer arrays (len(tokens) must be cfg["vocab"]); else synthetic token strings."""
    D, F, H, KVH, L, V = cfg["dim"], cfg["ffn"], cfg["heads"], cfg["kv_heads"], cfg["layers"], cfg["vocab"]
    HD = D // H
    rng = np.random.default_rng(seed)
    seeds = rng.integers(0, 2**63 - 1, size=16 * L + 16)
    k = iter(seeds)

    def q4(n_rows, n_cols, s):
        return lambda: G.q4_0_quantize(_normal(np.random.default_rng(s), n_rows * n_cols))

    def f32_normal(n, s):
        return lambda: _normal(np.random.default_rng(s), n).tobytes()

    ones = lambda n: (lambda: np.ones(n, dtype=np.float32).tobytes())
    t = []
    emb_seed = int(next(k))
    t.append(("token_embd.weight", [D, V], G.TYPE["Q4_0"], q4(V, D, emb_seed)))
    for l in range(L):
        p = f"blk.{l}."
        t.append((p + "attn_norm.weight", [D], G.TYPE["F32"], ones(D)))
        t.append((p + "attn_q.weight", [D, D], G.TYPE["Q4_0"], q4(D, D, int(next(k)))))
        t.append((p + "attn_q.bias", [D], G.TYPE["F32"], f32_normal(D, int(next(k)))))
        t.append((p + "attn_k.weight", [D, KVH * HD], G.TYPE["Q4_0"], q4(KVH * HD, D, int(next(k)))))
        t.append((p + "attn_k.bias", [KVH * HD], G.TYPE["F32"], f32_normal(KVH * HD, int(next(k)))))
        t.append((p + "attn_v.weight", [D, KVH * HD], G.TYPE["Q4_0"], q4(KVH * HD, D, int(next(k)))))
        t.append((p + "attn_v.bias", [KVH * HD], G.TYPE["F32"], f32_normal(KVH * HD, int(next(k)))))
        t.append((p + "attn_output.weight", [D, D], G.TYPE["Q4_0"], q4(D, D, int(next(k)))))
        t.append((p + "ffn_norm.weight", [D], G.TYPE["F32"], ones(D)))
        t.append((p + "ffn_gate.weight", [D, F], G.TYPE["Q4_0"], q4(F, D, int(next(k)))))
        t.append((p + "ffn_up.weight", [D, F], G.TYPE["Q4_0"], q4(F, D, int(next(k)))))
        t.append((p + "ffn_down.weight", [F, D], G.TYPE["Q4_0"], q4(D, F, int(next(k)))))
    t.append(("output_norm.weight", [D], G.TYPE["F32"], ones(D)))
    mode = cfg.get("lm_head", "tied")
    if mode == "q8":
        t.append(("output.weight", [D, V], G.TYPE["Q8_0"],
                  lambda: G.q8_0_quantize(_normal(np.random.default_rng(emb_seed), V * D))))
    elif mode == "q4":
        t.append(("output.weight", [D, V], G.TYPE["Q4_0"], q4(V, D, int(next(k)))))
    elif mode != "tied":
        raise ValueError(f"unknown lm_head mode {mode}")

    kv = [
        ("general.architecture", 8, "qwen2"),
        ("general.alignment", 4, 32),
        ("qwen2.block_count", 4, L),
        ("qwen2.context_length", 4, 32768),
        ("qwen2.embedding_length", 4, D),
        ("qwen2.feed_forward_length", 4, F),
        ("qwen2.attention.head_count", 4, H),
        ("qwen2.attention.head_count_kv", 4, KVH),
        ("qwen2.rope.freq_base", 6, float(cfg["rope_theta"])),
        ("qwen2.attention.layer_norm_rms_epsilon", 6, float(cfg["eps"])),
        ("tokenizer.ggml.model", 8, "gpt2"),
    ]
    if tokenizer is None:
        kv += [("tokenizer.ggml.tokens", 9, (8, [f"<t{i}>" for i in range(V)])), ("tokenizer.ggml.eos_token_id", 4, V - 1)]
    else:
        toks, merges, types = tokenizer
        if len(toks) != V:
            raise ValueError(f"tokenizer has {len(toks)} tokens, the model's vocabulary {V}")
        eos = toks.index("<|endoftext|>") if "<|endoftext|>" in toks else V - 1
        kv += [("tokenizer.ggml.tokens", 9, (8, list(toks))), ("tokenizer.ggml.merges", 9, (8, list(merges))),
               ("tokenizer.ggml.token_type", 9, (5, [int(t) for t in types])), ("tokenizer.ggml.eos_token_id", 4, eos)]
    G.write_gguf(path, kv, t)


def cache_dir() -> str:
    d = os.environ.get("H2_MODEL_CACHE") or os.path.join(os.environ.get("TMPDIR", "/tmp"), "h2b200_models")
    os.makedirs(d, exist_ok=True)
    return d


def ensure(name: str, seed: int = 0, **overrides) -> str:
    """Path of the seeded model `name` (a CONFIGS key), building it once into the cache directory."""
    cfg = dict(CONFIGS[name], **overrides)
    key = hashlib.sha256(json.dumps([cfg, seed, 1], sort_keys=True).encode()).hexdigest()[:16]
    path = os.path.join(cache_dir(), f"{name}-s{seed}-{key}.gguf")
    if not os.path.exists(path):
        build(path, cfg, seed)
    return path


def prompt_ids(vocab: int, n: int, seed: int = 1) -> np.ndarray:
    """n uniform-random prompt token ids in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int32)


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


def device_tensors(name: str, seed: int = 0, device: int = 0):
    """A seeded synthetic model of CONFIGS[name] generated on the GPU without a file (the full 7B configuration's
    3.98 GB of Q4_0 would take minutes to write with numpy): returns (cfg, source) with source(tensor name) ->
    (ggml type, raw GGUF bytes as a host array) or None, for backend.CudaBackend(source, None, cfg). Linear and
    embedding weights ~ N(0, 0.02) (torch's generator, seeded per tensor) quantized to Q4_0 with the ggml reference
    algorithm (the one of gguf.q4_0_quantize, on the GPU); norm weights 1.0; q/k/v biases ~ N(0, 0.02)."""
    import torch

    c = CONFIGS[name]
    D, F, H, KVH, L, V = c["dim"], c["ffn"], c["heads"], c["kv_heads"], c["layers"], c["vocab"]
    HD = D // H
    dev = torch.device("cuda", device)
    shapes = {"token_embd.weight": (V, D), "output.weight": (V, D)}
    for l in range(L):
        p = f"blk.{l}."
        shapes.update({p + "attn_q.weight": (D, D), p + "attn_k.weight": (KVH * HD, D),
                       p + "attn_v.weight": (KVH * HD, D), p + "attn_output.weight": (D, D),
                       p + "ffn_gate.weight": (F, D), p + "ffn_up.weight": (F, D), p + "ffn_down.weight": (D, F),
                       p + "attn_q.bias": (D,), p + "attn_k.bias": (KVH * HD,), p + "attn_v.bias": (KVH * HD,)})
    names = sorted(shapes)

    def normal(n, key):
        g = torch.Generator(device=dev)
        g.manual_seed((seed * 1000003 + names.index(key) * 7919 + 17) & 0x7FFFFFFFFFFFFFFF)
        return torch.randn(n, generator=g, device=dev, dtype=torch.float32) * 0.02

    def q4_0(x):
        x = x.reshape(-1, 32)
        idx = torch.argmax(x.abs(), dim=1)                  # first of equal magnitudes
        m = x.gather(1, idx[:, None])[:, 0]
        d = m / -8.0
        inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
        q = torch.clamp((x * inv[:, None] + 8.5).to(torch.int32), max=15).to(torch.uint8)  # trunc toward zero
        out = torch.empty(x.shape[0], 18, dtype=torch.uint8, device=dev)
        out[:, 0:2] = d.to(torch.float16).view(torch.uint8).reshape(-1, 2)
        out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
        return out.reshape(-1).cpu().numpy()

    def source(tname: str):
        if tname.endswith("norm.weight"):
            return G.TYPE["F32"], np.ones(D, dtype=np.float32).view(np.uint8)
        if tname == "output.weight" and c.get("lm_head", "tied") == "tied":
            return None
        if tname not in shapes:
            return None
        sh = shapes[tname]
        n = int(np.prod(sh))
        if len(sh) == 1:
            return G.TYPE["F32"], normal(n, tname).cpu().numpy().view(np.uint8)
        return G.TYPE["Q4_0"], q4_0(normal(n, tname))

    cfg = {"arch": "qwen2", "dim": D, "layers": L, "ffn": F, "heads": H, "kv_heads": KVH, "vocab": V,
           "eps": c["eps"], "rope_theta": c["rope_theta"]}
    return cfg, source
