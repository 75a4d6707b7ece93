"""Test infrastructure: drives the CPU parity oracle. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import this module, and only as the checker or the timed CPU baseline; the product never does.

Two interchangeable kernel libraries sit behind the same driver:
  - "oracle": oracle/_build/libh2oracle.so, the scalar restatement of the reference's kernels (h2_oracle.c);
  - "ref_st" / "ref_mt": oracle/_ref/libh2ref_{st,mt}.so, the reference's own kernels.c compiled natively
    through oracle/shim (single-threaded, or the -DMT barrier pool on pthreads).

The driver restates the reference's CPU backend host (h2-own-inference-engine/engine/cpu-worker.js):
`RefEngine.__init__` follows init (cpu-worker.js:46-151: repack GGUF Q4_0/Q8_0 blocks into separate value and
fp32 scale arrays, concatenate [q;k;v] and [gate;up], copy norms and biases, build the RoPE table in double
precision, lay out the scratch buffers), `forward` follows forward (cpu-worker.js:169-182: context check,
chunks of at most `mt` tokens, logits on the last chunk only) and `sample` follows sample (cpu-worker.js:154-167).

Tied embeddings: the reference requires a Q8_0 output.weight (cpu-worker.js:126). For a model without one, the
driver hands the reference library the lossless Q8_0 re-encoding of token_embd (same fp16 scales, int8 q - 8),
on which dot_q8_q8 computes exactly what dot_q4_q8 computes on the Q4_0 blocks; the restatement can also take
the Q4_0 blocks directly (tensor kind 10).
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
import time
from typing import Dict, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBS = {
    "oracle": os.path.join(HERE, "_build", "libh2oracle.so"),
    "ref_st": os.path.join(HERE, "_ref", "libh2ref_st.so"),
    "ref_mt": os.path.join(HERE, "_ref", "libh2ref_mt.so"),
}
_loaded: Dict[str, C.CDLL] = {}
_owner: Dict[str, object] = {}


def build() -> None:
    """Compile the restatement and, when the reference sources are present, the reference library."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def available(kind: str) -> bool:
    return os.path.exists(LIBS[kind])


def lib(kind: str) -> C.CDLL:
    if kind in _loaded:
        return _loaded[kind]
    path = LIBS[kind]
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
    L = C.CDLL(path)
    p, i, f, d, u32 = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_uint32
    if kind == "oracle":
        pre = "h2o_"
        L.h2o_set_config.restype = i
        L.h2o_set_tensor.restype = i
        L.h2o_sample.argtypes = [p, i, d, u32]
        L.h2o_sample.restype = i
        L.h2o_fast_exp.argtypes = [f]
        L.h2o_fast_exp.restype = f
        L.h2o_quantize_row.argtypes = [p, p, p, p, i]
        L.h2o_rmsnorm.argtypes = [p, p, p, i, f]
        L.h2o_matvec_q4.argtypes = [p, p, i, i, i, p, p, i, p, i, p, p, p]
    else:
        pre = ""
        L.h2shim_start_helpers.argtypes = [i]
        L.h2shim_start_helpers.restype = i
        L.run_barrier_test.argtypes = [i, i]
        L.run_barrier_test.restype = i
        L.run_read_test.argtypes = [i]
    getattr(L, pre + "set_config").argtypes = [i, i, i, i, i, i, i, i, f]
    getattr(L, pre + "set_tensor").argtypes = [i, i, p, p]
    getattr(L, pre + "set_buffers").argtypes = [p] * 15
    getattr(L, pre + "run").argtypes = [i, i, i, i]
    _loaded[kind] = L
    return L


def _ptr(a: Optional[np.ndarray]) -> Optional[int]:
    return None if a is None else a.ctypes.data


def _aligned(n: int, dtype, align: int = 64) -> np.ndarray:
    """Zeroed array whose data starts on an `align`-byte boundary (the reference lays buffers out on 64 B)."""
    dt = np.dtype(dtype)
    raw = np.zeros(n * dt.itemsize + align, dtype=np.uint8)
    off = (-raw.ctypes.data) % align
    return raw[off:off + n * dt.itemsize].view(dt)


def rope_table(ctx: int, hd: int, theta: float) -> np.ndarray:
    """cpu-worker.js:131-135: cos/sin of pos / theta^(2i/hd), in double precision, stored as float32."""
    out = np.empty(ctx * hd, dtype=np.float32)
    for i in range(hd // 2):
        inv = math.pow(theta, (2 * i) / hd)
        for pos in range(ctx):
            a = pos / inv
            out[pos * hd + 2 * i] = math.cos(a)
            out[pos * hd + 2 * i + 1] = math.sin(a)
    return out


class RefEngine:
    """The reference CPU backend over one oracle library (see the module docstring)."""

    def __init__(self, kind: str, parsed, data, ctx: int = 2048, mt: int = 16, threads: int = 1,
                 decode_threads: Optional[int] = None, tied_as_q4: bool = False):
        from e2e_browser_voice_agent_b200 import gguf as G  # the loader (gguf.js restated)

        self.kind = kind
        self.L = lib(kind)
        self.pre = "h2o_" if kind == "oracle" else ""
        cfg = G.qwen2_config(parsed["meta"])
        self.cfg = cfg
        D, NL, F, H, KVH, V = cfg["dim"], cfg["layers"], cfg["ffn"], cfg["heads"], cfg["kv_heads"], cfg["vocab"]
        HD = D // H
        QKV = D + 2 * KVH * HD
        if kind != "oracle" and HD > 64:
            raise ValueError("the reference's attention accumulator holds head_dim <= 64 (kernels.c:370)")
        if kind == "ref_st":
            threads = 1
        self.threads = threads
        self.decode_threads = min(threads, decode_threads or threads)
        self.ctx, self.mt = ctx, mt
        T = parsed["tensors"]
        TYPE = G.TYPE
        keep = []  # arrays the library points into

        self._calls = []

        def call(name, *args):
            self._calls.append((name, args))
            return getattr(self.L, self.pre + name)(*args)

        def q4(names):
            qs_l, d_l = [], []
            for n in names:
                t = T[n]
                if t["type"] != TYPE["Q4_0"]:
                    raise ValueError(f"{n}: expected Q4_0")  # cpu-worker.js:112
                qs, d = G.q4_0_split(G.tensor_view(data, t))
                qs_l.append(qs)
                d_l.append(d)
            qs = _aligned(sum(a.size for a in qs_l), np.uint8)
            qs[:] = np.concatenate([a.reshape(-1) for a in qs_l])
            d = _aligned(sum(a.size for a in d_l), np.float32)
            d[:] = np.concatenate(d_l)
            keep.extend([qs, d])
            return qs, d

        def f32(names):
            parts = []
            for n in names:
                t = T[n]
                if t["type"] != TYPE["F32"]:
                    raise ValueError(n)  # cpu-worker.js:105
                parts.append(G.tensor_view(data, t).view(np.float32))
            a = _aligned(sum(p.size for p in parts), np.float32)
            a[:] = np.concatenate(parts)
            keep.append(a)
            return a

        for l in range(NL):
            p = f"blk.{l}."
            for kind_id, names in ((0, ["attn_q.weight", "attn_k.weight", "attn_v.weight"]), (1, ["attn_output.weight"]),
                                   (2, ["ffn_gate.weight", "ffn_up.weight"]), (3, ["ffn_down.weight"])):
                qs, d = q4([p + n for n in names])
                call("set_tensor", kind_id, l, _ptr(qs), _ptr(d))
            call("set_tensor", 4, l, None, _ptr(f32([p + "attn_norm.weight"])))
            call("set_tensor", 5, l, None, _ptr(f32([p + "ffn_norm.weight"])))
            call("set_tensor", 6, l, None, _ptr(f32([p + "attn_q.bias", p + "attn_k.bias", p + "attn_v.bias"])))
        eqs, ed = q4(["token_embd.weight"])
        call("set_tensor", 7, 0, _ptr(eqs), _ptr(ed))
        out = T.get("output.weight")
        if out is None:  # tied embeddings
            if tied_as_q4:
                if kind != "oracle":
                    raise ValueError("only the restatement takes a Q4_0 output matrix")
                call("set_tensor", 10, 0, _ptr(eqs), _ptr(ed))
            else:
                emb = G.tensor_view(data, T["token_embd.weight"])
                oq, od = G.q8_0_split(G.q4_0_to_q8_0(emb))
                oq2, od2 = _aligned(oq.size, np.int8), _aligned(od.size, np.float32)
                oq2[:], od2[:] = oq.reshape(-1), od
                keep.extend([oq2, od2])
                call("set_tensor", 8, 0, _ptr(oq2), _ptr(od2))
        elif out["type"] == TYPE["Q8_0"]:
            oq, od = G.q8_0_split(G.tensor_view(data, out))
            oq2, od2 = _aligned(oq.size, np.int8), _aligned(od.size, np.float32)
            oq2[:], od2[:] = oq.reshape(-1), od
            keep.extend([oq2, od2])
            call("set_tensor", 8, 0, _ptr(oq2), _ptr(od2))
        elif out["type"] == TYPE["Q4_0"] and kind == "oracle":
            qs, d = q4(["output.weight"])
            call("set_tensor", 10, 0, _ptr(qs), _ptr(d))
        else:
            raise ValueError("output.weight: expected Q8_0")  # cpu-worker.js:126
        call("set_tensor", 9, 0, None, _ptr(f32(["output_norm.weight"])))

        self.rope = rope_table(ctx, HD, float(cfg["rope_theta"]))
        MT = mt
        B = {
            "x": _aligned(MT * D, np.float32), "xn": _aligned(MT * D, np.float32), "qkv": _aligned(MT * QKV, np.float32),
            "att": _aligned(MT * D, np.float32), "gu": _aligned(MT * 2 * F, np.float32), "act": _aligned(MT * F, np.float32),
            "logits": _aligned(V, np.float32), "kc": _aligned(NL * KVH * ctx * HD, np.float32),
            "vc": _aligned(NL * KVH * ctx * HD, np.float32), "scores": _aligned(max(threads, 1) * ctx, np.float32),
            "aq": _aligned(MT * max(F, D), np.int8), "ad": _aligned(MT * max(F, D) // 32, np.float32),
            "as": _aligned(MT * max(F, D) // 32, np.float32), "tokens": _aligned(ctx + 1, np.int32),
        }
        self.B = B
        call("set_config", D, NL, F, H, KVH, V, ctx, MT, float(cfg["eps"]))
        call("set_buffers", *[_ptr(B[k]) for k in ("x", "xn", "qkv", "att", "gu", "act", "logits", "kc", "vc", "scores",
                                                     "aq", "ad", "as")], _ptr(self.rope), _ptr(B["tokens"]))
        self._keep = keep
        _owner[kind] = self
        if kind == "ref_mt" and threads > 1:
            if self.L.h2shim_start_helpers(max(threads, os.cpu_count() or 1)) != 0:
                raise RuntimeError("the helper pool of this process is smaller than the requested thread count")

    def _activate(self):
        """Each library holds one model in global state (kernels.c:30-41): re-point it at this engine's tensors
        and buffers if another engine on the same library was set up since."""
        if _owner.get(self.kind) is not self:
            for name, args in self._calls:
                getattr(self.L, self.pre + name)(*args)
            _owner[self.kind] = self

    def sample(self, temperature: float, seed: int) -> int:
        return int(lib("oracle").h2o_sample(_ptr(self.B["logits"]), self.cfg["vocab"], float(temperature),
                                            seed & 0xFFFFFFFF))

    def forward(self, ids: Sequence[int], pos: int, temperature: float = 0.0, seed: int = 1,
                want_logits: bool = False, nth: Optional[int] = None) -> Dict:
        """cpu-worker.js:169-182."""
        ids = [int(t) for t in ids]
        if nth is None:
            nth = self.threads if len(ids) > 1 else self.decode_threads
        if pos + len(ids) >= self.ctx:
            raise RuntimeError("context full")
        self._activate()
        self.B["tokens"][pos:pos + len(ids)] = ids
        t0 = time.perf_counter()
        run = getattr(self.L, self.pre + "run")
        for c in range(0, len(ids), self.mt):
            n = min(self.mt, len(ids) - c)
            run(pos + c, n, 1 if c + n >= len(ids) else 0, nth)
        nxt = self.sample(temperature, (seed + pos) & 0xFFFFFFFF)
        ms = (time.perf_counter() - t0) * 1e3
        return {"next": nxt, "ms": ms, "logits": self.B["logits"].copy() if want_logits else None}

    def logits(self) -> np.ndarray:
        return self.B["logits"].copy()


def open_model(kind: str, path: str, **kw) -> RefEngine:
    from e2e_browser_voice_agent_b200 import gguf as G
    parsed, data = G.load_file(path)
    return RefEngine(kind, parsed, data, **kw)


# ------------------------------------------------------------------ kernel-level entry points (restatement)

def quantize_row(x: np.ndarray):
    """kernels.c:90-114 on one row: (int8 q, float32 d per 32, float32 d*sum(q) per 32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    q = np.zeros(n, np.int8)
    d = np.zeros(n // 32, np.float32)
    s = np.zeros(n // 32, np.float32)
    lib("oracle").h2o_quantize_row(_ptr(q), _ptr(d), _ptr(s), _ptr(x), n)
    return q, d, s


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    lib("oracle").h2o_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.size, float(eps))
    return out


def matvec_q4(blocks: np.ndarray, N: int, K: int, x: np.ndarray, op: int = 0, bias=None, y=None, nth: int = 1):
    """The Q4_0 matvec microbench on the CPU path: quantize_row on each of the M rows of x, then matmul_q4.
    blocks: GGUF Q4_0 bytes of an N x K matrix; x: float32 [M][K]. Returns y float32 [M][N]."""
    from e2e_browser_voice_agent_b200 import gguf as G
    qs, d = G.q4_0_split(blocks)
    qs = np.ascontiguousarray(qs)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    M = x.shape[0]
    y = np.zeros((M, N), np.float32) if y is None else np.ascontiguousarray(y, dtype=np.float32).copy()
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    aq = np.zeros(M * K, np.int8)
    ad = np.zeros(M * K // 32, np.float32)
    as_ = np.zeros(M * K // 32, np.float32)
    lib("oracle").h2o_matvec_q4(_ptr(qs), _ptr(d), N, K, M, _ptr(x), _ptr(y), op, _ptr(b), nth, _ptr(aq), _ptr(ad),
                                _ptr(as_))
    return y


def fast_exp(x: float) -> float:
    return float(lib("oracle").h2o_fast_exp(float(x)))
