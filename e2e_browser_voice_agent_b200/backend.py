"""The "cuda" backend object: the shape of the reference's CPU / WebGPU backends over libh2cuda.

createCPU (h2-own-inference-engine/engine/cpu.js:17-69) returns
  {name, ctx, threads, build, memoryBytes, info, forward, readLogits, rawForward, profile, readTest, barrierTest,
   destroy};
create_cuda returns an object with the same members (snake_case) whose work runs in libh2cuda on a B200:
  forward(ids, pos, temperature=0, seed=1, want_logits=False) -> next token id
      writes ids at pos; raises RuntimeError("context full") when pos + len(ids) >= ctx (cpu-worker.js:173);
      prompts run in chunks of prefill_chunk tokens; logits exist for the last id only.
  read_logits() -> float32 array of the last forward's logits, or None (cpu.js:60-62: the CPU backend keeps them
      only when asked with want_logits / keep_logits)
  raw_forward(ids, pos) -> {"next", "ms", "logits"} (cpu.js:63)
  profile(ids, pos) -> {op name: ms} (cpu-worker.js:31-37 names)
  destroy()
Added for the multi-session configuration: every call takes an optional `seq` (an independent KV cache).
Added for the 7B configuration: tp=(world, rank, group id) makes this object one rank of a tensor-parallel group
(h2c_create_tp): every rank loads the same full tensors (the library keeps its rows) and makes the same calls; each
returns the same tokens and logits as one GPU would.

Weight upload follows the CPU host's init (cpu-worker.js:57-128): per layer the [q;k;v] and [gate;up] Q4_0
matrices are concatenated row-wise, norms and [bq;bk;bv] biases are F32, token_embd is Q4_0 and output.weight is
Q8_0 (the reference's requirement) or Q4_0; a model without output.weight uses tied embeddings.
"""
from __future__ import annotations

import ctypes as C
import time
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from . import gguf as G


class CudaBackend:
    """parsed, data: the GGUF file (parse_gguf result and its bytes), or parsed = a callable name -> (ggml type, raw
    tensor bytes) or None, with data unused (models generated without a file, e.g. synth.device_tensors)."""

    name = "cuda"

    def __init__(self, parsed, data, cfg: Dict, ctx: int = 2048, prefill_chunk: int = 16, max_seqs: int = 1,
                 device: int = 0, keep_logits: bool = False, on_progress=None, decode_mode: str = "auto",
                 tp: Optional[Tuple[int, int, bytes]] = None, tp_timeout_ms: int = 0):
        L = _lib.load()
        self._L = L
        D, NL, F, H, KVH, V = cfg["dim"], cfg["layers"], cfg["ffn"], cfg["heads"], cfg["kv_heads"], cfg["vocab"]
        self.cfg = cfg
        self.ctx = int(ctx)
        self.prefill_chunk = int(prefill_chunk)
        self.max_seqs = int(max_seqs)
        self.keep_logits = keep_logits
        c = _lib.Config(dim=D, layers=NL, ffn=F, heads=H, kv_heads=KVH, vocab=V, ctx=self.ctx,
                        max_chunk=self.prefill_chunk, max_seqs=self.max_seqs, eps=float(cfg["eps"]),
                        rope_theta=float(cfg["rope_theta"]))
        h = C.c_void_p()
        if tp is None:
            _lib.check(L.h2c_create(int(device), C.byref(c), C.byref(h)), None)
        else:  # one rank of a tensor-parallel group: (world, rank, group id from _lib.tp_unique_id on rank 0)
            world, rank, gid = tp
            if len(gid) != _lib.TP_ID_BYTES:
                raise ValueError(f"tensor-parallel id must be {_lib.TP_ID_BYTES} bytes")
            idbuf = (C.c_uint8 * _lib.TP_ID_BYTES).from_buffer_copy(gid)
            _lib.check(L.h2c_create_tp(int(device), C.byref(c), int(world), int(rank), C.cast(idbuf, C.c_void_p),
                                       int(tp_timeout_ms), C.byref(h)), None)
        self.tp_world = int(L.h2c_tp_world(h))
        self.tp_rank = int(L.h2c_tp_rank(h))
        self._h = h
        self._next = C.c_int32()
        self._last_logits: Dict[int, Optional[np.ndarray]] = {}
        # tensor source: name -> (ggml type, raw bytes), from the GGUF file (parsed, data) or a callable
        if callable(parsed):
            source = parsed
        else:
            T = parsed["tensors"]

            def source(name: str):
                t = T.get(name)
                return None if t is None else (t["type"], G.tensor_view(data, t))

        def raw(name: str, want: int) -> np.ndarray:
            t = source(name)
            if t is None:
                raise ValueError(f"{name}: missing")
            if t[0] != want:
                kind = {G.TYPE["Q4_0"]: "Q4_0", G.TYPE["F32"]: "F32"}.get(want, str(want))
                raise ValueError(f"{name}: expected {kind}")  # cpu-worker.js:105, 112
            return t[1]

        def put(kind: int, layer: int, ggml_type: int, blob: np.ndarray) -> None:
            blob = np.ascontiguousarray(blob)
            _lib.check(L.h2c_set_tensor(self._h, kind, layer, ggml_type, blob.ctypes.data, blob.nbytes), self._h)

        q4, f32 = G.TYPE["Q4_0"], G.TYPE["F32"]
        for l in range(NL):
            p = f"blk.{l}."
            put(_lib.KIND_QKV, l, q4, np.concatenate([raw(p + n, q4) for n in ("attn_q.weight", "attn_k.weight", "attn_v.weight")]))
            put(_lib.KIND_O, l, q4, raw(p + "attn_output.weight", q4))
            put(_lib.KIND_GATE_UP, l, q4, np.concatenate([raw(p + n, q4) for n in ("ffn_gate.weight", "ffn_up.weight")]))
            put(_lib.KIND_DOWN, l, q4, raw(p + "ffn_down.weight", q4))
            put(_lib.KIND_ATTN_NORM, l, f32, raw(p + "attn_norm.weight", f32))
            put(_lib.KIND_FFN_NORM, l, f32, raw(p + "ffn_norm.weight", f32))
            put(_lib.KIND_QKV_BIAS, l, f32, np.concatenate([raw(p + n, f32) for n in ("attn_q.bias", "attn_k.bias", "attn_v.bias")]))
            if on_progress:
                on_progress(l + 1, NL)
        put(_lib.KIND_EMBED, 0, q4, raw("token_embd.weight", q4))
        out = source("output.weight")
        if out is not None:
            if out[0] not in (G.TYPE["Q8_0"], G.TYPE["Q4_0"]):
                raise ValueError("output.weight: expected Q8_0")  # cpu-worker.js:126
            put(_lib.KIND_OUTPUT, 0, out[0], out[1])
        put(_lib.KIND_OUTPUT_NORM, 0, f32, raw("output_norm.weight", f32))
        if decode_mode != "auto":
            self.set_decode_mode(decode_mode)
        self.memory_bytes = int(L.h2c_device_bytes(self._h))
        self.build = _lib.LIB_PATH
        self.threads = 1
        self.info = (f"B200 sm_100a, {self.max_seqs} sequence(s) x {self.ctx} positions, prefill chunk "
                     f"{self.prefill_chunk}, {self.memory_bytes / 2**20:.0f} MiB on device")

    # ---------------------------------------------------------------- backend API (cpu.js:52-68)
    def forward(self, ids: Sequence[int], pos: int, temperature: float = 0.0, seed: int = 1,
                want_logits: bool = False, seq: int = 0) -> int:
        if self._h is None:
            raise RuntimeError("backend destroyed")
        arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        if pos + arr.size >= self.ctx:
            raise RuntimeError("context full")
        rc = self._L.h2c_forward(self._h, int(seq), arr.ctypes.data, int(arr.size), int(pos), float(temperature),
                                 int(seed) & 0xFFFFFFFF, C.byref(self._next))
        if rc == _lib.ERR_CONTEXT_FULL:
            raise RuntimeError("context full")
        _lib.check(rc, self._h)
        self._last_logits = {}
        if want_logits or self.keep_logits:
            self._last_logits[seq] = self._read(seq)
        return int(self._next.value)

    def forward_batch(self, seqs: Sequence[int], ids: Sequence[int], pos: Sequence[int], temperature: float = 0.0,
                      seed: int = 1, want_logits: bool = False) -> List[int]:
        """One decode step of several sessions at once: token ids[m] of sequence seqs[m] at position pos[m];
        returns each session's next token (the same tokens and logits as separate forward calls)."""
        if self._h is None:
            raise RuntimeError("backend destroyed")
        s = np.ascontiguousarray(np.asarray(seqs, dtype=np.int32).reshape(-1))
        t = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        p = np.ascontiguousarray(np.asarray(pos, dtype=np.int32).reshape(-1))
        if not (s.size == t.size == p.size) or s.size == 0:
            raise ValueError("seqs, ids and pos must have the same non-zero length")
        if int(p.max()) + 1 >= self.ctx:
            raise RuntimeError("context full")
        out = np.empty(s.size, dtype=np.int32)
        rc = self._L.h2c_forward_batch(self._h, int(s.size), s.ctypes.data, t.ctypes.data, p.ctypes.data,
                                       float(temperature), int(seed) & 0xFFFFFFFF, out.ctypes.data)
        if rc == _lib.ERR_CONTEXT_FULL:
            raise RuntimeError("context full")
        _lib.check(rc, self._h)
        self._last_logits = {}
        if want_logits or self.keep_logits:
            for q in s.tolist():
                self._last_logits[q] = self._read(q)
        return out.tolist()

    def generate_batch(self, seqs: Sequence[int], ids: Sequence[int], pos: Sequence[int], steps: int):
        """Greedy decode of `steps` tokens of every session on the device (batched steps chained without the
        host). Returns ([n][steps] token array, device milliseconds)."""
        s = np.ascontiguousarray(np.asarray(seqs, dtype=np.int32).reshape(-1))
        t = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        p = np.ascontiguousarray(np.asarray(pos, dtype=np.int32).reshape(-1))
        if not (s.size == t.size == p.size) or s.size == 0:
            raise ValueError("seqs, ids and pos must have the same non-zero length")
        out = np.empty((s.size, int(steps)), dtype=np.int32)
        ms = C.c_float()
        rc = self._L.h2c_generate_batch(self._h, int(s.size), s.ctypes.data, t.ctypes.data, p.ctypes.data, int(steps),
                                        out.ctypes.data, C.byref(ms))
        if rc == _lib.ERR_CONTEXT_FULL:
            raise RuntimeError("context full")
        _lib.check(rc, self._h)
        self._last_logits = {}
        return out, float(ms.value)

    def _read(self, seq: int) -> np.ndarray:
        out = np.empty(self.cfg["vocab"], dtype=np.float32)
        _lib.check(self._L.h2c_read_logits(self._h, int(seq), out.ctypes.data, out.size), self._h)
        return out

    def read_logits(self, seq: int = 0) -> Optional[np.ndarray]:
        return self._last_logits.get(seq)

    def raw_forward(self, ids: Sequence[int], pos: int, seq: int = 0) -> Dict:
        t0 = time.perf_counter()
        nxt = self.forward(ids, pos, want_logits=True, seq=seq)
        return {"next": nxt, "ms": (time.perf_counter() - t0) * 1e3, "logits": self._last_logits.get(seq)}

    def profile(self, ids: Sequence[int], pos: int, seq: int = 0) -> Dict[str, float]:
        arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        ms = (C.c_double * _lib.NPROF)()
        _lib.check(self._L.h2c_profile(self._h, int(seq), arr.ctypes.data, int(arr.size), int(pos), ms), self._h)
        return {n: float(ms[i]) for i, n in enumerate(_lib.PROFILE_NAMES)}

    def generate(self, first_id: int, pos: int, steps: int, seq: int = 0):
        """Greedy decode of `steps` tokens on the device (h2c_generate). Returns (ids, device milliseconds)."""
        out = np.empty(steps, dtype=np.int32)
        ms = C.c_float()
        rc = self._L.h2c_generate(self._h, int(seq), int(first_id), int(pos), int(steps), out.ctypes.data, C.byref(ms))
        if rc == _lib.ERR_CONTEXT_FULL:
            raise RuntimeError("context full")
        _lib.check(rc, self._h)
        self._last_logits = {}
        return out, float(ms.value)

    def set_decode_mode(self, mode: str) -> None:
        """'auto' (persistent kernel when the model fits it), 'graph' or 'persistent'."""
        code = {"auto": _lib.DECODE_AUTO, "graph": _lib.DECODE_GRAPH, "persistent": _lib.DECODE_PERSISTENT}[mode]
        _lib.check(self._L.h2c_set_decode_mode(self._h, code), self._h)

    @property
    def decode_path(self) -> str:
        n = self._L.h2c_decode_path(self._h)
        if n < 0:
            _lib.check(n, self._h)
        return {_lib.DECODE_GRAPH: "graph", _lib.DECODE_PERSISTENT: "persistent"}[n]

    def trace_decode(self, first_id: int, pos: int, steps: int, seq: int = 0) -> np.ndarray:
        """Stage timestamps (ns) of the persistent kernel: array [CTAs][steps][layers + 1][16]."""
        L = self.cfg["layers"]
        n = self._L.h2c_decode_ctas(self._h)
        if n < 0:
            _lib.check(n, self._h)
        if n == 0:
            raise RuntimeError("this model takes the graph decode path (no persistent kernel to trace)")
        out = np.zeros((n, steps, L + 1, 16), dtype=np.uint64)
        _lib.check(self._L.h2c_trace_decode(self._h, int(seq), int(first_id), int(pos), int(steps), out.ctypes.data,
                                            out.size), self._h)
        return out

    def set_decode_fault(self, stall_cta: int = -1, timeout_ns: int = 2_000_000_000) -> None:
        """Test aid: make one CTA of the persistent kernel withhold its results so the bounded waits expire."""
        _lib.check(self._L.h2c_set_decode_fault(self._h, int(stall_cta), int(timeout_ns)), self._h)

    def batch_kernels(self, n: int) -> int:
        """Kernels one batched decode step of n sessions launches (0 before the first such step)."""
        k = self._L.h2c_batch_kernels(self._h, int(n))
        if k < 0:
            _lib.check(k, self._h)
        return k

    def decode_kernels(self) -> int:
        n = self._L.h2c_decode_kernels(self._h)
        if n < 0:
            _lib.check(n, self._h)
        return n

    def destroy(self) -> None:
        if self._h is not None:
            self._L.h2c_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def create_cuda(parsed, data, cfg: Dict, **opts) -> CudaBackend:
    """The counterpart of createCPU(gguf, bytes, cfg, opts) (cpu.js:17)."""
    return CudaBackend(parsed, data, cfg, **opts)


def open_model(path: str, **opts) -> CudaBackend:
    parsed, data = G.load_file(path)
    cfg = G.qwen2_config(parsed["meta"])
    if cfg["arch"] != "qwen2":
        raise ValueError(f"unsupported architecture {cfg['arch']}")  # llm.js:19
    return CudaBackend(parsed, data, cfg, **opts)
