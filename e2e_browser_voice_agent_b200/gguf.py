"""GGUF reader (the engine's loader) and a minimal writer for seeded test models.

The reader mirrors the reference loader h2-own-inference-engine/engine/gguf.js: `parse_gguf` follows
parseGGUF (gguf.js:15-69) and returns the same table (name, shape, type, offset, count, start, bytes), and
`qwen2_config` follows qwen2Config (gguf.js:72-88). Tensor bytes are not copied: `tensor_view` slices the file
buffer, as the reference's backends read `bytes.subarray(t.start, …)`.

The writer emits GGUF v3 (the layout parseGGUF reads: magic, version, counts, metadata, tensor table, aligned
data) and is used to produce the seeded models of the benchmark configurations.
"""
from __future__ import annotations

import mmap
import os
import struct
from typing import Any, Dict, List, Sequence, Tuple

import numpy as np

# gguf.js:6-7
TYPE = {"F32": 0, "F16": 1, "Q4_0": 2, "Q8_0": 8}
BLOCK = {TYPE["Q4_0"]: (32, 18), TYPE["Q8_0"]: (32, 34), TYPE["F32"]: (1, 4), TYPE["F16"]: (1, 2)}
GGUF_MAGIC = 0x46554747


class GGUFError(ValueError):
    """Malformed, truncated or unsupported GGUF data."""


def tensor_bytes(ggml_type: int, count: int) -> int:
    """gguf.js:9-13."""
    if ggml_type not in BLOCK:
        raise GGUFError(f"unsupported tensor type {ggml_type}")
    per, size = BLOCK[ggml_type]
    if count % per:
        raise GGUFError(f"element count {count} is not a multiple of the block size {per}")
    return (count // per) * size


class _Cursor:
    def __init__(self, buf: memoryview):
        self.buf = buf
        self.p = 0

    def take(self, n: int) -> memoryview:
        if n < 0 or self.p + n > len(self.buf):
            raise GGUFError("truncated GGUF file")
        v = self.buf[self.p:self.p + n]
        self.p += n
        return v

    def unpack(self, fmt: str):
        size = struct.calcsize(fmt)
        return struct.unpack("<" + fmt, self.take(size))[0]

    def string(self) -> str:
        n = self.unpack("Q")
        return bytes(self.take(n)).decode("utf-8", errors="replace")


_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}


def _read_value(c: _Cursor, vtype: int) -> Any:
    """gguf.js:24-46."""
    if vtype in _SCALAR:
        return c.unpack(_SCALAR[vtype])
    if vtype == 8:
        return c.string()
    if vtype == 9:
        etype = c.unpack("I")
        n = c.unpack("Q")
        if etype in (4, 5, 6) and n > 0:
            dt = {4: "<u4", 5: "<i4", 6: "<f4"}[etype]
            return np.frombuffer(c.take(4 * n), dtype=dt).copy()
        return [_read_value(c, etype) for _ in range(n)]
    raise GGUFError(f"unknown GGUF value type {vtype}")


def parse_gguf(buffer) -> Dict[str, Any]:
    """Parse a GGUF buffer (bytes, bytearray, mmap or uint8 array): gguf.js:15-69.

    Returns {"version", "meta", "tensors", "data_start"}; each tensor is a dict with name, shape (shape[0] is
    the row length), type, offset, count, start (absolute byte offset) and bytes.
    """
    buf = memoryview(buffer).cast("B")
    c = _Cursor(buf)
    if c.unpack("I") != GGUF_MAGIC:
        raise GGUFError("not a GGUF file")
    version = c.unpack("I")
    n_tensors = c.unpack("Q")
    n_kv = c.unpack("Q")
    meta: Dict[str, Any] = {}
    for _ in range(n_kv):
        k = c.string()
        meta[k] = _read_value(c, c.unpack("I"))
    tensors: Dict[str, Dict[str, Any]] = {}
    for _ in range(n_tensors):
        name = c.string()
        nd = c.unpack("I")
        shape = [c.unpack("Q") for _ in range(nd)]
        ttype = c.unpack("I")
        offset = c.unpack("Q")
        count = 1
        for s in shape:
            count *= s
        tensors[name] = {"name": name, "shape": shape, "type": ttype, "offset": offset, "count": count}
    align = int(meta.get("general.alignment", 32) or 32)
    data_start = -(-c.p // align) * align
    for t in tensors.values():
        t["start"] = data_start + t["offset"]
        t["bytes"] = tensor_bytes(t["type"], t["count"])
        if t["start"] + t["bytes"] > len(buf):
            raise GGUFError(f"tensor {t['name']} extends past the end of the file")
    return {"version": version, "meta": meta, "tensors": tensors, "data_start": data_start}


def qwen2_config(meta: Dict[str, Any]) -> Dict[str, Any]:
    """gguf.js:72-88 (same keys, snake_case for kv_heads / rope_theta / context_max)."""
    a = meta.get("general.architecture")

    def g(k):
        return meta.get(f"{a}.{k}")

    toks = meta.get("tokenizer.ggml.tokens")
    if toks is None:
        raise GGUFError("tokenizer.ggml.tokens missing: the vocabulary size is read from it")
    return {
        "arch": a,
        "dim": g("embedding_length"),
        "layers": g("block_count"),
        "ffn": g("feed_forward_length"),
        "heads": g("attention.head_count"),
        "kv_heads": g("attention.head_count_kv"),
        "rope_theta": g("rope.freq_base") or 10000,
        "eps": g("attention.layer_norm_rms_epsilon"),
        "vocab": len(toks),
        "eos": meta.get("tokenizer.ggml.eos_token_id"),
        "context_max": g("context_length"),
    }


def load_file(path: str):
    """Memory-map a GGUF file read-only and parse it. Returns (parsed, buffer)."""
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    return parse_gguf(mm), mm


def tensor_view(buffer, t: Dict[str, Any]) -> np.ndarray:
    """The raw bytes of tensor t as a uint8 array view (no copy)."""
    return np.frombuffer(buffer, dtype=np.uint8, count=t["bytes"], offset=t["start"])


# ------------------------------------------------------------------ writer (GGUF v3)

def _pack_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _pack_value(vtype: int, v: Any) -> bytes:
    if vtype in _SCALAR:
        return struct.pack("<" + _SCALAR[vtype], v)
    if vtype == 8:
        return _pack_string(v)
    raise GGUFError(f"cannot write value type {vtype}")


def write_gguf(path: str, kv: Sequence[Tuple[str, int, Any]], tensors: Sequence[Tuple[str, List[int], int, Any]],
               alignment: int = 32) -> None:
    """Write a GGUF v3 file.

    kv: (key, value_type, value); value_type 9 takes (element_type, list) for arrays.
    tensors: (name, shape with shape[0] = row length, ggml type, bytes-like data); data can also be a callable
    returning the bytes, so large tensors are produced one at a time while writing.
    """
    head = bytearray()
    head += struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kv))
    for key, vtype, v in kv:
        head += _pack_string(key) + struct.pack("<I", vtype)
        if vtype == 9:
            etype, items = v
            head += struct.pack("<IQ", etype, len(items))
            if etype == 8:
                head += b"".join(_pack_string(s) for s in items)
            else:
                head += b"".join(_pack_value(etype, x) for x in items)
        else:
            head += _pack_value(vtype, v)
    offsets = []
    off = 0
    for name, shape, ttype, _ in tensors:
        count = 1
        for s in shape:
            count *= s
        offsets.append(off)
        head += _pack_string(name) + struct.pack("<I", len(shape))
        head += b"".join(struct.pack("<Q", s) for s in shape)
        head += struct.pack("<IQ", ttype, off)
        off += -(-tensor_bytes(ttype, count) // alignment) * alignment
    pad = (-len(head)) % alignment
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(head)
        f.write(b"\0" * pad)
        pos = 0
        for (name, shape, ttype, data), o in zip(tensors, offsets):
            if pos < o:
                f.write(b"\0" * (o - pos))
                pos = o
            blob = data() if callable(data) else data
            blob = memoryview(blob).cast("B")
            count = 1
            for s in shape:
                count *= s
            if len(blob) != tensor_bytes(ttype, count):
                raise GGUFError(f"{name}: {len(blob)} bytes, expected {tensor_bytes(ttype, count)}")
            f.write(blob)
            pos += len(blob)
        tail = (-pos) % alignment
        f.write(b"\0" * tail)
    os.replace(tmp, path)


# ------------------------------------------------------------------ block formats

def q4_0_quantize(x: np.ndarray) -> np.ndarray:
    """Quantize float32 rows (length a multiple of 32) to GGUF Q4_0 blocks (18 B: fp16 d + 16 nibble bytes).

    The published ggml reference algorithm: per 32 values take the value m of largest magnitude (first one on
    ties), d = m / -8, q = min(15, trunc(x / d + 8.5)); byte j holds value j (low nibble) and j+16 (high).
    """
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.argmax(np.abs(x), axis=1)
    m = x[np.arange(x.shape[0]), idx]
    d = (m / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = (x * inv[:, None] + np.float32(8.5)).astype(np.int8)  # C (int8_t) cast: truncation toward zero
    q = np.minimum(q, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    """Quantize float32 rows to GGUF Q8_0 blocks (34 B: fp16 d + 32 int8), ggml's reference algorithm:
    d = amax / 127, q = round-half-away(x / d)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.max(np.abs(x), axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = x * inv[:, None]
    q = (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def q4_0_split(blocks: np.ndarray):
    """GGUF Q4_0 blocks -> (qs uint8 [nb][16], d float32 [nb]): the reference's repack (cpu-worker.js:97-104)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 18)
    d = b[:, 0:2].copy().view(np.float16).reshape(-1).astype(np.float32)
    return np.ascontiguousarray(b[:, 2:]), d


def q8_0_split(blocks: np.ndarray):
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 34)
    d = b[:, 0:2].copy().view(np.float16).reshape(-1).astype(np.float32)
    return np.ascontiguousarray(b[:, 2:]).view(np.int8), d


def q4_0_dequantize(blocks: np.ndarray) -> np.ndarray:
    """Q4_0 blocks -> float32 values, w = (q - 8) * d (kernels.c:319-320)."""
    qs, d = q4_0_split(blocks)
    lo = (qs & 15).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


def q4_0_to_q8_0(blocks: np.ndarray) -> np.ndarray:
    """Lossless re-encoding of Q4_0 blocks as Q8_0 blocks (int8 q - 8, same fp16 scale). A Q8_0 matrix built this
    way gives the reference's dot_q8_q8 exactly the per-lane integer sums dot_q4_q8 computes on the original."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 18)
    qs = b[:, 2:]
    lo = (qs & 15).astype(np.int16) - 8
    hi = (qs >> 4).astype(np.int16) - 8
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = b[:, 0:2]
    out[:, 2:] = np.concatenate([lo, hi], axis=1).astype(np.int8).view(np.uint8)
    return out.reshape(-1)
