"""The GGUF loader (gguf.js restated) and the seeded-model writer."""
import numpy as np
import pytest

from e2e_browser_voice_agent_b200 import gguf as G
from e2e_browser_voice_agent_b200 import synth


def test_roundtrip_and_config():
    path = synth.ensure("small")
    parsed, data = G.load_file(path)
    cfg = G.qwen2_config(parsed["meta"])
    assert cfg == {"arch": "qwen2", "dim": 256, "layers": 3, "ffn": 640, "heads": 4, "kv_heads": 2,
                   "rope_theta": 1e6, "eps": pytest.approx(1e-6), "vocab": 2048, "eos": 2047, "context_max": 32768}
    t = parsed["tensors"]["blk.0.ffn_down.weight"]
    assert t["shape"] == [640, 256] and t["type"] == G.TYPE["Q4_0"] and t["bytes"] == 640 * 256 // 32 * 18
    assert t["start"] % 32 == 0
    assert "output.weight" not in parsed["tensors"]  # tied


def test_against_gguf_package_reader():
    """Cross-check the tensor table with the independent `gguf` package reader."""
    gg = pytest.importorskip("gguf")
    path = synth.ensure("tiny")
    parsed, data = G.load_file(path)
    r = gg.GGUFReader(path)
    assert len(r.tensors) == len(parsed["tensors"])
    for t in r.tensors:
        mine = parsed["tensors"][t.name]
        assert int(t.tensor_type) == mine["type"]
        assert list(int(x) for x in t.shape) == mine["shape"]
        assert int(t.data_offset) == mine["start"]


def test_q4_0_quantizer_matches_gguf_package():
    gg = pytest.importorskip("gguf")
    x = np.random.default_rng(3).standard_normal((64, 96)).astype(np.float32) * 0.02
    mine = G.q4_0_quantize(x)
    theirs = gg.quants.quantize(x, gg.GGMLQuantizationType.Q4_0).reshape(-1)
    assert np.array_equal(mine, theirs)


def test_q4_unpack_bit_exact():
    """Nibble order (wiki 02: byte j holds value j low, j+16 high) and w = (q - 8) * d, exactly."""
    x = np.random.default_rng(4).standard_normal(32 * 10).astype(np.float32)
    blocks = G.q4_0_quantize(x)
    b = blocks.reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    w = G.q4_0_dequantize(blocks).reshape(-1, 32)
    for i in range(10):
        for j in range(16):
            assert w[i, j] == np.float32((int(b[i, 2 + j]) & 15) - 8) * d[i]
            assert w[i, 16 + j] == np.float32((int(b[i, 2 + j]) >> 4) - 8) * d[i]


def test_q4_to_q8_lossless():
    x = np.random.default_rng(5).standard_normal(32 * 7).astype(np.float32)
    q4 = G.q4_0_quantize(x)
    q8 = G.q4_0_to_q8_0(q4)
    qs, d = G.q8_0_split(q8)
    assert np.array_equal((qs.astype(np.float32) * d[:, None]).reshape(-1), G.q4_0_dequantize(q4))


def test_malformed_files(tmp_path):
    with pytest.raises(G.GGUFError, match="not a GGUF"):
        G.parse_gguf(b"GGML" + b"\0" * 64)
    path = synth.ensure("tiny")
    raw = open(path, "rb").read()
    with pytest.raises(G.GGUFError, match="truncated|past the end"):
        G.parse_gguf(raw[: len(raw) // 2])
    with pytest.raises(G.GGUFError, match="truncated"):
        G.parse_gguf(raw[:100])
    with pytest.raises(G.GGUFError, match="unsupported tensor type"):
        G.tensor_bytes(12, 256)


def test_prompt_ids_seeded():
    a = synth.prompt_ids(151936, 32, seed=1)
    assert a.dtype == np.int32 and a.min() >= 0 and a.max() < 151936
    assert np.array_equal(a, synth.prompt_ids(151936, 32, seed=1))
