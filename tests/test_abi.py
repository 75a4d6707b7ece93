"""The C-ABI library: loads without a GPU, exports exactly what include/h2cuda.h declares, and its host-only
entry points behave. No compute calls here (no GPU in this process)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from e2e_browser_voice_agent_b200 import _lib, build
from e2e_browser_voice_agent_b200 import gguf as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"\b(h2c_\w+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (h2c_\w+)", out))
    assert declared() <= exported, declared() - exported
    assert set(_lib.EXPORTS) <= declared()


def test_q4_pack_layout(lib):
    N, K = 3, 64
    x = np.random.default_rng(0).standard_normal(N * K).astype(np.float32)
    blocks = G.q4_0_quantize(x)
    nbytes = lib.h2c_q4_matrix_bytes(N, K)
    nb = N * K // 32
    assert nbytes >= nb * 18
    out = np.zeros(nbytes, np.uint8)
    assert lib.h2c_q4_pack(blocks.ctypes.data, N, K, out.ctypes.data) == 0
    qs, d = G.q4_0_split(blocks)
    assert np.array_equal(out[: nb * 16], qs.reshape(-1))
    off = (nb * 16 + 255) // 256 * 256
    assert np.array_equal(out[off: off + 2 * nb].view(np.float16).astype(np.float32), d)


def test_invalid_arguments_return_status(lib):
    assert lib.h2c_q4_pack(None, 1, 32, None) == _lib.ERR_INVALID
    assert lib.h2c_q4_matvec(None, 1, 32, None, 1, None, 0, None, None, None) == _lib.ERR_INVALID
    h = C.c_void_p()
    bad = _lib.Config(dim=100, layers=1, ffn=64, heads=2, kv_heads=1, vocab=10, ctx=8, max_chunk=4, max_seqs=1,
                      eps=1e-6, rope_theta=1e4)
    assert lib.h2c_create(0, C.byref(bad), C.byref(h)) == _lib.ERR_INVALID
    assert b"invalid" in lib.h2c_last_error(None)
    assert lib.h2c_destroy(None) == 0
    assert lib.h2c_q4_matvec_scratch_bytes(2, 64) >= 2 * 64 + 2 * 2 * 8


def test_create_without_gpu_reports_error(lib):
    """On a machine without a CUDA device, creation fails with a status, not a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    cfg = _lib.Config(dim=128, layers=1, ffn=256, heads=2, kv_heads=1, vocab=64, ctx=16, max_chunk=4, max_seqs=1,
                      eps=1e-6, rope_theta=1e4)
    rc = lib.h2c_create(0, C.byref(cfg), C.byref(h))
    assert rc == _lib.ERR_CUDA and not h.value
