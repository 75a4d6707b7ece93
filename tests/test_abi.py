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


PERM = [((p & 3) >> 1) * 8 + (p >> 2) * 2 + (p & 1) for p in range(16)]  # byte p <- GGUF byte PERM[p]


def pack_ref(blocks, N, K):
    """Independent restatement of the device layout: 32-row groups, [group][block][row][16 permuted bytes],
    then fp16 scales [group][block][row]."""
    nb, Np = K // 32, (N + 31) // 32 * 32
    b = blocks.reshape(N, nb, 18)
    qs = np.zeros((Np, nb, 16), np.uint8)
    d = np.zeros((Np, nb), np.uint16)
    qs[:N] = b[:, :, 2:][:, :, PERM]
    d[:N] = b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)
    qs = qs.reshape(Np // 32, 32, nb, 16).transpose(0, 2, 1, 3).reshape(-1)
    d = d.reshape(Np // 32, 32, nb).transpose(0, 2, 1).reshape(-1)
    return qs, d


@pytest.mark.parametrize("N,K", [(3, 64), (40, 96), (64, 32)])
def test_q4_pack_layout(lib, N, K):
    x = np.random.default_rng(N).standard_normal(N * K).astype(np.float32)
    blocks = G.q4_0_quantize(x)
    nbytes = lib.h2c_q4_matrix_bytes(N, K)
    out = np.zeros(nbytes, np.uint8)
    assert lib.h2c_q4_pack(blocks.ctypes.data, N, K, out.ctypes.data) == 0
    qs, d = pack_ref(blocks, N, K)
    assert np.array_equal(out[: qs.size], qs)
    off = (qs.size + 255) // 256 * 256
    assert np.array_equal(out[off: off + 2 * d.size].view(np.uint16), d)


def test_permuted_lane_arithmetic_matches_oracle(oracle_built):
    """Emulate, in numpy float32, what k_matvec computes on the packed layout (word l of a permuted block paired
    with word l of the permuted int8 activations, minus 8 x the lane sum, products then lane chains in block
    order, ((l0 + l1) + l2) + l3) and check it bit-for-bit against the oracle's quantize_row + matmul_q4."""
    import oracle as O
    N, K = 40, 96
    nb = K // 32
    rng = np.random.default_rng(7)
    blocks = G.q4_0_quantize(rng.standard_normal(N * K, dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(K, dtype=np.float32)
    ref = O.matvec_q4(blocks, N, K, x[None, :])[0]
    q, xd, _ = O.quantize_row(x)
    qs, d = pack_ref(blocks, N, K)
    qs = qs.reshape(-1, nb, 32, 16)
    dd = d.view(np.float16).astype(np.float32).reshape(-1, nb, 32)
    xb = q.reshape(nb, 32)
    xp0 = xb[:, :16][:, PERM].reshape(nb, 4, 4).astype(np.int32)   # word l = lane l's 4 values, first half
    xp1 = xb[:, 16:][:, PERM].reshape(nb, 4, 4).astype(np.int32)
    for n in range(N):
        g, r = n // 32, n % 32
        acc = [np.float32(0)] * 4
        for b in range(nb):
            w = qs[g, b, r].reshape(4, 4).astype(np.int32)
            sc = np.float32(dd[g, b, r] * xd[b])
            for l in range(4):
                p = int(((w[l] & 15) * xp0[b, l]).sum() + ((w[l] >> 4) * xp1[b, l]).sum()
                        - 8 * (xp0[b, l].sum() + xp1[b, l].sum()))
                acc[l] = np.float32(acc[l] + np.float32(np.float32(p) * sc))
        v = np.float32(np.float32(np.float32(acc[0] + acc[1]) + acc[2]) + acc[3])
        assert v.view(np.uint32) == ref[n].view(np.uint32), n


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
