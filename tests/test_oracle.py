"""The CPU oracle: the restatement (oracle/h2_oracle.c) pinned against the reference's own kernels.c.

Pins, in order of strength:
  1. golden fixtures produced by the reference library (tests/golden, make_golden.py): bit-identical logits;
  2. the reference library itself (oracle/_ref, built here from the reference sources): bit-identical logits over
     several configurations, prompt chunkings and thread counts;
  3. properties the reference documents: results independent of threads and chunking (wiki 04:75-77).
"""
import glob
import os

import numpy as np
import pytest

import oracle as O
from e2e_browser_voice_agent_b200 import synth
from e2e_browser_voice_agent_b200 import gguf as G

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run_stream(eng, prompt, forced):
    out = [eng.forward(prompt, 0, want_logits=True)]
    pos = len(prompt)
    for t in forced:
        out.append(eng.forward([int(t)], pos, want_logits=True))
        pos += 1
    return np.stack([r["logits"] for r in out]), [r["next"] for r in out]


@pytest.mark.parametrize("fx", GOLDEN, ids=[os.path.basename(f)[:-4] for f in GOLDEN])
def test_restatement_matches_golden(fx, oracle_built):
    g = np.load(fx)
    path = synth.ensure(str(g["model"]))
    assert synth.file_sha256(path) == str(g["sha256"]), "seeded model generator changed"
    eng = O.open_model("oracle", path, ctx=64, mt=int(g["mt"]))
    lg, nxt = run_stream(eng, g["prompt"], g["forced"])
    assert np.array_equal(bits(lg), bits(g["logits"]))
    assert nxt == list(g["next"])


need_ref = pytest.mark.skipif(not O.available("ref_st"), reason="reference library not built (no reference sources)")


@need_ref
@pytest.mark.parametrize("model,mt,threads", [("tiny", 16, 1), ("small", 5, 3), ("gqa7", 2, 4), ("small-q8", 16, 2)])
def test_restatement_matches_reference(model, mt, threads, oracle_built):
    path = synth.ensure(model)
    ref = O.open_model("ref_mt", path, ctx=48, mt=mt, threads=threads)
    res = O.open_model("oracle", path, ctx=48, mt=mt, threads=threads)
    V = ref.cfg["vocab"]
    prompt = synth.prompt_ids(V, 13, seed=5)
    forced = synth.prompt_ids(V, 6, seed=6)
    a, na = run_stream(ref, prompt, forced)
    b, nb = run_stream(res, prompt, forced)
    assert np.array_equal(bits(a), bits(b))
    assert na == nb


@need_ref
def test_reference_threads_and_chunking_invariant(oracle_built):
    """wiki 04:75-77: logits are bit-identical for any thread count and any chunking of the prompt."""
    path = synth.ensure("small")
    V = 2048
    prompt = synth.prompt_ids(V, 11, seed=7)
    base = O.open_model("ref_st", path, ctx=32, mt=16).forward(prompt, 0, want_logits=True)["logits"]
    res = O.open_model("oracle", path, ctx=32, mt=4, threads=2)
    r = res.forward(prompt[:5], 0)
    r = res.forward(prompt[5:], 5, want_logits=True)
    assert np.array_equal(bits(base), bits(r["logits"]))
    one = O.open_model("oracle", path, ctx=32, mt=1, threads=1)
    for i, t in enumerate(prompt):
        r = one.forward([int(t)], i, want_logits=True)
    assert np.array_equal(bits(base), bits(r["logits"]))


def test_tied_q4_equals_q8_expansion(oracle_built):
    """A Q4_0 lm_head (tied embeddings) and its lossless Q8_0 re-encoding give bit-identical logits."""
    path = synth.ensure("tiny")
    a = O.open_model("oracle", path, ctx=16, mt=4, tied_as_q4=True)
    b = O.open_model("oracle", path, ctx=16, mt=4, tied_as_q4=False)
    p = synth.prompt_ids(512, 5, seed=9)
    assert np.array_equal(bits(a.forward(p, 0, want_logits=True)["logits"]),
                          bits(b.forward(p, 0, want_logits=True)["logits"]))


@need_ref
def test_reference_barrier_selftest():
    """kernels.c:281-288: the MT barrier keeps every thread in step (the reference's own self-test)."""
    L = O.lib("ref_mt")
    L.h2shim_start_helpers(os.cpu_count() or 2)
    assert L.run_barrier_test(2000, min(4, os.cpu_count() or 2)) == 0


def test_context_full(oracle_built):
    eng = O.open_model("oracle", synth.ensure("tiny"), ctx=8, mt=4)
    eng.forward([1, 2, 3], 0)
    with pytest.raises(RuntimeError, match="context full"):
        eng.forward([4, 5, 6, 7, 8], 3)


def test_fast_exp_matches_reference_formula(oracle_built):
    # kernels.c:69-78: clamps below -87 to 0, above 88 to e^88; ~1e-7 relative error elsewhere
    assert O.fast_exp(-100.0) == 0.0
    assert O.fast_exp(100.0) == O.fast_exp(88.0)
    for x in np.linspace(-80, 80, 321):
        assert abs(O.fast_exp(float(x)) / np.exp(np.float64(x)) - 1) < 1e-6


def test_quantize_row_exact(oracle_built):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(96).astype(np.float32)
    x[32:64] = 0.0  # an all-zero block: d = 0, q = 0
    q, d, s = O.quantize_row(x)
    assert d[1] == 0 and not q[32:64].any()
    for b in (0, 2):
        blk = x[32 * b:32 * b + 32]
        dd = np.float32(np.abs(blk).max()) / np.float32(127)
        inv = np.float32(1) / dd
        exp = np.rint(blk * inv).astype(np.int32)  # nearest-even
        assert d[b] == dd and np.array_equal(q[32 * b:32 * b + 32], exp.astype(np.int8))
        assert s[b] == dd * np.float32(exp.sum())


def test_sampler_greedy_and_temperature(oracle_built):
    lg = np.zeros(10, np.float32)
    lg[[3, 7]] = 2.0
    L = O.lib("oracle")
    assert L.h2o_sample(lg.ctypes.data, 10, 0.0, 1) == 3  # ties -> lowest index (strict >)
    # temperature sampling is a deterministic function of (logits, temperature, seed)
    lg = np.random.default_rng(1).standard_normal(50).astype(np.float32)
    a = [L.h2o_sample(lg.ctypes.data, 50, 0.8, s) for s in range(20)]
    b = [L.h2o_sample(lg.ctypes.data, 50, 0.8, s) for s in range(20)]
    assert a == b and len(set(a)) > 3


def test_mulberry32_known_values():
    """The first outputs of mulberry32 for seed 1, from the JavaScript definition (cpu-worker.js:160)."""
    def js_mulberry(seed):
        s = seed
        while True:
            s = (s + 0x6D2B79F5) & 0xFFFFFFFF
            t = s
            t = ((t ^ (t >> 15)) * (t | 1)) & 0xFFFFFFFF
            t ^= (t + ((t ^ (t >> 7)) * (t | 61) & 0xFFFFFFFF)) & 0xFFFFFFFF
            yield ((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296
    g = js_mulberry(1)
    first = [next(g) for _ in range(3)]
    # sampling with a one-hot-like distribution picks by the first random number
    lg = np.array([0.0, 0.0], np.float32)
    L = O.lib("oracle")
    # r = u * 2 (two equal weights): index 0 when u <= 0.5
    assert L.h2o_sample(lg.ctypes.data, 2, 1.0, 1) == (0 if first[0] * 2 - 1 <= 0 else 1)
