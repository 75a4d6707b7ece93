"""Tensor parallelism on GPUs: h2c_create_tp (row-split matrices, NCCL all-gathers inside the decode step's CUDA
graph), one process per GPU.

- Two or more GPUs: G ranks run prompt chunks (mma.sync and tcgen05 pass sizes), device-chained greedy decode, a
  single step with logits and a sampled step. Every rank's tokens and logits equal one GPU's bit for bit (and the
  prompt's logits equal the oracle's), for a tied Q4_0, a Q8_0 and an untied Q4_0 lm_head, head_dim 64 and 128,
  and the 7B layer shapes. Skipped on a box with fewer GPUs (NCCL rejects two ranks on one GPU).
- One GPU: a group whose second rank never joins ends in H2C_ERR_TIMEOUT within the deadline (a host-side wait in
  NCCL's set-up; no kernel runs) and the process can open an engine afterwards."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _script(be, vocab):
    p = np.random.default_rng(3).integers(0, vocab, size=70).astype(np.int32)
    t0 = be.forward(p, 0, want_logits=True)  # chunks of prefill_chunk tokens, logits of the last
    lg0 = be.read_logits()
    ids, _ = be.generate(t0, 70, 12)          # device-chained steps on the CUDA graph
    t1 = be.forward([int(ids[-1])], 82, want_logits=True)
    lg1 = be.read_logits()
    t2 = be.forward([t1], 83, temperature=0.8, seed=7)  # sampled on the device from the gathered logits
    return {"t0": t0, "ids": [int(i) for i in ids], "t1": t1, "t2": t2, "lg0": lg0, "lg1": lg1}


def _rank(rank, world, name, chunk, qid, qout):
    try:
        import torch
        from e2e_browser_voice_agent_b200 import _lib, backend, synth
        torch.cuda.set_device(rank)
        if rank == 0:
            gid = _lib.tp_unique_id()
            for _ in range(world - 1):
                qid.put(gid)
        else:
            gid = qid.get(timeout=120)
        be = backend.open_model(synth.ensure(name), ctx=160, prefill_chunk=chunk, device=rank, tp=(world, rank, gid),
                                tp_timeout_ms=60000)
        assert (be.tp_world, be.tp_rank) == (world, rank)
        out = _script(be, be.cfg["vocab"])
        try:
            be.forward_batch([0], [1], [90])
            out["batch"] = "accepted"
        except RuntimeError as ex:
            out["batch"] = str(ex)
        out["path"] = be.decode_path
        be.destroy()
        qout.put((rank, out))
    except BaseException as ex:  # reported to the parent
        qout.put((rank, repr(ex)))


@pytest.mark.parametrize("name,chunk,world", [("small", 8, 2), ("small-q8", 16, 2), ("hd128", 64, 2),
                                              ("qwen2-7b-2l", 64, 2), ("qwen2-7b-2l", 32, 4)])
def test_tensor_parallel_ranks_equal_one_gpu(name, chunk, world, oracle_built):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from e2e_browser_voice_agent_b200 import backend, synth
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # inherited by the ranks
    ctx = mp.get_context("spawn")
    qid, qout = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, name, chunk, qid, qout)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(qout.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert isinstance(got[r], dict), got[r]
    path = synth.ensure(name)
    one = backend.open_model(path, ctx=160, prefill_chunk=chunk, device=0)
    ref = _script(one, one.cfg["vocab"])
    one.destroy()
    for r in range(world):
        g = got[r]
        assert g["path"] == "graph" and "tensor parallelism" in g["batch"]
        assert (g["t0"], g["ids"], g["t1"], g["t2"]) == (ref["t0"], ref["ids"], ref["t1"], ref["t2"]), r
        for k in ("lg0", "lg1"):
            assert np.array_equal(g[k].view(np.uint32), ref[k].view(np.uint32)), (r, k)
    O = oracle_built
    o = O.open_model("oracle", path, ctx=160, mt=chunk, threads=8)
    p = np.random.default_rng(3).integers(0, one.cfg["vocab"], size=70).astype(np.int32)
    r0 = o.forward(p, 0, want_logits=True)
    assert r0["next"] == ref["t0"]
    assert np.array_equal(r0["logits"].view(np.uint32), ref["lg0"].view(np.uint32))


_NEVER_JOINS = r"""
import json, time
from e2e_browser_voice_agent_b200 import _lib, backend, synth
gid = _lib.tp_unique_id()
t0 = time.time()
try:
    backend.open_model(synth.ensure("small"), ctx=64, prefill_chunk=8, device=0, tp=(2, 0, gid), tp_timeout_ms=3000)
    res = {"code": 0}
except _lib.H2CError as ex:
    res = {"code": ex.code, "msg": str(ex)}
res["s"] = time.time() - t0
be = backend.open_model(synth.ensure("small"), ctx=64, prefill_chunk=8, device=0)
res["after"] = be.forward([1, 2, 3], 0)
be.destroy()
print(json.dumps(res))
"""


def test_group_set_up_times_out_when_a_rank_never_joins():
    from e2e_browser_voice_agent_b200 import _lib, synth
    synth.ensure("small")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", _NEVER_JOINS], capture_output=True, text=True, timeout=300, env=env,
                       cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["code"] == _lib.ERR_TIMEOUT, res
    assert "aborted" in res["msg"] and res["s"] < 60
    assert isinstance(res["after"], int)
