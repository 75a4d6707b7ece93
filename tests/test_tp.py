"""Tensor parallelism's host logic on CPU (tp.py: the row split libh2cuda applies in h2c_set_tensor, the group plan,
the id exchange), with two gloo ranks for the N > 1 path.

The split is by output rows: each rank computes whole rows of every matrix and an all-gather assembles the vector.
The gloo test shows, on the oracle (the reference's matmul restated), that this is bit-exact: every rank computes
its rows of each matrix kind of a seeded model, the ranks all-gather them, and the assembled outputs equal the
single-process product bit for bit. The GPU form (NCCL, libh2cuda) is tests/test_gpu_tp.py."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from e2e_browser_voice_agent_b200 import gguf as G
from e2e_browser_voice_agent_b200 import synth, tp


def full_rows(cfg):
    D, F, KVH, V = cfg["dim"], cfg["ffn"], cfg["kv_heads"], cfg["vocab"]
    HD = D // cfg["heads"]
    return {"qkv": D + 2 * KVH * HD, "o": D, "gate_up": 2 * F, "down": D, "output": V}


@pytest.mark.parametrize("name", ["qwen2-7b", "qwen2-0.5b", "small", "hd128", "qwen2-7b-2l"])
def test_every_row_owned_once(name):
    cfg = synth.CONFIGS[name]
    n = full_rows(cfg)
    for world in (1, 2, 4, 8):
        try:
            tp.check(cfg, world)
        except ValueError:
            continue
        for kind, N in n.items():
            owned = [r for rank in range(world) for (a, c) in tp.rows(cfg, world, rank)[kind] for r in range(a, a + c)]
            assert sorted(owned) == list(range(N)), (name, world, kind)
        # gathered in rank order, the outputs of O, down and the lm_head are the full vector in row order
        for kind in ("o", "down", "output"):
            owned = [r for rank in range(world) for (a, c) in tp.rows(cfg, world, rank)[kind] for r in range(a, a + c)]
            assert owned == list(range(n[kind]))


def test_group_plan_and_rejected_sizes():
    c7, c05 = synth.CONFIGS["qwen2-7b"], synth.CONFIGS["qwen2-0.5b"]
    assert [tp.plan(c7, n) for n in (1, 2, 4, 8)] == [(1, 1), (2, 1), (4, 1), (4, 2)]
    assert tp.plan(c05, 8) == (2, 4)
    with pytest.raises(ValueError, match="kv heads"):
        tp.check(c7, 8)  # 4 kv heads cannot be split 8 ways
    with pytest.raises(ValueError):
        tp.check(c7, 3)
    # the lm_head rows: vocab / G rounded up to 32 rows, the last rank takes the rest
    assert tp.rows(c7, 4, 3)["output"] == [(3 * 38016, 152064 - 3 * 38016)]
    assert tp.rows(c05, 2, 1)["output"] == [(75968, 151936 - 75968)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _matrices(cfg, seed):
    """Seeded Q4_0 matrices of every split kind, with the reduction length each multiplies."""
    rng = np.random.default_rng(seed)
    n = full_rows(cfg)
    D, F = cfg["dim"], cfg["ffn"]
    out = {}
    for kind, N in n.items():
        K = F if kind == "down" else D
        out[kind] = (G.q4_0_quantize(rng.standard_normal(N * K).astype(np.float32) * 0.02), N, K)
    return out


def _take(blocks, K, ranges):
    rb = K // 32 * 18
    return np.concatenate([blocks[a * rb:(a + c) * rb] for a, c in ranges])


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import datetime
    import torch
    import torch.distributed as dist
    import oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    cfg = synth.CONFIGS["small"]
    mats = _matrices(cfg, seed=7)
    rng = np.random.default_rng(11)
    M = 3  # tokens
    res = {}
    for kind, (blocks, N, K) in mats.items():
        x = rng.standard_normal((M, K)).astype(np.float32)
        ranges = tp.rows(cfg, world, rank)[kind]
        mine = O.matvec_q4(_take(blocks, K, ranges), sum(c for _, c in ranges), K, x)
        # all-gather the row blocks (equal sizes except the lm_head's last rank: pad to the pitch)
        pitch = max(sum(c for _, c in tp.rows(cfg, world, r)[kind]) for r in range(world))
        send = np.zeros((M, pitch), np.float32)
        send[:, :mine.shape[1]] = mine
        parts = [torch.zeros(M, pitch) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(send))
        y = np.zeros((M, N), np.float32)
        for r in range(world):
            o = 0
            for a, c in tp.rows(cfg, world, r)[kind]:
                y[:, a:a + c] = parts[r].numpy()[:, o:o + c]
                o += c
        full = O.matvec_q4(blocks, N, K, x)
        res[kind] = bool(np.array_equal(y.view(np.uint32), full.view(np.uint32)))
    gid = tp.exchange_ids(world, rank, world, lambda: bytes([rank + 1]) * 128)
    out.put((rank, res, gid[:2]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_row_split_is_bit_exact(oracle_built):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, ok, gid in res:
        assert ok == {k: True for k in ("qkv", "o", "gate_up", "down", "output")}, (rank, ok)
        assert gid == b"\x01\x01"  # rank 0's id reached both ranks


def test_library_group_id_and_rejected_groups():
    """The C ABI without a GPU: group ids (NCCL's bootstrap, host only) and the split checks of h2c_create_tp."""
    import ctypes as C
    from e2e_browser_voice_agent_b200 import _lib
    a, b = _lib.tp_unique_id(), _lib.tp_unique_id()
    assert len(a) == len(b) == _lib.TP_ID_BYTES and a != b
    L = _lib.load()
    c7 = synth.CONFIGS["qwen2-7b"]
    cfg = _lib.Config(dim=c7["dim"], layers=c7["layers"], ffn=c7["ffn"], heads=c7["heads"], kv_heads=c7["kv_heads"],
                      vocab=c7["vocab"], ctx=64, max_chunk=8, max_seqs=1, eps=1e-6, rope_theta=1e6)
    idbuf = (C.c_uint8 * _lib.TP_ID_BYTES).from_buffer_copy(a)
    h = C.c_void_p()
    for world, rank in ((8, 0), (3, 1), (2, 2), (0, 0)):
        rc = L.h2c_create_tp(0, C.byref(cfg), world, rank, C.cast(idbuf, C.c_void_p), 1000, C.byref(h))
        assert rc == _lib.ERR_INVALID and not h.value, (world, rank)
    assert b"kv_heads" in L.h2c_last_error(None) or b"rank" in L.h2c_last_error(None)
