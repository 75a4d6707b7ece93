"""Multi-GPU host logic on CPU: session sharding and the max-over-ranks timing reduction, with two gloo ranks
(the same code bench.py runs under torchrun with NCCL, one rank per GPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from e2e_browser_voice_agent_b200 import sessions


def test_shard_covers_every_session_once():
    for world in (1, 2, 3, 8):
        got = sorted(s for r in range(world) for s in sessions.shard(256, world, r))
        assert got == list(range(256))
        assert all(len(sessions.shard(256, world, r)) in (256 // world, 256 // world + 1) for r in range(world))
    with pytest.raises(ValueError):
        sessions.shard(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    sessions.init("gloo", timeout_s=30)
    w, r, _ = sessions.env_rank()
    mine = sessions.shard(256, w, r)
    sessions.barrier()
    # each rank reports a different "device time"; every rank must see the slowest one
    mx = sessions.max_over_ranks(10.0 + 5.0 * r)
    n = sessions.max_over_ranks(float(len(mine)))
    out.put((r, mine[:3], mx, n))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [r[1] for r in res] == [[0, 2, 4], [1, 3, 5]]
    assert all(r[2] == 15.0 and r[3] == 128.0 for r in res)
