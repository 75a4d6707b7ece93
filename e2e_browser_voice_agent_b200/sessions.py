"""Multi-GPU host logic for serving independent sessions: one process per GPU, sessions sharded across ranks, no
collective on the data path.

The reference serves one conversation per backend (cpu.js keeps a single outstanding request per backend); a
node with several B200s serves several sessions by giving each rank its own engine and its own share of the
sessions. The only cross-rank steps are the ones measurement needs: a barrier around the timed region and the
maximum of the per-rank device times (the job finishes when its slowest rank does).
"""
from __future__ import annotations

import datetime
import os
from typing import List


def shard(n_sessions: int, world: int, rank: int) -> List[int]:
    """Session ids of `rank`: round-robin over ranks, so every session is served by exactly one rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_sessions, world))


def session_seed(session: int) -> int:
    """Prompt seed of a session (session 0 uses the seed of the single-session workload)."""
    return 1 + session


def env_rank():
    """(world, rank, local_rank) from the torchrun environment (1, 0, 0 without one)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, timeout_s: float = 120.0) -> None:
    """Join the process group (rendezvous from the environment, as torchrun sets it) with a short timeout, so ranks
    that wait for a missing peer end with an error instead of hanging."""
    import torch
    import torch.distributed as dist
    kw = {}
    if backend == "nccl":  # bind the group to this rank's GPU (set as current before init)
        kw["device_id"] = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)


def max_over_ranks(x: float, device=None) -> float:
    """The maximum of x over all ranks (x itself without a process group)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
