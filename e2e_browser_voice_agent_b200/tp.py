"""Tensor parallelism for the 7B configuration: which rows of each matrix a rank owns, and the group set-up.

The split is the one libh2cuda applies inside h2c_set_tensor when an engine was created with h2c_create_tp (the
host passes full tensors; the library keeps its rows). Every matrix is split by OUTPUT rows, never by the reduction
dimension, so each output value is one rank's dot product over the whole row, in the reference's lane order
(kernels.c:121-155, 200-273), and the model's results stay bit-identical to one GPU's. The reference has no
multi-device code (it runs one CPU process); an all-reduce of partial sums over split rows, the usual form, would
change the float32 summation order, so the exchange here is an all-gather of whole rows' results instead:

  per layer  attention output (H/G heads each)  -> all-gather, then every rank quantizes the full vector
             residual after O (D/G rows each)   -> all-gather
             FFN activation, quantized (F/G)    -> all-gather of the int8 values, block scales and lane sums
             residual after down (D/G rows)     -> all-gather
  per step   logits (Vp rows each)              -> all-gather, then every rank takes the same argmax / sample

The q/k/v rows of a rank are those of its heads, so RoPE, the KV cache and attention stay per rank with no
exchange. Requirements: kv_heads, dim / 32 and ffn / 32 divisible by G. For Qwen2-7B (28 query / 4 kv heads) that
allows G = 1, 2, 4: 4 kv heads cannot be split 8 ways, so 8 GPUs run two replicas of a TP-4 group (plan()).
"""
from __future__ import annotations

from typing import Dict, List, Tuple

Ranges = List[Tuple[int, int]]  # (first row, rows)


def check(cfg: Dict, world: int) -> None:
    """Raise ValueError when the model cannot be split over `world` ranks."""
    D, F, H, KVH, V = cfg["dim"], cfg["ffn"], cfg["heads"], cfg["kv_heads"], cfg["vocab"]
    if world < 1 or world > 8:
        raise ValueError("tensor-parallel group size must be 1..8")
    if KVH % world:
        raise ValueError(f"{KVH} kv heads cannot be split over {world} ranks")
    if D % (32 * world) or F % (32 * world):
        raise ValueError(f"dim {D} and ffn {F} must split into whole 32-value blocks over {world} ranks")
    if world > 1 and V <= (world - 1) * lm_pitch(V, world):
        raise ValueError("vocabulary too small for the group size")


def lm_pitch(vocab: int, world: int) -> int:
    """Rows of the lm_head per rank (the last rank may have fewer): vocab / world rounded up to 32 rows."""
    return vocab if world == 1 else -(-vocab // (32 * world)) * 32


def rows(cfg: Dict, world: int, rank: int) -> Dict[str, Ranges]:
    """Row ranges of the full tensors that rank `rank` of `world` keeps, per kind of tensor (in the order they are
    stored on the device): "qkv" the [q; k; v] matrix and bias, "o", "gate_up" the [gate; up] matrix, "down",
    "output" the lm_head (rows of token_embd when tied)."""
    check(cfg, world)
    D, F, H, KVH, V = cfg["dim"], cfg["ffn"], cfg["heads"], cfg["kv_heads"], cfg["vocab"]
    HD = D // H
    Hl, KVl, Dl, Fl = H // world, KVH // world, D // world, F // world
    Vp = lm_pitch(V, world)
    r = rank
    return {
        "qkv": [(r * Hl * HD, Hl * HD), (D + r * KVl * HD, KVl * HD), (D + (KVH + r * KVl) * HD, KVl * HD)],
        "o": [(r * Dl, Dl)],
        "gate_up": [(r * Fl, Fl), (F + r * Fl, Fl)],
        "down": [(r * Dl, Dl)],
        "output": [(r * Vp, min(Vp, V - r * Vp))],
    }


def plan(cfg: Dict, n_gpus: int) -> Tuple[int, int]:
    """(group size G, replicas) for n_gpus GPUs: the largest G <= n_gpus that check() accepts and divides n_gpus;
    the groups run independent sequences (Qwen2-7B on 8 GPUs: two TP-4 groups)."""
    for g in range(min(n_gpus, 8), 0, -1):
        if n_gpus % g:
            continue
        try:
            check(cfg, g)
        except ValueError:
            continue
        return g, n_gpus // g
    return 1, n_gpus


def exchange_ids(world: int, rank: int, group: int, make_id) -> bytes:
    """Under torch.distributed (every process one rank, world ranks in consecutive groups of `group`): the first
    rank of each group creates its id with make_id() (_lib.tp_unique_id); returns the id of this rank's group."""
    import torch.distributed as dist
    mine = make_id() if rank % group == 0 else None
    got: List = [None] * world
    dist.all_gather_object(got, mine)
    return got[rank - rank % group]
