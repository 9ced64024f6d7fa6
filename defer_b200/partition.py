"""Session-level data parallelism across GPUs (one process per GPU).

A single decode step does not shard usefully at these model sizes, so the
work that spreads over several GPUs is a set of independent sessions:
generations to run, or checkpoints (WALs) to replay with Divergence
verification (engine.rs:241-274). Each rank takes a contiguous block of the
session index, the blocks balanced by token count; every rank holds the
whole model, runs its block with the batched token loop, and only the small
per-session outcomes are gathered on the host. There is no collective on the
data path, and a session's result does not depend on where it ran (the token
loop is bit-identical across batch compositions).
"""
from __future__ import annotations

import bisect
from typing import Callable, List, Optional, Sequence, Tuple


def partition(weights: Sequence[int], world: int) -> List[range]:
    """Contiguous blocks of range(len(weights)), one per rank, balanced by
    total weight: rank r starts at the first index whose exclusive prefix sum
    reaches r * total / world. Deterministic; every index lands in exactly
    one block; blocks may be empty when there are fewer sessions than ranks."""
    if world < 1:
        raise ValueError("world size must be positive")
    n = len(weights)
    if any(w < 0 for w in weights):
        raise ValueError("weights must be non-negative")
    prefix = [0]
    for w in weights:
        prefix.append(prefix[-1] + int(w))
    total = prefix[-1]
    starts = []
    for r in range(world):
        if total == 0:
            starts.append((n * r) // world)
        else:
            # smallest i with prefix[i] * world >= r * total
            target = r * total
            i = bisect.bisect_left([p * world for p in prefix], target)
            starts.append(min(i, n))
    starts.append(n)
    for r in range(world):
        starts[r + 1] = max(starts[r + 1], starts[r])
    return [range(starts[r], starts[r + 1]) for r in range(world)]


def checkpoint_tokens(ck) -> int:
    """Token steps a verified checkout of `ck` runs (its history length)."""
    return len(ck.history_tokens)


def _gpu_replay(model, cks, batch):
    from . import replay_batch
    return replay_batch(model, cks, batch=batch, fingerprints=True)


def replay_sharded(model, ckpts: Sequence, rank: int, world: int, batch: int = 64,
                   group=None, worker: Optional[Callable] = None) -> Tuple[list, float, List[range]]:
    """Batched verified replay of `ckpts` over `world` ranks.

    Rank `rank` replays its block (partition by history length) with
    `worker(model, block, batch) -> (outcomes, device_ms)` (default: the GPU
    batched replay); with `group` (a torch.distributed process group) the
    outcomes of every rank are gathered into session order on every rank and
    the device time is the maximum over ranks. Returns (outcomes, device_ms,
    blocks)."""
    blocks = partition([checkpoint_tokens(c) for c in ckpts], world)
    mine = blocks[rank]
    work = worker or _gpu_replay
    out, ms = work(model, [ckpts[i] for i in mine], batch) if len(mine) else ([], 0.0)
    if group is None or world == 1:
        return list(out), float(ms), blocks
    import torch.distributed as dist
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, list(out), float(ms)), group=group)
    by_rank = {r: (o, t) for r, o, t in gathered}
    outcomes = []
    for r in range(world):
        outcomes.extend(by_rank[r][0])
    return outcomes, max(t for _, t in by_rank.values()), blocks
