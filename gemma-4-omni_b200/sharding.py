"""Session sharding across GPUs: one process (and one listener context) per GPU.

Every session's streaming state -- mel row, subsampler row, K/V ring, conv
ring, valid bits, PCM tail -- is private to it, and the weights are read-only,
so the step partitions by session with no exchange between GPUs: ingress routes
each session's rows to ``shard_of(session_id, n_gpus)`` and each rank packs and
steps only its own rows.  The only collectives are end-of-run host reductions
of counters and timings (max over ranks for time, sum for work).
"""
from __future__ import annotations

from typing import Callable, Iterable, Sequence

_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x100000001B3


def shard_of(session_id, n_shards: int) -> int:
    """Stable shard of a session: integer ids by value mod n, other ids by the
    64-bit FNV-1a hash of their UTF-8 text mod n (identical in every process,
    unlike Python's salted ``hash``)."""
    if n_shards < 1:
        raise ValueError("n_shards must be >= 1")
    if isinstance(session_id, bool):
        raise TypeError("session ids are str or int")
    if isinstance(session_id, int):
        return session_id % n_shards
    h = _FNV_OFFSET
    for b in str(session_id).encode("utf-8"):
        h ^= b
        h = (h * _FNV_PRIME) & 0xFFFFFFFFFFFFFFFF
    return h % n_shards


def split_rows(rows: Iterable, n_shards: int, key: Callable = lambda r: r.session_id) -> list[list]:
    """Route one tick's rows to their shards, keeping the tick's row order
    within every shard."""
    out: list[list] = [[] for _ in range(n_shards)]
    for r in rows:
        out[shard_of(key(r), n_shards)].append(r)
    return out


def local_sessions(candidates: Iterable, rank: int, world: int, count: int) -> list:
    """The first ``count`` ids of ``candidates`` that shard to ``rank``: a fixed
    number of sessions per GPU (weak scaling) under the real routing rule."""
    out = []
    for sid in candidates:
        if shard_of(sid, world) == rank:
            out.append(sid)
            if len(out) == count:
                break
    if len(out) < count:
        raise ValueError(f"only {len(out)} of {count} sessions route to rank {rank}")
    return out


def reduce_over_ranks(times: Sequence[float], counts: Sequence[int], device=None) -> tuple[list, list]:
    """End-of-run reduction across ranks: max of each time, sum of each count.

    Works on any initialised process group (``gloo`` on CPU tensors, ``nccl``
    on ``device``); with no process group it returns the inputs unchanged."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(times), list(counts)
    t = torch.tensor(list(times), dtype=torch.float64, device=device)
    c = torch.tensor(list(counts), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(c, op=dist.ReduceOp.SUM)
    return t.tolist(), [int(v) for v in c.tolist()]
