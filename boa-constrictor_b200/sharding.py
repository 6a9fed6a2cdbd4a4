"""Chunk sharding across ranks (one process per GPU) and assembly of one BOA2
container from the shards.

Chunks are independent (fresh state and a raw first byte per chunk,
boa.cpp:420-435), so a stream is split into contiguous chunk ranges, one per
rank, with no data exchange while coding.  The container only needs every
chunk's first byte and word count plus the streams in chunk order; rank 0
gathers them (torch.distributed, any backend) and writes the file.
"""
from __future__ import annotations

import numpy as np


def shard_range(n_chunks: int, rank: int, world: int):
    """(first_chunk, n_chunks) of `rank`: contiguous, sizes differ by <= 1."""
    a = n_chunks * rank // world
    b = n_chunks * (rank + 1) // world
    return a, b - a


class ShardError(RuntimeError):
    """A rank could not deliver its shard: it reported an error, or it left
    the job (the gather's collective failed or timed out)."""


def gather_container(total_size: int, chunk_len: int, first_bytes, sizes_words, payload_words, dist=None,
                     group=None, dst: int = 0, error: str | None = None):
    """Collect every rank's shard (in rank order = chunk order) on rank `dst`
    and return the BOA2 bytes there (None elsewhere).  Works with one rank and
    no process group too.

    A rank whose coding failed calls this with `error` (a message) and no
    data, so that its peers are not left waiting in the collective: every
    rank then raises ShardError naming the failed ranks.  A rank that left
    the job without calling it makes the collective fail (a closed
    connection, or the process group's timeout), which is raised as
    ShardError as well."""
    from . import boa2_build
    if error is None:
        mine = ("ok", (np.asarray(first_bytes, np.uint8), np.asarray(sizes_words, np.uint32),
                       np.asarray(payload_words, np.uint32)))
    else:
        mine = ("failed", str(error))
    if dist is None or not dist.is_initialized() or dist.get_world_size(group) == 1:
        parts = [mine]
    else:
        parts = [None] * dist.get_world_size(group)
        try:
            dist.all_gather_object(parts, mine, group=group)
        except Exception as e:  # a peer left: gloo / NCCL report it as a runtime error
            raise ShardError(f"shard gather failed, a rank left or timed out: {e}") from e
    failed = [(r, p[1]) for r, p in enumerate(parts) if p[0] != "ok"]
    if failed:
        raise ShardError("; ".join(f"rank {r} failed: {msg}" for r, msg in failed))
    if dist is not None and dist.is_initialized() and dist.get_world_size(group) > 1 and dist.get_rank(group) != dst:
        return None
    fb = np.concatenate([p[1][0] for p in parts])
    sz = np.concatenate([p[1][1] for p in parts])
    pay = np.concatenate([p[1][2] for p in parts])
    return boa2_build(total_size, chunk_len, fb, sz, pay)
