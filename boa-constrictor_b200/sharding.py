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


def gather_container(total_size: int, chunk_len: int, first_bytes, sizes_words, payload_words, dist=None,
                     group=None, dst: int = 0):
    """Collect every rank's shard (in rank order = chunk order) on rank `dst`
    and return the BOA2 bytes there (None elsewhere).  Works with one rank and
    no process group too."""
    from . import boa2_build
    mine = (np.asarray(first_bytes, np.uint8), np.asarray(sizes_words, np.uint32),
            np.asarray(payload_words, np.uint32))
    if dist is None or not dist.is_initialized() or dist.get_world_size(group) == 1:
        parts = [mine]
    else:
        parts = [None] * dist.get_world_size(group)
        dist.all_gather_object(parts, mine, group=group)
        if dist.get_rank(group) != dst:
            return None
    fb = np.concatenate([p[0] for p in parts])
    sz = np.concatenate([p[1] for p in parts])
    pay = np.concatenate([p[2] for p in parts])
    return boa2_build(total_size, chunk_len, fb, sz, pay)
