"""Multi-rank path on CPU: two gloo ranks each code a contiguous chunk range
(the CPU oracle stands in for the GPU so the test runs anywhere), rank 0
assembles one BOA2 container, and the whole container decodes back to the
input.  Mirrors what bench.py / a torchrun job does on GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, load_package


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, wpath, out_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle as O
    boa = load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    chunk = 300
    data = boa.synth.particle_stream(7 * chunk + 41, 9)
    n_chunks = (len(data) + chunk - 1) // chunk
    c0, n = boa.sharding.shard_range(n_chunks, rank, world)
    end = min(len(data), (c0 + n) * chunk)
    m = O.OracleModel(wpath, 0, 64, 1)
    fb, streams = m.compress(data[c0 * chunk:end], chunk, threads=1)
    sizes = np.array([len(s) for s in streams], np.uint32)
    pay = np.concatenate(streams) if streams else np.zeros(0, np.uint32)
    blob = boa.sharding.gather_container(len(data), chunk, fb, sizes, pay, dist=dist)
    if rank == 0:
        open(out_path, "wb").write(blob)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shards_build_one_container(boa, oracle, boa2, weights, tmp_path):
    w = weights("mamba", 64, 1, 5)
    out = str(tmp_path / "x.boa")
    mp.spawn(_worker, args=(2, _free_port(), w, out), nprocs=2, join=True)
    blob = open(out, "rb").read()
    p = boa2.parse(blob)
    data = boa.synth.particle_stream(7 * 300 + 41, 9)
    assert p["n_chunks"] == 8 and p["total_size"] == len(data) and p["last_chunk_len"] == 41
    m = oracle.OracleModel(w, 0, 64, 1)
    back = m.decompress(p["first_bytes"], [np.frombuffer(s, "<u4") for s in p["streams"]], len(data), 300)
    assert back == data


def test_shard_ranges_cover_exactly(boa):
    for n in (1, 7, 16384, 262144):
        for world in (1, 2, 3, 8):
            got = [boa.sharding.shard_range(n, r, world) for r in range(world)]
            assert sum(k for _, k in got) == n
            assert all(got[r][0] + got[r][1] == got[r + 1][0] for r in range(world - 1))


def _worker_failing(rank, world, port, mode, out_dir):
    """Rank 1 fails: with mode "error" it reports a coder failure through the
    gather, with mode "leave" it exits without joining it.  Every rank writes
    what it saw to out_dir/rank<r>.txt."""
    import datetime
    boa = load_package()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    if rank == 1 and mode == "leave":
        os._exit(0)
    fb = np.full(2, rank, np.uint8)
    sizes = np.array([1, 1], np.uint32)
    pay = np.array([rank, rank + 1], np.uint32)
    err = "simulated coder failure" if (rank == 1 and mode == "error") else None
    try:
        boa.sharding.gather_container(2 * world * 10, 10, fb, sizes, pay, dist=dist, error=err)
        seen = "ok"
    except boa.sharding.ShardError as e:
        seen = f"ShardError: {e}"
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(seen)
    if mode == "error":
        dist.destroy_process_group()
    else:
        os._exit(0)  # the group lost a member; leave without a collective teardown


@pytest.mark.parametrize("mode", ["error", "leave"])
def test_failed_rank_is_reported_not_waited_for(boa, tmp_path, mode):
    """Failure detection on the host: a rank that reports an error, or that
    leaves the job, makes the gather raise ShardError on the ranks still
    running (naming the failed rank when it reported), instead of leaving
    them blocked in the collective."""
    import time
    t0 = time.monotonic()
    mp.spawn(_worker_failing, args=(2, _free_port(), mode, str(tmp_path)), nprocs=2, join=True)
    assert time.monotonic() - t0 < 60
    r0 = (tmp_path / "rank0.txt").read_text()
    assert r0.startswith("ShardError")
    if mode == "error":
        assert "rank 1 failed: simulated coder failure" in r0
        assert (tmp_path / "rank1.txt").read_text().startswith("ShardError")
    else:
        assert not (tmp_path / "rank1.txt").exists()
