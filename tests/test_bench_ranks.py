"""Multi-rank host logic of bench.py on CPU (gloo, world size 2).

On the GPU box `bench.py --gpus N` runs one process per GPU over NCCL; frames
are independent, so the only cross-rank operations are the barrier around the
timed region and a max-reduce of the elapsed times. These tests run the same
RankGroup over gloo on 127.0.0.1 with two spawned ranks.
"""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench
    r, lr, w = bench.dist_env()
    ranks = bench.RankGroup(w, backend="gloo", timeout_s=60)
    ranks.barrier()
    ms = 10.0 + 5.0 * r                      # rank 1 is the slower one
    ms_max = ranks.max(ms)
    seeds = list(range(bench.frame_seed_base(r, 4), bench.frame_seed_base(r, 4) + 4))
    value = bench.aggregate_frames_per_s(w, 4, 3, ms_max)
    ranks.barrier()
    ranks.close()
    out.put((r, lr, w, ms_max, seeds, value))


def test_two_ranks_barrier_max_and_disjoint_frames():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, l0, w0, m0, s0, v0), (r1, l1, w1, m1, s1, v1) = results
    assert (r0, r1, w0, w1) == (0, 1, 2, 2) and (l0, l1) == (0, 1)
    assert m0 == m1 == 15.0                    # every rank reports the slowest rank's time
    assert not set(s0) & set(s1) and sorted(s0 + s1) == list(range(8))
    assert v0 == v1 == pytest.approx(2 * 4 * 3 / 0.015)


def test_single_rank_needs_no_group():
    import bench
    g = bench.RankGroup(1)
    g.barrier()
    assert g.max(3.5) == 3.5 and not g.pg
    assert bench.aggregate_frames_per_s(1, 256, 10, 1000.0) == 2560.0
    assert bench.frame_seed_base(3, 256) == 768


def _gather_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import numpy as np
    import torch

    import bench
    ranks = bench.RankGroup(world, backend="gloo", timeout_s=60)
    first, count = bench.shard(16, rank, world)
    # stand-in per-frame checksums: a function of the frame index only
    local = torch.tensor([(f * 0x9E3779B97F4A7C15) & 0x7FFFFFFFFFFFFFFF for f in range(first, first + count)],
                         dtype=torch.int64)
    gathered = ranks.all_gather(local)
    ranks.close()
    out.put((rank, bench.checksum_digest(gathered.numpy().astype(np.uint64)), list(range(first, first + count))))


def test_checksum_gather_is_rank_ordered_and_digest_independent_of_world():
    """The streaming workload's final gather: rank-ordered concatenation of
    each rank's contiguous frame block, so the digest equals a single rank's."""
    import numpy as np
    import torch.multiprocessing as mp

    import bench
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    single = np.array([(f * 0x9E3779B97F4A7C15) & 0x7FFFFFFFFFFFFFFF for f in range(16)], np.uint64)
    assert res[0][1] == res[1][1] == bench.checksum_digest(single)
    assert res[0][2] == list(range(8)) and res[1][2] == list(range(8, 16))
