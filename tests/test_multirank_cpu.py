"""CPU, world size 2 over gloo: the bench's N>1 logic -- every rank draws the
same global batch, takes its share from the library's LPT planner
(pkc_shard_plan: utterance sharding, no data-path collective), and the job's
time is the MAX over ranks while the audio is the SUM of the shares (the
whole global batch: strong scaling)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [repo, os.path.join(repo, "parakeet.cpp_b200", "python"), os.path.join(repo, "oracle")]
    import datetime
    import torch
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        pcm_all, info = bench.workload("c2_0.6b_f16", batch=7)
        mine = bench.my_share(pcm_all, world, rank)
        audio = sum(len(pcm_all[i]) for i in mine) / 16000
        ms, e2e, tot, wall = bench.combine_ranks(10.0 * (rank + 1), 20.0 * (rank + 1), audio, 5.0 + rank, world,
                                                 torch.device("cpu"))
        total = sum(len(p) for p in pcm_all) / 16000
        q.put((rank, audio, ms, e2e, tot, wall, mine, total))
    finally:
        dist.destroy_process_group()


def test_two_rank_combine_and_sharding():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, a0, ms0, e0, t0, w0, m0, g0), (r1, a1, ms1, e1, t1, w1, m1, g1) = res
    assert not set(m0) & set(m1)                 # disjoint shares ...
    assert sorted(m0 + m1) == list(range(7))     # ... covering the global batch
    assert ms0 == ms1 == 20.0                    # MAX over ranks
    assert e0 == e1 == 40.0
    assert w0 == w1 == 6.0
    assert abs(t0 - (a0 + a1)) < 1e-9            # SUM of audio ...
    assert abs(t0 - g0) < 1e-9 and g0 == g1      # ... = the whole global batch
    assert t0 == t1
    # LPT keeps the two shares' audio within one clip of each other
    assert abs(a0 - a1) <= 35.0


def test_workload_is_the_same_global_batch_on_every_rank():
    import bench
    a, _ = bench.workload("c2_0.6b_f16", batch=2)
    b, _ = bench.workload("c2_0.6b_f16", batch=2)
    assert all((x == y).all() for x, y in zip(a, b))
    assert bench.my_share(a, 1, 0) == [0, 1]
