"""Clip sharding across GPUs (one process per device, no collective on the data path): the shard plan, a 2-rank
gloo run whose merged results equal the single-process run, and a rank failure that every rank learns of."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from mimizuku_b200.shard import ShardError, merge, run_sharded, shard


@pytest.mark.parametrize("n,world", [(0, 1), (1, 1), (7, 2), (256, 8), (5, 8), (33, 4)])
def test_shard_plan_covers_every_clip_once(n, world):
    seen = []
    for r in range(world):
        s, c = shard(n, world, r)
        seen.extend(range(s, s + c))
        assert c in (n // world, n // world + 1)
    assert seen == list(range(n))


def _work_fn(start, count):
    """Host-side stand-in for one rank's transcription: token timestamps of synthetic alignment rows per clip."""
    import mimizuku_b200 as m
    times, lens = [], []
    for i in range(start, start + count):
        rng = np.random.default_rng(i)
        w = rng.random((6, 2, 200)).astype(np.float32)
        times.append(m.jump_times(w, 150))
        lens.append(6)
    return {"tokens": np.arange(start, start + count)[:, None].repeat(3, 1), "lens": np.array(lens, np.int32),
            "times": np.array(times).reshape(count, 6)}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, n, fail_rank, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        def work(s, c):
            if rank == fail_rank:
                raise RuntimeError("simulated GPU loss")
            return _work_fn(s, c)
        parts = run_sharded(work, n)
        q.put((rank, "ok", merge(parts)))
    except ShardError as e:
        q.put((rank, "error", str(e)))
    finally:
        dist.destroy_process_group()


def _run(world, n, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, n, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


def test_two_ranks_merge_to_the_single_process_result():
    n = 7
    out = _run(2, n)
    single = _work_fn(0, n)
    for _, st, res in out:
        assert st == "ok"
        for k in ("tokens", "lens", "times"):
            assert np.array_equal(res[k], single[k])


def test_a_failed_rank_is_reported_to_every_rank():
    out = _run(2, 5, fail_rank=1)
    for _, st, msg in out:
        assert st == "error" and "rank 1 failed" in msg and "simulated GPU loss" in msg
