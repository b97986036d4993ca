"""Host-side sharding logic on CPU: the assignment, the batches, and world-size-2 runs over gloo,
including a rank whose shard fails (the failure is made on the host; no GPU is involved)."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from telmo_b200 import sharding, synthetic


def test_assignment_partitions_and_balances():
    secs = synthetic.lengths_log_uniform(4096, 1.0, 30.0, seed=0)
    samples = (secs * 16000).astype(np.int64)
    for world in [1, 2, 4, 8]:
        shards = sharding.assign(samples, world)
        flat = sorted(u for s in shards for u in s)
        assert flat == list(range(4096))
        loads = [samples[s].sum() for s in shards]
        # Longest-first greedy is within one longest utterance of the mean.
        assert max(loads) - min(loads) <= samples.max()
        assert max(loads) / np.mean(loads) < 1.01


def test_batches_are_length_sorted_and_bounded():
    samples = np.array([16000 * s for s in [5, 1, 30, 2, 12, 40]])
    b = sharding.batches(range(6), samples, max_seconds=20.0)
    lengths = [[samples[u] // 16000 for u in batch] for batch in b]
    assert lengths == [[1, 2, 5, 12], [30], [40]]
    assert sum(len(x) for x in b) == 6


def test_batches_split_the_audio_evenly():
    # 100 s in batches of at most 40 s: three batches of about a third each, not 40 + 40 + 20.
    samples = np.full(10, 10 * 16000)
    b = sharding.batches(range(10), samples, max_seconds=40.0)
    assert [len(x) for x in b] == [4, 3, 3]
    secs = synthetic.lengths_log_uniform(4096, 1.0, 30.0, seed=0)
    samples = (secs * 16000).astype(np.int64)
    for world in (1, 8):
        shard = sharding.assign(samples, world)[0]
        b = sharding.batches(shard, samples, 2048.0)
        loads = [samples[x].sum() / 16000 for x in b]
        assert max(loads) <= 2048.0 and len(b) == int(np.ceil(samples[shard].sum() / 16000 / 2048.0))
        assert min(loads) > 0.9 * max(loads), loads


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    samples = np.array([16000 * (1 + (u * 7) % 30) for u in range(64)])
    shard = sharding.assign(samples, world)[rank]

    def work():
        if rank == fail_rank:
            raise RuntimeError("injected shard failure")
        return [int(u) for b in sharding.batches(shard, samples, 100.0) for u in b]

    try:
        results = sharding.run_shard(rank, world, work)
        q.put((rank, "ok", sorted(u for r in results for u in r)))
    except sharding.ShardError as e:
        q.put((rank, "error", str(e)))
    dist.destroy_process_group()


def _run(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out)


def test_two_ranks_cover_every_utterance_over_gloo():
    out = _run(fail_rank=-1)
    assert [o[1] for o in out] == ["ok", "ok"]
    assert out[0][2] == out[1][2] == list(range(64))


def test_a_failed_rank_is_reported_on_every_rank():
    out = _run(fail_rank=1)
    assert [o[1] for o in out] == ["error", "error"]
    for _, _, msg in out:
        assert "rank 1 failed" in msg and "injected shard failure" in msg
