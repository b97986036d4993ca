"""Utterance sharding across GPUs: the work splits by utterance with no data-path collective.

Each rank takes the utterances that a longest-first greedy assignment gives it (cost linear in
length, the matrix products' share), processes them in length-sorted batches, and keeps its own
tokens. The only cross-rank traffic is host-side: an optional gather of token ids and the
status of every rank's shard, so that one rank's failure is reported on all ranks instead of
leaving them waiting.
"""

from __future__ import annotations

from typing import Callable, List, Sequence

import numpy as np

SAMPLE_RATE = 16000


def assign(samples: Sequence[int], world: int) -> List[List[int]]:
    """Longest-first greedy assignment of utterances (by sample count) to `world` ranks: each
    utterance, longest first, goes to the least-loaded rank (lowest rank on ties). Returns each
    rank's utterance indices."""
    if world < 1:
        raise ValueError("world must be at least 1")
    samples = np.asarray(samples, dtype=np.int64)
    order = np.argsort(-samples, kind="stable")
    load = np.zeros(world, dtype=np.int64)
    shards: List[List[int]] = [[] for _ in range(world)]
    for u in order:
        r = int(np.argmin(load))
        shards[r].append(int(u))
        load[r] += samples[u]
    return shards


def batches(utts: Sequence[int], samples: Sequence[int], max_seconds: float) -> List[List[int]]:
    """Length-sorted batches of about equal audio: ceil(total / max_seconds) of them, none above
    `max_seconds` (a longer utterance gets a batch of its own), so a batch's utterances have
    similar lengths and the last batch is not a small remainder. The cut rule is the one
    telmo_granite_transcribe applies to its groups, so the sorted utterances passed to it in one
    call are transcribed in exactly these batches."""
    samples = np.asarray(samples, dtype=np.int64)
    ordered = sorted(utts, key=lambda u: (int(samples[u]), u))
    limit = int(max_seconds * SAMPLE_RATE)
    total = int(samples[ordered].sum()) if ordered else 0
    groups = max(1, -(-total // limit))
    out, cur = [], []
    acc = in_batch = 0
    g = 1
    for u in ordered:
        n = int(samples[u])
        if cur and (in_batch + n > limit or acc >= g * total // groups):
            out.append(cur)
            cur, in_batch = [], 0
            g += 1
        cur.append(u)
        acc += n
        in_batch += n
    if cur:
        out.append(cur)
    return out


class ShardError(RuntimeError):
    """Raised on every rank when any rank's shard failed."""


def run_shard(rank: int, world: int, work: Callable[[], object], group=None):
    """Runs this rank's `work`, then exchanges every rank's status on the host (one
    all_gather_object over `group`, a gloo or NCCL process group; none when world is 1). Returns
    the list of every rank's result, or raises ShardError naming the ranks that failed."""
    try:
        result, status = work(), None
    except Exception as e:  # the shard's failure is reported, not swallowed
        result, status = None, f"{type(e).__name__}: {e}"
    if world == 1:
        if status:
            raise ShardError(f"rank 0 failed: {status}")
        return [result]
    import torch.distributed as dist
    gathered = [None] * world
    dist.all_gather_object(gathered, (status, result), group=group)
    failed = [(r, s) for r, (s, _) in enumerate(gathered) if s]
    if failed:
        raise ShardError("; ".join(f"rank {r} failed: {s}" for r, s in failed))
    return [res for _, res in gathered]
