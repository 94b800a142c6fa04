"""Sharded search plumbing on CPU ranks (gloo, world_size 2): per-shard top-k with global ids, the
all-gather layout, padding of short shards and the merge tie rule. The merge ranks candidates with
the oracle here; on GPUs the same code path uses the library's top-k over NCCL."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import maxsim_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_topk(scores, k, ids=None):
    v, i = O.topk(scores.numpy(), k, ids=None if ids is None else ids.numpy())
    return torch.from_numpy(v), torch.from_numpy(i)


def shard_scores(world: int, n_per: list[int], rows: int) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(123)
    full = (torch.randint(0, 40, (rows, sum(n_per)), generator=g).float() / 4.0)  # many ties
    out, c = [], 0
    for n in n_per:
        out.append(full[:, c:c + n].clone())
        c += n
    return out


def _worker(rank, world, port, n_per, rows, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from tilemaxsim_b200.sharded import merge_topk
        scores = shard_scores(world, n_per, rows)[rank]
        base = sum(n_per[:rank])
        kk = min(k, n_per[rank])
        v, i = oracle_topk(scores, kk)
        v, i = merge_topk(v, i + base, k, group=dist.group.WORLD, topk_fn=oracle_topk)
        q.put((rank, v.numpy(), i.numpy()))
    finally:
        dist.destroy_process_group()


def run(n_per, rows=3, k=50):
    world = len(n_per)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_per, rows, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = torch.cat(shard_scores(world, n_per, rows), dim=1)
    want_v, want_i = O.topk(full.numpy(), k)
    for rank, v, i in res:  # identical on every rank, equal to the single-corpus top-k
        np.testing.assert_array_equal(i, want_i)
        np.testing.assert_array_equal(v, want_v)


def test_merge_two_ranks():
    run([400, 300])


def test_merge_short_shard_padded():
    run([30, 500], k=50)  # rank 0 has fewer documents than k: padded with (NaN, max id)


def _exit_flushed(q):
    """os._exit skips the queue's feeder thread: flush what was put before leaving."""
    q.close()
    q.join_thread()
    os._exit(0)


def _faulty_worker(rank, world, port, mode, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        dist.barrier()  # both ranks are up; the fault comes after this step
    except Exception as e:
        if rank == 0:
            q.put(("setup failed: " + type(e).__name__, -1.0))
        _exit_flushed(q)
    if rank == 1:  # leaves between steps, with no collective in flight
        if mode == "stalls":
            time.sleep(10)
        os._exit(0)
    from tilemaxsim_b200.sharded import merge_topk
    v = torch.arange(20, dtype=torch.float32).view(2, 10)
    i = torch.arange(20, dtype=torch.int64).view(2, 10)
    t0 = time.monotonic()
    try:
        merge_topk(v, i, 10, group=dist.group.WORLD, topk_fn=oracle_topk)
        q.put(("completed", time.monotonic() - t0))
    except Exception as e:  # the failure reaches the host as an exception, not a hang
        q.put((type(e).__name__, time.monotonic() - t0))
    _exit_flushed(q)  # no process-group teardown: it would wait for the missing rank


@pytest.mark.parametrize("mode", ["dies", "stalls"])
def test_missing_rank_fails_the_merge_within_the_timeout(mode):
    """Failure detection on the host: a rank that exits (or stops responding) between search
    steps makes the surviving rank's top-k merge raise within the process group's timeout."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_faulty_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        outcome, seconds = q.get(timeout=90)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert outcome != "completed" and not outcome.startswith("setup failed"), outcome
    assert 0 <= seconds < 30
