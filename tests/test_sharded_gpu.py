"""Sharded search on real GPUs: two ranks (one process per GPU, NCCL), each scoring its shard of a
ragged corpus, merging per-shard top-k with one all-gather. The merged result must equal a
single-GPU top-k over the whole corpus exactly (per-document scores do not depend on how the
corpus is split: same kernel arithmetic per document). Skipped with fewer than two GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _corpus(n_docs=3000, seed=5):
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(0, 300, (n_docs,), generator=g)
    off = torch.zeros(n_docs + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(lengths, 0)
    D = torch.nn.functional.normalize(torch.randn(int(off[-1]), 128, generator=g), dim=-1).half()
    Qb = torch.nn.functional.normalize(torch.randn(8, 32, 128, generator=g), dim=-1).half()
    return Qb, D, off


def _worker(rank, world, port, k, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from tilemaxsim_b200.sharded import ShardedIndex
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        Qb, D, off = _corpus()
        n = off.numel() - 1
        cuts = [n * r // world for r in range(world + 1)]
        lo, hi = cuts[rank], cuts[rank + 1]
        t0, t1 = int(off[lo]), int(off[hi])
        idx = ShardedIndex(D[t0:t1].to(dev), (off[lo:hi + 1] - t0).to(dev), doc_id_base=lo,
                           group=dist.group.WORLD)
        v, i = idx.search(Qb.to(dev), k)
        q.put((rank, v.cpu().numpy(), i.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("k", [10, 1000])
def test_two_gpu_sharded_search_equals_single_gpu(k):
    from tilemaxsim_b200 import maxsim_topk
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, k, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    Qb, D, off = _corpus()
    dev = torch.device("cuda", 0)
    wv, wi = maxsim_topk(Qb.to(dev), D.to(dev), off.to(dev), k)
    for rank, v, i in res:
        np.testing.assert_array_equal(i, wi.cpu().numpy())
        np.testing.assert_array_equal(v, wv.cpu().numpy())
