"""GraphedStep: a search step captured as a CUDA graph gives the eager step's results exactly, for
fresh host inputs on every call (dense and PQ)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R

pytestmark = pytest.mark.gpu


def test_graphed_dense_search_equals_eager(cuda_device):
    from tilemaxsim_b200 import GraphedStep
    from tilemaxsim_b200.sharded import ShardedIndex
    lengths = R.ragged_lengths(3000, 0, 200, seed=3)
    off = torch.from_numpy(R.offsets_from_lengths(lengths)).to(cuda_device)
    D = R.normalized((int(off[-1]), 128), 4).to(cuda_device)
    idx = ShardedIndex(D, off, doc_id_base=500)
    q0 = R.normalized((6, 32, 128), 5)
    step = GraphedStep(lambda Q: idx.search(Q, 50), q0.to(cuda_device))
    for seed in (5, 6, 7):
        qh = R.normalized((6, 32, 128), seed).pin_memory()
        v, i = step(qh)
        ev, ei = idx.search(qh.to(cuda_device), 50)
        assert torch.equal(v, ev.cpu()) and torch.equal(i, ei.cpu())
    with pytest.raises(ValueError):
        step(R.normalized((5, 32, 128), 8))  # the captured shape is fixed


def test_graphed_pq_step_equals_eager(cuda_device):
    from tilemaxsim_b200 import GraphedStep, TileMaxSimPQ, topk
    lengths = R.ragged_lengths(500, 0, 150, seed=9)
    off = torch.from_numpy(R.offsets_from_lengths(lengths)).to(cuda_device)
    codes = torch.randint(0, 256, (int(off[-1]), 16), generator=R.gen(5), dtype=torch.uint8).to(cuda_device)
    cb = R.randn((16, 256, 8), 3, torch.float32).to(cuda_device)

    # token-rows kernel, decoder-warp kernel (exact=False); the table-lookup kernel (default)
    for nq_, exact in ((1, False), (5, False), (3, True)):
        pq = TileMaxSimPQ(cb, exact=exact)

        def fn(Q):
            return topk(pq.score_queries(Q, codes, off), 20)

        q0 = R.normalized((nq_, 32, 128), 4)
        step = GraphedStep(fn, q0.to(cuda_device))
        qh = R.normalized((nq_, 32, 128), 11).pin_memory()
        v, i = step(qh)
        ev, ei = fn(qh.to(cuda_device))
        np.testing.assert_array_equal(v.numpy(), ev.cpu().numpy())
        assert torch.equal(i, ei.cpu())
