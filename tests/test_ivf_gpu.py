"""Candidate generation (IVFIndex: centroid probe -> inverted lists -> exact MaxSim over the
candidates) against the oracle's restatement. Integer stages are checked exactly: the inverted
lists, and the candidate sets built from the GPU's probes; the probes themselves against the
oracle's top-nprobe up to fp32 near-ties of the centroid scores; the final top-k against the
full-corpus scores masked to each query's candidates, bit for bit (a document's score does not
depend on which other documents are scored with it)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def _corpus(n_docs, n_cent, d, seed, lo=0, hi=120):
    g = R.gen(seed)
    cent = torch.nn.functional.normalize(torch.randn(n_cent, d, generator=g), dim=-1).half()
    lens = R.ragged_lengths(n_docs, lo, hi, seed)
    off = R.offsets_from_lengths(lens)
    T = int(off[-1])
    # tokens near their centroid, as after k-means assignment
    codes = torch.randint(0, n_cent, (T,), generator=g, dtype=torch.int32)
    D = torch.nn.functional.normalize(cent[codes.long()].float() + 0.3 * torch.randn(T, d, generator=g), dim=-1).half()
    return cent, codes, D, off


@pytest.mark.parametrize("n_docs,n_cent,nprobe,bq,nq", [(600, 64, 2, 3, 32), (2000, 256, 4, 5, 20),
                                                       (300, 16, 16, 2, 8), (1500, 1024, 1, 4, 32)])
def test_ivf_lists_probe_and_candidates(n_docs, n_cent, nprobe, bq, nq, cuda_device):
    from tilemaxsim_b200 import IVFIndex
    cent, codes, D, off = _corpus(n_docs, n_cent, 128, seed=n_docs + n_cent)
    codes[::53] = n_cent + 7  # ids outside the table belong to no list
    idx = IVFIndex(cent.to(cuda_device), codes.to(cuda_device), torch.from_numpy(off).to(cuda_device))
    lists = O.ivf_lists(codes, off, n_cent)
    got_off = idx.ivf_offsets.cpu().numpy()
    got_docs = idx.ivf_docs.cpu().numpy()
    for c in range(n_cent):
        np.testing.assert_array_equal(got_docs[got_off[c]:got_off[c + 1]], lists[c])
    Q = R.normalized((bq, nq, 128), 5)
    probe = idx.probe(Q.to(cuda_device), nprobe).cpu().numpy()
    # every probed centroid is among the oracle's best nprobe, up to fp32 near-ties
    S = Q.float().reshape(bq * nq, 128).numpy() @ cent.float().numpy().T
    kth = np.sort(S, axis=1)[:, -nprobe]
    chosen = np.take_along_axis(S, probe.reshape(bq * nq, nprobe), axis=1)
    assert np.all(chosen >= kth[:, None] - 1e-5)
    want_probe = O.ivf_probe(Q, cent, nprobe)
    assert np.mean(want_probe == probe) > 0.99
    # candidate sets from the GPU's probes: exact
    bitmaps, cand = idx.candidates(Q.to(cuda_device), nprobe)
    want = O.ivf_candidates(probe, lists)
    union = np.unique(np.concatenate(want))
    np.testing.assert_array_equal(cand.cpu().numpy(), union)
    bm = bitmaps.cpu().numpy().view(np.uint32)
    for q in range(bq):
        bits = np.unpackbits(bm[q].view(np.uint8), bitorder="little")[:n_docs]
        np.testing.assert_array_equal(np.nonzero(bits)[0], want[q])


@pytest.mark.parametrize("k,nprobe", [(10, 2), (100, 4), (5, 1)])
def test_ivf_search_equals_masked_full_scoring(k, nprobe, cuda_device):
    from tilemaxsim_b200 import IVFIndex, maxsim_batched
    cent, codes, D, off = _corpus(3000, 128, 128, seed=7, lo=1, hi=200)
    dev = cuda_device
    offs = torch.from_numpy(off).to(dev)
    idx = IVFIndex(cent.to(dev), codes.to(dev), offs)
    Q = R.normalized((6, 32, 128), 9).to(dev)
    vals, ids = idx.search(Q, D.to(dev), k, nprobe)
    full = maxsim_batched(Q, D.to(dev), offs).cpu().numpy()
    probe = idx.probe(Q, nprobe).cpu().numpy()
    lists = O.ivf_lists(codes, off, 128)
    for q, cands in enumerate(O.ivf_candidates(probe, lists)):
        s = np.full(full.shape[1], np.nan, np.float32)
        s[cands] = full[q, cands]
        wv, wi = O.topk(s, min(k, len(cands)))
        kk = len(wi)
        np.testing.assert_array_equal(ids[q, :kk].cpu().numpy(), wi)
        np.testing.assert_array_equal(vals[q, :kk].cpu().numpy(), wv)
        assert torch.all(ids[q, kk:] == -1) and torch.all(torch.isneginf(vals[q, kk:]))
    # the exact scores of the candidates against the CPU oracle
    np.testing.assert_allclose(full[:2, :500], O.maxsim_ragged(Q[:2].cpu(), D, off)[:, :500], rtol=1e-3, atol=1e-3)


def test_ivf_no_candidates_and_empty_lists(cuda_device):
    """Queries whose probed centroids hold no document get (-inf, -1) everywhere."""
    from tilemaxsim_b200 import IVFIndex
    cent, codes, D, off = _corpus(200, 32, 128, seed=3)
    codes[:] = 0  # every token on centroid 0: all other lists are empty
    idx = IVFIndex(cent.to(cuda_device), codes.to(cuda_device), torch.from_numpy(off).to(cuda_device))
    # a query equal to centroid 5 probes centroid 5 only (nprobe = 1)
    Q = cent[5].float().expand(1, 4, 128).contiguous().half().to(cuda_device)
    vals, ids = idx.search(Q, D.to(cuda_device), 10, 1)
    assert torch.all(ids == -1) and torch.all(torch.isneginf(vals))
