"""BASELINE configurations at full size on one GPU, checked against exact scores.

Top-k parity rule (north star: "top-k document IDs identical except for exact-score ties"): the
kernel sums the d products of each dot product in fp32 in the tensor core's order, so its scores
carry rounding error and two documents whose exact scores are closer than that error may swap. The
checker scores the same fp16 inputs in float64 (exact for this purpose), derives for every
(query, document) a bound E on the fp32 kernel's error (``oracle.maxsim_error_bound``:
(gamma_d(2^-22) + gamma_Nq(2^-24)) * sum_i |q_i| * max_j |x_j| + 2^-24 |s|), and asserts that every
score lies within E of the exact one and that every position where the kernel's top-k differs from
the exact ranking holds two documents whose exact scores are within the sum of their bounds. The
number of such positions is printed. Sizes that the CPU oracle cannot score whole use
``exact_f64.maxsim_f64_device`` (the same float64 computation on the GPU, checked against the CPU
oracle in the C1 test); the C3 corpora are checked through document independence.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from exact_f64 import maxsim_f64_device
from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def corpus(n_docs, lo, hi, d, seed, dev):
    lengths = R.ragged_lengths(n_docs, lo, hi, seed)
    off = R.offsets_from_lengths(lengths)
    g = torch.Generator(device=dev).manual_seed(seed)
    D = torch.empty(int(off[-1]), d, dtype=torch.float16, device=dev)
    for t0 in range(0, D.shape[0], 1 << 22):
        x = torch.randn(min(1 << 22, D.shape[0] - t0), d, device=dev, generator=g)
        D[t0:t0 + x.shape[0]] = torch.nn.functional.normalize(x, dim=-1).half()
    return D, off, lengths


def queries(bq, nq, d, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.nn.functional.normalize(torch.randn(bq, nq, d, device=dev, generator=g), dim=-1).half()


def ranking_check(Q, scores, ids, exact, dmax, k, d):
    """Every query row: scores within the derived bound of the exact ones, top-k ranking equal to
    the exact one except between documents closer than their bounds. Returns (#differing positions,
    largest error / bound)."""
    qn = torch.linalg.vector_norm(Q.double(), dim=-1).cpu().numpy()
    bound = O.maxsim_error_bound(qn, dmax, exact, d)
    scores = scores.cpu().numpy()
    ids = ids.cpu().numpy()
    swaps = 0
    for r in range(exact.shape[0]):
        swaps += O.check_ranking_within_bound(ids[r], scores[r], exact[r], bound[r], k)
    fin = np.isfinite(exact)
    ratio = float(np.max(np.abs(scores[fin] - exact[fin]) / bound[fin]))
    return swaps, ratio


def test_c1_cpu_reference_config_top10(cuda_device):
    """Config 1: 1 query x 32 tokens, 1000 docs x 180 tokens: scores and top-10 ids."""
    from tilemaxsim_b200 import maxsim_topk, maxsim_batched
    D, off, _ = corpus(1000, 180, 180, 128, 42, cuda_device)
    Q = queries(1, 32, 128, 1, cuda_device)
    offs = torch.from_numpy(off).to(cuda_device)
    want = O.maxsim_ragged(Q.cpu(), D.cpu(), off)
    scores = maxsim_batched(Q, D, offs)
    np.testing.assert_allclose(scores.cpu().numpy(), want, rtol=1e-3, atol=1e-3)
    exact = O.maxsim_ragged_f64(Q.cpu(), D.cpu(), off)
    dmax = O.doc_max_norm(D.cpu(), off)
    exact_dev, dmax_dev = maxsim_f64_device(Q, D, off, chunk_tokens=50_000)
    np.testing.assert_allclose(exact_dev, exact, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dmax_dev, dmax, rtol=1e-12)
    _, ids = maxsim_topk(Q, D, offs, 10)
    swaps, ratio = ranking_check(Q, scores, ids, exact, dmax, 10, 128)
    print(f"C1 top-10: {swaps} positions differ from the exact ranking; max error/bound {ratio:.2e}")
    assert swaps == 0


def test_c2_rerank_top1000_full_corpus(cuda_device):
    """Config 2 at full size (64 queries x 100k ragged docs): the top-1000 of every query against
    the exact float64 ranking over the whole corpus."""
    from tilemaxsim_b200 import maxsim_topk, maxsim_batched
    D, off, _ = corpus(100_000, 64, 300, 128, 42, cuda_device)
    Q = queries(64, 32, 128, 7, cuda_device)
    offs = torch.from_numpy(off).to(cuda_device)
    _, ids = maxsim_topk(Q, D, offs, 1000)
    scores = maxsim_batched(Q, D, offs)
    exact, dmax = maxsim_f64_device(Q, D, off, chunk_tokens=1 << 19)
    # the device float64 scores agree with the CPU oracle's float64 on a sample of queries
    np.testing.assert_allclose(exact[[0, 63], :2000],
                               O.maxsim_ragged_f64(Q[[0, 63]].cpu(), D[: int(off[2000])].cpu(), off[:2001]),
                               rtol=1e-12, atol=1e-12)
    swaps, ratio = ranking_check(Q, scores, ids, exact, dmax, 1000, 128)
    print(f"C2 top-1000 x 64 queries: {swaps} of {64 * 1000} positions differ from the exact ranking, "
          f"all within the fp32 error bound; max error/bound {ratio:.2e}")


@pytest.mark.parametrize("d", [256, 768])
def test_c3_dsweep_full_size_document_independence(d, cuda_device):
    """Config 3 at full size (16 queries x 50k docs x 256 tokens, d = 256 / 768)."""
    from tilemaxsim_b200 import maxsim_batched
    D, off, lengths = corpus(50_000, 256, 256, d, 3, cuda_device)
    Q = queries(16, 32, d, 4, cuda_device)
    full = maxsim_batched(Q, D, torch.from_numpy(off).to(cuda_device))
    pick = np.sort(np.random.default_rng(1).choice(50_000, 64, replace=False))
    tok = np.concatenate([np.arange(off[i], off[i + 1]) for i in pick])
    sub_off = R.offsets_from_lengths(lengths[pick])
    Dsub = D[torch.from_numpy(tok).to(cuda_device)]
    sub = maxsim_batched(Q, Dsub, torch.from_numpy(sub_off).to(cuda_device))
    assert torch.equal(full[:, torch.from_numpy(pick).to(cuda_device)], sub)
    np.testing.assert_allclose(sub.cpu().numpy(), O.maxsim_ragged(Q.cpu(), Dsub.cpu(), sub_off),
                               rtol=1e-3, atol=1e-3)


def test_c5_shard_full_size_document_independence(cuda_device):
    """One GPU's shard of config 5 (1.25M docs, N_d ~ U[96,160], 256 queries, top-100)."""
    from tilemaxsim_b200 import maxsim_batched, topk
    D, off, lengths = corpus(1_250_000, 96, 160, 128, 42, cuda_device)
    Q = queries(256, 32, 128, 7, cuda_device)
    full = maxsim_batched(Q, D, torch.from_numpy(off).to(cuda_device))
    vals, ids = topk(full, 100)
    # four queries against the exact float64 ranking of the whole shard
    exact, dmax = maxsim_f64_device(Q[:4], D, off, chunk_tokens=1 << 22)
    swaps, ratio = ranking_check(Q[:4], full[:4], ids[:4], exact, dmax, 100, 128)
    print(f"C5 shard top-100 x 4 queries: {swaps} positions differ from the exact ranking; "
          f"max error/bound {ratio:.2e}")
    pick = np.sort(np.random.default_rng(2).choice(1_250_000, 48, replace=False))
    tok = np.concatenate([np.arange(off[i], off[i + 1]) for i in pick])
    sub_off = R.offsets_from_lengths(lengths[pick])
    Dsub = D[torch.from_numpy(tok).to(cuda_device)]
    sub = maxsim_batched(Q, Dsub, torch.from_numpy(sub_off).to(cuda_device))
    assert torch.equal(full[:, torch.from_numpy(pick).to(cuda_device)], sub)
    np.testing.assert_allclose(sub[:8].cpu().numpy(), O.maxsim_ragged(Q[:8].cpu(), Dsub.cpu(), sub_off),
                               rtol=1e-3, atol=1e-3)
