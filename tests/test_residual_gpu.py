"""Residual-compressed corpora (ColBERTv2 layout): tokens decoded on chip by the dense kernel's
decoder warps and scored on the tensor cores, against the oracle's decompress-then-score."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def _corpus(d, nbits, seed, n_docs=400, hi=150, n_cent=1000):
    g = R.gen(seed)
    cent = torch.nn.functional.normalize(torch.randn(n_cent, d, generator=g), dim=-1).half()
    lens = R.ragged_lengths(n_docs, 0, hi, seed)
    lens[::97] = 0  # a few empty documents in every corpus
    off = R.offsets_from_lengths(lens)
    T = int(off[-1])
    codes = torch.randint(0, n_cent, (T,), generator=g, dtype=torch.int32)
    res = torch.randint(0, 256, (T, d * nbits // 8), generator=g, dtype=torch.uint8)
    bw = torch.sort(torch.randn(1 << nbits, generator=g) * 0.05).values
    return cent, codes, res, bw, off


@pytest.mark.parametrize("nqry,nq,nbits,normalize,d", [
    (1, 32, 2, True, 128), (5, 32, 2, True, 128), (3, 32, 1, False, 128), (2, 32, 4, True, 128),
    (1, 40, 2, True, 128), (1, 32, 2, True, 64), (6, 20, 4, False, 64), (2, 32, 1, True, 64),
    (4, 32, 2, True, 128), (1, 100, 4, True, 64), (2, 32, 2, False, 128)])
def test_residual_vs_oracle(nqry, nq, nbits, normalize, d, cuda_device):
    """Up to four 32-row query chunks take the token-rows kernel (decoded tokens in TMEM, one
    document stream per lane, the unit-length scale applied to each token's products); larger
    batches the dense kernel's residual decoder warps."""
    from tilemaxsim_b200 import ResidualMaxSim
    cent, codes, res, bw, off = _corpus(d, nbits, seed=nqry + 10 * nbits + d)
    Q = R.normalized((nqry, nq, d), 7)
    scorer = ResidualMaxSim(cent.to(cuda_device), bw.to(cuda_device), nbits, normalize)
    got = scorer.score_queries(Q.to(cuda_device), codes.to(cuda_device), res.to(cuda_device),
                               torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    D = O.residual_decompress(cent, codes, res, bw, nbits, normalize)
    want = O.maxsim_ragged(Q, torch.from_numpy(D), off)
    inf = np.isinf(want)
    assert inf.any()  # empty documents are in the corpus
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=1e-3)


def test_residual_empty_corpus_and_code_clamp(cuda_device):
    """A corpus of empty documents scores -inf; centroid ids out of range are clamped, never read
    outside the centroid table."""
    from tilemaxsim_b200 import ResidualMaxSim
    cent, codes, res, bw, off = _corpus(128, 2, seed=3, n_docs=50)
    scorer = ResidualMaxSim(cent.to(cuda_device), bw.to(cuda_device), 2)
    Q = R.normalized((2, 32, 128), 8).to(cuda_device)
    empty = scorer.score_queries(Q, codes[:0].to(cuda_device), res[:0].to(cuda_device),
                                 torch.zeros(6, dtype=torch.int64, device=cuda_device))
    assert empty.shape == (2, 5) and torch.all(torch.isneginf(empty))
    wild = codes.clone()
    wild[::7] = 10**6
    wild[1::7] = -5
    got = scorer.score_queries(Q, wild.to(cuda_device), res.to(cuda_device), torch.from_numpy(off).to(cuda_device))
    want = O.maxsim_ragged(Q.cpu(), torch.from_numpy(O.residual_decompress(cent, wild, res, bw, 2)), off)
    inf = np.isinf(want)
    np.testing.assert_allclose(got.cpu().numpy()[~inf], want[~inf], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("d,nbits,misalign", [(64, 1, 0), (128, 2, 4), (128, 4, 0)])
def test_residual_long_ranges_and_copy_widths(d, nbits, misalign, cuda_device):
    """Dozens of 128-token tiles per CTA (the shared-memory ring wraps many times), residual rows
    copied 4 bytes at a time (8-byte rows, or a residual buffer that is only 4-byte aligned) or 16
    at a time."""
    from tilemaxsim_b200 import ResidualMaxSim
    cent, codes, res, bw, off = _corpus(d, nbits, seed=21 + d + nbits, n_docs=8000, n_cent=4096)
    rb = res.shape[1]
    res_d = res.to(cuda_device)
    if misalign:
        buf = torch.zeros(res.numel() + 16, dtype=torch.uint8, device=cuda_device)
        res_d = buf[misalign:misalign + res.numel()].view(-1, rb)
        res_d.copy_(res.to(cuda_device))
        assert res_d.data_ptr() % 16 == misalign
    Q = R.normalized((2, 32, d), 9)
    scorer = ResidualMaxSim(cent.to(cuda_device), bw.to(cuda_device), nbits)
    got = scorer.score_queries(Q.to(cuda_device), codes.to(cuda_device), res_d,
                               torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.maxsim_ragged(Q, torch.from_numpy(O.residual_decompress(cent, codes, res, bw, nbits)), off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("nbits", [1, 2, 4])
def test_residual_colbert_encoded_corpus(nbits, cuda_device):
    """End to end from a restatement of ColBERTv2's encoder: seeded embeddings near their centroids
    are compressed (nearest centroid, quantile buckets, bits least-significant first, packbits),
    scored on the GPU straight from the compressed form, and checked (a) against the oracle's
    decompress-then-score to 1e-3 and (b) against MaxSim over the original embeddings to the
    codec's quantisation error: |score(decoded) - score(X)| <= sum_i |q_i| * max_j |decoded_j - x_j|."""
    import colbert_codec as CC
    from tilemaxsim_b200 import ResidualMaxSim
    rng = np.random.default_rng(nbits)
    d, n_cent, n_docs = 128, 256, 300
    C = rng.standard_normal((n_cent, d)).astype(np.float32)
    C /= np.linalg.norm(C, axis=1, keepdims=True)
    lens = R.ragged_lengths(n_docs, 1, 120, seed=nbits)
    off = R.offsets_from_lengths(lens)
    T = int(off[-1])
    X = C[rng.integers(0, n_cent, T)] + 0.05 * rng.standard_normal((T, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    codes = np.argmax(X @ C.T, axis=1)
    cut, w = CC.train_buckets(X - C[codes], nbits)
    codes, packed = CC.compress(X, C, cut, nbits)
    cent = torch.from_numpy(C).half()
    Q = R.normalized((3, 32, d), 9)
    scorer = ResidualMaxSim(cent.to(cuda_device), torch.from_numpy(w).to(cuda_device), nbits, True)
    got = scorer.score_queries(Q.to(cuda_device), torch.from_numpy(codes).to(cuda_device),
                               torch.from_numpy(packed).to(cuda_device),
                               torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    dec = O.residual_decompress(cent, codes, packed, w, nbits, normalize=True)
    np.testing.assert_allclose(got, O.maxsim_ragged(Q, torch.from_numpy(dec), off), rtol=1e-3, atol=1e-3)
    err = np.linalg.norm(dec.astype(np.float32) - X, axis=1)  # per token
    per_doc = np.maximum.reduceat(err, off[:-1])
    bound = torch.linalg.vector_norm(Q.float(), dim=-1).sum(-1).numpy()[:, None] * per_doc[None, :]
    exact = O.maxsim_ragged(Q, torch.from_numpy(X), off)
    assert np.all(np.abs(got - exact) <= bound + 1e-3)


@pytest.mark.parametrize("nqry", [1, 5])
def test_residual_offsets_not_starting_at_zero(nqry, cuda_device):
    """A corpus given as a window of larger code / residual arrays (offsets start past 0), on the
    token-rows kernel (one query) and the dense kernel's decoder warps (five queries)."""
    from tilemaxsim_b200 import ResidualMaxSim
    cent, codes, res, bw, off = _corpus(128, 2, seed=31 + nqry, n_docs=500)
    pad = 777
    T = codes.numel()
    codes_w = torch.cat([torch.randint(0, cent.shape[0], (pad,), generator=R.gen(1), dtype=torch.int32), codes,
                         torch.zeros(40, dtype=torch.int32)])
    res_w = torch.cat([torch.randint(0, 256, (pad, res.shape[1]), generator=R.gen(2), dtype=torch.uint8), res,
                       torch.zeros(40, res.shape[1], dtype=torch.uint8)])
    off_w = off + pad
    Q = R.normalized((nqry, 32, 128), 12)
    scorer = ResidualMaxSim(cent.to(cuda_device), bw.to(cuda_device), 2)
    got = scorer.score_queries(Q.to(cuda_device), codes_w.to(cuda_device), res_w.to(cuda_device),
                               torch.from_numpy(off_w).to(cuda_device)).cpu().numpy()
    assert codes_w.numel() == T + pad + 40
    want = O.maxsim_ragged(Q, torch.from_numpy(O.residual_decompress(cent, codes, res, bw, 2)), off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=1e-3)
