"""The CPU oracle against the golden outputs of the reference's own PyTorch functions."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import load_golden
from oracle import maxsim_oracle as O


@pytest.mark.parametrize("i", range(len(R.EXP10_CONFIGS)))
def test_exp10_padded(i):
    meta, g = load_golden(f"exp10_{i}")
    c = R.exp10_case(i)
    assert R.sha256(c["Q"], c["D"]) == meta["sha256"], "input recipe drifted from the fixture"
    np.testing.assert_allclose(O.maxsim_padded(c["Q"], c["D"]), g["scores"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(O.token_max_padded(c["Q"], c["D"]), g["token_max"], rtol=1e-5, atol=1e-5)


def test_v1_selfcheck_naive_equals_loop():
    meta, g = load_golden("v1_selfcheck")
    c = R.v1_selfcheck_case()
    assert R.sha256(c["Q"], c["D"]) == meta["sha256"]
    np.testing.assert_allclose(O.maxsim_padded(c["Q"], c["D"]), g["naive"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(g["loop"], g["naive"], rtol=1e-5, atol=1e-4)


RAGGED = {"ragged_f16": {}, "ragged_bf16": {"dtype": torch.bfloat16, "seed": 11},
          "ragged_nq20": {"nq": 20, "n_queries": 2, "seed": 13},
          "ragged_nq40": {"nq": 40, "n_queries": 2, "n_docs": 120, "seed": 17}}


@pytest.mark.parametrize("name", list(RAGGED))
def test_ragged(name):
    meta, g = load_golden(name)
    c = R.ragged_case(**RAGGED[name])
    assert R.sha256(c["Qb"], c["D"], c["offsets"].numpy()) == meta["sha256"]
    s = O.maxsim_ragged(c["Qb"], c["D"], c["offsets"].numpy(), chunk_docs=37)
    assert np.isneginf(g["scores"]).sum() >= 3 * c["Qb"].shape[0]  # the forced empty documents
    np.testing.assert_allclose(s, g["scores"], rtol=1e-5, atol=1e-4)
    tm = O.token_max_ragged(c["Qb"], c["D"], c["offsets"].numpy())
    np.testing.assert_allclose(tm, g["token_max"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name,cb_dtype", [("pq_f32", torch.float32), ("pq_f16", torch.float16)])
def test_pq(name, cb_dtype):
    meta, g = load_golden(name)
    c = R.pq_case(cb_dtype)
    assert R.sha256(c["codebook"], c["Q"], c["codes"]) == meta["sha256"]
    np.testing.assert_allclose(O.pq_maxsim_adc(c["Q"], c["codebook"], c["codes"]), g["adc"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(O.pq_maxsim_decompress(c["Q"], c["codebook"], c["codes"]), g["decompress"],
                               rtol=1e-5, atol=1e-4)
    # ragged ADC form on the same codes (every doc the same length) agrees with the padded form
    B, Nd, M = c["codes"].shape
    off = np.arange(B + 1, dtype=np.int64) * Nd
    r = O.pq_maxsim_adc_ragged(c["Q"][None], c["codebook"], c["codes"].reshape(B * Nd, M), off)[0]
    np.testing.assert_allclose(r, g["adc"], rtol=1e-5, atol=1e-4)


def test_topk_ties():
    meta, g = load_golden("topk_ties")
    s = R.topk_case()["scores"]
    assert R.sha256(s) == meta["sha256"]
    vals, ids = O.topk(s, 1000)
    np.testing.assert_array_equal(ids, g["order"])
    np.testing.assert_array_equal(vals[:, :100][~np.isnan(vals[:, :100])],
                                  g["torch_topk_values"][~np.isnan(vals[:, :100])])


def test_segment_max_ignores_rows_past_the_last_document():
    """Rows after the last offset (a corpus window inside a larger token array) belong to no
    document; empty documents score -inf."""
    S = np.arange(10, dtype=np.float32).reshape(10, 1)
    got = O._segment_max(S, np.array([2, 4, 4, 6]), 0).ravel()
    np.testing.assert_array_equal(got, np.array([3, -np.inf, 5], np.float32))
    codes = np.zeros((12, 2), np.uint8)
    codes[10:] = 1  # trailing rows with a larger table entry must not reach the last document
    table = np.zeros((1, 2, 2), np.float32)
    table[:, :, 1] = 100.0
    tok = O.pq_token_scores(table, codes)
    np.testing.assert_array_equal(O._segment_max(tok, np.array([0, 5, 10]), 0).ravel(), [0, 0])


def test_residual_decompress_bit_order():
    """Known answer for the residual layout: one 8-dimension token, nbits = 2, residual bytes
    0b00011011 and 0b11100100. MSB-first pairs give fields 00,01,10,11 / 11,10,01,00; bit k of a
    dimension's index is its pair's k-th bit, so the indices are 0,2,1,3 / 3,1,2,0."""
    centroids = np.zeros((2, 8), np.float16)
    centroids[1] = np.arange(8, dtype=np.float16)
    bw = np.array([-1.0, -0.25, 0.25, 1.0], np.float32)
    R = np.array([[0b00011011, 0b11100100]], np.uint8)
    got = O.residual_decompress(centroids, np.array([1]), R, bw, 2, normalize=False)
    idx = np.array([0, 2, 1, 3, 3, 1, 2, 0])
    np.testing.assert_array_equal(got[0], (np.arange(8) + bw[idx]).astype(np.float16))
    unit = O.residual_decompress(centroids, np.array([1]), R, bw, 2, normalize=True).astype(np.float32)
    np.testing.assert_allclose(np.linalg.norm(unit[0]), 1.0, rtol=2e-3)
    one = O.residual_decompress(np.zeros((1, 8), np.float16), np.array([0]), np.array([[0b10000000]], np.uint8),
                                np.array([0.0, 1.0], np.float32), 1, normalize=False)
    np.testing.assert_array_equal(one[0], np.array([1, 0, 0, 0, 0, 0, 0, 0], np.float16))


def test_exact_f64_scores_and_error_bound():
    """The float64 scorer matches the fp32 oracle to fp32 rounding; the derived error bound covers
    the fp32 oracle's own deviation on every (query, document); the ranking check accepts the fp32
    oracle's top-k and rejects a real inversion."""
    g = torch.Generator().manual_seed(3)
    Q = torch.nn.functional.normalize(torch.randn(4, 32, 128, generator=g), dim=-1).half()
    lengths = R.ragged_lengths(400, 0, 60, 5)
    off = R.offsets_from_lengths(lengths)
    D = torch.nn.functional.normalize(torch.randn(int(off[-1]), 128, generator=g), dim=-1).half()
    exact = O.maxsim_ragged_f64(Q, D, off)
    f32 = O.maxsim_ragged(Q, D, off)
    fin = np.isfinite(exact)
    assert np.array_equal(np.isinf(f32), ~fin) and (~fin).sum() == 4 * (lengths == 0).sum()
    qn = np.linalg.norm(Q.double().numpy(), axis=-1)
    bound = O.maxsim_error_bound(qn, O.doc_max_norm(D, off), exact, 128)
    assert np.all(np.abs(f32[fin] - exact[fin]) <= bound[fin])
    for r in range(4):
        _, ids = O.topk(f32[r], 50)
        O.check_ranking_within_bound(ids, f32[r], exact[r], bound[r], 50)
    # a top-k that swaps two documents far apart is rejected
    _, ids = O.topk(f32[0], 50)
    bad_scores = f32[0].copy()
    bad_scores[ids[0]], bad_scores[ids[40]] = bad_scores[ids[40]], bad_scores[ids[0]]
    _, bad_ids = O.topk(bad_scores, 50)
    with pytest.raises(AssertionError):
        O.check_ranking_within_bound(bad_ids, bad_scores, exact[0], bound[0], 50)


def _encoded_corpus(nbits: int, d: int = 128, T: int = 3000, n_cent: int = 64, seed: int = 0):
    import colbert_codec as CC
    rng = np.random.default_rng(seed)
    C = rng.standard_normal((n_cent, d)).astype(np.float32)
    C /= np.linalg.norm(C, axis=1, keepdims=True)
    # embeddings near the centroids, as after k-means: centroid + small noise, unit length
    X = C[rng.integers(0, n_cent, T)] + 0.05 * rng.standard_normal((T, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    codes = np.argmax(X @ C.T, axis=1)
    cut, w = CC.train_buckets(X - C[codes], nbits)
    codes, packed = CC.compress(X, C, cut, nbits)
    return X, C, codes, packed, cut, w


@pytest.mark.parametrize("nbits", [1, 2, 4])
def test_residual_layout_matches_colbert_encoder(nbits):
    """Pins the residual bit layout to a restatement of ColBERTv2's encoder (bucketize, bits spread
    least-significant first, np.packbits): decoding with weights w[b] = b returns exactly the bucket
    index the encoder chose for every dimension; with the trained weights the decoded vectors are
    within the codec's quantisation error of the encoder's inputs."""
    import colbert_codec as CC
    X, C, codes, packed, cut, w = _encoded_corpus(nbits)
    resid = X - C[codes]
    b = np.searchsorted(cut, resid, side="left")
    ident = np.arange(1 << nbits, dtype=np.float32)
    dec = O.residual_decompress(np.zeros_like(C, dtype=np.float16), codes, packed, ident, nbits, normalize=False)
    np.testing.assert_array_equal(dec.astype(np.int64), b)
    # quantisation error: inner buckets are bounded by their cutoffs, outer ones by the data range
    edges = np.concatenate([[resid.min()], cut, [resid.max()]])
    half = np.maximum(np.abs(w - edges[:-1]), np.abs(edges[1:] - w))  # per bucket
    raw = O.residual_decompress(C.astype(np.float16), codes, packed, w, nbits, normalize=False).astype(np.float32)
    tol = half[b] + 2e-3  # + fp16 rounding of the centroid and of the result
    assert np.all(np.abs(raw - X) <= tol)
    unit = O.residual_decompress(C.astype(np.float16), codes, packed, w, nbits, normalize=True).astype(np.float32)
    cos = (unit * X).sum(axis=1)
    assert cos.min() > 0.9


def test_ivf_oracle_lists_and_candidates():
    """The IVF restatement on a hand-made corpus: three documents over four centroids."""
    codes = np.array([0, 2, 2, 1, 3, 0, 9], dtype=np.int32)  # 9 is outside the table
    off = np.array([0, 3, 5, 7])  # doc0: {0, 2}, doc1: {1, 3}, doc2: {0}
    lists = O.ivf_lists(codes, off, 4)
    assert [list(x) for x in lists] == [[0, 2], [1], [0], [1]]
    cands = O.ivf_candidates(np.array([[2, 3], [1, 1], [7, 0]]), lists)
    assert [list(c) for c in cands] == [[0, 1], [1], [0, 2]]
