"""Top-k (tms_topk) and PQ-ADC (tms_pq_table, tms_pq_maxsim) kernels against the oracle and the
reference's golden outputs. Top-k ids must be identical (score descending, id ascending); PQ scores
within 1e-3 relative of the reference's ADC path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import load_golden
from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def test_topk_ties_golden(cuda_device):
    from tilemaxsim_b200 import topk
    _, g = load_golden("topk_ties")
    s = R.topk_case()["scores"].to(cuda_device)
    for k in (1, 10, 100, 1000):
        vals, ids = topk(s, k)
        np.testing.assert_array_equal(ids.cpu().numpy(), g["order"][:, :k])
        want, _ = O.topk(s.cpu(), k)
        np.testing.assert_array_equal(vals.cpu().numpy(), want)


@pytest.mark.parametrize("rows,n,k", [(3, 100_000, 1000), (64, 100_000, 1000), (2, 20_000, 10),
                                      (1, 1_250_003, 100), (5, 16_385, 2048), (4, 7, 7),
                                      (1, 400_000, 10), (1, 16_400, 1000), (300, 40_000, 5),
                                      (1, 10_000_000, 1000)])
def test_topk_random(rows, n, k, cuda_device):
    from tilemaxsim_b200 import topk
    g = torch.Generator().manual_seed(rows * n + k)
    s = torch.randn(rows, n, generator=g)
    s[:, ::97] = s[:, :1]  # exact ties across the row
    vals, ids = topk(s.to(cuda_device), k, id_base=5)
    wv, wi = O.topk(s, k)
    np.testing.assert_array_equal(ids.cpu().numpy(), wi + 5)
    np.testing.assert_array_equal(vals.cpu().numpy(), wv)


def test_topk_merge_with_ids(cuda_device):
    from tilemaxsim_b200 import topk
    g = torch.Generator().manual_seed(1)
    s = torch.randn(6, 8 * 100, generator=g).round(decimals=1)
    ids = torch.randperm(10_000, generator=g)[: 6 * 800].reshape(6, 800)
    vals, out = topk(s.to(cuda_device), 100, ids=ids.to(cuda_device))
    wv, wi = O.topk(s, 100, ids=ids.numpy())
    np.testing.assert_array_equal(out.cpu().numpy(), wi)
    np.testing.assert_array_equal(vals.cpu().numpy(), wv)


PATHS = ["tensor", "exact"]  # tensor-core decode path (default) / fp32 table-lookup path
# tensor path (exact=False): codebook rounded to fp16 -> |error| <= 1e-3*|score| + 5e-3
# exact path (the default): the reference's fp32 table arithmetic, summed in another order
TOL = {"tensor": (1e-3, 5e-3), "exact": (1e-5, 1e-4)}


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("name,cb_dtype", [("pq_f32", torch.float32), ("pq_f16", torch.float16)])
def test_pq_golden(name, cb_dtype, path, cuda_device):
    rtol, atol = TOL[path]
    from tilemaxsim_b200 import TileMaxSimPQ
    _, g = load_golden(name)
    c = R.pq_case(cb_dtype)
    pq = TileMaxSimPQ(c["codebook"].to(cuda_device), exact=(path == "exact"))
    Q, codes = c["Q"].to(cuda_device), c["codes"].to(cuda_device)
    got = pq.score_batch(Q, codes).cpu().numpy()
    np.testing.assert_allclose(got, g["adc"], rtol=rtol, atol=atol)
    np.testing.assert_allclose(got, g["decompress"], rtol=rtol, atol=atol)
    s1 = pq.score_single(Q, codes[3])
    assert s1.dim() == 0
    np.testing.assert_allclose(s1.item(), g["adc"][3], rtol=rtol, atol=atol)
    T = pq.build_distance_table(Q).cpu().numpy()
    np.testing.assert_allclose(T, O.pq_table(c["Q"], c["codebook"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("M,K,dsub,nq", [(16, 256, 8, 32), (8, 256, 16, 32), (32, 256, 4, 32),
                                         (16, 100, 8, 5), (12, 256, 8, 40), (16, 256, 8, 1),
                                         (32, 256, 8, 64)])
def test_pq_ragged_multiquery(M, K, dsub, nq, path, cuda_device):
    rtol, atol = TOL[path]
    from tilemaxsim_b200 import TileMaxSimPQ
    lengths = R.ragged_lengths(400, 0, 200, seed=M + K)
    off = R.offsets_from_lengths(lengths)
    cb = R.randn((M, K, dsub), 3, torch.float32)
    Qb = R.normalized((5, nq, M * dsub), 4)
    codes = torch.randint(0, K, (int(off[-1]), M), generator=R.gen(5), dtype=torch.uint8)
    pq = TileMaxSimPQ(cb.to(cuda_device), exact=(path == "exact"))
    got = pq.score_queries(Qb.to(cuda_device), codes.to(cuda_device), torch.from_numpy(off).to(cuda_device))
    want = O.pq_maxsim_adc_ragged(Qb, cb, codes, off)
    got = got.cpu().numpy()
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=rtol, atol=atol)


@pytest.mark.parametrize("nqry,M,K,dsub,nq,lengths", [
    (1, 16, 256, 8, 32, "ragged"), (2, 16, 256, 8, 32, "ragged"), (4, 16, 256, 8, 32, "ragged"),
    (3, 16, 256, 8, 20, "ragged"), (1, 16, 256, 8, 64, "ragged"), (2, 32, 256, 8, 40, "ragged"),
    (1, 32, 256, 8, 32, "ragged"), (1, 8, 256, 8, 32, "ragged"), (2, 8, 256, 8, 30, "tiny"),
    (1, 8, 256, 16, 32, "ragged"), (1, 16, 100, 8, 5, "ragged"), (1, 16, 256, 8, 32, "tiny"),
    (2, 16, 256, 8, 32, "one_long"), (4, 16, 256, 8, 32, "tiny"), (3, 16, 256, 8, 32, "one_long"),
    (1, 16, 256, 8, 128, "ragged"), (5, 16, 256, 8, 32, "ragged")])
def test_pq_small_batch_token_rows(nqry, M, K, dsub, nq, lengths, cuda_device):
    """Small query batches (1-4 chunks of 32 query rows) take the token-rows tensor kernel: decoded
    tokens in TMEM as the MMA's A operand, one document stream per TMEM lane, per-lane running
    maxima summed when the lane's document ends (5 queries check the decoder-warp kernel). Ragged
    corpora with empty documents, documents of 1-3 tokens (several documents per lane), and one
    document longer than a CTA's share of the corpus."""
    from tilemaxsim_b200 import TileMaxSimPQ
    if lengths == "ragged":
        lens = R.ragged_lengths(700, 0, 300, seed=nqry + M)
    elif lengths == "tiny":
        lens = R.ragged_lengths(3000, 0, 3, seed=7)
    else:
        lens = R.ragged_lengths(300, 0, 40, seed=8)
        lens[100] = 20_000
    off = R.offsets_from_lengths(lens)
    cb = R.randn((M, K, dsub), 3, torch.float32)
    Qb = R.normalized((nqry, nq, M * dsub), 4)
    codes = torch.randint(0, K, (int(off[-1]), M), generator=R.gen(5), dtype=torch.uint8)
    pq = TileMaxSimPQ(cb.to(cuda_device), exact=False)
    got = pq.score_queries(Qb.to(cuda_device), codes.to(cuda_device),
                           torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.pq_maxsim_adc_ragged(Qb, cb, codes, off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=5e-3)


@pytest.mark.parametrize("nqry", [1, 2, 5])
def test_pq_offsets_not_starting_at_zero_and_empty_corpus(nqry, cuda_device):
    """A corpus given as a window of a larger code array (offsets start past 0), and a corpus of
    empty documents only (every score -inf), on every PQ kernel the query count selects."""
    from tilemaxsim_b200 import TileMaxSimPQ
    cb = R.randn((16, 256, 8), 3, torch.float32)
    Qb = R.normalized((nqry, 32, 128), 4)
    lens = R.ragged_lengths(300, 0, 150, seed=11)
    off = R.offsets_from_lengths(lens) + 777
    codes = torch.randint(0, 256, (int(off[-1]) + 50, 16), generator=R.gen(5), dtype=torch.uint8)
    pq = TileMaxSimPQ(cb.to(cuda_device), exact=False)
    got = pq.score_queries(Qb.to(cuda_device), codes.to(cuda_device),
                           torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.pq_maxsim_adc_ragged(Qb, cb, codes, off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=5e-3)
    empty = torch.full((41,), 5, dtype=torch.int64)
    s = pq.score_queries(Qb.to(cuda_device), codes.to(cuda_device), empty.to(cuda_device)).cpu()
    assert s.shape == (nqry, 40) and torch.all(torch.isneginf(s))


@pytest.mark.parametrize("qdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nqry", [1, 5])
def test_pq_fast_mode_rounds_wider_queries_to_fp16(qdtype, nqry, cuda_device):
    """Fast mode takes fp32 / bf16 queries on the tensor-core path (rounded to fp16) and stays
    within the fast-mode tolerance of the fp32 table-lookup oracle."""
    from tilemaxsim_b200 import TileMaxSimPQ
    lens = R.ragged_lengths(300, 0, 150, seed=21)
    off = R.offsets_from_lengths(lens)
    cb = R.randn((16, 256, 8), 3, torch.float32)
    Qb = R.normalized((nqry, 32, 128), 4).float().to(qdtype)
    codes = torch.randint(0, 256, (int(off[-1]), 16), generator=R.gen(5), dtype=torch.uint8)
    got = TileMaxSimPQ(cb.to(cuda_device), exact=False).score_queries(
        Qb.to(cuda_device), codes.to(cuda_device), torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.pq_maxsim_adc_ragged(Qb.float(), cb, codes, off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-3, atol=5e-3)


def test_pq_single_query_full_size_property(cuda_device):
    """Single query over a 400k-document slice of BASELINE config 4 (51.2M code rows) on the
    token-rows kernel agrees with the exact table-lookup path on every score."""
    from tilemaxsim_b200 import TileMaxSimPQ
    g = torch.Generator(device=cuda_device).manual_seed(6)
    n, nd = 400_000, 128
    codes = torch.randint(0, 256, (n * nd, 16), generator=g, device=cuda_device, dtype=torch.uint8)
    off = torch.arange(n + 1, device=cuda_device, dtype=torch.int64) * nd
    cb = torch.randn(16, 256, 8, generator=g, device=cuda_device)
    Q = torch.nn.functional.normalize(torch.randn(1, 32, 128, generator=g, device=cuda_device), dim=-1).half()
    fast = TileMaxSimPQ(cb, exact=False).score_queries(Q, codes, off)
    exact = TileMaxSimPQ(cb, exact=True).score_queries(Q, codes, off)
    torch.testing.assert_close(fast, exact, rtol=1e-3, atol=5e-3)


def test_pq_tensor_path_full_size_property(cuda_device):
    """BASELINE config 4 shape on a 200k-document slice (25.6M code rows): the tensor-core path
    agrees with the exact table-lookup path on every score (1e-3 relative + 5e-3)."""
    from tilemaxsim_b200 import TileMaxSimPQ
    g = torch.Generator(device=cuda_device).manual_seed(4)
    n, nd = 200_000, 128
    codes = torch.randint(0, 256, (n * nd, 16), generator=g, device=cuda_device, dtype=torch.uint8)
    off = torch.arange(n + 1, device=cuda_device, dtype=torch.int64) * nd
    cb = torch.randn(16, 256, 8, generator=g, device=cuda_device)
    Qb = torch.nn.functional.normalize(torch.randn(16, 32, 128, generator=g, device=cuda_device), dim=-1).half()
    fast = TileMaxSimPQ(cb, exact=False).score_queries(Qb, codes, off)
    exact = TileMaxSimPQ(cb, exact=True).score_queries(Qb, codes, off)
    torch.testing.assert_close(fast, exact, rtol=1e-3, atol=5e-3)


def test_pq_exact_c4_shape_vs_oracle(cuda_device):
    """BASELINE config 4 shape (16 queries x 32 tokens, M=16, K=256, dsub=8, 128-token documents,
    fp32 codebook) on a 1000-document slice: the default (exact) path agrees with the reference's
    ADC arithmetic within 1e-5 relative."""
    from tilemaxsim_b200 import TileMaxSimPQ
    g = torch.Generator().manual_seed(12)
    n, nd = 1000, 128
    codes = torch.randint(0, 256, (n * nd, 16), generator=g, dtype=torch.uint8)
    off = np.arange(n + 1, dtype=np.int64) * nd
    cb = torch.randn(16, 256, 8, generator=g)
    Qb = torch.nn.functional.normalize(torch.randn(16, 32, 128, generator=g), dim=-1).half()
    got = TileMaxSimPQ(cb.to(cuda_device)).score_queries(
        Qb.to(cuda_device), codes.to(cuda_device), torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.pq_maxsim_adc_ragged(Qb, cb, codes, off)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-4)


def test_pq_exact_c4_full_size_document_independence(cuda_device):
    """BASELINE config 4 at full size (16 queries x 1M documents x 128 codes): the full corpus
    scored at once equals sampled documents scored alone, bit for bit, and the samples agree with
    the reference's ADC arithmetic within 1e-5 relative."""
    from tilemaxsim_b200 import TileMaxSimPQ
    g = torch.Generator(device=cuda_device).manual_seed(4)
    n, nd = 1_000_000, 128
    codes = torch.randint(0, 256, (n * nd, 16), generator=g, device=cuda_device, dtype=torch.uint8)
    off = torch.arange(n + 1, device=cuda_device, dtype=torch.int64) * nd
    cb = torch.randn(16, 256, 8, generator=g, device=cuda_device)
    Qb = torch.nn.functional.normalize(torch.randn(16, 32, 128, generator=g, device=cuda_device), dim=-1).half()
    pq = TileMaxSimPQ(cb)
    full = pq.score_queries(Qb, codes, off)
    pick = torch.from_numpy(np.sort(np.random.default_rng(3).choice(n, 200, replace=False))).to(cuda_device)
    sub_codes = codes.view(n, nd, 16)[pick].reshape(-1, 16)
    sub_off = torch.arange(201, device=cuda_device, dtype=torch.int64) * nd
    sub = pq.score_queries(Qb, sub_codes, sub_off)
    assert torch.equal(full[:, pick], sub)
    want = O.pq_maxsim_adc_ragged(Qb.cpu(), cb.cpu(), sub_codes.cpu(), sub_off.cpu().numpy())
    np.testing.assert_allclose(sub.cpu().numpy(), want, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("nqry,nq,lengths", [(1, 32, "c4"), (2, 32, "c4"), (1, 64, "ragged"),
                                              (2, 20, "ragged"), (1, 5, "tiny"), (3, 32, "c4"),
                                              (4, 32, "ragged"), (7, 16, "ragged"), (5, 40, "c4"),
                                              (1, 128, "ragged"), (3, 100, "tiny"), (6, 8, "ragged")])
def test_pq_precise_tensor_path_vs_oracle(nqry, nq, lengths, cuda_device):
    """fp16 queries at the default precision run on the tensor cores with the codebook split into
    fp16 hi + lo, in passes of up to four 32-row query chunks (three chunks on the four-chunk
    kernel, partial last passes, 128-row queries); batches of <= 8-token queries needing several
    passes take the fp32 table lookups. Scores within 1e-5 relative of the reference's fp32 ADC
    arithmetic either way."""
    from tilemaxsim_b200 import TileMaxSimPQ, _lib
    if lengths == "c4":
        off = np.arange(2001, dtype=np.int64) * 128
    elif lengths == "ragged":
        off = R.offsets_from_lengths(R.ragged_lengths(900, 0, 300, seed=nq))
    else:
        off = R.offsets_from_lengths(R.ragged_lengths(3000, 0, 3, seed=7))
    cb = R.randn((16, 256, 8), 3, torch.float32)
    Qb = R.normalized((nqry, nq, 128), 4)
    codes = torch.randint(0, 256, (int(off[-1]), 16), generator=R.gen(5), dtype=torch.uint8)
    pq = TileMaxSimPQ(cb.to(cuda_device))
    assert pq._mode() == _lib.TMS_PQ_PRECISE
    got = pq.score_queries(Qb.to(cuda_device), codes.to(cuda_device),
                           torch.from_numpy(off).to(cuda_device)).cpu().numpy()
    want = O.pq_maxsim_adc_ragged(Qb, cb, codes, off)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("world,rows,k", [(3, 5, 100), (8, 64, 1000), (2, 3, 7)])
def test_packed_merge_equals_topk_of_candidates(world, rows, k, cuda_device):
    """The shard merge's pack and merge kernels, with the all-gather emulated on one GPU (ranks'
    packed rows concatenated rank-major): equal to the oracle's top-k of all ranks' candidates,
    ties (many) and NaN padding included."""
    import ctypes
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    g = torch.Generator().manual_seed(world * rows + k)
    vals = (torch.randint(0, 50, (world, rows, k), generator=g).float() / 4.0)
    vals[:, :, -2:] = float("nan")  # padded lists
    ids = torch.randint(0, 10**12, (world, rows, k), generator=g)
    packed = torch.empty(world, rows, 2 * k, dtype=torch.int64, device=cuda_device)
    vd, idd = vals.to(cuda_device), ids.to(cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for r in range(world):
        assert lib.tms_topk_pack(ctypes.c_void_p(vd[r].data_ptr()), ctypes.c_void_p(idd[r].data_ptr()), rows, k,
                                 ctypes.c_void_p(packed[r].data_ptr()), stream) == 0
    out_v = torch.empty(rows, k, device=cuda_device)
    out_i = torch.empty(rows, k, dtype=torch.int64, device=cuda_device)
    assert lib.tms_topk_merge_packed(ctypes.c_void_p(packed.data_ptr()), world, rows, k,
                                     ctypes.c_void_p(out_v.data_ptr()), ctypes.c_void_p(out_i.data_ptr()),
                                     stream) == 0
    cand_v = vals.permute(1, 0, 2).reshape(rows, world * k)
    cand_i = ids.permute(1, 0, 2).reshape(rows, world * k)
    wv, wi = O.topk(cand_v.numpy(), k, ids=cand_i.numpy())
    np.testing.assert_array_equal(out_i.cpu().numpy(), wi)
    np.testing.assert_array_equal(out_v.cpu().numpy(), wv)
