"""Dense MaxSim kernel (tms_dense_maxsim, tcgen05 + TMA) against the reference's outputs and the
oracle. Tolerance: |gpu - ref| <= 1e-3 * |ref| + 1e-3 for fp16/bf16 inputs (fp32 accumulation; the
absolute term covers scores near zero), 2e-3 relative for fp32 inputs (TF32 multiply, as the
reference's tl.dot)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from conftest import load_golden
from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-3


def close(got, want, rtol=RTOL, atol=ATOL):
    got = got.detach().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (got.shape, want.shape)
    inf = np.isinf(want)
    np.testing.assert_array_equal(got[inf], want[inf])
    np.testing.assert_allclose(got[~inf], want[~inf], rtol=rtol, atol=atol)


@pytest.mark.parametrize("i", range(len(R.EXP10_CONFIGS)))
def test_exp10_all_entry_points(i, cuda_device):
    from tilemaxsim_b200 import (flash_maxsim_batch, flash_maxsim_token_max, flash_maxsim_v2,
                                 flash_maxsim_v2_multiquery)
    _, g = load_golden(f"exp10_{i}")
    c = R.exp10_case(i)
    Q, D = c["Q"].to(cuda_device), c["D"].to(cuda_device)
    for fn in (flash_maxsim_v2_multiquery, flash_maxsim_v2, flash_maxsim_batch):
        close(fn(Q, D), g["scores"])
    close(flash_maxsim_token_max(Q, D), g["token_max"])


def test_v1_single_and_selfcheck(cuda_device):
    from tilemaxsim_b200 import flash_maxsim_single
    _, g = load_golden("v1_selfcheck")
    c = R.v1_selfcheck_case()
    Q, D = c["Q"].to(cuda_device), c["D"].to(cuda_device)
    s = flash_maxsim_single(Q, D[0])
    assert s.dim() == 0 and s.dtype == torch.float32
    close(s.reshape(1), g["naive"][:1])
    empty = flash_maxsim_single(Q, D[0, :0])
    assert torch.isneginf(empty).item()


RAGGED = {"ragged_f16": {}, "ragged_bf16": {"dtype": torch.bfloat16, "seed": 11},
          "ragged_nq20": {"nq": 20, "n_queries": 2, "seed": 13},
          "ragged_nq40": {"nq": 40, "n_queries": 2, "n_docs": 120, "seed": 17}}


@pytest.mark.parametrize("name", list(RAGGED))
def test_ragged_batched(name, cuda_device):
    from tilemaxsim_b200 import _lib, maxsim_batched
    _, g = load_golden(name)
    c = R.ragged_case(**RAGGED[name])
    Qb, D, off = c["Qb"].to(cuda_device), c["D"].to(cuda_device), c["offsets"].to(cuda_device)
    close(maxsim_batched(Qb, D, off), g["scores"])
    close(maxsim_batched(Qb, D, off, out_mode=_lib.TMS_OUT_TOKEN_MAX), g["token_max"])


def test_multi_doc_offsets_not_starting_at_zero(cuda_device):
    from tilemaxsim_b200 import flash_maxsim_multi_doc
    c = R.ragged_case(n_queries=1, n_docs=50, seed=21)
    off = c["offsets"].clone()
    off = off[10:]  # documents 10..49 only; offsets start mid-matrix
    want = O.maxsim_ragged(c["Qb"][0], c["D"], off.numpy())
    got = flash_maxsim_multi_doc(c["Qb"][0].to(cuda_device), c["D"].to(cuda_device), off.to(cuda_device))
    close(got, want)


@pytest.mark.parametrize("bq,nq,n_docs,lo,hi,d", [
    (64, 32, 3000, 64, 300, 128),   # the multi-query rerank shape, smaller corpus (16 query tiles)
    (5, 32, 2000, 1, 40, 128),      # many short documents per tile
    (7, 17, 700, 0, 600, 128),      # documents longer than two tiles, odd Nq
    (3, 100, 300, 10, 200, 128),    # Nq > 96: four 32-row chunks per query
    (16, 32, 400, 200, 300, 256),   # d-sweep shapes (K loop)
    (4, 32, 200, 200, 300, 768),
    (2, 32, 300, 5, 120, 64),
    (1, 8, 500, 1, 50, 96),         # d not a multiple of 64 (zero-filled K tail)
    (1, 1, 100, 1, 9, 128),         # Nq = 1
])
def test_ragged_random_vs_oracle(bq, nq, n_docs, lo, hi, d, cuda_device):
    from tilemaxsim_b200 import maxsim_batched
    lengths = R.ragged_lengths(n_docs, lo, hi, seed=bq * 1000 + nq)
    off = R.offsets_from_lengths(lengths)
    Qb = R.normalized((bq, nq, d), 5)
    D = R.normalized((int(off[-1]), d), 6)
    got = maxsim_batched(Qb.to(cuda_device), D.to(cuda_device), torch.from_numpy(off).to(cuda_device))
    close(got, O.maxsim_ragged(Qb, D, off))


def test_fp32_inputs_tf32(cuda_device):
    from tilemaxsim_b200 import flash_maxsim_v2_multiquery
    Q = R.normalized((32, 128), 1, torch.float32)
    D = R.normalized((40, 130, 128), 2, torch.float32)
    close(flash_maxsim_v2_multiquery(Q.to(cuda_device), D.to(cuda_device)), O.maxsim_padded(Q, D),
          rtol=2e-3, atol=2e-3)


def test_bf16_padded(cuda_device):
    from tilemaxsim_b200 import flash_maxsim_v2_multiquery
    Q = R.normalized((32, 128), 3, torch.bfloat16)
    D = R.normalized((64, 180, 128), 4, torch.bfloat16)
    close(flash_maxsim_v2_multiquery(Q.to(cuda_device), D.to(cuda_device)), O.maxsim_padded(Q, D))


def test_zero_padding_participates(cuda_device):
    """Padded API: zero rows are real rows (dot = 0), so a doc whose real tokens all score < 0 gets
    max 0 from its padding, exactly as the reference (src/flash_maxsim_v2.py:120)."""
    from tilemaxsim_b200 import flash_maxsim_v2_multiquery
    Q = torch.ones(4, 64, dtype=torch.float16)
    D = torch.zeros(3, 10, 64, dtype=torch.float16)
    D[:, :5] = -1.0
    got = flash_maxsim_v2_multiquery(Q.to(cuda_device), D.to(cuda_device))
    close(got, O.maxsim_padded(Q, D))
    assert torch.all(got == 0)


def test_edge_cases(cuda_device):
    from tilemaxsim_b200 import maxsim_batched
    Qb = R.normalized((2, 32, 128), 8).to(cuda_device)
    # all documents empty
    off = torch.zeros(6, dtype=torch.int64, device=cuda_device)
    D = torch.zeros(0, 128, dtype=torch.float16, device=cuda_device)
    assert torch.all(torch.isneginf(maxsim_batched(Qb, D, off)))
    # one token, one document
    D1 = R.normalized((1, 128), 9).to(cuda_device)
    off1 = torch.tensor([0, 1], dtype=torch.int64, device=cuda_device)
    close(maxsim_batched(Qb, D1, off1), O.maxsim_ragged(Qb.cpu(), D1.cpu(), off1.cpu().numpy()))
    # zero documents
    off0 = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    assert maxsim_batched(Qb, D1, off0).shape == (2, 0)


def test_deterministic(cuda_device):
    from tilemaxsim_b200 import maxsim_batched
    c = R.ragged_case(n_queries=9, n_docs=800, seed=31)
    args = [c["Qb"].to(cuda_device), c["D"].to(cuda_device), c["offsets"].to(cuda_device)]
    a = maxsim_batched(*args)
    b = maxsim_batched(*args)
    assert torch.equal(a, b)


def test_full_size_rerank_consistency(cuda_device):
    """BASELINE config 2 at full size (64 queries x 100k ragged docs, Nd ~ U[64, 300]): scoring the
    whole corpus equals scoring sampled documents alone (document independence), and the sampled
    documents match the oracle."""
    from tilemaxsim_b200 import maxsim_batched
    lengths = R.ragged_lengths(100_000, 64, 300, seed=42)
    off = R.offsets_from_lengths(lengths)
    g = torch.Generator(device=cuda_device).manual_seed(42)
    D = torch.randn(int(off[-1]), 128, device=cuda_device, generator=g)
    D = torch.nn.functional.normalize(D, dim=-1).half()
    Qb = torch.nn.functional.normalize(torch.randn(64, 32, 128, device=cuda_device, generator=g), dim=-1).half()
    full = maxsim_batched(Qb, D, torch.from_numpy(off).to(cuda_device))
    pick = np.sort(np.random.default_rng(0).choice(100_000, 300, replace=False))
    sub_tok = np.concatenate([np.arange(off[i], off[i + 1]) for i in pick])
    sub_off = R.offsets_from_lengths(lengths[pick])
    Dsub = D[torch.from_numpy(sub_tok).to(cuda_device)]
    sub = maxsim_batched(Qb, Dsub, torch.from_numpy(sub_off).to(cuda_device))
    assert torch.equal(full[:, torch.from_numpy(pick).to(cuda_device)], sub)
    close(sub, O.maxsim_ragged(Qb.cpu(), Dsub.cpu(), sub_off))


@pytest.mark.parametrize("case", ["single_query", "multi_query", "pq_tensor", "pq_token_rows", "pq_precise",
                                  "pq_precise4", "residual_rows"])
def test_bounded_wait_reports_timeout(case, cuda_device):
    """Fault knob: the producer issues no load, so every consumer wait runs out after the (short)
    limit; the kernel returns, the host reads TMS_ERR_TIMEOUT, and the context stays usable."""
    from tilemaxsim_b200 import TileMaxSimPQ, _lib, maxsim_batched
    lib = _lib.load()
    if case == "residual_rows":
        from tilemaxsim_b200 import ResidualMaxSim
        cent = torch.nn.functional.normalize(torch.randn(64, 128, generator=R.gen(4)), dim=-1).half()
        codes = torch.randint(0, 64, (40 * 64,), generator=R.gen(4), dtype=torch.int32)
        res = torch.randint(0, 256, (40 * 64, 32), generator=R.gen(4), dtype=torch.uint8)
        bw = torch.tensor([-0.05, -0.01, 0.01, 0.05])
        off = (torch.arange(41, dtype=torch.int64) * 64)
        scorer = ResidualMaxSim(cent.to(cuda_device), bw.to(cuda_device), 2)
        Qb = R.normalized((1, 32, 128), 5)
        args = [Qb.to(cuda_device), codes.to(cuda_device), res.to(cuda_device), off.to(cuda_device)]
        run = lambda: scorer.score_queries(*args)  # noqa: E731
        want = O.maxsim_ragged(Qb, torch.from_numpy(O.residual_decompress(cent, codes, res, bw, 2)), off.numpy())
        tol = (1e-3, 1e-3)
    elif case.startswith("pq"):
        cb = R.randn((16, 256, 8), 3, torch.float32).to(cuda_device)
        pq = TileMaxSimPQ(cb, exact=case.startswith("pq_precise"))
        codes = torch.randint(0, 256, (40 * 64, 16), generator=R.gen(4), dtype=torch.uint8).to(cuda_device)
        off = (torch.arange(41, dtype=torch.int64) * 64).to(cuda_device)
        # 5 queries: decoder-warp variant of the dense kernel; 1 query: token-rows kernel; 4 queries
        # at the default precision: the four-chunk token-rows kernel (MMAs issued by a decoder warp)
        nqry = {"pq_tensor": 5, "pq_precise4": 4}.get(case, 1)
        Qb = R.normalized((nqry, 32, 128), 5).to(cuda_device)
        run = lambda: pq.score_queries(Qb, codes, off)  # noqa: E731
        want = O.pq_maxsim_adc_ragged(Qb.cpu(), cb.cpu(), codes.cpu(), off.cpu().numpy())
        tol = (1e-3, 5e-3)
    else:
        c = R.ragged_case(n_queries=1 if case == "single_query" else 9, n_docs=20, seed=3)
        args = [c["Qb"].to(cuda_device), c["D"].to(cuda_device), c["offsets"].to(cuda_device)]
        run = lambda: maxsim_batched(*args)  # noqa: E731
        want = O.maxsim_ragged(c["Qb"], c["D"], c["offsets"].numpy())
        tol = (RTOL, ATOL)
    assert _lib.last_device_error(cuda_device)[0] == _lib.TMS_OK
    lib.tms_set_debug(50_000_000, 1)  # 50 ms limit, producer / decoders silent
    try:
        run()
        rc, word = _lib.last_device_error(cuda_device)
    finally:
        lib.tms_set_debug(2_000_000_000, 0)
    assert rc == _lib.TMS_ERR_TIMEOUT and word & 0x80000000
    # the context still works and the error word was cleared
    close(run(), want, *tol)
    assert _lib.last_device_error(cuda_device)[0] == _lib.TMS_OK


def test_validate_offsets(cuda_device, monkeypatch):
    """tms_validate_offsets flags negative, decreasing and out-of-range offsets through the device
    error word (then cleared); TMS_CHECK_OFFSETS=1 runs it before ragged scoring, so malformed
    offsets raise on the host before any scoring kernel is launched."""
    from tilemaxsim_b200 import _lib, maxsim_batched, validate_offsets
    t = lambda x: torch.tensor(x, dtype=torch.int64, device=cuda_device)  # noqa: E731
    validate_offsets(t([0, 3, 3, 10]), 10)
    validate_offsets(t([4, 4]), 10)
    for bad, idx in (([0, 5, 3, 10], 2), ([0, 3, 12], 2), ([-1, 3], 0)):
        with pytest.raises(ValueError, match=rf"doc_offsets\[{idx}\]"):
            validate_offsets(t(bad), 10)
        assert _lib.last_device_error(cuda_device)[0] == _lib.TMS_OK  # read and cleared
    Q = R.normalized((2, 32, 128), 5).to(cuda_device)
    D = R.normalized((10, 128), 6).to(cuda_device)
    monkeypatch.setenv("TMS_CHECK_OFFSETS", "1")
    with pytest.raises(ValueError):
        maxsim_batched(Q, D, t([0, 5, 3, 10]))
    assert maxsim_batched(Q, D, t([0, 3, 3, 10])).shape == (2, 3)
