"""tms_dense_maxsim_noalloc: the dense MaxSim entry point for callers that cannot give the library
any device memory (for instance a serving engine that has reserved the whole GPU for its own
memory pool, or a host plug-in that must never call cudaMalloc). Its scratch lives in a static
4 MiB device array inside the library instead of a caller workspace.

The test calls it through the C ABI, twice in a row on different inputs, and checks each result
against the workspace entry point (tms_dense_maxsim, reached through maxsim_batched) within the
tolerance the other dense tests use. The file name sorts last so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process (the first call sets up the
array's device address itself).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import recipes as R

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-3


def _noalloc(lib, Qb, D, off, out_mode, out):
    from tilemaxsim_b200 import _lib
    Bq, Nq, d = Qb.shape
    return lib.tms_dense_maxsim_noalloc(
        ctypes.c_void_p(Qb.data_ptr()), _lib.DTYPE_CODE[D.dtype], Bq, Nq, d, ctypes.c_void_p(D.data_ptr()),
        D.shape[0], ctypes.c_void_p(off.data_ptr()), off.numel() - 1, 0, ctypes.c_void_p(out.data_ptr()),
        out_mode, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("n_queries,nq,seed", [(3, 32, 51), (2, 40, 52)])
def test_noalloc_matches_workspace_entry_point_twice(n_queries, nq, seed, cuda_device):
    from tilemaxsim_b200 import _lib, maxsim_batched
    lib = _lib.load()
    results = []
    for call in range(2):  # two calls in a row on different inputs: no state leaks between calls
        c = R.ragged_case(n_queries=n_queries, nq=nq, n_docs=250, seed=seed + 10 * call)
        Qb, D, off = c["Qb"].to(cuda_device), c["D"].to(cuda_device), c["offsets"].to(cuda_device)
        out = torch.full((n_queries, off.numel() - 1), float("nan"), dtype=torch.float32, device=cuda_device)
        rc = _noalloc(lib, Qb, D, off, _lib.TMS_OUT_SCORE, out)
        assert rc == _lib.TMS_OK, _lib.strerror(rc)
        want = maxsim_batched(Qb, D, off)
        got, exp = out.cpu().numpy(), want.cpu().numpy()
        inf = np.isinf(exp)
        assert inf.any()  # the recipe has empty documents (-inf)
        np.testing.assert_array_equal(got[inf], exp[inf])
        np.testing.assert_allclose(got[~inf], exp[~inf], rtol=RTOL, atol=ATOL)
        results.append(got)
    assert not np.array_equal(results[0], results[1])


def test_noalloc_token_max_matches_workspace_entry_point(cuda_device):
    """Per-query-token maxima (TMS_OUT_TOKEN_MAX) go through the same static scratch."""
    from tilemaxsim_b200 import _lib, maxsim_batched
    lib = _lib.load()
    for call in range(2):
        c = R.ragged_case(n_queries=2, nq=40, n_docs=120, seed=61 + call)
        Qb, D, off = c["Qb"].to(cuda_device), c["D"].to(cuda_device), c["offsets"].to(cuda_device)
        out = torch.full((2, off.numel() - 1, 40), float("nan"), dtype=torch.float32, device=cuda_device)
        rc = _noalloc(lib, Qb, D, off, _lib.TMS_OUT_TOKEN_MAX, out)
        assert rc == _lib.TMS_OK, _lib.strerror(rc)
        want = maxsim_batched(Qb, D, off, out_mode=_lib.TMS_OUT_TOKEN_MAX).cpu().numpy()
        got = out.cpu().numpy()
        inf = np.isinf(want)
        np.testing.assert_array_equal(got[inf], want[inf])
        np.testing.assert_allclose(got[~inf], want[~inf], rtol=RTOL, atol=ATOL)


def test_noalloc_limit_boundary(cuda_device):
    """The documented limit: 512 queries of 32 tokens at d = 128 fp16 pack into exactly 4 MiB and
    run; 513 do not fit and are rejected before any launch."""
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    D = R.normalized((64, 128), 5).to(cuda_device)
    off = torch.tensor([0, 30, 64], dtype=torch.int64, device=cuda_device)
    assert lib.tms_dense_workspace_size(_lib.TMS_F16, 512, 32, 128, 2, _lib.TMS_OUT_SCORE) == 4 << 20
    Qb = R.normalized((512, 32, 128), 6).to(cuda_device)
    out = torch.zeros(512, 2, dtype=torch.float32, device=cuda_device)
    assert _noalloc(lib, Qb, D, off, _lib.TMS_OUT_SCORE, out) == _lib.TMS_OK
    from tilemaxsim_b200 import maxsim_batched
    np.testing.assert_allclose(out.cpu().numpy(), maxsim_batched(Qb, D, off).cpu().numpy(), rtol=RTOL, atol=ATOL)
    Qb = R.normalized((513, 32, 128), 6).to(cuda_device)
    out = torch.zeros(513, 2, dtype=torch.float32, device=cuda_device)
    assert _noalloc(lib, Qb, D, off, _lib.TMS_OUT_SCORE, out) == _lib.TMS_ERR_TOO_LARGE


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    # 2048 queries of 32 tokens at d = 128 fp16 pack into 512 query tiles = 16 MiB > 4 MiB
    Qb = torch.zeros(2048, 32, 128, dtype=torch.float16, device=cuda_device)
    D = torch.zeros(16, 128, dtype=torch.float16, device=cuda_device)
    off = torch.tensor([0, 16], dtype=torch.int64, device=cuda_device)
    out = torch.zeros(2048, 1, dtype=torch.float32, device=cuda_device)
    assert _noalloc(lib, Qb, D, off, _lib.TMS_OUT_SCORE, out) == _lib.TMS_ERR_TOO_LARGE
