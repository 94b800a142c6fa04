"""Scoring + top-k in bounded memory (tms_dense_maxsim_topk): documents are scored a chunk at a
time and each chunk's top-k is merged into a running list. The result must equal the top-k of the
full score matrix exactly (values and ids), whatever the chunk size, including chunks smaller
than k (their lists are padded) and empty documents (-inf)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import recipes as R

pytestmark = pytest.mark.gpu


def _corpus(n_docs, seed, dev):
    lengths = R.ragged_lengths(n_docs, 0, 120, seed)
    off = R.offsets_from_lengths(lengths)
    g = torch.Generator().manual_seed(seed)
    D = torch.nn.functional.normalize(torch.randn(int(off[-1]), 128, generator=g), dim=-1).half()
    return D.to(dev), torch.from_numpy(off).to(dev)


@pytest.mark.parametrize("bq,k,chunk", [(1, 10, None), (1, 10, 7), (3, 100, 333), (3, 100, 57),
                                        (64, 1, 50), (5, 40, 1000), (2, 300, 900)])
def test_streamed_topk_equals_full_matrix_topk(bq, k, chunk, cuda_device):
    from tilemaxsim_b200 import maxsim_batched, maxsim_topk, topk
    D, off = _corpus(2000, 3, cuda_device)
    lengths = off[1:] - off[:-1]
    assert int((lengths == 0).sum()) > 0  # the corpus holds empty documents
    Qb = R.normalized((bq, 32, 128), 5).to(cuda_device)
    want_v, want_i = topk(maxsim_batched(Qb, D, off), k, id_base=1000)
    got_v, got_i = maxsim_topk(Qb, D, off, k, id_base=1000, chunk_docs=chunk)
    torch.testing.assert_close(got_v, want_v, rtol=0, atol=0, equal_nan=True)
    assert torch.equal(got_i, want_i)


@pytest.mark.parametrize("nq,dtype", [(40, torch.float16), (32, torch.bfloat16), (100, torch.bfloat16)])
def test_streamed_topk_long_queries_and_bf16(nq, dtype, cuda_device):
    """Queries longer than 32 tokens (per-chunk partial sums inside every document chunk) and
    bf16 inputs, chunked, against the full-matrix top-k."""
    from tilemaxsim_b200 import maxsim_batched, maxsim_topk, topk
    D, off = _corpus(1500, 7, cuda_device)
    D = D.to(dtype)
    Qb = R.normalized((3, nq, 128), 8).to(dtype).to(cuda_device)
    want_v, want_i = topk(maxsim_batched(Qb, D, off), 64)
    got_v, got_i = maxsim_topk(Qb, D, off, 64, chunk_docs=211)
    torch.testing.assert_close(got_v, want_v, rtol=0, atol=0)
    assert torch.equal(got_i, want_i)


def test_streamed_topk_uniform_documents_c_abi(cuda_device):
    """The uniform-length layout (no offsets array) through the C ABI, chunked."""
    from tilemaxsim_b200 import _lib, maxsim_padded, topk
    lib = _lib.load()
    B, Nd, k = 700, 40, 25
    D = torch.nn.functional.normalize(torch.randn(B, Nd, 128, generator=R.gen(6)), dim=-1).half().to(cuda_device)
    Qb = R.normalized((4, 32, 128), 7).to(cuda_device)
    want_v, want_i = topk(maxsim_padded(Qb, D), k)
    vals = torch.empty((4, k), dtype=torch.float32, device=cuda_device)
    ids = torch.empty((4, k), dtype=torch.int64, device=cuda_device)
    ws_bytes = lib.tms_dense_topk_workspace_size(_lib.TMS_F16, 4, 32, 128, B, k, 64)
    ws, ws_ptr = _lib.workspace(ws_bytes, cuda_device)
    rc = lib.tms_dense_maxsim_topk(
        ctypes.c_void_p(Qb.data_ptr()), _lib.TMS_F16, 4, 32, 128, ctypes.c_void_p(D.data_ptr()), B * Nd,
        None, B, Nd, k, 64, 0, ctypes.c_void_p(vals.data_ptr()), ctypes.c_void_p(ids.data_ptr()),
        ctypes.c_void_p(ws_ptr), ws_bytes, ctypes.c_void_p(_lib.stream_handle(cuda_device)))
    assert rc == _lib.TMS_OK
    torch.testing.assert_close(vals, want_v, rtol=0, atol=0)
    assert torch.equal(ids, want_i)


def test_streamed_topk_argument_errors(cuda_device):
    from tilemaxsim_b200 import maxsim_topk
    D, off = _corpus(50, 4, cuda_device)
    Qb = R.normalized((2, 32, 128), 5).to(cuda_device)
    with pytest.raises(ValueError):
        maxsim_topk(Qb, D, off, 51)
    with pytest.raises(ValueError):
        maxsim_topk(Qb, D, off, 0)
    v, i = maxsim_topk(Qb[0], D, off, 5)  # a single 2-D query
    assert v.shape == (5,) and i.shape == (5,)
    assert np.all(np.diff(v.cpu().numpy()) <= 0)
