"""Drop-in replacement for the reference's ``src/flash_maxsim_kernel.py`` (the V1 API).

``flash_maxsim_single`` / ``flash_maxsim_batch`` / ``flash_maxsim_multi_doc`` keep the reference's
signatures and results (src/flash_maxsim_kernel.py:167-273); the scoring runs in the sm_100a
tcgen05 kernel. ``flash_maxsim_multi_doc`` scores every variable-length document in ONE launch
(the reference launched one kernel and made two host syncs per document). ``pytorch_maxsim_naive``
and ``pytorch_maxsim_loop`` are the reference's plain-PyTorch baselines (:280-303), kept because
callers import them from this module; they are ordinary torch code on any device.
"""
from __future__ import annotations

import torch

from . import _lib
from .maxsim import _dense_call, maxsim_padded


def flash_maxsim_single(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """MaxSim of one query (Nq, d) and one document (Nd, d) -> 0-d fp32 tensor
    (reference: src/flash_maxsim_kernel.py:167-197). An empty document gives -inf."""
    Nq, d = Q.shape
    assert D.shape[1] == d
    Nd = D.shape[0]
    return _dense_call(Q.unsqueeze(0), D, None, 1, Nd, _lib.TMS_OUT_SCORE)[0, 0]


def flash_maxsim_batch(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """MaxSim of one query (Nq, d) against B padded documents (B, Nd, d) -> (B,) fp32
    (reference: src/flash_maxsim_kernel.py:200-245)."""
    B, Nd, d = D.shape
    assert Q.shape[1] == d
    return maxsim_padded(Q.unsqueeze(0), D)[0]


def flash_maxsim_token_max(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """The V1 kernel's intermediate: per-query-token maxima (B, Nq) fp32, max_j <Q_i, D_bj>
    (reference: src/flash_maxsim_kernel.py:95-148, before _sum_reduce_kernel)."""
    B, Nd, d = D.shape
    assert Q.shape[1] == d
    return maxsim_padded(Q.unsqueeze(0), D, out_mode=_lib.TMS_OUT_TOKEN_MAX)[0]


def flash_maxsim_multi_doc(Q: torch.Tensor, D_flat: torch.Tensor, doc_offsets: torch.Tensor) -> torch.Tensor:
    """MaxSim of one query against variable-length documents: D_flat (total_tokens, d), document i
    = D_flat[doc_offsets[i]:doc_offsets[i+1]] -> (num_docs,) fp32
    (reference: src/flash_maxsim_kernel.py:248-273)."""
    n_docs = doc_offsets.shape[0] - 1
    if doc_offsets.device != D_flat.device:
        doc_offsets = doc_offsets.to(D_flat.device)
    return _dense_call(Q.unsqueeze(0), D_flat, doc_offsets, n_docs, 0, _lib.TMS_OUT_SCORE)[0]


def pytorch_maxsim_naive(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """Plain-PyTorch MaxSim that materialises the (B, Nq, Nd) similarity tensor
    (reference: src/flash_maxsim_kernel.py:280-288)."""
    S = torch.einsum("qd,bnd->bqn", Q.float(), D.float())
    return S.max(dim=-1).values.sum(dim=-1)


def pytorch_maxsim_loop(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """Plain-PyTorch MaxSim looping over query tokens (reference: src/flash_maxsim_kernel.py:291-303)."""
    B = D.shape[0]
    scores = torch.zeros(B, dtype=torch.float32, device=Q.device)
    for i in range(Q.shape[0]):
        scores += torch.einsum("d,bnd->bn", Q[i].float(), D.float()).max(dim=-1).values
    return scores
