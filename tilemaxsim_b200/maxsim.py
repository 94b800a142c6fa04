"""Batched, ragged MaxSim scoring and top-k on B200 -- the additive API over the C ABI.

``maxsim_batched`` scores B_q queries against a ragged corpus stored as one concatenated token
matrix plus int64 document offsets (the layout of the reference's ``flash_maxsim_multi_doc``,
src/flash_maxsim_kernel.py:248-273) in a single tcgen05 kernel launch; ``maxsim_topk`` adds the
per-query top-k (the reference ranks with ``torch.topk``, src/cycle3_experiments.py:215).
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib


def validate_offsets(doc_offsets: torch.Tensor, n_tokens: int) -> None:
    """Checks a document offsets array on its GPU (tms_validate_offsets): every entry in
    [0, n_tokens] and the array non-decreasing. Raises ValueError naming a bad index. Synchronises
    the current stream. The scoring calls never read outside their arrays whatever the offsets;
    this only tells a caller that its offsets are malformed. Setting TMS_CHECK_OFFSETS=1 runs it
    before every ragged scoring call."""
    lib = _lib.load()
    dev = _lib.require_cuda(doc_offsets)
    off = _as_contig(doc_offsets.to(torch.int64))
    with torch.cuda.device(dev):
        rc = lib.tms_validate_offsets(ctypes.c_void_p(off.data_ptr()), off.numel() - 1, int(n_tokens),
                                      ctypes.c_void_p(_lib.stream_handle(dev)))
        _lib.check(rc, "tms_validate_offsets")
        status, word = _lib.last_device_error(dev)
    if status == _lib.TMS_ERR_BAD_OFFSETS:
        raise ValueError(f"doc_offsets[{word & 0x3FFFFFFF}] is negative, smaller than the entry before "
                         f"it, or past n_tokens={n_tokens}")
    if status != _lib.TMS_OK:
        raise _lib.TileMaxSimError(status, "device error word")


def _check_offsets_enabled() -> bool:
    return os.environ.get("TMS_CHECK_OFFSETS", "0") not in ("", "0")


def _as_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def _dense_call(Qb: torch.Tensor, D_tokens: torch.Tensor, doc_offsets: torch.Tensor | None,
                n_docs: int, nd_uniform: int, out_mode: int) -> torch.Tensor:
    """Runs tms_dense_maxsim. Qb (B_q, Nq, d); D_tokens (T, d). Returns fp32 scores (B_q, n_docs)
    or per-token maxima (B_q, n_docs, Nq)."""
    lib = _lib.load()
    dev = _lib.require_cuda(Qb, D_tokens, *( [doc_offsets] if doc_offsets is not None else []))
    if Qb.dim() != 3 or D_tokens.dim() != 2:
        raise ValueError(f"expected Q (B_q, Nq, d) and D (T, d); got {tuple(Qb.shape)}, {tuple(D_tokens.shape)}")
    Bq, Nq, d = Qb.shape
    if D_tokens.shape[1] != d:
        raise ValueError(f"embedding dims differ: Q has d={d}, D has d={D_tokens.shape[1]}")
    if D_tokens.dtype not in _lib.DTYPE_CODE:
        raise TypeError(f"unsupported dtype {D_tokens.dtype}; use float16, bfloat16 or float32")
    if Qb.dtype != D_tokens.dtype:
        Qb = Qb.to(D_tokens.dtype)
    Qb = _as_contig(Qb)
    D_tokens = _as_contig(D_tokens)
    if doc_offsets is not None:
        if doc_offsets.dtype != torch.int64:
            doc_offsets = doc_offsets.to(torch.int64)
        doc_offsets = _as_contig(doc_offsets)
        if _check_offsets_enabled():
            validate_offsets(doc_offsets, D_tokens.shape[0])
    dt = _lib.DTYPE_CODE[D_tokens.dtype]
    shape = (Bq, n_docs) if out_mode == _lib.TMS_OUT_SCORE else (Bq, n_docs, Nq)
    with torch.cuda.device(dev):
        out = torch.empty(shape, dtype=torch.float32, device=dev)
        if Bq == 0 or n_docs == 0:
            return out
        ws_bytes = lib.tms_dense_workspace_size(dt, Bq, Nq, d, n_docs, out_mode)
        if ws_bytes == 0:
            raise _lib.TileMaxSimError(_lib.TMS_ERR_UNSUPPORTED, f"dense MaxSim with d={d}, dtype={D_tokens.dtype}")
        ws, ws_ptr = _lib.workspace(ws_bytes, dev)
        rc = lib.tms_dense_maxsim(
            ctypes.c_void_p(Qb.data_ptr()), dt, Bq, Nq, d, ctypes.c_void_p(D_tokens.data_ptr()),
            D_tokens.shape[0], ctypes.c_void_p(doc_offsets.data_ptr() if doc_offsets is not None else 0),
            n_docs, nd_uniform, ctypes.c_void_p(out.data_ptr()), out_mode, ctypes.c_void_p(ws_ptr),
            ws_bytes, ctypes.c_void_p(_lib.stream_handle(dev)))
        _lib.check(rc, "tms_dense_maxsim")
        del ws  # returned to torch's caching allocator; stream-ordered reuse is safe
    return out


def maxsim_padded(Qb: torch.Tensor, D: torch.Tensor, out_mode: int = _lib.TMS_OUT_SCORE) -> torch.Tensor:
    """Qb (B_q, Nq, d) against padded docs D (B, Nd, d): every one of the Nd rows participates,
    zero padding included (src/flash_maxsim_v2.py:105-124). Returns (B_q, B) fp32."""
    if D.dim() != 3:
        raise ValueError(f"expected D (B, Nd, d); got {tuple(D.shape)}")
    B, Nd, d = D.shape
    D = _as_contig(D)
    return _dense_call(Qb, D.view(B * Nd, d), None, B, Nd, out_mode)


def maxsim_batched(Qb: torch.Tensor, D_tokens: torch.Tensor, doc_offsets: torch.Tensor,
                   out_mode: int = _lib.TMS_OUT_SCORE) -> torch.Tensor:
    """MaxSim of every query against every document of a ragged corpus.

    Qb: (B_q, Nq, d) or (Nq, d); D_tokens: (T, d); doc_offsets: (n_docs + 1,) int64 with document i
    owning tokens [doc_offsets[i], doc_offsets[i+1]). Returns fp32 (B_q, n_docs) (or (n_docs,) for a
    single 2-D query). An empty document scores -inf.
    """
    single = Qb.dim() == 2
    if single:
        Qb = Qb.unsqueeze(0)
    if doc_offsets.dim() != 1 or doc_offsets.numel() < 1:
        raise ValueError("doc_offsets must be 1-D with n_docs + 1 entries")
    out = _dense_call(Qb, D_tokens, doc_offsets, doc_offsets.numel() - 1, 0, out_mode)
    return out[0] if single else out


def topk(scores: torch.Tensor, k: int, ids: torch.Tensor | None = None, id_base: int = 0
         ) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row top-k of (rows, n) fp32 scores, ordered by score descending then id ascending (NaN
    last). Ids are column + id_base, or ids[r, c] when given. Returns (values (rows, k) fp32,
    ids (rows, k) int64)."""
    lib = _lib.load()
    single = scores.dim() == 1
    if single:
        scores = scores.unsqueeze(0)
        if ids is not None:
            ids = ids.unsqueeze(0)
    dev = _lib.require_cuda(scores, *([ids] if ids is not None else []))
    if scores.dtype != torch.float32:
        scores = scores.float()
    if scores.stride(-1) != 1:
        scores = scores.contiguous()
    rows, n = scores.shape
    if not (0 < k <= n):
        raise ValueError(f"k={k} must be in [1, n={n}]")
    if ids is not None:
        if ids.shape != scores.shape:
            raise ValueError("ids must have the shape of scores")
        ids = ids.to(torch.int64)
        if ids.stride(-1) != 1:
            ids = ids.contiguous()
    with torch.cuda.device(dev):
        vals = torch.empty((rows, k), dtype=torch.float32, device=dev)
        out_ids = torch.empty((rows, k), dtype=torch.int64, device=dev)
        ws_bytes = lib.tms_topk_workspace_size(rows, n, k)
        ws, ws_ptr = _lib.workspace(ws_bytes, dev, align=256)
        rc = lib.tms_topk(ctypes.c_void_p(scores.data_ptr()), rows, n, scores.stride(0), k,
                          ctypes.c_void_p(ids.data_ptr() if ids is not None else 0),
                          ids.stride(0) if ids is not None else 0, id_base,
                          ctypes.c_void_p(vals.data_ptr()), ctypes.c_void_p(out_ids.data_ptr()),
                          ctypes.c_void_p(ws_ptr), ws_bytes, ctypes.c_void_p(_lib.stream_handle(dev)))
        _lib.check(rc, "tms_topk")
        del ws
    if single:
        return vals[0], out_ids[0]
    return vals, out_ids


def maxsim_topk(Qb: torch.Tensor, D_tokens: torch.Tensor, doc_offsets: torch.Tensor, k: int,
                id_base: int = 0, chunk_docs: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Scores B_q queries against a ragged corpus and returns each query's k best documents:
    (scores (B_q, k) fp32, doc ids (B_q, k) int64), ties broken by the smaller doc id.

    The full (B_q, n) score matrix is never held: documents are scored `chunk_docs` at a time
    (default: a 1 GiB score buffer) and each chunk's top-k is merged into a running list, which
    gives exactly the top-k of the full matrix (tms_dense_maxsim_topk)."""
    lib = _lib.load()
    single = Qb.dim() == 2
    if single:
        Qb = Qb.unsqueeze(0)
    dev = _lib.require_cuda(Qb, D_tokens, doc_offsets)
    if Qb.dim() != 3 or D_tokens.dim() != 2 or doc_offsets.dim() != 1 or doc_offsets.numel() < 1:
        raise ValueError("expected Q (B_q, Nq, d), D (T, d) and 1-D offsets (n_docs + 1,)")
    Bq, Nq, d = Qb.shape
    if D_tokens.shape[1] != d:
        raise ValueError(f"embedding dims differ: Q has d={d}, D has d={D_tokens.shape[1]}")
    if D_tokens.dtype not in _lib.DTYPE_CODE:
        raise TypeError(f"unsupported dtype {D_tokens.dtype}; use float16, bfloat16 or float32")
    n_docs = doc_offsets.numel() - 1
    if not (0 < k <= n_docs):
        raise ValueError(f"k={k} must be in [1, n_docs={n_docs}]")
    Qb = _as_contig(Qb.to(D_tokens.dtype))
    D_tokens = _as_contig(D_tokens)
    doc_offsets = _as_contig(doc_offsets.to(torch.int64))
    dt = _lib.DTYPE_CODE[D_tokens.dtype]
    chunk = 0 if chunk_docs is None else int(chunk_docs)
    with torch.cuda.device(dev):
        vals = torch.empty((Bq, k), dtype=torch.float32, device=dev)
        ids = torch.empty((Bq, k), dtype=torch.int64, device=dev)
        if Bq > 0:
            ws_bytes = lib.tms_dense_topk_workspace_size(dt, Bq, Nq, d, n_docs, k, chunk)
            if ws_bytes == 0:
                raise _lib.TileMaxSimError(_lib.TMS_ERR_UNSUPPORTED, f"dense MaxSim top-k with d={d}")
            ws, ws_ptr = _lib.workspace(ws_bytes, dev)
            rc = lib.tms_dense_maxsim_topk(
                ctypes.c_void_p(Qb.data_ptr()), dt, Bq, Nq, d, ctypes.c_void_p(D_tokens.data_ptr()),
                D_tokens.shape[0], ctypes.c_void_p(doc_offsets.data_ptr()), n_docs, 0, k, chunk, id_base,
                ctypes.c_void_p(vals.data_ptr()), ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(ws_ptr),
                ws_bytes, ctypes.c_void_p(_lib.stream_handle(dev)))
            _lib.check(rc, "tms_dense_maxsim_topk")
            del ws
    if single:
        return vals[0], ids[0]
    return vals, ids
