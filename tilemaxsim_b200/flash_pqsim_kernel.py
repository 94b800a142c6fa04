"""Drop-in replacement for the reference's ``src/flash_pqsim_kernel.py`` (PQ / ADC MaxSim).

``TileMaxSimPQ(codebook)`` keeps the reference's attributes (``codebook, M, K, dsub, d``) and
methods (``build_distance_table``, ``score_batch``, ``score_single``; src/flash_pqsim_kernel.py:
176-280). Scoring goes through the C ABI ``tms_pq_maxsim`` and reads the uint8 codes directly:
neither the (Nq, M, K) table nor an int32 copy of the codes is written to HBM (the reference wrote
both). ``score_queries`` is the additive multi-query, ragged-corpus entry point. By default
(``exact=True``) scoring keeps the reference's precision, agreeing with its ADC path to fp32
rounding (1e-5 relative): each CTA builds an fp32 distance table for eight query tokens in shared
memory and sums table entries straight from the uint8 codes (no reconstruction); fp16 queries of
up to 128 tokens instead run on the tensor cores, in passes of up to four 32-row query chunks, with
each token rebuilt from the codebook split into fp16 hi + fp16 lo parts, which carry about 22
significant bits (the codebook must lie inside the fp16 range, checked at construction; otherwise
the table lookups take every shape; batches of <= 8-token queries that need several passes keep
the table lookups too).
``exact=False`` is the faster tensor-core mode: queries in fp16 (fp32 / bf16 ones are rounded to
fp16) and each token rebuilt on chip from an fp16 copy of the codebook; for up to four 32-row
query chunks the rebuilt tokens go to tensor memory as the MMA's A operand (token-rows kernel), for
larger batches into the dense kernel's shared-memory operand tiles. Rounding the codebook to fp16
costs about 1e-3 relative (|error| <= 1e-3*|score| + 5e-3).
``pytorch_pqsim_baseline`` is the reference's decompress-then-score PyTorch baseline (:283-313).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .maxsim import _check_offsets_enabled, validate_offsets


def _codes_u8(codes: torch.Tensor) -> torch.Tensor:
    if codes.dtype != torch.uint8:
        codes = codes.to(torch.uint8)  # the reference also accepts int32 codes (< 256)
    return codes if codes.is_contiguous() else codes.contiguous()


class TileMaxSimPQ:
    """MaxSim over product-quantized documents (reference: src/flash_pqsim_kernel.py:176-280)."""

    def __init__(self, codebook: torch.Tensor, exact: bool = True):
        """codebook: (M, K, dsub) centroids (fp16, bf16 or fp32), K <= 256.

        exact=True (default): fp32 table lookups, the reference's arithmetic (scores within fp32
        rounding of the reference's ADC path). exact=False: queries of a supported shape are
        scored on the tensor cores in fp16 (fp32 / bf16 queries are rounded to fp16), codes decoded
        on chip through the codebook rounded to fp16 (|error| <= 1e-3*|score| + 5e-3); other shapes
        fall back to the table lookups."""
        self.exact = bool(exact)
        self.codebook = codebook.contiguous()
        # the tensor-core route to the reference's precision stores the codebook as fp16 hi + lo,
        # which needs every centroid value inside the fp16 range (checked once here)
        self._split_ok = bool(self.codebook.abs().max().item() < 65504.0) if self.codebook.numel() else False
        self.M, self.K, self.dsub = codebook.shape
        self.d = self.M * self.dsub
        if self.codebook.dtype not in _lib.DTYPE_CODE:
            raise TypeError(f"codebook dtype {codebook.dtype} not supported")

    def _tensor_shape(self) -> bool:
        """The tensor-core path's shape rule (csrc: pq_mma_codebook_bytes): dsub % 8 == 0,
        d % 64 == 0, d <= 512, K <= 256 and an fp16 codebook of at most 96 KB."""
        return (self.dsub % 8 == 0 and self.d % 64 == 0 and self.d <= 512 and self.K <= 256
                and self.M * self.K * self.dsub * 2 <= 96 * 1024)

    def _q(self, Q: torch.Tensor) -> torch.Tensor:
        if Q.dtype not in _lib.DTYPE_CODE:
            Q = Q.float()
        return Q if Q.is_contiguous() else Q.contiguous()

    def build_distance_table(self, Q: torch.Tensor) -> torch.Tensor:
        """(Nq, d) queries -> (Nq, M, K) fp32 table, T[q,m,k] = <Q[q, m-slice], C[m,k]>
        (reference: src/flash_pqsim_kernel.py:190-211)."""
        Nq = Q.shape[0]
        assert Q.shape[1] == self.d
        lib = _lib.load()
        dev = _lib.require_cuda(Q, self.codebook)
        Q = self._q(Q)
        with torch.cuda.device(dev):
            table = torch.empty(Nq, self.M, self.K, dtype=torch.float32, device=dev)
            rc = lib.tms_pq_table(ctypes.c_void_p(Q.data_ptr()), _lib.DTYPE_CODE[Q.dtype], 1, Nq,
                                  ctypes.c_void_p(self.codebook.data_ptr()), _lib.DTYPE_CODE[self.codebook.dtype],
                                  self.M, self.K, self.dsub, ctypes.c_void_p(table.data_ptr()),
                                  ctypes.c_void_p(_lib.stream_handle(dev)))
            _lib.check(rc, "tms_pq_table")
        return table

    def _score(self, Qb: torch.Tensor, codes_tokens: torch.Tensor, offsets: torch.Tensor | None,
               n_docs: int, nd: int) -> torch.Tensor:
        lib = _lib.load()
        tensors = [Qb, codes_tokens, self.codebook] + ([offsets] if offsets is not None else [])
        dev = _lib.require_cuda(*tensors)
        Bq, Nq, d = Qb.shape
        if d != self.d:
            raise ValueError(f"queries have d={d}, codebook expects d={self.d}")
        if codes_tokens.shape[-1] != self.M:
            raise ValueError(f"codes have {codes_tokens.shape[-1]} sub-quantizers, codebook has {self.M}")
        Qb = self._q(Qb)
        if not self.exact and Qb.dtype != torch.float16 and self._tensor_shape():
            Qb = Qb.half()  # the tensor-core path multiplies fp16 queries (fast-mode tolerance)
        codes_tokens = _codes_u8(codes_tokens)
        if offsets is not None and _check_offsets_enabled():
            validate_offsets(offsets, codes_tokens.shape[0])
        with torch.cuda.device(dev):
            out = torch.empty(Bq, n_docs, dtype=torch.float32, device=dev)
            if Bq == 0 or n_docs == 0:
                return out
            ws_bytes = lib.tms_pq_workspace_size(Bq, Nq, self.M, self.K, self.dsub, n_docs)
            ws, ws_ptr = _lib.workspace(ws_bytes, dev, align=1024)
            rc = lib.tms_pq_maxsim(
                ctypes.c_void_p(Qb.data_ptr()), _lib.DTYPE_CODE[Qb.dtype], Bq, Nq,
                ctypes.c_void_p(self.codebook.data_ptr()), _lib.DTYPE_CODE[self.codebook.dtype],
                self.M, self.K, self.dsub, ctypes.c_void_p(codes_tokens.data_ptr()), codes_tokens.shape[0],
                ctypes.c_void_p(offsets.data_ptr() if offsets is not None else 0), n_docs, nd,
                ctypes.c_void_p(out.data_ptr()), self._mode(),
                ctypes.c_void_p(ws_ptr), ws_bytes,
                ctypes.c_void_p(_lib.stream_handle(dev)))
            _lib.check(rc, "tms_pq_maxsim")
            del ws
        return out

    def _mode(self) -> int:
        if not self.exact:
            return _lib.TMS_PQ_FAST
        return _lib.TMS_PQ_PRECISE if self._split_ok else _lib.TMS_PQ_EXACT

    def score_batch(self, Q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        """(Nq, d) query vs (B, Nd, M) codes -> (B,) fp32 (reference: src/flash_pqsim_kernel.py:213-252)."""
        B, Nd, M = codes.shape
        assert M == self.M
        return self._score(Q.unsqueeze(0), codes.reshape(B * Nd, M), None, B, Nd)[0]

    def score_single(self, Q: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
        """(Nq, d) query vs one document's (Nd, M) codes -> 0-d fp32 (reference: :254-280)."""
        Nd, M = codes.shape
        assert M == self.M
        return self._score(Q.unsqueeze(0), codes, None, 1, Nd)[0, 0]

    def score_queries(self, Qb: torch.Tensor, codes_tokens: torch.Tensor, doc_offsets: torch.Tensor) -> torch.Tensor:
        """B_q queries (B_q, Nq, d) vs a ragged corpus of codes (T, M) with int64 offsets (n+1,)
        -> (B_q, n) fp32; an empty document scores -inf."""
        if doc_offsets.dtype != torch.int64:
            doc_offsets = doc_offsets.to(torch.int64)
        return self._score(Qb, codes_tokens, doc_offsets.contiguous(), doc_offsets.numel() - 1, 0)


def pytorch_pqsim_baseline(Q: torch.Tensor, codebook: torch.Tensor, codes: torch.Tensor) -> torch.Tensor:
    """Decompress-then-score PyTorch baseline (reference: src/flash_pqsim_kernel.py:283-313)."""
    M, K, dsub = codebook.shape
    B, Nd, _ = codes.shape
    d = Q.shape[1]
    D_approx = torch.zeros(B, Nd, d, dtype=torch.float32, device=Q.device)
    for m in range(M):
        D_approx[:, :, m * dsub:(m + 1) * dsub] = codebook[m][codes[:, :, m].long()].float()
    S = torch.einsum("qd,bnd->bqn", Q.float(), D_approx)
    return S.max(dim=-1).values.sum(dim=-1)
