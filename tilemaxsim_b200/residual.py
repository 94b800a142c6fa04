"""MaxSim over a residual-compressed corpus (the ColBERTv2 / PLAID storage layout).

Each document token is stored as a centroid id plus an nbits-per-dimension residual:

    token = centroids[code] + bucket_weights[b_j]   for every dimension j (then optionally
                                                     scaled to unit length, as ColBERTv2 does)

where bit k of dimension j's bucket index b_j is bit (j * nbits + k) of the token's residual row,
bits numbered from the most significant bit of byte 0. ``ResidualMaxSim.score_queries`` scores
queries against such a corpus in one launch of the dense tensor-core kernel: its decoder warps
rebuild each token in shared memory from the centroid row (read through L2) and the residual bits,
so the decompressed embeddings are never written to HBM (C ABI ``tms_residual_maxsim``).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .maxsim import _check_offsets_enabled, validate_offsets


class ResidualMaxSim:
    def __init__(self, centroids: torch.Tensor, bucket_weights: torch.Tensor, nbits: int,
                 normalize: bool = True):
        """centroids (n_centroids, d) with d = 64 or 128 (kept as fp16); bucket_weights
        (2**nbits,) (kept as fp32); nbits 1, 2 or 4; normalize: scale each decoded token to unit
        length (ColBERTv2's decompression does)."""
        if nbits not in (1, 2, 4):
            raise ValueError(f"nbits must be 1, 2 or 4, got {nbits}")
        if centroids.dim() != 2 or centroids.shape[1] not in (64, 128):
            raise ValueError(f"centroids must be (n, 64) or (n, 128), got {tuple(centroids.shape)}")
        if bucket_weights.numel() != 1 << nbits:
            raise ValueError(f"expected {1 << nbits} bucket weights, got {bucket_weights.numel()}")
        self.centroids = centroids.to(torch.float16).contiguous()
        self.bucket_weights = bucket_weights.to(torch.float32).contiguous().view(-1)
        self.nbits = int(nbits)
        self.normalize = bool(normalize)
        self.d = self.centroids.shape[1]

    def score_queries(self, Qb: torch.Tensor, codes: torch.Tensor, residuals: torch.Tensor,
                      doc_offsets: torch.Tensor) -> torch.Tensor:
        """Qb (B_q, Nq, d) queries (rounded to fp16), codes (T,) int32 centroid ids, residuals
        (T, d * nbits / 8) uint8, doc_offsets (n + 1,) int64 -> (B_q, n) fp32 scores; an empty
        document scores -inf."""
        lib = _lib.load()
        single = Qb.dim() == 2
        if single:
            Qb = Qb.unsqueeze(0)
        dev = _lib.require_cuda(Qb, codes, residuals, doc_offsets, self.centroids, self.bucket_weights)
        Bq, Nq, d = Qb.shape
        if d != self.d:
            raise ValueError(f"queries have d={d}, centroids d={self.d}")
        T = codes.numel()
        if residuals.shape != (T, d * self.nbits // 8):
            raise ValueError(f"residuals must be ({T}, {d * self.nbits // 8}) uint8, got {tuple(residuals.shape)}")
        Qb = Qb.to(torch.float16).contiguous()
        codes = codes.to(torch.int32).contiguous()
        residuals = residuals.to(torch.uint8).contiguous()
        offsets = doc_offsets.to(torch.int64).contiguous()
        if _check_offsets_enabled():
            validate_offsets(offsets, T)
        n_docs = offsets.numel() - 1
        with torch.cuda.device(dev):
            out = torch.empty(Bq, n_docs, dtype=torch.float32, device=dev)
            if Bq > 0 and n_docs > 0:
                ws_bytes = lib.tms_residual_workspace_size(Bq, Nq, d, n_docs)
                ws, ws_ptr = _lib.workspace(ws_bytes, dev)
                rc = lib.tms_residual_maxsim(
                    ctypes.c_void_p(Qb.data_ptr()), Bq, Nq, d, ctypes.c_void_p(self.centroids.data_ptr()),
                    self.centroids.shape[0], ctypes.c_void_p(codes.data_ptr()),
                    ctypes.c_void_p(residuals.data_ptr()), ctypes.c_void_p(self.bucket_weights.data_ptr()),
                    self.nbits, int(self.normalize), T, ctypes.c_void_p(offsets.data_ptr()), n_docs, 0,
                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws_ptr), ws_bytes,
                    ctypes.c_void_p(_lib.stream_handle(dev)))
                _lib.check(rc, "tms_residual_maxsim")
                del ws
        return out[0] if single else out
