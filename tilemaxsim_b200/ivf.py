"""Candidate generation upstream of MaxSim: an inverted-file (IVF) probe over token centroids.

The reference scores candidates that external searchers produce (PLAID's ``dense_search``,
src/plaid_integration_benchmark.py:186-211 and :309-317; WARP, baselines/bench_warp.py); it has no
candidate stage of its own. ``IVFIndex`` is that stage, built on the same corpus layout the
library scores (one token matrix + int64 document offsets) and the per-token centroid ids that a
ColBERTv2 / PLAID index stores (the ``codes`` of ``ResidualMaxSim``):

1. every query token scores all centroids (one fp32 GEMM, Q . C^T) and probes its ``nprobe`` best
   (the library's top-k: score descending, then centroid id ascending);
2. a document is a candidate of a query when one of its tokens is assigned to a probed centroid
   (``tms_ivf_candidates``: per-query candidate bitmaps and their union, from inverted lists);
3. the union's documents are gathered into one contiguous ragged corpus (``tms_gather_docs``) and
   scored for the whole query batch by ONE dense MaxSim launch; a query's scores of documents that
   only other queries probed are masked (``tms_mask_candidates``), and each query keeps its top-k.

A document's MaxSim score does not depend on the rest of the corpus, so the scores equal those of
scoring the full corpus, bit for bit; the search returns the exact top-k of each query's own
candidate set.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .maxsim import maxsim_batched, topk


class IVFIndex:
    """Inverted lists of a ragged corpus's token centroids.

    centroids: (n_centroids, d) fp16 / bf16 / fp32 on a CUDA device; codes: (T,) centroid id of
    every token (int32 or int64; ids outside the table are left out of every list); doc_offsets:
    (n_docs + 1,) int64. The lists (the sorted ids of the documents holding a token of each
    centroid) are built once on the device with torch sorting operations -- index construction,
    not the search path."""

    def __init__(self, centroids: torch.Tensor, codes: torch.Tensor, doc_offsets: torch.Tensor):
        dev = _lib.require_cuda(centroids, codes, doc_offsets)
        self.device = dev
        self.centroids = centroids.contiguous()
        self.n_centroids, self.d = self.centroids.shape
        off = doc_offsets.to(torch.int64).contiguous()
        self.doc_offsets = off
        self.n_docs = off.numel() - 1
        lengths = (off[1:] - off[:-1]).clamp_min(0)
        t0 = int(off[0].item()) if self.n_docs >= 0 else 0
        doc_of_tok = torch.repeat_interleave(torch.arange(self.n_docs, device=dev), lengths)
        c = codes[t0:t0 + doc_of_tok.numel()].to(torch.int64)
        keep = (c >= 0) & (c < self.n_centroids)
        key = torch.unique(c[keep] * max(self.n_docs, 1) + doc_of_tok[keep])  # sorted
        cent = key // max(self.n_docs, 1)
        counts = torch.bincount(cent, minlength=self.n_centroids)
        self.ivf_offsets = torch.zeros(self.n_centroids + 1, dtype=torch.int64, device=dev)
        torch.cumsum(counts, 0, out=self.ivf_offsets[1:])
        self.ivf_docs = (key - cent * max(self.n_docs, 1)).to(torch.int32).contiguous()

    def probe(self, Qb: torch.Tensor, nprobe: int) -> torch.Tensor:
        """(B_q, Nq, d) queries -> (B_q, Nq * nprobe) int64 ids of every token's nprobe best
        centroids."""
        Bq, Nq, d = Qb.shape
        if d != self.d:
            raise ValueError(f"queries have d={d}, centroids have d={self.d}")
        nprobe = max(1, min(int(nprobe), self.n_centroids))
        S = Qb.reshape(Bq * Nq, d).float() @ self.centroids.float().T  # plain fp32 GEMM (cuBLAS)
        _, ids = topk(S.contiguous(), nprobe)
        return ids.view(Bq, Nq * nprobe)

    def candidates(self, Qb: torch.Tensor, nprobe: int) -> tuple[torch.Tensor, torch.Tensor]:
        """-> (bitmaps (B_q + 1, ceil(n_docs / 32)) int32: row q = query q's candidates, last row
        = their union; union ids (n_cand,) int64 in increasing order)."""
        lib = _lib.load()
        probe = self.probe(Qb, nprobe).contiguous()
        Bq = probe.shape[0]
        words = (self.n_docs + 31) // 32
        with torch.cuda.device(self.device):
            bitmaps = torch.empty((Bq + 1, max(words, 1)), dtype=torch.int32, device=self.device)
            cand = torch.empty(max(self.n_docs, 1), dtype=torch.int64, device=self.device)
            count = torch.empty(1, dtype=torch.int64, device=self.device)
            rc = lib.tms_ivf_candidates(
                ctypes.c_void_p(probe.data_ptr()), Bq, probe.shape[1],
                ctypes.c_void_p(self.ivf_offsets.data_ptr()), ctypes.c_void_p(self.ivf_docs.data_ptr()),
                self.n_centroids, self.n_docs, ctypes.c_void_p(bitmaps.data_ptr()),
                ctypes.c_void_p(cand.data_ptr()), cand.numel(), ctypes.c_void_p(count.data_ptr()),
                ctypes.c_void_p(_lib.stream_handle(self.device)))
            _lib.check(rc, "tms_ivf_candidates")
            n_cand = int(count.item())  # sizes the gathered corpus: one host synchronisation
        return bitmaps, cand[:n_cand]

    def search(self, Qb: torch.Tensor, D_tokens: torch.Tensor, k: int, nprobe: int
               ) -> tuple[torch.Tensor, torch.Tensor]:
        """Top-k of each query among its own candidates, by exact MaxSim over D_tokens (the corpus
        the index was built for). Returns (scores (B_q, k) fp32, doc ids (B_q, k) int64); a query
        with fewer than k candidates is padded with (-inf, -1)."""
        lib = _lib.load()
        _lib.require_cuda(Qb, D_tokens)
        Bq = Qb.shape[0]
        bitmaps, cand = self.candidates(Qb, nprobe)
        n_cand = cand.numel()
        vals = torch.full((Bq, k), float("-inf"), dtype=torch.float32, device=self.device)
        ids = torch.full((Bq, k), -1, dtype=torch.int64, device=self.device)
        if n_cand == 0 or Bq == 0:
            return vals, ids
        D_tokens = D_tokens.contiguous()
        row_bytes = D_tokens.shape[1] * D_tokens.element_size()
        with torch.cuda.device(self.device):
            stream = ctypes.c_void_p(_lib.stream_handle(self.device))
            g_off = torch.empty(n_cand + 1, dtype=torch.int64, device=self.device)
            rc = lib.tms_gather_offsets(ctypes.c_void_p(self.doc_offsets.data_ptr()), self.n_docs,
                                        ctypes.c_void_p(cand.data_ptr()), n_cand,
                                        ctypes.c_void_p(g_off.data_ptr()), stream)
            _lib.check(rc, "tms_gather_offsets")
            total = int(g_off[-1].item())
            G = torch.empty((max(total, 1), D_tokens.shape[1]), dtype=D_tokens.dtype, device=self.device)
            rc = lib.tms_gather_docs(ctypes.c_void_p(D_tokens.data_ptr()), row_bytes,
                                     ctypes.c_void_p(self.doc_offsets.data_ptr()), self.n_docs,
                                     D_tokens.shape[0], ctypes.c_void_p(cand.data_ptr()), n_cand,
                                     ctypes.c_void_p(g_off.data_ptr()), total,
                                     ctypes.c_void_p(G.data_ptr()), stream)
            _lib.check(rc, "tms_gather_docs")
            scores = maxsim_batched(Qb, G[:total], g_off)
            rc = lib.tms_mask_candidates(ctypes.c_void_p(scores.data_ptr()), Bq, n_cand, n_cand,
                                         ctypes.c_void_p(cand.data_ptr()),
                                         ctypes.c_void_p(bitmaps.data_ptr()), self.n_docs,
                                         ctypes.c_float(float("nan")), stream)
            _lib.check(rc, "tms_mask_candidates")
        kk = min(k, n_cand)
        v, col = topk(scores, kk)  # columns ascend with document id: the tie rule carries over
        pad = torch.isnan(v)  # ranks after every candidate: not a candidate of this query
        vals[:, :kk] = v.masked_fill(pad, float("-inf"))
        ids[:, :kk] = cand[col].masked_fill(pad, -1)
        return vals, ids
