"""Exact (float64) MaxSim on the GPU for the full-size ranking tests: test infrastructure.

The same computation as ``oracle.maxsim_oracle.maxsim_ragged_f64`` (float64 products and sums of
the fp16 inputs, max over each document's tokens, sum over query tokens), run with torch float64
on the device so that whole BASELINE corpora (18M-160M tokens) can be checked in seconds. The C1
test checks it against the CPU oracle. Nothing in the library imports it.
"""
from __future__ import annotations

import numpy as np
import torch


def maxsim_f64_device(Qb: torch.Tensor, D: torch.Tensor, offsets: np.ndarray,
                      chunk_tokens: int = 1 << 20) -> tuple[np.ndarray, np.ndarray]:
    """Qb (B_q, Nq, d), D (T, d) on the device, offsets (n+1,) numpy int64.
    Returns (exact (B_q, n) float64 with -inf for empty docs, per-doc max token norm (n,))."""
    dev = D.device
    bq, nq, d = Qb.shape
    off = np.asarray(offsets, dtype=np.int64)
    n = len(off) - 1
    Qf = Qb.reshape(bq * nq, d).double()
    m = torch.empty((n, bq * nq), dtype=torch.float64, device=dev)
    dmax = torch.empty(n, dtype=torch.float64, device=dev)
    c0 = 0
    while c0 < n:  # chunks of whole documents, about chunk_tokens tokens each
        c1 = int(np.searchsorted(off, off[c0] + chunk_tokens, side="right")) - 1
        c1 = min(n, max(c1, c0 + 1))
        t0, t1 = int(off[c0]), int(off[c1])
        lengths = torch.from_numpy(np.diff(off[c0:c1 + 1])).to(dev)
        X = D[t0:t1].double()
        m[c0:c1] = torch.segment_reduce(X @ Qf.T, "max", lengths=lengths, axis=0)
        dmax[c0:c1] = torch.segment_reduce(X.norm(dim=1), "max", lengths=lengths, axis=0).clamp_min(0)
        c0 = c1
    exact = m.view(n, bq, nq).sum(dim=-1).T
    return exact.cpu().numpy(), dmax.cpu().numpy()
