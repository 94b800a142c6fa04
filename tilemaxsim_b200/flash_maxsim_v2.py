"""Drop-in replacement for the reference's ``src/flash_maxsim_v2.py`` entry points.

Same names, arguments and return values as ashutoshuiuc/tilemaxsim: ``Q`` is (Nq, d), ``D`` is a
padded (B, Nd, d) batch, the result is a fresh (B,) fp32 tensor on Q's device. Every Nd row of D
participates (zero padding included), as in the reference (src/flash_maxsim_v2.py:105-124). Both
functions run the same sm_100a tcgen05 kernel (C ABI ``tms_dense_maxsim``); unlike the reference
there is no Nq >= 16 restriction, no d <= 128 / d-tiled split and no atomics (deterministic).
"""
from __future__ import annotations

import torch

from .maxsim import maxsim_padded


def _check(Q: torch.Tensor, D: torch.Tensor) -> None:
    if Q.dim() != 2 or D.dim() != 3:
        raise ValueError(f"expected Q (Nq, d) and D (B, Nd, d); got {tuple(Q.shape)} and {tuple(D.shape)}")
    if Q.shape[1] != D.shape[2]:
        raise ValueError(f"Q has d={Q.shape[1]} but D has d={D.shape[2]}")


def flash_maxsim_v2(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """MaxSim scores (B,) of one query against B padded documents
    (reference: src/flash_maxsim_v2.py:193-224)."""
    _check(Q, D)
    return maxsim_padded(Q.unsqueeze(0), D)[0]


def flash_maxsim_v2_multiquery(Q: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """MaxSim scores (B,) of one query against B padded documents; the reference's recommended
    entry point (src/flash_maxsim_v2.py:227-289). Any d that is a multiple of 8 (16-bit) or 4
    (fp32) is handled by the same kernel's K loop (the reference's d-tiled variant, :133-190)."""
    _check(Q, D)
    return maxsim_padded(Q.unsqueeze(0), D)[0]
