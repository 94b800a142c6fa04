"""PLAID / ColBERT adapter: a native ``colbert_score_packed`` over the ragged kernel.

PLAID scores candidate passages with ``colbert_score_packed(Q, D_packed, D_lengths, config)``:
``D_packed`` holds the candidates' token embeddings back to back, ``D_lengths`` their lengths.
The reference's drop-in (src/plaid_integration_benchmark.py:154-183) pads them into a (B, max_Nd, d)
tensor through StridedTensor, multiplies by the mask and calls the padded kernel, so zero padding
rows take part in the max. This adapter passes the packed layout straight to the ragged kernel:
no padded copy, and each passage's max runs over its own tokens only, as PLAID's own scorer does
with its mask.

Install it over PLAID the way the reference's benchmark does (src/plaid_integration_benchmark.py:
328-333)::

    import colbert.modeling.colbert as m, colbert.search.index_storage as s
    from tilemaxsim_b200.plaid import colbert_score_packed
    m.colbert_score_packed = s.colbert_score_packed = colbert_score_packed
"""
from __future__ import annotations

import torch

from .maxsim import maxsim_batched


def colbert_score_packed(Q: torch.Tensor, D_packed: torch.Tensor, D_lengths: torch.Tensor,
                         config=None) -> torch.Tensor:
    """Q (1, Nq, d) or (Nq, d); D_packed (sum(D_lengths), d); D_lengths (n,) -> (n,) fp32 scores.

    `config` is accepted for signature compatibility; tensors on the CPU are moved to the current
    CUDA device (the scoring itself has no CPU path)."""
    if Q.dim() == 3:
        if Q.shape[0] != 1:
            raise ValueError("colbert_score_packed scores one query; got Q of shape %s" % (tuple(Q.shape),))
        Q = Q[0]
    dev = D_packed.device if D_packed.is_cuda else torch.device("cuda", torch.cuda.current_device())
    Q, D_packed, D_lengths = Q.to(dev), D_packed.to(dev), D_lengths.to(dev)
    if D_packed.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        D_packed = D_packed.half()
    offsets = torch.zeros(D_lengths.numel() + 1, dtype=torch.int64, device=dev)
    torch.cumsum(D_lengths.to(torch.int64), 0, out=offsets[1:])
    return maxsim_batched(Q.to(D_packed.dtype), D_packed, offsets)
