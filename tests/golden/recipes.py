"""Deterministic input recipes shared by the golden-fixture generator and the tests.

Inputs are regenerated from seeds with torch's CPU generator (bit-reproducible across machines);
every fixture stores a SHA-256 of the inputs it was made from, so a recipe that drifted fails
loudly instead of comparing against the wrong numbers. Conventions follow the reference's own
synthetic data: i.i.d. Gaussian (``torch.randn``, src/run_all_experiments.py:622-623) or Gaussian
then L2-normalised per token in fp32 and cast (src/encode_msmarco.py:147-186), ragged lengths from
``numpy.random.default_rng(seed).integers`` (src/run_all_todo_experiments.py:227-229).
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def randn(shape, seed: int, dtype=torch.float16) -> torch.Tensor:
    """Plain i.i.d. N(0, 1) in fp32, cast to dtype (the reference's exp10 inputs)."""
    return torch.randn(*shape, generator=gen(seed), dtype=torch.float32).to(dtype)


def normalized(shape, seed: int, dtype=torch.float16) -> torch.Tensor:
    """N(0, 1) in fp32, L2-normalised along the last dim, cast to dtype."""
    x = torch.randn(*shape, generator=gen(seed), dtype=torch.float32)
    x = x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    return x.to(dtype)


def ragged_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, n).astype(np.int64)


def offsets_from_lengths(lengths: np.ndarray) -> np.ndarray:
    off = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(lengths, out=off[1:])
    return off


def codes_u8(shape, seed: int) -> torch.Tensor:
    return torch.randint(0, 256, shape, generator=gen(seed), dtype=torch.uint8)


def sha256(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = a.contiguous().view(torch.uint8).numpy() if a.dtype != torch.bfloat16 else \
                a.contiguous().view(torch.int16).numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------------------------
# Cases. Each returns a dict of CPU tensors / arrays; names are stable (fixtures key on them).
# ---------------------------------------------------------------------------------------------

# (Nq, Nd, d, B): the reference's "correctness at scale" sweep, src/run_all_experiments.py:617-626
EXP10_CONFIGS = [
    (8, 32, 64, 100),
    (16, 64, 128, 100),
    (32, 128, 128, 100),
    (32, 128, 256, 100),
    (32, 256, 128, 100),
    (64, 128, 128, 100),
    (32, 128, 384, 50),
    (32, 128, 768, 20),
]


def exp10_case(i: int) -> dict:
    nq, nd, d, b = EXP10_CONFIGS[i]
    return {"Q": randn((nq, d), 4200 + 2 * i), "D": randn((b, nd, d), 4201 + 2 * i)}


def v1_selfcheck_case() -> dict:
    """Shape of the reference's own self-check, src/flash_maxsim_kernel.py:306-330."""
    return {"Q": randn((32, 128), 42), "D": randn((16, 128, 128), 43)}


def ragged_case(n_queries: int = 3, nq: int = 32, d: int = 128, n_docs: int = 300,
                lo: int = 0, hi: int = 300, seed: int = 7, dtype=torch.float16) -> dict:
    lengths = ragged_lengths(n_docs, lo, hi, seed)
    lengths[[5, 6, n_docs - 1]] = 0  # empty documents, two adjacent and one at the very end
    off = offsets_from_lengths(lengths)
    return {"Qb": normalized((n_queries, nq, d), seed + 1, dtype),
            "D": normalized((int(off[-1]), d), seed + 2, dtype),
            "offsets": torch.from_numpy(off)}


def pq_case(cb_dtype=torch.float32, seed: int = 42, B: int = 8, Nd: int = 128, nq: int = 32,
            M: int = 16, K: int = 256, dsub: int = 8) -> dict:
    """Shape of the reference's PQ self-check, src/flash_pqsim_kernel.py:320-333."""
    return {"codebook": randn((M, K, dsub), seed, cb_dtype),
            "Q": normalized((nq, M * dsub), seed + 1, torch.float16),
            "codes": codes_u8((B, Nd, M), seed + 2)}


def topk_case() -> dict:
    """Scores with many exact ties and a NaN, to pin the (score desc, id asc) rule."""
    g = gen(99)
    s = torch.randint(0, 50, (4, 3000), generator=g).float() / 8.0
    s[1, 17] = float("nan")
    s[2, :] = 1.0  # all tied
    return {"scores": s}
