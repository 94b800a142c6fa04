"""Restatement of the ColBERTv2 residual encoder, the producer of the residual-compressed corpora
that ``tms_residual_maxsim`` decodes: test infrastructure only.

The format is the one ColBERTv2 / PLAID store (named by the reference at
src/full_scale_benchmark.py:364-366 and src/review_experiments.py:148). The encoder follows the
published ResidualCodec of stanford-futuredata/ColBERT (colbert/indexing/codecs/residual.py,
v0.2.x; not present in this container), restated here from its documented steps:

1. each embedding's code is its nearest centroid by inner product;
2. the residual is the embedding minus that centroid;
3. with 2^nbits buckets, the bucket cutoffs are the residual quantiles at 1/2^nbits, ...,
   (2^nbits - 1)/2^nbits, and each bucket's weight is the quantile at its middle
   ((b + 0.5)/2^nbits), both over all dimensions of a training sample;
4. every residual value is bucketized against the cutoffs (index b in [0, 2^nbits));
5. the index's bits are spread least-significant first, (b >> k) & 1 for k = 0 .. nbits-1, so
   dimension j's bits take positions j*nbits .. j*nbits + nbits - 1 of the row;
6. the bit row is packed into bytes most-significant bit first (numpy.packbits).

Decompression (the inverse the library implements on the GPU) adds the bucket weights to the
centroid and normalises the result to unit length.
"""
from __future__ import annotations

import numpy as np


def train_buckets(residuals: np.ndarray, nbits: int) -> tuple[np.ndarray, np.ndarray]:
    """Bucket cutoffs (2^nbits - 1,) and weights (2^nbits,) from residual quantiles."""
    n = 1 << nbits
    flat = np.asarray(residuals, dtype=np.float32).ravel()
    cutoffs = np.quantile(flat, np.arange(1, n) / n).astype(np.float32)
    weights = np.quantile(flat, (np.arange(n) + 0.5) / n).astype(np.float32)
    return cutoffs, weights


def compress(X: np.ndarray, centroids: np.ndarray, cutoffs: np.ndarray, nbits: int
             ) -> tuple[np.ndarray, np.ndarray]:
    """X (T, d) fp32 embeddings -> (codes (T,) int32, packed residuals (T, d*nbits/8) uint8)."""
    X = np.asarray(X, dtype=np.float32)
    C = np.asarray(centroids, dtype=np.float32)
    codes = np.argmax(X @ C.T, axis=1).astype(np.int32)
    resid = X - C[codes]
    # bucketize: index = number of cutoffs strictly below the value (torch.bucketize, right=False)
    b = np.searchsorted(cutoffs, resid, side="left").astype(np.uint8)
    bits = (b[:, :, None] >> np.arange(nbits, dtype=np.uint8)) & 1  # (T, d, nbits), LSB first
    packed = np.packbits(bits.reshape(X.shape[0], -1), axis=1)     # MSB first within each byte
    return codes, packed
