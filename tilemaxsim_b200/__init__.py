"""tilemaxsim_b200 -- B200-native (sm_100a) late-interaction MaxSim scoring.

Drop-in modules with the reference's (ashutoshuiuc/tilemaxsim) entry points:
  tilemaxsim_b200.flash_maxsim_v2      flash_maxsim_v2, flash_maxsim_v2_multiquery
  tilemaxsim_b200.flash_maxsim_kernel  flash_maxsim_single / _batch / _multi_doc, pytorch_maxsim_*
  tilemaxsim_b200.flash_pqsim_kernel   TileMaxSimPQ, pytorch_pqsim_baseline
Additive API: maxsim_batched, maxsim_topk, topk (tilemaxsim_b200.maxsim), sharded_search
(tilemaxsim_b200.sharded), GraphedStep (a search step captured as a CUDA graph), ResidualMaxSim
(ColBERTv2 residual-compressed corpora) and IVFIndex (candidate generation by a centroid probe).
All scoring runs in libtilemaxsim_b200.so (hand-written sm_100a CUDA behind a C ABI,
include/tilemaxsim.h); there is no CPU fallback.
"""
from .flash_maxsim_kernel import (flash_maxsim_batch, flash_maxsim_multi_doc, flash_maxsim_single,
                                  flash_maxsim_token_max, pytorch_maxsim_loop, pytorch_maxsim_naive)
from .flash_maxsim_v2 import flash_maxsim_v2, flash_maxsim_v2_multiquery
from .flash_pqsim_kernel import TileMaxSimPQ, pytorch_pqsim_baseline
from .graphed import GraphedStep
from .ivf import IVFIndex
from .maxsim import maxsim_batched, maxsim_padded, maxsim_topk, topk, validate_offsets
from .residual import ResidualMaxSim

__version__ = "0.1.0"
__all__ = [
    "flash_maxsim_single", "flash_maxsim_batch", "flash_maxsim_multi_doc", "flash_maxsim_token_max",
    "pytorch_maxsim_naive", "pytorch_maxsim_loop", "flash_maxsim_v2", "flash_maxsim_v2_multiquery",
    "TileMaxSimPQ", "pytorch_pqsim_baseline", "maxsim_batched", "maxsim_padded", "maxsim_topk", "topk",
    "GraphedStep", "validate_offsets", "ResidualMaxSim", "IVFIndex",
]
