"""Corpus-sharded MaxSim search over several GPUs (one process per GPU).

Each rank holds a contiguous shard of the corpus (its documents' tokens + int64 offsets) and the
global id of its first document. A search scores every query against the local shard (one
tcgen05 launch), keeps the local top-k with global ids, and merges the shards' lists with ONE
all-gather of a packed (ids, score bits) buffer (NCCL over NVLink/NVSwitch in production, gloo in
the CPU tests) followed by a top-k of the world*k candidates under the same rule: score
descending, then global id ascending. The result is identical on every rank and equal to a
single-GPU top-k over the whole corpus.

The reference has no distributed path (its "multi-GPU" experiment ran independent halves from one
process with no merge, src/run_all_experiments.py:355-443); this is additive API.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .maxsim import maxsim_batched, topk

PAD_ID = torch.iinfo(torch.int64).max


def _pad_to_k(vals: torch.Tensor, ids: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Pads (rows, kk) lists to k columns with (NaN, PAD_ID), which rank after every real entry
    (NaN ranks last, and among NaN the padding's id is the largest)."""
    rows, kk = vals.shape
    if kk == k:
        return vals.contiguous(), ids.contiguous()
    pv = torch.full((rows, k), float("nan"), dtype=vals.dtype, device=vals.device)
    pi = torch.full((rows, k), PAD_ID, dtype=ids.dtype, device=ids.device)
    pv[:, :kk] = vals
    pi[:, :kk] = ids
    return pv, pi


def merge_topk(vals: torch.Tensor, ids: torch.Tensor, k: int, group=None,
               topk_fn: Callable | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merges every rank's (rows, k) top-k list into the global (rows, k) top-k.

    One all-gather of a packed (rows, 2k) int64 buffer per rank (the k global ids, then the k
    scores' fp32 bit patterns). On CUDA tensors the library packs (`tms_topk_pack`) and merges
    straight from the gathered buffer (`tms_topk_merge_packed`, the tms_topk rule); `topk_fn(scores,
    k, ids=...)` replaces that merge (the CPU tests pass the oracle's) and then the candidates are
    unpacked with torch."""
    vals, ids = _pad_to_k(vals, ids, k)
    if group is None or dist.get_world_size(group) == 1:
        return vals, ids
    world = dist.get_world_size(group)
    rows = vals.shape[0]
    native = topk_fn is None and vals.is_cuda
    packed = torch.empty((rows, 2 * k), dtype=torch.int64, device=vals.device)
    if native:
        lib = _lib.load()
        stream = ctypes.c_void_p(_lib.stream_handle(vals.device))
        _lib.check(lib.tms_topk_pack(ctypes.c_void_p(vals.data_ptr()), ctypes.c_void_p(ids.data_ptr()),
                                     rows, k, ctypes.c_void_p(packed.data_ptr()), stream), "tms_topk_pack")
    else:
        packed[:, :k] = ids
        packed[:, k:] = vals.view(torch.int32).to(torch.int64)
    gathered = torch.empty((world * rows, 2 * k), dtype=torch.int64, device=vals.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)  # rank-major along dim 0
    if native:
        out_v = torch.empty((rows, k), dtype=torch.float32, device=vals.device)
        out_i = torch.empty((rows, k), dtype=torch.int64, device=vals.device)
        _lib.check(lib.tms_topk_merge_packed(ctypes.c_void_p(gathered.data_ptr()), world, rows, k,
                                             ctypes.c_void_p(out_v.data_ptr()),
                                             ctypes.c_void_p(out_i.data_ptr()), stream),
                   "tms_topk_merge_packed")
        return out_v, out_i
    g = gathered.view(world, rows, 2 * k).permute(1, 0, 2)  # (rows, world, 2k)
    cand_i = g[:, :, :k].reshape(rows, world * k)
    cand_v = g[:, :, k:].reshape(rows, world * k).to(torch.int32).view(torch.float32)
    fn = topk_fn or topk
    return fn(cand_v.contiguous(), k, ids=cand_i.contiguous())


class ShardedIndex:
    """One rank's shard of a ragged corpus: tokens (T, d), offsets (n+1,) int64, global id base."""

    def __init__(self, D_tokens: torch.Tensor, doc_offsets: torch.Tensor, doc_id_base: int = 0,
                 group=None):
        self.D = D_tokens
        self.offsets = doc_offsets.to(torch.int64)
        self.n_docs = self.offsets.numel() - 1
        self.doc_id_base = int(doc_id_base)
        self.group = group

    def search_scores(self, scores: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Local (B_q, n) scores -> global top-k (scores (B_q, k), global doc ids (B_q, k))."""
        kk = min(k, self.n_docs)
        if kk > 0:
            vals, ids = topk(scores, kk, id_base=self.doc_id_base)
        else:
            vals = scores.new_empty((scores.shape[0], 0))
            ids = torch.empty((scores.shape[0], 0), dtype=torch.int64, device=scores.device)
        return merge_topk(vals, ids, k, self.group)

    def search(self, Qb: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Queries (B_q, Nq, d) -> global top-k over all shards."""
        return self.search_scores(maxsim_batched(Qb, self.D, self.offsets), k)


def sharded_search(Qb: torch.Tensor, D_tokens: torch.Tensor, doc_offsets: torch.Tensor, k: int,
                   group=None, doc_id_base: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Functional form of ShardedIndex(D_tokens, doc_offsets, doc_id_base, group).search(Qb, k)."""
    return ShardedIndex(D_tokens, doc_offsets, doc_id_base, group).search(Qb, k)
