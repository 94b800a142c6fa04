"""On-disk corpus shard format (replaces the reference's ``torch.save`` embedding caches,
src/encode_real_msmarco.py:163-173).

A shard is a directory::

    shard.json       {"format": "tilemaxsim-shard", "version": 1, "n_docs", "n_tokens", "d",
                      "dtype", "doc_id_base", "files": {name: {"dtype", "shape"}}}
    tokens.bin       (n_tokens, d) row-major fp16 / bf16 / fp32 token embeddings
    offsets.bin      (n_docs + 1,) int64 document offsets
    codes.bin        optional (n_tokens, M) uint8 PQ codes
    codebook.bin     optional (M, K, dsub) fp32 PQ codebook

Every file is raw little-endian data padded to a 4 KiB multiple, so it can be memory-mapped and
copied to the GPU in large page-aligned transfers (`load_shard(..., device="cuda")`).
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import torch

FORMAT, VERSION, ALIGN = "tilemaxsim-shard", 1, 4096
_NP = {"float16": np.float16, "float32": np.float32, "int64": np.int64, "uint8": np.uint8,
       "bfloat16": np.uint16}
_TORCH = {"float16": torch.float16, "float32": torch.float32, "int64": torch.int64, "uint8": torch.uint8,
          "bfloat16": torch.bfloat16}


def _dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).replace("torch.", "")


def _write(path: Path, t: torch.Tensor) -> dict:
    t = t.detach().contiguous().cpu()
    name = _dtype_name(t)
    arr = t.view(torch.uint16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    raw = arr.tobytes()
    with open(path, "wb") as f:
        f.write(raw)
        pad = (-len(raw)) % ALIGN
        if pad:
            f.write(b"\0" * pad)
    return {"dtype": name, "shape": list(t.shape)}


def save_shard(path: str | os.PathLike, D_tokens: torch.Tensor, doc_offsets: torch.Tensor,
               doc_id_base: int = 0, codes: torch.Tensor | None = None,
               codebook: torch.Tensor | None = None) -> Path:
    """Writes one corpus shard (see the module docstring) and returns its directory."""
    p = Path(path)
    p.mkdir(parents=True, exist_ok=True)
    if D_tokens.dim() != 2 or doc_offsets.dim() != 1:
        raise ValueError("expected D_tokens (T, d) and doc_offsets (n+1,)")
    files = {"tokens": _write(p / "tokens.bin", D_tokens),
             "offsets": _write(p / "offsets.bin", doc_offsets.to(torch.int64))}
    if codes is not None:
        files["codes"] = _write(p / "codes.bin", codes.to(torch.uint8))
    if codebook is not None:
        files["codebook"] = _write(p / "codebook.bin", codebook.float())
    meta = {"format": FORMAT, "version": VERSION, "n_docs": int(doc_offsets.numel() - 1),
            "n_tokens": int(D_tokens.shape[0]), "d": int(D_tokens.shape[1]),
            "dtype": _dtype_name(D_tokens), "doc_id_base": int(doc_id_base), "files": files}
    (p / "shard.json").write_text(json.dumps(meta, indent=1))
    return p


def load_shard(path: str | os.PathLike, device: str | torch.device = "cpu") -> dict:
    """Reads a shard (memory-mapped) -> {"tokens", "offsets", "codes"?, "codebook"?, "doc_id_base",
    "meta"} with tensors on `device`."""
    p = Path(path)
    meta = json.loads((p / "shard.json").read_text())
    if meta.get("format") != FORMAT or meta.get("version") != VERSION:
        raise ValueError(f"{p} is not a {FORMAT} v{VERSION} directory")
    out = {"doc_id_base": meta["doc_id_base"], "meta": meta}
    for name, info in meta["files"].items():
        shape = tuple(info["shape"])
        count = int(np.prod(shape)) if shape else 1
        mm = np.memmap(p / f"{name}.bin", dtype=_NP[info["dtype"]], mode="r", shape=(count,))
        t = torch.from_numpy(np.array(mm)).reshape(shape)
        if info["dtype"] == "bfloat16":
            t = t.view(torch.bfloat16)
        out[name] = t.to(device)
    if out["offsets"][-1].item() > meta["n_tokens"] or out["offsets"].numel() != meta["n_docs"] + 1:
        raise ValueError(f"{p}: offsets do not match the token count")
    return out
