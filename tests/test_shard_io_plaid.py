"""Shard format round trip (CPU) and the PLAID adapter against the oracle (GPU)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import recipes as R
from oracle import maxsim_oracle as O


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_shard_round_trip(tmp_path, dtype):
    from tilemaxsim_b200.shard_io import load_shard, save_shard
    c = R.ragged_case(n_queries=1, n_docs=50, seed=3, dtype=dtype if dtype != torch.float32 else torch.float16)
    D = c["D"].to(dtype)
    codes = torch.randint(0, 256, (D.shape[0], 16), dtype=torch.uint8)
    cb = torch.randn(16, 256, 8)
    save_shard(tmp_path / "s0", D, c["offsets"], doc_id_base=1000, codes=codes, codebook=cb)
    s = load_shard(tmp_path / "s0")
    assert s["doc_id_base"] == 1000
    assert torch.equal(s["tokens"], D) and s["tokens"].dtype == dtype
    assert torch.equal(s["offsets"], c["offsets"]) and torch.equal(s["codes"], codes)
    assert torch.equal(s["codebook"], cb)
    assert (tmp_path / "s0" / "tokens.bin").stat().st_size % 4096 == 0


def test_shard_rejects_foreign_directory(tmp_path):
    from tilemaxsim_b200.shard_io import load_shard
    (tmp_path / "shard.json").write_text('{"format": "other"}')
    with pytest.raises(ValueError):
        load_shard(tmp_path)


@pytest.mark.gpu
def test_colbert_score_packed_matches_oracle(cuda_device, tmp_path):
    from tilemaxsim_b200.plaid import colbert_score_packed
    from tilemaxsim_b200.shard_io import load_shard, save_shard
    c = R.ragged_case(n_queries=1, n_docs=120, lo=1, hi=180, seed=9)
    lengths = c["offsets"][1:] - c["offsets"][:-1]
    got = colbert_score_packed(c["Qb"][:1], c["D"], lengths)  # CPU inputs, PLAID style (1, Nq, d)
    want = O.maxsim_ragged(c["Qb"][0], c["D"], c["offsets"].numpy())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-3, atol=1e-3)
    # the same corpus through the shard format, loaded onto the GPU
    save_shard(tmp_path / "s", c["D"], c["offsets"])
    s = load_shard(tmp_path / "s", device=cuda_device)
    from tilemaxsim_b200 import maxsim_batched
    np.testing.assert_allclose(maxsim_batched(c["Qb"][0].to(cuda_device), s["tokens"], s["offsets"]).cpu().numpy(),
                               want, rtol=1e-3, atol=1e-3)
