"""Host-side checks of the drop-in Python API (no GPU): argument validation happens before any
kernel call, and CPU tensors are rejected loudly (there is no CPU fallback)."""
from __future__ import annotations

import pytest
import torch


def test_cpu_tensors_are_rejected():
    from tilemaxsim_b200 import flash_maxsim_v2_multiquery, maxsim_batched, topk
    Q = torch.zeros(32, 128, dtype=torch.float16)
    D = torch.zeros(4, 10, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        flash_maxsim_v2_multiquery(Q, D)
    with pytest.raises(ValueError, match="CUDA"):
        maxsim_batched(Q, D.view(40, 128), torch.tensor([0, 10, 40]))
    with pytest.raises(ValueError, match="CUDA"):
        topk(torch.zeros(3, 50), 5)


def test_shape_errors_match_the_reference():
    from tilemaxsim_b200 import flash_maxsim_batch, flash_maxsim_single, flash_maxsim_v2
    Q = torch.zeros(32, 128, dtype=torch.float16)
    with pytest.raises(AssertionError):  # src/flash_maxsim_kernel.py:180
        flash_maxsim_single(Q, torch.zeros(10, 64, dtype=torch.float16))
    with pytest.raises(AssertionError):  # src/flash_maxsim_kernel.py:213
        flash_maxsim_batch(Q, torch.zeros(2, 10, 64, dtype=torch.float16))
    with pytest.raises(ValueError):
        flash_maxsim_v2(Q, torch.zeros(10, 128, dtype=torch.float16))


def test_pq_shape_errors():
    from tilemaxsim_b200 import TileMaxSimPQ
    pq = TileMaxSimPQ(torch.zeros(16, 256, 8))
    assert (pq.M, pq.K, pq.dsub, pq.d) == (16, 256, 8, 128)
    with pytest.raises(AssertionError):  # src/flash_pqsim_kernel.py:226
        pq.score_batch(torch.zeros(32, 128, dtype=torch.float16), torch.zeros(2, 10, 8, dtype=torch.uint8))
    with pytest.raises(AssertionError):  # src/flash_pqsim_kernel.py:201
        pq.build_distance_table(torch.zeros(32, 64))


def test_reference_baselines_run_on_cpu():
    """pytorch_maxsim_naive / _loop / pytorch_pqsim_baseline are the reference's plain-torch
    baselines, kept in the drop-in modules; they agree with the oracle on CPU."""
    import numpy as np
    import recipes as R
    from oracle import maxsim_oracle as O
    from tilemaxsim_b200 import pytorch_maxsim_loop, pytorch_maxsim_naive, pytorch_pqsim_baseline
    c = R.v1_selfcheck_case()
    want = O.maxsim_padded(c["Q"], c["D"])
    np.testing.assert_allclose(pytorch_maxsim_naive(c["Q"], c["D"]).numpy(), want, rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(pytorch_maxsim_loop(c["Q"], c["D"]).numpy(), want, rtol=1e-5, atol=1e-4)
    p = R.pq_case()
    np.testing.assert_allclose(pytorch_pqsim_baseline(p["Q"], p["codebook"], p["codes"]).numpy(),
                               O.pq_maxsim_decompress(p["Q"], p["codebook"], p["codes"]), rtol=1e-5, atol=1e-4)


def test_bench_reference_arm_prints_one_json_line():
    """The reference arm runs on host cores: `bench.py --impl reference` prints exactly one JSON
    line on standard output with the contract's keys (anything a library prints goes to stderr)."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--config", "c1",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, cwd=root, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["e2e"]["h2d_bytes_per_step"] == 0


def test_graphed_step_needs_device_inputs():
    """GraphedStep captures GPU work only: CPU example inputs are refused before any capture."""
    import pytest
    import torch
    from tilemaxsim_b200 import GraphedStep
    with pytest.raises(ValueError):
        GraphedStep(lambda q: q, torch.zeros(2, 32, 128))
    with pytest.raises(ValueError):
        GraphedStep(lambda: None)


def test_residual_scorer_validates_before_any_kernel():
    """ResidualMaxSim checks nbits, the centroid width, the bucket-weight count and the residual
    row width on the host, and refuses CPU tensors (no CPU fallback)."""
    from tilemaxsim_b200 import ResidualMaxSim
    cent = torch.zeros(16, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="nbits"):
        ResidualMaxSim(cent, torch.zeros(8), 3)
    with pytest.raises(ValueError, match="centroids"):
        ResidualMaxSim(torch.zeros(16, 96, dtype=torch.float16), torch.zeros(4), 2)
    with pytest.raises(ValueError, match="bucket weights"):
        ResidualMaxSim(cent, torch.zeros(3), 2)
    sc = ResidualMaxSim(cent, torch.zeros(4), 2)
    assert sc.d == 128 and sc.nbits == 2 and sc.centroids.dtype == torch.float16
    Q = torch.zeros(1, 32, 128, dtype=torch.float16)
    codes = torch.zeros(10, dtype=torch.int32)
    res = torch.zeros(10, 32, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        sc.score_queries(Q, codes, res, torch.tensor([0, 10]))


@pytest.mark.parametrize("nqry,nq,exact,route,launches", [
    (16, 32, True, "tokrows", 4),   # C4 at the reference precision: four passes of four queries
    (1, 32, True, "tokrows", 1),    # single query, hi/lo token rows
    (5, 40, True, "tokrows", 6),    # 2 + 2 + 1 queries of two chunks: three passes + chunk sums
    (6, 8, True, "lut", 1),         # <= 8-token queries needing several passes: table lookups
    (1, 32, False, "tokrows", 1),   # fast mode, one chunk
    (4, 32, False, "tokrows", 1),   # fast mode, four chunks in one pass
    (16, 32, False, "decoder", 2),  # fast mode, more than four chunks: packing + decoder kernel
])
def test_bench_pq_route_matches_the_library_routing(nqry, nq, exact, route, launches):
    """bench.py's kernel-launch claim follows csrc/pq_adc.cu's routing (M=16, K=256, dsub=8)."""
    import bench
    assert bench.pq_route(nqry, nq, 16, 256, 8, exact) == route
    assert bench.pq_score_launches(nqry, nq, 16, 256, 8, exact) == launches


def test_bench_residual_launches_match_the_library_routing():
    """Up to four query chunks: the token-rows kernel (+ the chunk sum for > 32-token queries);
    more: packing + the dense kernel's residual decoder warps."""
    import bench
    assert bench.res_score_launches(1, 32) == 1
    assert bench.res_score_launches(2, 64) == 2
    assert bench.res_score_launches(5, 32) == 2
