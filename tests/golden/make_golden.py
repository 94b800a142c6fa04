"""Generates tests/golden/*.npz from the REFERENCE implementation's own PyTorch functions.

Run once in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_golden.py --reference /path/to/tilemaxsim

It imports ``pytorch_maxsim_naive`` / ``pytorch_maxsim_loop`` (src/flash_maxsim_kernel.py:280-303),
``pytorch_pqsim_baseline`` (src/flash_pqsim_kernel.py:283-313) and ``pytorch_pq_adc_table``
(src/from_retcompiler/benchmark_pq_adc.py:95-114) from the reference, runs them on CPU on the
seeded inputs of recipes.py, and stores their outputs with a SHA-256 of the inputs. Inputs are not
stored: tests regenerate them from the recipe and check the hash. Ragged documents are scored one
slice at a time, as the reference's ``flash_maxsim_multi_doc`` does (src/flash_maxsim_kernel.py:
248-273); an empty document is -inf (running max initialised to -inf, :48 and :92).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import recipes as R  # noqa: E402


def save(name: str, meta: dict, **arrays) -> None:
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
    print(f"wrote {path.name}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in arrays.items()))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    a = ap.parse_args()
    src = Path(a.reference) / "src"
    sys.path.insert(0, str(src))
    sys.path.insert(0, str(src / "from_retcompiler"))
    import flash_maxsim_kernel as ref_v1  # noqa: E402
    import flash_pqsim_kernel as ref_pq  # noqa: E402
    import benchmark_pq_adc as ref_adc  # noqa: E402

    torch.set_num_threads(max(1, torch.get_num_threads()))

    # 1. exp10 sweep (padded docs): pytorch_maxsim_naive and the per-token maxima.
    for i, (nq, nd, d, b) in enumerate(R.EXP10_CONFIGS):
        c = R.exp10_case(i)
        scores = ref_v1.pytorch_maxsim_naive(c["Q"], c["D"]).numpy()
        tokmax = torch.einsum("qd,bnd->bqn", c["Q"].float(), c["D"].float()).max(-1).values.numpy()
        save(f"exp10_{i}", {"case": "exp10", "index": i, "Nq": nq, "Nd": nd, "d": d, "B": b,
                            "sha256": R.sha256(c["Q"], c["D"]),
                            "source": "src/flash_maxsim_kernel.py:280-288 pytorch_maxsim_naive"},
             scores=scores, token_max=tokmax)

    # 2. V1 self-check shape: naive and loop oracles must agree.
    c = R.v1_selfcheck_case()
    naive = ref_v1.pytorch_maxsim_naive(c["Q"], c["D"]).numpy()
    loop = ref_v1.pytorch_maxsim_loop(c["Q"], c["D"]).numpy()
    save("v1_selfcheck", {"case": "v1_selfcheck", "sha256": R.sha256(c["Q"], c["D"]),
                          "source": "src/flash_maxsim_kernel.py:280-303"}, naive=naive, loop=loop)

    # 3. Ragged corpora (multi-query, empty docs), fp16 and bf16.
    for name, kw in [("ragged_f16", {}), ("ragged_bf16", {"dtype": torch.bfloat16, "seed": 11}),
                     ("ragged_nq20", {"nq": 20, "n_queries": 2, "seed": 13}),
                     ("ragged_nq40", {"nq": 40, "n_queries": 2, "n_docs": 120, "seed": 17})]:
        c = R.ragged_case(**kw)
        off = c["offsets"].numpy()
        n = len(off) - 1
        out = np.full((c["Qb"].shape[0], n), -np.inf, dtype=np.float32)
        tm = np.full((c["Qb"].shape[0], n, c["Qb"].shape[1]), -np.inf, dtype=np.float32)
        for q in range(c["Qb"].shape[0]):
            for i in range(n):
                s, e = int(off[i]), int(off[i + 1])
                if e > s:
                    doc = c["D"][s:e].unsqueeze(0)
                    out[q, i] = ref_v1.pytorch_maxsim_naive(c["Qb"][q], doc)[0].item()
                    tm[q, i] = torch.einsum("qd,bnd->bqn", c["Qb"][q].float(), doc.float()).max(-1).values[0].numpy()
        save(name, {"case": "ragged", "kwargs": {k: (str(v) if isinstance(v, torch.dtype) else v) for k, v in kw.items()},
                    "sha256": R.sha256(c["Qb"], c["D"], off),
                    "source": "src/flash_maxsim_kernel.py:248-273 (per-doc pytorch_maxsim_naive)"},
             scores=out, token_max=tm)

    # 4. PQ: decompress baseline and the reference's table (ADC) restatement.
    for name, cb_dtype in [("pq_f32", torch.float32), ("pq_f16", torch.float16)]:
        c = R.pq_case(cb_dtype)
        base = ref_pq.pytorch_pqsim_baseline(c["Q"], c["codebook"], c["codes"]).numpy()
        B, Nd, M = c["codes"].shape
        tok = ref_adc.pytorch_pq_adc_table(c["Q"], c["codes"].reshape(B * Nd, M), c["codebook"])
        adc = tok.reshape(-1, B, Nd).max(dim=-1).values.sum(dim=0).numpy()
        save(name, {"case": "pq", "cb_dtype": str(cb_dtype),
                    "sha256": R.sha256(c["codebook"], c["Q"], c["codes"]),
                    "source": "src/flash_pqsim_kernel.py:283-313; src/from_retcompiler/benchmark_pq_adc.py:95-114"},
             decompress=base, adc=adc)

    # 5. top-k with ties: reference ranks with torch.topk (src/cycle3_experiments.py:215); the
    #    fixture stores the (score desc, id asc) order and torch.topk's values.
    c = R.topk_case()
    s = c["scores"]
    order = np.stack([np.lexsort((np.arange(s.shape[1]), np.isnan(r), np.where(np.isnan(r), np.inf, -r)))
                      for r in s.numpy()])
    tv = torch.topk(torch.nan_to_num(s, nan=-np.inf), k=100, dim=1).values.numpy()
    save("topk_ties", {"case": "topk", "sha256": R.sha256(s)}, order=order[:, :1000].astype(np.int64),
         torch_topk_values=tv)
    return 0


if __name__ == "__main__":
    sys.exit(main())
