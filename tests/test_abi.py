"""CPU-side checks of the C ABI: the in-tree library loads, exports exactly what
include/tilemaxsim.h declares, and rejects bad arguments before touching the GPU."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    hdr = (ROOT / "include" / "tilemaxsim.h").read_text()
    return set(re.findall(r"TMS_API\s+[\w\s\*]+?\b(tms_\w+)\s*\(", hdr))


def test_library_exports_every_declared_symbol():
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    decl = declared_symbols()
    assert len(decl) >= 12
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert decl == set(_lib.SIGNATURES), "ctypes signatures and header disagree"


def test_strerror_and_version():
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    assert _lib.strerror(_lib.TMS_ERR_TIMEOUT) == "device wait timed out"
    assert b"sm_100a" in lib.tms_version()


def test_invalid_arguments_rejected_without_gpu():
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    # bad dtype, bad mode, negative sizes: rejected before any CUDA call
    assert lib.tms_dense_maxsim(nul, 99, 1, 32, 128, nul, 10, nul, 1, 10, nul, 0, nul, 0, nul) == _lib.TMS_ERR_INVALID
    assert lib.tms_dense_maxsim(nul, 0, 1, 32, 128, nul, 10, nul, 1, 10, nul, 7, nul, 0, nul) == _lib.TMS_ERR_INVALID
    assert lib.tms_dense_maxsim(nul, 0, -1, 32, 128, nul, 10, nul, 1, 10, nul, 0, nul, 0, nul) == _lib.TMS_ERR_INVALID
    # nothing to do is OK
    assert lib.tms_dense_maxsim(nul, 0, 0, 32, 128, nul, 10, nul, 1, 10, nul, 0, nul, 0, nul) == _lib.TMS_OK
    assert lib.tms_topk(nul, 1, 10, 5, 3, nul, 0, 0, nul, nul, nul, 0, nul) == _lib.TMS_ERR_INVALID  # ld < n
    assert lib.tms_pq_maxsim(nul, 0, 1, 32, nul, 2, 16, 300, 8, nul, 0, nul, 1, 0, nul, 0, nul, 0, nul) == _lib.TMS_ERR_UNSUPPORTED
    assert lib.tms_pq_maxsim(nul, 0, 1, 32, nul, 2, 16, 256, 8, nul, 0, nul, 1, 0, nul, 7, nul, 0, nul) == _lib.TMS_ERR_INVALID


@pytest.mark.parametrize("d,ok", [(128, True), (64, True), (768, True), (96, True), (100, False)])
def test_dense_workspace_query(d, ok):
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    n = lib.tms_dense_workspace_size(_lib.TMS_F16, 64, 32, d, 100_000, _lib.TMS_OUT_SCORE)
    assert (n > 0) == ok
    if ok:  # packed query tiles: 16 tiles x 128 rows x d x 2 bytes, 1024-aligned
        assert n >= 16 * 128 * d * 2


def test_dense_plans():
    """Launch plans on a 148-SM B200: single query -> one Q-resident group over all SMs;
    64-query rerank -> 16 query tiles in groups, CTAs a whole number of waves; d=768 -> streaming."""
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    info = (ctypes.c_int64 * 10)()
    assert lib.tms_dense_plan_info(0, 1, 32, 128, 100_000, 18_000_000, 0, 148, info) == 0
    tn, qres, g, st, ng, nr, nm, kc, smem, ctas = list(info)
    assert (tn, qres, g, ng, nm, kc, ctas) == (256, 1, 1, 1, 1, 2, 148) and st >= 2 and smem <= 232448
    assert lib.tms_dense_plan_info(0, 64, 32, 128, 100_000, 18_000_000, 0, 148, info) == 0
    tn, qres, g, st, ng, nr, nm, kc, smem, ctas = list(info)
    assert nm == 16 and qres == 1 and g * ng >= nm and ctas % 148 == 0 and smem <= 232448
    assert lib.tms_dense_plan_info(0, 16, 32, 768, 50_000, 12_800_000, 0, 148, info) == 0
    assert info[1] == 0 and info[8] <= 232448


def test_dense_topk_workspace_is_bounded_by_the_chunk():
    """tms_dense_topk_workspace_size: the score buffer scales with chunk_docs, not with the corpus;
    0 for arguments no call could take (host-side sizing, no GPU needed)."""
    from tilemaxsim_b200 import _lib
    lib = _lib.load()
    f = lib.tms_dense_topk_workspace_size
    small = f(_lib.TMS_F16, 64, 32, 128, 10_000_000, 100, 5000)
    big = f(_lib.TMS_F16, 64, 32, 128, 10_000_000, 100, 50_000)
    assert 0 < small < big
    assert big - small >= 64 * 45_000 * 4  # the (B_q, chunk) fp32 score buffer grows with the chunk
    assert small < 64 * 5000 * 4 + (8 << 20)  # scores + query tiles + candidate lists, no corpus term
    default = f(_lib.TMS_F16, 256, 32, 128, 10_000_000, 100, 0)
    assert (1 << 30) <= default < (1 << 30) + (16 << 20)  # the 1 GiB default score buffer
    assert f(_lib.TMS_F16, 64, 32, 128, 0, 100, 0) == 0
    assert f(_lib.TMS_F16, 64, 32, 128, 1000, 0, 0) == 0
    assert f(_lib.TMS_F16, 0, 32, 128, 1000, 10, 0) == 0
