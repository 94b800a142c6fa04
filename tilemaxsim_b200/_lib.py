"""ctypes binding of libtilemaxsim_b200.so (the C ABI declared in include/tilemaxsim.h).

The library is loaded from this package directory only; if it is missing the import of any scoring
entry point raises -- there is no CPU or eager fallback. Buffers are passed as raw device pointers
(``tensor.data_ptr()``) and every call runs on ``torch.cuda.current_stream()``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libtilemaxsim_b200.so"

TMS_OK = 0
TMS_ERR_INVALID = 1
TMS_ERR_UNSUPPORTED = 2
TMS_ERR_CUDA = 3
TMS_ERR_TIMEOUT = 4
TMS_ERR_WORKSPACE = 5
TMS_ERR_TOO_LARGE = 6
TMS_ERR_BAD_OFFSETS = 7

TMS_F16, TMS_BF16, TMS_F32 = 0, 1, 2
TMS_OUT_SCORE, TMS_OUT_TOKEN_MAX = 0, 1
TMS_PQ_FAST, TMS_PQ_EXACT, TMS_PQ_PRECISE = 0, 1, 2

DTYPE_CODE = {torch.float16: TMS_F16, torch.bfloat16: TMS_BF16, torch.float32: TMS_F32}

# (name, restype, argtypes) of every exported symbol; test_abi checks the header declares the same.
_i64, _i32, _u64, _sz, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_void_p
SIGNATURES = {
    "tms_strerror": (ctypes.c_char_p, [_i32]),
    "tms_version": (ctypes.c_char_p, []),
    "tms_last_device_error": (_i32, [_vp, ctypes.POINTER(ctypes.c_uint32)]),
    "tms_set_debug": (None, [_u64, _i32]),
    "tms_validate_offsets": (_i32, [_vp, _i64, _i64, _vp]),
    "tms_dense_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i64, _i32]),
    "tms_topk_pack": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp]),
    "tms_topk_merge_packed": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "tms_ivf_candidates": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp]),
    "tms_gather_offsets": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp]),
    "tms_gather_docs": (_i32, [_vp, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp]),
    "tms_mask_candidates": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, ctypes.c_float, _vp]),
    "tms_dense_maxsim": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _vp, _i32,
                                _vp, _sz, _vp]),
    "tms_dense_maxsim_noalloc": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _vp,
                                        _i32, _vp]),
    "tms_dense_plan_info": (_i32, [_i32, _i64, _i64, _i64, _i64, _i64, _i32, _i32,
                                   ctypes.POINTER(ctypes.c_int64)]),
    "tms_pq_table": (_i32, [_vp, _i32, _i64, _i64, _vp, _i32, _i64, _i64, _i64, _vp, _vp]),
    "tms_pq_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "tms_pq_maxsim": (_i32, [_vp, _i32, _i64, _i64, _vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64,
                             _i64, _vp, _i32, _vp, _sz, _vp]),
    "tms_dense_topk_workspace_size": (_sz, [_i32, _i64, _i64, _i64, _i64, _i64, _i64]),
    "tms_dense_maxsim_topk": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64,
                                     _i64, _vp, _vp, _vp, _sz, _vp]),
    "tms_residual_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "tms_residual_maxsim": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i64, _vp, _i64,
                                   _i64, _vp, _vp, _sz, _vp]),
    "tms_topk_workspace_size": (_sz, [_i64, _i64, _i64]),
    "tms_topk": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _sz, _vp]),
}

_lib = None


class TileMaxSimError(RuntimeError):
    """A non-OK status from the C ABI."""

    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {strerror(code)} (status {code})")


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads (once) and returns the shared library, with argtypes/restypes set."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build it with `python -m tilemaxsim_b200.build` (nvcc, sm_100a). "
            "tilemaxsim_b200 has no CPU fallback.")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def strerror(code: int) -> str:
    return load().tms_strerror(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != TMS_OK:
        raise TileMaxSimError(code, what)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("tilemaxsim_b200 scores CUDA tensors only (no CPU fallback); "
                             f"got {getattr(t, 'device', type(t))}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def workspace(nbytes: int, device: torch.device, align: int = 1024) -> tuple[torch.Tensor, int]:
    """A device byte buffer from torch's caching allocator and its `align`-aligned address."""
    if nbytes <= 0:
        return torch.empty(0, dtype=torch.uint8, device=device), 0
    buf = torch.empty(nbytes + align, dtype=torch.uint8, device=device)
    addr = buf.data_ptr()
    return buf, (addr + align - 1) // align * align


def last_device_error(device: torch.device | None = None) -> tuple[int, int]:
    """(status, raw word) of the device error word; synchronises the current stream."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    word = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        rc = load().tms_last_device_error(ctypes.c_void_p(stream_handle(dev)), ctypes.byref(word))
    return rc, word.value
