"""ctypes binding of ``libv1x.so`` (the C ABI declared in include/v1x.h).

The library is required: there is no CPU or Triton fallback.  Importing this
module does not load it; the first call does, and raises if the shared
library is missing or fails to load.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("V1X_LIB", Path(__file__).resolve().parent / "libv1x.so"))

V1X_OK = 0
V1X_ERR_INVALID = -1
V1X_ERR_CUDA = -2
V1X_ERR_UNSUPPORTED = -3
V1X_STATUS_ARENA_EXHAUSTED = 1
V1X_STATUS_TIMEOUT = 2
V1X_STATUS_BAD_PAGE = 3
V1X_STATUS_CAPACITY = 4

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float

# name -> argument types (return type is int unless noted)
SIGNATURES = {
    "v1x_version": [],
    "v1x_last_error": [],
    "v1x_route": [P, I64, I64, P, P, P, I32, I64, I64, P, P, I64, P, I64, I32, I64, P],
    "v1x_topk": [P, I64, I64, P, P, I64, P, P, I64, P, I32, I64, P, P, P, P, P, I64, I64, I32, P,
                 I64, I32, I32, P, I64, I32, I64, P],
    "v1x_sort_segments": [P, P, P, P, I64, I64, I64, P],
    "v1x_group_offsets": [P, P, I64, I64, I64, I64, P],
    "v1x_sort_segments_grouped": [P, P, P, P, P, I64, I64, I64, I64, P],
    "v1x_fingerprint": [P, P, P, P, I64, P],
    "v1x_match_pages": [P, P, P, P, P, P, P, P, P, I64, I64, P],
    "v1x_allocate": [P, P, P, P, P, P, P, P, P],
    "v1x_publish": [P, P, P, P, P, P, P, P, P, P, P, P, P, P],
    "v1x_release": [P, P, P, P, P],
    "v1x_release_many": [P, P, P, I64, P, P, P, P],
    "v1x_prepare_buckets": [P, P, P, P, P, P, I64, I64, P, P, P, P, P, P, P, P, P, P, P, P, P, P, I64, P, I64, I64,
                            P, P, P],
    "v1x_query_metadata": [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, P, I64, P],
    "v1x_query_lengths": [P, P, P, I64, I64, I64, I64, I64, I64, P],
    "v1x_fine_table_shared": [P, P, I32, P, P, P, I64, I64, I64, I64, I64, I64, P],
    "v1x_stage_tail_shared": [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, P],
    "v1x_mask_fine": [P, P, I32, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, P],
    "v1x_reduce_centers": [P, P, P, I64, I64, I64, I64, P],
    "v1x_output_ids": [P, P, P, P, P, P, I32, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I32,
                       I32, I64, I64, P],
    "v1x_expand_logical": [P, P, I64, I64, I64, P],
    "v1x_topk_transform": [P, I64, I64, P, P, I64, I64, P, P, P, I64, I64, P],
    "v1x_mask_scores": [P, I64, I64, P, I64, P, I64, P, I64, I64, I64, P],
    "v1x_query_stage": [P, P, P, P, I64, P, P, P, I64, P, P, P, P, P, P, I64, I64, I64, I64, P],
    "v1x_score_fp8": [P, P, P, I64, P, P, I64, P, I64, I64, P, I64, I64, I32, I32, I32, P, I64, P],
    "v1x_score_fp8_ex": [P, P, P, I64, P, P, I64, P, I64, I64, P, I64, I64, I32, I32, I32, I32, I64, P, I64, P],
    "v1x_mqa_logits_fp8": [P, P, P, P, I64, P, P, P, I64, I64, I32, I32, I64, P],
    "v1x_mqa_logits_fp8_grouped": [P, P, P, P, I64, P, P, P, I64, I64, I64, I64, I32, P, P],
    "v1x_score_fp8_grouped": [P, P, P, I64, I64, P, P, I64, I64, P, P, P, P, P, I64, I64, I64, I64, I32, P, P],
    "v1x_pack_q": [P, I32, I64, I64, I64, I64, I64, I64, F32, P, P, P],
    "v1x_selftest_wait_timeout": [I64, P, P, P],
    "v1x_query_prepare": [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, P, P, P, P, P, I64, I64, I64, P],
    "v1x_route_pages": [P, I64, P, P, P, I32, I64, I64, P, P, I64, P, I64, I32, I64, P],
    "v1x_gather_slots": [P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                         P],
    "v1x_build_workspace_bytes": [I64],
    "v1x_build_buckets": [P, I64, P, P, P, P, P, P, P, P, I64, P],
    "v1x_build_buckets_noalloc": [P, I64, P, P, P, P, P, P, P, I64, P],
    "v1x_initialize": [P, I64, P, P, P, P, P, P, P],
    "v1x_group_init": [P, I32, P, P, P, P, I64, I64, I64, I64, P],
    "v1x_group_dots": [P, P, P, P, P, I64, I64, I32, I64, I64, P],
    "v1x_group_anchor": [P, P, P, P, I64, I32, I64, I64, P],
    "v1x_assemble": [P, I64, P, P, P, P, P, P, P],
    "v1x_stage_union": [P, I64, P, I64, P, I64, P, P, I64, P, P, I64, I64, P, P],
    "v1x_shared_tables": [P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I32, I64, P],
    "v1x_shared_normalize": [P, I64, P, P, P, P, P, I64, P, I64, I64, I64, I64, I32, I64, P],
    "v1x_shared_map_topk": [P, P, P, P, P, P, P, I64, P, I64, P, P, I64, I64, I64, I64, I64, P],
    "v1x_route_physical": [P, I64, P, P, P, P, P, I64, I64, I64, P],
    "v1x_select_fused": [P, P, I64, P, P, I64, I64, P, P, I64, P, I64, P, I64, P, I64, P, I64, I64, I64, I64, I64,
                         I64, P, P, P, P, P, P, P, P, P, P, P, I64, P, I64, I64, P, P],
}
# entry points whose return type is not int
RESTYPES = {"v1x_last_error": ctypes.c_char_p, "v1x_build_workspace_bytes": ctypes.c_int64}

_lock = threading.Lock()
_lib = None


class V1xError(RuntimeError):
    """A v1x entry point rejected its arguments or failed to launch."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise V1xError(f"v1x CUDA library not built: {LIB_PATH} is missing "
                                   "(run __graft_entry__.build() or python 10_20_b200/build.py)")
                h = ctypes.CDLL(str(LIB_PATH))
                for name, args in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = RESTYPES.get(name, ctypes.c_int)
                _lib = h
    return _lib


def call(name: str, *args, device: torch.device | None = None):
    """Invoke an entry point (with `device` current) and raise on a non-zero code."""
    fn = getattr(lib(), name)
    if device is not None and device.index is not None and device.index != torch.cuda.current_device():
        with torch.cuda.device(device):
            rc = fn(*args)
    else:
        rc = fn(*args)
    if rc != V1X_OK:
        msg = lib().v1x_last_error().decode(errors="replace")
        if rc == V1X_ERR_INVALID:
            raise ValueError(f"{name}: {msg}")
        raise V1xError(f"{name} failed ({rc}): {msg}")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"expected a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError("v1x kernels take CUDA tensors only (there is no CPU path)")
    return t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def same_device(*ts):
    devs = {t.device for t in ts if t is not None}
    require(len(devs) <= 1, f"tensors on different devices: {devs}")
