"""CPU: the C-ABI library loads, exports every declared entry point, and the
Python shims refuse to run without CUDA tensors (there is no CPU path)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "v1x.h").read_text()
    return sorted(set(re.findall(r"V1X_API\s+[\w\s\*]*?\b(v1x_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 20
    assert "v1x_route" in syms and "v1x_topk" in syms and "v1x_gather_slots" in syms


def test_library_exports_every_declared_symbol(v1x):
    lib = ctypes.CDLL(v1x.library_path())
    for s in declared_symbols():
        assert hasattr(lib, s), f"missing export {s}"
    assert lib.v1x_version() == 0x000100


def test_ctypes_table_covers_header(v1x):
    from importlib import import_module
    _lib = import_module("10_20_b200._lib")
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def declared_arg_counts():
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "v1x.h").read_text(), flags=re.S)
    out = {}
    for name, args in re.findall(r"V1X_API\s+[\w\s\*]*?\b(v1x_\w+)\s*\(([^)]*)\)", text):
        args = args.strip()
        out[name] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_ctypes_argument_counts_match_header(v1x):
    from importlib import import_module
    _lib = import_module("10_20_b200._lib")
    for name, n in declared_arg_counts().items():
        assert len(_lib.SIGNATURES[name]) == n, name


def test_shims_reject_cpu_tensors(v1x):
    from importlib import import_module
    qf = import_module("10_20_b200.query_fused")
    B, P = 4, 64
    scores = torch.zeros((B, P * 8))
    i32 = lambda *s: torch.zeros(s, dtype=torch.int32)
    with pytest.raises(ValueError):
        qf.module().route(scores, i32(B), i32(B), i32(B, 8), P, i32(B, P), i32(B, 76), i32(B), 1, True)
    gather = import_module("10_20_b200.gather")
    ws = gather.GatherWorkspace(2, "cpu", torch.bfloat16)
    with pytest.raises(ValueError):
        ws.gather(torch.zeros((8, 1, 128), dtype=torch.bfloat16), None, None,
                  torch.zeros((2, 2048), dtype=torch.int32), 0)


def test_signed_path_shims_reject_cpu_tensors(v1x):
    """The signed-score operators check their arguments on the host and refuse
    CPU tensors (there is no CPU path)."""
    from importlib import import_module
    NS = import_module("10_20_b200.native_scoring")
    T = import_module("10_20_b200.topk2048")
    G = import_module("10_20_b200.gather")
    R = import_module("10_20_b200.native_route")
    S = import_module("10_20_b200.scoring")
    i32 = lambda *s: torch.zeros(s, dtype=torch.int32)
    with pytest.raises(ValueError):
        NS.pack_q(torch.zeros((2, 4, 128), dtype=torch.bfloat16), 0.1)
    with pytest.raises(ValueError):
        NS.pack_q(torch.zeros((2, 4, 64), dtype=torch.bfloat16), 0.1)          # head dim 128 only
    with pytest.raises(ValueError):
        T.transform(torch.zeros((2, 4096)), i32(2), i32(2, 64), i32(2, 2048), 64)
    with pytest.raises(ValueError):
        T.transform(torch.zeros((2, 4096)), i32(2), i32(2, 64), i32(2, 2048), 48)  # page size not 2^k
    with pytest.raises(ValueError):
        G.mask_scores(torch.zeros((2, 128)), i32(2, 2), i32(4, 64), i32(2))
    with pytest.raises(ValueError):
        R.rank_pages(torch.zeros((2, 800)), 100, 10)
    with pytest.raises(ValueError):
        R.extension(64, 4).route(torch.zeros((2, 800)), i32(2, 10), 100, 10)
    with pytest.raises(ValueError):
        R.extension(96, 4)
    q8 = torch.zeros((32, 4, 128), dtype=torch.uint8)
    with pytest.raises(ValueError):
        S.paged_logits_grouped(q8, torch.zeros((32, 4)), torch.zeros((2, 8448), dtype=torch.uint8), i32(2), 128,
                               torch.zeros((32, 128)))
    with pytest.raises(ValueError):
        S.mqa_logits_grouped(q8, torch.zeros((32, 4)), (torch.zeros((100, 128), dtype=torch.uint8),
                             torch.zeros(100)), i32(32), i32(32))


def test_triton_style_launcher_requires_grid(v1x):
    from importlib import import_module
    K = import_module("10_20_b200.kernels")
    with pytest.raises(TypeError):
        K.release(None, None, None, None)


def test_batched_lifecycle_rejects_bad_arguments_before_any_launch(v1x):
    """Argument checks of the batched lifecycle entry points run on the host
    before any CUDA call, so they are exercised here without a GPU: NULL
    buffers and oversize batches return V1X_ERR_INVALID with a message."""
    from importlib import import_module
    _lib = import_module("10_20_b200._lib")
    lib = _lib.lib()
    nulls = [None] * 5
    rc = lib.v1x_prepare_buckets(*nulls, None, 0, 1, *([None] * 14), 16, None, 2, 4096, None, None, None)
    assert rc == _lib.V1X_ERR_INVALID
    assert b"NULL" in lib.v1x_last_error()
    rc = lib.v1x_prepare_buckets(*nulls, None, 0, 65, *([None] * 14), 16, None, 2, 4096, None, None, None)
    assert rc == _lib.V1X_ERR_INVALID and b"at most 64 buckets" in lib.v1x_last_error()
    rc = lib.v1x_prepare_buckets(*([1] * 5), 16, 0, 1, *([16] * 14), 16, None, 2, 4096, None, None, None)
    assert rc == _lib.V1X_ERR_INVALID and b"src_buckets" in lib.v1x_last_error()
    # host meta records and source ids: an id outside [0, src_buckets) is
    # rejected before anything is launched (the device pointers are never used)
    import numpy as np
    meta = np.zeros((2, 4), np.int32)
    src = np.array([0, 5], np.int32)
    rc = lib.v1x_prepare_buckets(16, 16, 16, 16, meta.ctypes.data, src.ctypes.data, 5, 2, *([16] * 13), None, 0,
                                 None, 0, 4096, 16, None, None)
    assert rc == _lib.V1X_ERR_INVALID and b"source id 5 of bucket 1" in lib.v1x_last_error()
    rc = lib.v1x_release_many(None, None, None, 3, None, None, None, None)
    assert rc == _lib.V1X_ERR_INVALID and b"NULL" in lib.v1x_last_error()
    assert lib.v1x_release_many(None, None, None, 0, None, None, None, None) == _lib.V1X_OK
