"""v1x_build_buckets_noalloc (the index build with its workspace inside the
library) against v1x_build_buckets (caller-supplied workspace): two calls in a
row give identical outputs; more buckets than the fixed scratch holds are
rejected.  Collected last on purpose: it must also pass after every other test
has run in the same process."""
import ctypes
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ib = importlib.import_module("10_20_b200.index_build")
_lib = importlib.import_module("10_20_b200._lib")


def _pool(seed, pages):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn((pages, 64, 128), generator=gen).to(torch.float8_e4m3fn)
    buf = torch.zeros((pages, 8448), dtype=torch.uint8)
    buf[:, :8192] = k.view(torch.uint8).reshape(pages, 8192)
    buf.view(torch.float32)[:, 2048:] = torch.rand((pages, 64), generator=gen) + 0.25
    return buf


def _noalloc(native, source, starts, status, n):
    d = native.device
    tmp = torch.empty((n, 16, 8448), dtype=torch.uint8, device=d)
    centers = torch.empty((n, 2, 8448), dtype=torch.uint8, device=d)
    mapping = torch.empty((n, 16, 64), dtype=torch.int32, device=d)
    perm = torch.empty((n, 1024), dtype=torch.int32, device=d)
    _lib.call("v1x_build_buckets_noalloc", native.data_ptr(), native.shape[0], source.data_ptr(),
              starts.data_ptr(), tmp.data_ptr(), centers.data_ptr(), mapping.data_ptr(), perm.data_ptr(),
              status.data_ptr(), n, torch.cuda.current_stream().cuda_stream, device=d)
    return tmp, centers, mapping, perm


def test_noalloc_build_matches_workspace_build(cuda_dev):
    n, pages = 8, 200
    native = _pool(12, pages).cuda()
    rng = np.random.default_rng(12)
    source = torch.from_numpy(np.stack([rng.permutation(pages)[:16] for _ in range(n)]).astype(np.int32)).cuda()
    starts = torch.arange(n, dtype=torch.int32, device="cuda") * 1024 + 4096
    ref = ib.build_buckets(native, source, starts)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):                         # the scratch is reused by the second call
        got = _noalloc(native, source, starts, status, n)
        torch.cuda.synchronize()
        for x, y in zip(got, ref):
            assert torch.equal(x, y)
    # fewer buckets than the scratch holds
    got = _noalloc(native, source[:3].contiguous(), starts[:3].contiguous(), status, 3)
    for x, y in zip(got, ref):
        assert torch.equal(x, y[:3])
    assert int(status.item()) == 0


def test_noalloc_build_rejects_oversize(cuda_dev):
    native = _pool(13, 40).cuda()
    source = torch.zeros((9, 16), dtype=torch.int32, device="cuda")
    starts = torch.zeros(9, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="at most 8 buckets"):
        _noalloc(native, source, starts, status, 9)
    assert isinstance(_lib.lib().v1x_build_buckets_noalloc, ctypes._CFuncPtr)
