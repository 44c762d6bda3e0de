"""Failure detection on the GPU without a fault: a bounded device wait that
nothing satisfies must give up after its limit, report V1X_STATUS_TIMEOUT in the
status word, and leave the context usable for the next kernel."""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L = importlib.import_module("10_20_b200._lib")
G = importlib.import_module("10_20_b200.gather")


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    elapsed = torch.zeros(1, dtype=torch.int64, device="cuda")
    limit = 20_000_000  # 20 ms
    L.call("v1x_selftest_wait_timeout", limit, status.data_ptr(), elapsed.data_ptr(),
           torch.cuda.current_stream().cuda_stream, device=status.device)
    torch.cuda.synchronize()
    assert int(status.item()) == L.V1X_STATUS_TIMEOUT
    ns = int(elapsed.item())
    assert limit <= ns < limit + 500_000_000
    # the context still runs kernels: a small gather is exact afterwards
    k = torch.arange(8 * 128, dtype=torch.float32, device="cuda").reshape(8, 1, 128).to(torch.bfloat16)
    ids = torch.tensor([[3, -1, 7, 0]], dtype=torch.int32, device="cuda")
    ws = G.GatherWorkspace(1, "cuda:0", torch.bfloat16, dim=128, top=4)
    out = ws.gather(k, None, None, ids, 0)
    exp = np.zeros((4, 128), np.float32)
    for j, i in enumerate([3, -1, 7, 0]):
        if i >= 0:
            exp[j] = k[i, 0].float().cpu().numpy()
    assert np.array_equal(out.reshape(4, 128).float().cpu().numpy(), exp)


def test_bounded_wait_rejects_bad_limits(cuda_dev):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        L.call("v1x_selftest_wait_timeout", 0, status.data_ptr(), None, 0, device=status.device)
    with pytest.raises(ValueError):
        L.call("v1x_selftest_wait_timeout", 20_000_000_000, status.data_ptr(), None, 0, device=status.device)
