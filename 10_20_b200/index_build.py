"""Index build of 1024-token buckets: the first stages of the reference's
``Build.compute`` (sglang/srt/layers/attention/v1_deepseek/runtime.py:170-233).

Per bucket the reference runs ``initialize`` (DS/kernels.py:9-29), seven levels
of ``_dots`` x3 / ``_anchor`` x2 / ``_sort`` (NA/fused_grouping.py:39-76, n =
1024 .. 16) and ``assemble`` (DS/kernels.py:32-54): 44 dependent launches that
turn the bucket's 16 native pages into 16 reordered tmp pages (the members of
each 8-token group adjacent), 128 FP8 centres in 2 centre pages and the
logical position of every reordered slot.

``BucketBuilder.build`` does all of that for any number of buckets in one
launch of ``v1x_build_buckets`` (one 8-CTA thread-block cluster per bucket),
producing the reference's ``Build.tmp`` / ``.centers`` / ``.mapping`` (and the
final member order ``Build.perm[current]``) for every bucket.  The builder owns
its workspace and output buffers and reuses them between calls.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr, require

PAGE_BYTES = 8448


class BucketBuilder:
    """Reusable buffers for building up to `max_buckets` buckets per launch
    (larger requests are split into launches of that many)."""

    def __init__(self, device, max_buckets: int = 128):
        require(max_buckets >= 1, "max_buckets must be positive")
        self.device = torch.device(device)
        self.max_buckets = int(max_buckets)
        self._cap = 0

    def _ensure(self, n: int):
        if n <= self._cap:
            return
        d = self.device
        self.tmp = torch.empty((n, 16, PAGE_BYTES), dtype=torch.uint8, device=d)
        self.centers = torch.empty((n, 2, PAGE_BYTES), dtype=torch.uint8, device=d)
        self.mapping = torch.empty((n, 16, 64), dtype=torch.int32, device=d)
        self.perm = torch.empty((n, 1024), dtype=torch.int32, device=d)
        self.starts = torch.empty(n, dtype=torch.int32, device=d)
        nbytes = int(_lib.lib().v1x_build_workspace_bytes(n))
        self.work = torch.empty(nbytes, dtype=torch.uint8, device=d)
        self._cap = n

    def build(self, native: torch.Tensor, source: torch.Tensor, starts, status: torch.Tensor | None = None):
        """native: packed pool uint8 [P, 8448] (or its [P, 64, 1, 132] view);
        source: int32 [n, 16] native page of every bucket page (device);
        starts: the first logical token of every bucket (sequence of ints or an
        int32 device tensor).  Returns views (tmp [n, 16, 8448], centers
        [n, 2, 8448], mapping [n, 16, 64], perm [n, 1024]) valid until the next
        call.  A source page outside the pool reads as zeros and writes
        V1X_STATUS_BAD_PAGE to `status` (when given)."""
        require(native.dtype == torch.uint8 and native.is_cuda and native.is_contiguous()
                and native.numel() % PAGE_BYTES == 0, "native: contiguous uint8 packed page pool")
        require(source.dtype == torch.int32 and source.ndim == 2 and source.shape[1] == 16
                and source.is_contiguous() and source.device == native.device, "source: int32 [n, 16] on the pool's device")
        n = source.shape[0]
        require(n <= self.max_buckets, f"at most {self.max_buckets} buckets per call")
        self._ensure(max(n, 1))
        if isinstance(starts, torch.Tensor):
            require(starts.dtype == torch.int32 and starts.numel() == n, "starts: int32 [n]")
            st = starts.to(self.device, non_blocking=True)
        else:
            vals = [int(x) for x in starts]
            require(len(vals) == n, "starts: one value per bucket")
            st = self.starts[:n]
            st.copy_(torch.tensor(vals, dtype=torch.int32), non_blocking=False)
        if n:
            _lib.call("v1x_build_buckets", ptr(native), native.numel() // PAGE_BYTES, ptr(source), ptr(st),
                      ptr(self.tmp), ptr(self.centers), ptr(self.mapping), ptr(self.perm), ptr(self.work),
                      ptr(status), n, _lib.stream_of(native), device=native.device)
        return self.tmp[:n], self.centers[:n], self.mapping[:n], self.perm[:n]


def build_buckets(native, source, starts, status=None):
    """One-shot form of BucketBuilder.build (allocates its buffers)."""
    b = BucketBuilder(native.device, max(int(source.shape[0]), 1))
    tmp, centers, mapping, perm = b.build(native, source, starts, status)
    return tmp.clone(), centers.clone(), mapping.clone(), perm.clone()
