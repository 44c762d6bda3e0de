"""Drop-in for the v1_native backend's Top-2048 (``NA/deps/topk2048.py``,
which JIT-loads TopK-v2's ``topk_plan`` / ``topk_transform`` from the vendored
``topk_vendor/topk_v2.cuh``), backed by ``v1x_topk_transform`` of libv1x.so.

``module()`` returns an object with the two entry points and their argument
lists; ``topk2048(scores, need_values=True)`` is the wrapper the backend calls
(NA/deps/topk2048.py:15-32).  Selection: the 2048 largest of each row by
(value desc, index asc); outputs in ascending index order (TopK-v2 leaves the
order unspecified and breaks some boundary ties by atomic order).
"""
from __future__ import annotations

from functools import lru_cache

import torch

from . import _lib
from ._lib import ptr, require


def transform(scores, seq_lens, page_table, out, page_size, raw=None, original_ids=None):
    """TopKKernel::transform (topk_v2.cuh:354-430): checks as the reference's
    TensorMatcher, then one launch."""
    require(scores.dim() == 2 and scores.dtype == torch.float32 and scores.stride(1) == 1,
            "scores: float32 [B, L] with unit inner stride")
    B, L = scores.shape
    require(scores.stride(0) % 4 == 0, "score_stride must be a multiple of 4 (16-byte vectorized load)")
    require(seq_lens.shape == (B,) and seq_lens.dtype == torch.int32, "seq_lens: int32 [B]")
    require(page_table.dim() == 2 and page_table.shape[0] == B and page_table.dtype == torch.int32 and
            (page_table.stride(1) == 1 or page_table.shape[1] == 1), "page_table: int32 [B, -1], unit inner stride")
    require(out.dim() == 2 and out.shape[0] == B and out.dtype == torch.int32 and out.is_contiguous(),
            "page_indices: int32 [B, K]")
    K = out.shape[1]
    require(0 < K <= 2048, "topk must be in (0, 2048]")
    require(page_size > 0 and page_size & (page_size - 1) == 0, "page_size must be power of 2")
    if raw is not None:
        require(raw.shape == (B, K) and raw.dtype == torch.int32 and raw.is_contiguous(), "raw_indices: int32 [B, K]")
    if original_ids is not None:
        require(original_ids.dim() == 1 and original_ids.dtype == torch.int32, "original_ids: int32 [-1]")
    devs = {t.device for t in (scores, seq_lens, page_table, out, raw, original_ids) if t is not None}
    require(len(devs) == 1 and scores.is_cuda, "all tensors on one CUDA device")
    _lib.call("v1x_topk_transform", ptr(scores), scores.stride(0), L, ptr(seq_lens), ptr(page_table),
              page_table.stride(0), int(page_size), ptr(original_ids), ptr(out), ptr(raw), K, B,
              _lib.stream_of(scores), device=scores.device)


class _Module:
    """The JIT module's surface: ``topk_plan(seq_lens, metadata, _)`` and
    ``topk_transform(scores, seq_lens, page_table, page_indices, page_size,
    metadata, raw_indices)``."""

    def topk_plan(self, seq_lens, metadata, _unused=0):
        """Fills the plan buffer [B + 1, 2] as TopK-v2 lays it out (row 0 the
        batch size, then (batch id, length) per row); the transform here does
        not need it."""
        B = seq_lens.shape[0]
        require(metadata.shape == (B + 1, 2) and metadata.dtype == torch.int32, "invalid metadata shape")
        metadata[0, 0] = B
        metadata[0, 1] = 0
        metadata[1:, 0] = torch.arange(B, device=metadata.device, dtype=torch.int32)
        metadata[1:, 1] = seq_lens

    def topk_transform(self, scores, seq_lens, page_table, page_indices, page_size, metadata, raw_indices=None):
        require(metadata.shape == (scores.shape[0] + 1, 2), "invalid metadata shape")
        transform(scores, seq_lens, page_table, page_indices, page_size, raw_indices)


@lru_cache(None)
def module():
    return _Module()


def topk2048(scores, need_values=True):
    """NA/deps/topk2048.py:15-32: (values or None, raw indices as int64) of each
    row's Top-2048 (width >= 2048)."""
    assert scores.ndim == 2 and scores.is_cuda and scores.dtype == torch.float32
    rows, width = scores.shape
    assert width >= 2048
    lengths = torch.full((rows,), width, dtype=torch.int32, device=scores.device)
    # identity pages keep the raw candidate indices
    tables = torch.arange((width + 63) // 64, device=scores.device, dtype=torch.int32)[None].expand(rows, -1)
    out = torch.empty((rows, 2048), dtype=torch.int32, device=scores.device)
    raw = torch.empty_like(out)
    transform(scores, lengths, tables, out, 64, raw)
    indices = raw.long()
    return (scores.gather(1, indices) if need_values else None), indices
