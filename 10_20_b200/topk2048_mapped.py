"""Drop-in for the v1_native backend's Top-2048 with the original-position
mapping (``NA/deps/topk2048_mapped_20261012.py``: TopK-v2's transform whose
output goes through ``original_ids``), backed by ``v1x_topk_transform``."""
from __future__ import annotations

from functools import lru_cache

import torch

from .topk2048 import _Module, transform


class _MappedModule(_Module):
    def topk_transform(self, scores, seq_lens, page_table, page_indices, page_size, metadata, raw_indices=None,
                       original_ids=None):
        if metadata.shape != (scores.shape[0] + 1, 2):
            raise ValueError("invalid metadata shape")
        transform(scores, seq_lens, page_table, page_indices, page_size, raw_indices, original_ids)


@lru_cache(None)
def module():
    return _MappedModule()


def mapped_top2048(scores, table, original_ids, return_raw=False):
    """NA/deps/topk2048_mapped_20261012.py:13-21: out[r, t] = original_ids[
    table[r, raw // 64] * 64 + raw % 64] for each row's Top-2048 raw candidate
    (-1 for empty slots), plus the raw indices when return_raw."""
    assert original_ids.dtype == torch.int32 and original_ids.is_contiguous()
    rows, width = scores.shape
    lengths = torch.full((rows,), width, device=scores.device, dtype=torch.int32)
    out = torch.empty((rows, 2048), device=scores.device, dtype=torch.int32)
    raw = torch.empty_like(out) if return_raw else None
    transform(scores, lengths, table, out, 64, raw, original_ids)
    return (out, raw) if return_raw else out
