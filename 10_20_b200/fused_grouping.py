"""Drop-in for the ``_sort`` op of ``v1_native/fused_grouping.py`` (:64-76).

``_sort[(4096 // N, heads)](P, O, S, FLAG, N)`` stable-sorts every N-record
segment of the [heads, 4096] score layout by score descending (ties by
position, +0 == -0) and writes the permuted member ids to O; a no-op unless
FLAG < 0 on the device.  Backed by the sm_100a bitonic kernel of libv1x.so.

``group_offsets`` is an extension with no reference counterpart: for integer
group keys carried as float scores it returns each segment's descending
exclusive key offsets, i.e. where each group starts in the sorted output.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr, require
from .kernels import _Op


def _sort_impl(grid, P, O, S, FLAG, N):
    require(P.dtype == torch.int32 and O.dtype == torch.int32 and S.dtype == torch.float32,
            "_sort: P/O int32, S float32")
    require(FLAG.dtype == torch.int32, "_sort: FLAG int32")
    groups = int(grid[0])
    heads = int(grid[1]) if len(grid) > 1 else 1
    _lib.call("v1x_sort_segments", ptr(P), ptr(O), ptr(S), ptr(FLAG), int(N), groups, heads,
              _lib.stream_of(P), device=P.device)


_sort = _Op(_sort_impl)
_sort.__doc__ = __doc__


def group_offsets(S: torch.Tensor, N: int, heads: int, key_range: int) -> torch.Tensor:
    """[heads * 4096/N, key_range + 1] int32 offsets of descending integer keys."""
    groups = 4096 // N
    out = torch.empty((heads * groups, key_range + 1), dtype=torch.int32, device=S.device)
    _lib.call("v1x_group_offsets", ptr(S), ptr(out), int(N), groups, int(heads), int(key_range),
              _lib.stream_of(S), device=S.device)
    return out


def sort_grouped(P: torch.Tensor, O: torch.Tensor, S: torch.Tensor, FLAG: torch.Tensor, N: int, heads: int,
                 key_range: int, offsets: torch.Tensor | None = None) -> torch.Tensor:
    """Extension: ``_sort`` and ``group_offsets`` in one launch (N in 256..4096):
    writes the permutation to O and returns the offsets [heads * 4096/N,
    key_range + 1], equal to the two separate ops."""
    require(P.dtype == torch.int32 and O.dtype == torch.int32 and S.dtype == torch.float32,
            "sort_grouped: P/O int32, S float32")
    groups = 4096 // N
    if offsets is None:
        offsets = torch.empty((heads * groups, key_range + 1), dtype=torch.int32, device=S.device)
    _lib.call("v1x_sort_segments_grouped", ptr(P), ptr(O), ptr(S), ptr(FLAG), ptr(offsets), int(N), groups,
              int(heads), int(key_range), _lib.stream_of(S), device=S.device)
    return offsets
