"""Drop-in for ``v1_native/fused_grouping.py``: ``_init`` (:27-37), ``_dots``
(:39-54), ``_anchor`` (:56-63), ``_sort`` (:64-76) and ``FusedGroups`` (:78-111,
its fused mode), each op used as ``op[grid](*args)`` with the reference's
positional arguments and backed by sm_100a kernels of libv1x.so.

``_sort[(4096 // N, heads)](P, O, S, FLAG, N)`` stable-sorts every N-record
segment of the [heads, 4096] score layout by score descending (ties by
position, +0 == -0) and writes the permuted member ids to O; every op is a
no-op unless FLAG < 0 on the device.  Sums over the 128 dims follow one fixed
fp32 order (numpy's pairwise order, which the reference's kernels evaluate to
in the Triton interpreter), so repeated builds give identical groups.

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


def _heads(grid):
    return int(grid[1]) if len(grid) > 1 else 1


def _init_impl(grid, K, REQ, U, P, FLAG, START, KS0, KS1):
    """U[h, i] = K[REQ[START + i], h] / max(|.|, 1e-12), P[h, i] = START + i for
    the 4096 positions of each head (grid (256, heads))."""
    require(K.dtype in (torch.bfloat16, torch.float32), "_init: K bfloat16 or float32")
    require(U.dtype == torch.float32 and P.dtype == torch.int32 and REQ.dtype == torch.int32,
            "_init: U float32, P/REQ int32")
    _lib.call("v1x_group_init", ptr(K), int(K.dtype == torch.float32), ptr(REQ), ptr(U), ptr(P), ptr(FLAG),
              int(START), int(KS0), int(KS1), _heads(grid), _lib.stream_of(U), device=U.device)


def _dots_impl(grid, U, P, A, S, FLAG, N, START, MODE):
    """S[h, i] = dot(U[P[h, i]], anchor of the group) (MODE 2: minus S); grid
    (count // 16, heads)."""
    require(U.dtype == torch.float32 and S.dtype == torch.float32 and P.dtype == torch.int32 and
            A.dtype == torch.int32, "_dots: U/S float32, P/A int32")
    _lib.call("v1x_group_dots", ptr(U), ptr(P), ptr(A), ptr(S), ptr(FLAG), int(N), int(START), int(MODE),
              int(grid[0]) * 16, _heads(grid), _lib.stream_of(U), device=U.device)


def _anchor_impl(grid, P, A, S, FLAG, N, SLOT):
    """A[h, group, SLOT] = P at the leftmost minimum of S over the group; grid
    (count // N, heads)."""
    require(S.dtype == torch.float32 and P.dtype == torch.int32 and A.dtype == torch.int32,
            "_anchor: S float32, P/A int32")
    _lib.call("v1x_group_anchor", ptr(P), ptr(A), ptr(S), ptr(FLAG), int(N), int(SLOT), int(grid[0]) * int(N),
              _heads(grid), _lib.stream_of(S), device=S.device)


_init = _Op(_init_impl)
_dots = _Op(_dots_impl)
_anchor = _Op(_anchor_impl)


class FusedGroups:
    """Fixed-4K balanced cosine grouping over preallocated GPU scratch
    (NA/fused_grouping.py:78-111, fused mode): _init, then for n = 4096 .. 16
    three _dots, two _anchor and one _sort per level."""

    def __init__(self, heads, device):
        self.heads = heads
        self.mode = "fused"
        self.unit = torch.empty((heads, 4096, 128), device=device, dtype=torch.float32)
        self.perm = [torch.empty((heads, 4096), device=device, dtype=torch.int32) for _ in range(2)]
        self.anchor = torch.empty((heads, 256, 2), device=device, dtype=torch.int32)
        self.scores = torch.empty((heads, 4096), device=device, dtype=torch.float32)

    def run(self, k, slots, start, flag):
        if k.ndim != 3 or k.shape[1:] != (self.heads, 128) or k.stride(-1) != 1:
            raise ValueError("GPU grouping requires [slots, heads, 128] with contiguous dimensions")
        if slots.ndim != 1 or not slots.is_contiguous() or start < 0 or start + 4096 > slots.numel():
            raise ValueError("GPU grouping requires a complete 4096-key range and contiguous slot map")
        _init[(256, self.heads)](k, slots, self.unit, self.perm[0], flag, start, k.stride(0), k.stride(1))
        current = 0
        for n in (4096, 2048, 1024, 512, 256, 128, 64, 32, 16):
            p = self.perm[current]
            for mode in (0, 1, 2):
                _dots[(256, self.heads)](self.unit, p, self.anchor, self.scores, flag, n, start, mode)
                if mode < 2:
                    _anchor[(4096 // n, self.heads)](p, self.anchor, self.scores, flag, n, mode)
            _sort[(4096 // n, self.heads)](p, self.perm[1 - current], self.scores, flag, n)
            current = 1 - current
        return self.perm[current]


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
