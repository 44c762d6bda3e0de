"""Drop-in for the v1_native backend's page route (``NA/deps/route.py``:
``extension(threads, bits)`` with ``.route(scores, table, pages, take)`` and
``.route_mask(scores, table, pages, take, bitmap)``), backed by ``v1x_route``.

The reference sorts each row's page maxima (the max of a page's 8 centre
logits) descending with CUB over a blocked layout whose tie order -- page
p = rank / BASE + (rank % BASE) * 128, BASE = n / 128 for the smallest n in
{128, ..., 4096} holding the pages -- is fused.route's (VQ:26-30) for every
(threads, pages) it accepts, and writes the first `take` page ids of the
ranking to table[:, :take] (the columns after them are the caller's).  So the
ranking here is fused.route's, written through a row block allocated per call.  The
bitmap of ``route_mask`` marks the selected pages below ``pages``; the
reference also writes a 1 at row * pages + id for a padding id >= pages (an
all -inf tail of the ranking), which lands in the next row or past the buffer,
and that write is not repeated here.
"""
from __future__ import annotations

from functools import lru_cache

import torch

from . import _lib
from ._lib import ptr


def rank_pages(s, pages: int, take: int):
    """The first `take` page ids of each row's ranking (route.py's tie order,
    any 1 <= take <= pages <= 4096): a new int32 [rows, take] tensor.  s:
    float32 [rows, >= pages*8] of page centre logits, unit inner stride, row
    stride a multiple of 4.  Every buffer is allocated per call (from a captured
    graph's pool when captured), so nothing outlives the caller's references."""
    pages, take = int(pages), int(take)
    if not (0 < take <= pages <= 4096):
        raise ValueError("route: bad pages / take")
    if not (s.is_cuda and s.dtype == torch.float32 and s.dim() == 2 and s.shape[1] >= pages * 8
            and s.stride(1) == 1 and s.stride(0) % 4 == 0):
        raise ValueError("route: bad score layout")
    rows = s.shape[0]
    sel = torch.empty((rows, take), dtype=torch.int32, device=s.device)
    if rows == 0:
        return sel
    g = max(pages, 64)
    if g != pages:   # fewer than 64 pages: the route's smallest geometry, padded with -inf
        pad = torch.full((rows, g * 8), float("-inf"), dtype=torch.float32, device=s.device)
        pad[:, :pages * 8] = s[:, :pages * 8]
        s = pad
        score_cols = g * 8
    else:            # only the first `pages` pages are ranked, whatever the row holds after them
        score_cols = pages * 8
    # every page active ((n - 1) // 1024 * 16 >= pages for this length), and a
    # take below the page count (the route's identity branch is for take >= active)
    lens = torch.full((rows,), (g + 15) // 16 * 1024 + 1, dtype=torch.int32, device=s.device)
    takes = torch.full((rows,), take if take < g else g - 1, dtype=torch.int32, device=s.device)
    # without the fine-table fill the route reads neither rt nor tail_rows and
    # writes no ft: one int stands for each
    dummy = torch.zeros(1, dtype=torch.int32, device=s.device)
    _lib.call("v1x_route", ptr(s), s.stride(0), score_cols, ptr(lens), ptr(takes), ptr(sel), 0, take, g,
              ptr(dummy), ptr(dummy), take, ptr(dummy), 1, 0, rows, _lib.stream_of(s), device=s.device)
    return sel


class _Route:
    def __init__(self, threads: int, bits: int):
        if threads not in (64, 128, 256, 512) or bits not in (4, 5, 6):
            raise ValueError("threads in (64, 128, 256, 512), bits in (4, 5, 6)")
        self.threads = threads

    def route(self, s, t, pages, take):
        self._route(s, t, pages, take)

    def route_mask(self, s, t, pages, take, b):
        if not (b.is_cuda and b.dtype == torch.uint8 and b.is_contiguous() and b.shape == (s.shape[0], pages)):
            raise ValueError("bitmap: contiguous uint8 [rows, pages]")
        sel = self._route(s, t, pages, take)
        if sel is None:
            return
        # ranks past the row's pages (padding of the blocked layout, reached
        # only through -inf ties) mark the spare column, not the next row
        marks = torch.zeros((s.shape[0], int(pages) + 1), dtype=torch.uint8, device=s.device)
        marks.scatter_(1, torch.where(sel < pages, sel, pages).long(), 1)
        b.copy_(marks[:, :pages])

    def _route(self, s, t, pages, take):
        pages, take = int(pages), int(take)
        if not (s.is_cuda and t.is_cuda and s.device == t.device):
            raise ValueError("scores and table on one CUDA device")
        if s.dtype != torch.float32 or t.dtype != torch.int32 or s.dim() != 2 or t.dim() != 2 or \
                s.shape[0] != t.shape[0]:
            raise ValueError("scores float32 [rows, -1], table int32 [rows, -1]")
        if not (pages > self.threads // 2 and pages <= 4096 and 0 < take <= pages and t.shape[1] >= take):
            raise ValueError("route: bad pages / take")
        if not (s.shape[1] >= pages * 8 and s.stride(1) == 1 and s.stride(0) % 4 == 0 and t.stride(1) == 1):
            raise ValueError("route: bad score / table layout")
        if s.shape[0] == 0:
            return None
        sel = rank_pages(s, pages, take)
        t[:, :take].copy_(sel)
        return sel


@lru_cache(None)
def extension(threads: int = 256, bits: int = 4):
    return _Route(threads, bits)
