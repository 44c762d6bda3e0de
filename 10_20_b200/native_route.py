"""Drop-in for the v1_native backend's page route (``NA/deps/route.py``:
``extension(threads, bits)`` with ``.route(scores, table, pages, take)`` and
``.route_mask(scores, table, pages, take, bitmap)``), backed by ``v1x_route``.

The reference sorts each row's page maxima (the max of a page's 8 centre
logits) descending with CUB over a blocked layout whose tie order -- page
p = rank / BASE + (rank % BASE) * 128, BASE = n / 128 for the smallest n in
{128, ..., 4096} holding the pages -- is fused.route's (VQ:26-30) for every
(threads, pages) it accepts, and writes the first `take` page ids of the
ranking to table[:, :take] (the columns after them are the caller's).  So the
ranking here is fused.route's, written through a scratch row block.  The
bitmap of ``route_mask`` marks the selected pages below ``pages``; the
reference also writes a 1 at row * pages + id for a padding id >= pages (an
all -inf tail of the ranking), which lands in the next row or past the buffer,
and that write is not repeated here.
"""
from __future__ import annotations

from functools import lru_cache

import torch

from .query_fused import module as fused_module


_SCRATCH = {}
_SCRATCH_MAX = 32


def _buffers(device, rows, pages, take):
    key = (device, rows, pages, take)
    buf = _SCRATCH.get(key)
    if buf is None:
        if len(_SCRATCH) >= _SCRATCH_MAX:
            _SCRATCH.clear()
        g = max(pages, 64)
        # all pages active: (n - 1) // 1024 * 16 >= pages
        n = (g + 15) // 16 * 1024 + 1
        # take == pages ranks every page (the route's identity branch is for
        # take >= active only)
        k = take if take < g else g - 1
        buf = dict(lens=torch.full((rows,), n, dtype=torch.int32, device=device),
                   takes=torch.full((rows,), k, dtype=torch.int32, device=device),
                   sel=torch.empty((rows, take), dtype=torch.int32, device=device),
                   rt=torch.zeros((rows, g), dtype=torch.int32, device=device),
                   ft=torch.zeros((rows, take), dtype=torch.int32, device=device),
                   tail=torch.zeros(rows, dtype=torch.int32, device=device), g=g,
                   marks=torch.empty((rows, pages + 1), dtype=torch.uint8, device=device))
        _SCRATCH[key] = buf
    return buf


def rank_pages(s, pages: int, take: int):
    """The first `take` page ids of each row's ranking (route.py's tie order,
    any 1 <= take <= pages <= 4096): int32 [rows, take], a scratch buffer that
    the next call with the same shape overwrites.  s: float32 [rows, >= pages*8]
    of page centre logits, unit inner stride, row stride a multiple of 4."""
    pages, take = int(pages), int(take)
    if not (0 < take <= pages <= 4096):
        raise ValueError("route: bad pages / take")
    if not (s.is_cuda and s.dtype == torch.float32 and s.dim() == 2 and s.shape[1] >= pages * 8
            and s.stride(1) == 1 and s.stride(0) % 4 == 0):
        raise ValueError("route: bad score layout")
    rows = s.shape[0]
    buf = _buffers(s.device, rows, pages, take)
    if rows == 0:
        return buf["sel"]
    g = buf["g"]
    if g != pages:   # fewer than 64 pages: the route's smallest geometry, padded with -inf
        pad = torch.full((rows, g * 8), float("-inf"), dtype=torch.float32, device=s.device)
        pad[:, :pages * 8] = s[:, :pages * 8]
        s = pad
    else:            # only the first `pages` pages are ranked, whatever the row holds after them
        s = s[:, :pages * 8]
    fused_module().route(s, buf["lens"], buf["takes"], buf["sel"], g, buf["rt"], buf["ft"], buf["tail"], 1, False)
    return buf["sel"]


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
        marks = _buffers(s.device, s.shape[0], int(pages), int(take))["marks"]
        marks.zero_()
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
