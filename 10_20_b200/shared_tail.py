"""Drop-in for the reference's published-end shared-tail experiment: one
request's chunk of query rows shares one staged copy of its sink and tail pages.

Reference modules and the names kept here:
  experiments/tail_union_lab_20261021/union.py        stage_union[grid](...), launch(...),
                                                      PreparedStage (:16-83)
  experiments/fine_pool_shared_20261021/kernels.py    tables, normalize, map_topk (:13-76)
  experiments/fine_pool_shared_20261021/route_shared.py  route(...) over
                                                      route_shared.cu:12-80 (route_physical)

Every op launches an sm_100a kernel of libv1x.so on the current stream, reads
the published index end from its device word (so a captured graph follows it
when the word changes), allocates nothing and never synchronises.  A row's
candidates are its first min(n, S) tokens and [t, n) with t = max(s, min(end,
n, max(s, n - W))); the union copy holds the chunk's sink pages and tail pages
once for all rows.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr, require
from .kernels import _Op

PAGE_BYTES = 8448


def bounds(n, end, sink, window):
    """(s, t, count) of a row of n visible tokens (union.py:10-14)."""
    s = min(n, sink)
    t = max(s, min(min(max(end, 0), n), max(s, n - window)))
    return s, t, s + n - t


def _pages_of(t):
    return t.numel() * t.element_size() // PAGE_BYTES


def _stage_union(grid, SRC, NT, LENS, INDEXED_END, DST, META, DESC, R, S, W, B=512, PAGE=False):
    """union.py:16-40.  SRC / DST: int32 (or uint8) views of packed page pools."""
    require(SRC.is_contiguous() and DST.is_contiguous(), "stage_union: contiguous pools")
    require(NT.dtype == torch.int32 and LENS.dtype == torch.int32 and META.dtype == torch.int32
            and DESC.dtype == torch.int32 and INDEXED_END.dtype == torch.int32, "stage_union: int32 metadata")
    _lib.call("v1x_stage_union", ptr(SRC), _pages_of(SRC), ptr(NT), NT.numel(), ptr(LENS), int(R), ptr(INDEXED_END),
              ptr(DST), _pages_of(DST), ptr(META), ptr(DESC), int(S), int(W), None, _lib.stream_of(LENS),
              device=LENS.device)


stage_union = _Op(_stage_union)


def launch(src, nt, lens, indexed_end, dst, meta, desc, sink, window, block=512, page=False, warps=4):
    """union.py:46-48."""
    stage_union[(1,)](src.view(torch.int32), nt, lens, indexed_end, dst.view(torch.int32), meta, desc,
                      lens.numel(), sink, window, block, page)


class PreparedStage:
    """union.py:50-83: checked views and launch parameters bound once; calling it
    stages the union for the current lens / nt / indexed_end (graph-capturable).
    The caller sizes dst for every length it will replay and keeps src alive."""

    def __init__(self, src, nt, lens, indexed_end, dst, meta, desc, sink, window, block=None, warps=4):
        require(src.dtype == dst.dtype == torch.uint8, "src/dst: uint8 packed pools")
        require(src.is_contiguous() and dst.is_contiguous(), "src/dst: contiguous")
        require(src.ndim == dst.ndim == 2 and src.shape[1] == dst.shape[1] == PAGE_BYTES, "src/dst: [pages, 8448]")
        require(nt.ndim == lens.ndim == 1 and lens.numel() > 0, "nt/lens: 1-D, at least one row")
        require(nt.is_contiguous() and lens.is_contiguous(), "nt/lens: contiguous")
        require(nt.dtype == lens.dtype == meta.dtype == desc.dtype == indexed_end.dtype == torch.int32,
                "nt/lens/meta/desc/indexed_end: int32")
        require(indexed_end.shape == (1,) and indexed_end.is_contiguous(), "indexed_end: [1]")
        require(meta.shape == (lens.numel(), 3) and desc.numel() == 4, "meta: [rows, 3], desc: [4]")
        require(meta.is_contiguous() and desc.is_contiguous(), "meta/desc: contiguous")
        require(all(x.device == src.device for x in (nt, lens, indexed_end, dst, meta, desc)) and src.is_cuda,
                "all tensors on the source pool's CUDA device")
        require(sink >= 0 and window >= 0, "sink/window: non-negative")
        self.args = (src, nt, lens, indexed_end, dst, meta, desc, sink, window)

    def __call__(self):
        src, nt, lens, end, dst, meta, desc, sink, window = self.args
        _lib.call("v1x_stage_union", ptr(src), src.shape[0], ptr(nt), nt.numel(), ptr(lens), lens.numel(), ptr(end),
                  ptr(dst), dst.shape[0], ptr(meta), ptr(desc), int(sink), int(window), None,
                  _lib.stream_of(src), device=src.device)


def _tables(grid, LENS, END, TAKES, SELECTED, DESC, FT, DGLENS, CLENS, CAP, MAXTAKE, SCRATCH, FP, S, W, B=None,
            SHARED=True):
    """kernels.py:13-41; grid = (rows,)."""
    rows = int(grid[0])
    _lib.call("v1x_shared_tables", ptr(LENS), ptr(END), ptr(TAKES), ptr(SELECTED), ptr(DESC), ptr(FT), ptr(DGLENS),
              ptr(CLENS), int(CAP), int(MAXTAKE), int(SCRATCH), int(FP), int(S), int(W), int(bool(SHARED)), rows,
              _lib.stream_of(LENS), device=LENS.device)


def _normalize(grid, RAW, LENS, END, TAKES, SELECTED, MEMBERS, OUT, MAXTAKE, WIDTH, STRIDE, S, W, B=256,
               SHARED=True):
    """kernels.py:43-63; grid = (rows, cdiv(WIDTH, B))."""
    require(RAW.dtype == torch.float32 and OUT.dtype == torch.float32, "normalize: RAW/OUT float32")
    rows = int(grid[0])
    _lib.call("v1x_shared_normalize", ptr(RAW), int(STRIDE), ptr(LENS), ptr(END), ptr(TAKES), ptr(SELECTED),
              ptr(MEMBERS), MEMBERS.numel() // 64, ptr(OUT), int(MAXTAKE), int(WIDTH), int(S), int(W),
              int(bool(SHARED)), rows, _lib.stream_of(RAW), device=RAW.device)


def _map_topk(grid, IDS, VALUES, LENS, END, TAKES, SELECTED, MEMBERS, NT, LOGICAL, SLOTS, MAXTAKE, TOP, S, W,
              B=None):
    """kernels.py:65-76; grid = (rows,)."""
    require(IDS.dtype == torch.int64 and VALUES.dtype == torch.float32, "map_topk: IDS int64, VALUES float32")
    rows = int(grid[0])
    _lib.call("v1x_shared_map_topk", ptr(IDS), ptr(VALUES), ptr(LENS), ptr(END), ptr(TAKES), ptr(SELECTED),
              ptr(MEMBERS), MEMBERS.numel() // 64, ptr(NT), NT.numel(), ptr(LOGICAL), ptr(SLOTS), int(MAXTAKE),
              int(TOP), int(S), int(W), rows, _lib.stream_of(IDS), device=IDS.device)


tables = _Op(_tables)
normalize = _Op(_normalize)
map_topk = _Op(_map_topk)


def route(scores, published, budgets, rt, selected, takes):
    """route_shared.py:18-19 / route_shared.cu:56-80: the top published pages per
    row as physical ids.  scores f32 [R, P*8]; published, budgets, takes int32
    [R]; rt int32 [R, P]; selected int32 [R, M] (M <= P <= 4096)."""
    require(scores.is_cuda and scores.dtype == torch.float32 and scores.dim() == 2 and scores.is_contiguous(),
            "scores must be contiguous CUDA float32 [R,P*8]")
    require(rt.dim() == 2 and selected.dim() == 2, "rt/selected must be matrices")
    rows, pages, width = scores.shape[0], rt.shape[1], selected.shape[1]
    require(rows > 0 and 0 < pages <= 4096 and 0 < width <= pages,
            "invalid capacity (1..4096 pages, 1..pages output width)")
    require(scores.shape[1] == pages * 8 and rt.shape[0] == rows and selected.shape[0] == rows, "shape mismatch")
    for t in (published, budgets, rt, selected, takes):
        require(t.is_cuda and t.device == scores.device and t.dtype == torch.int32 and t.is_contiguous(),
                "metadata must be contiguous int32 on the scores device")
    require(published.numel() == rows and budgets.numel() == rows and takes.numel() == rows, "row metadata mismatch")
    _lib.call("v1x_route_physical", ptr(scores), scores.stride(0), ptr(published), ptr(budgets), ptr(rt),
              ptr(selected), ptr(takes), pages, width, rows, _lib.stream_of(scores), device=scores.device)
