"""Drop-in for ``v1_deepseek/query_fused.py``: ``module()`` exposing ``route`` and
``topk`` with the reference's argument lists (V1QueryKernel::route and ::topk,
sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:155-220), backed by the sm_100a
kernels of libv1x.so.

Tensors are validated like the reference's TensorMatcher checks (shape, dtype,
device, strides) and a violation raises ValueError before anything launches.
Both calls launch on the current CUDA stream, allocate nothing and never
synchronise, so they can be captured in a CUDA graph.
"""
from __future__ import annotations

import functools

import torch

from . import _lib
from ._lib import ptr, require


def _check_2d(t, name, rows, dtype, cols=None, row_stride_ok=False):
    require(isinstance(t, torch.Tensor) and t.is_cuda, f"{name}: CUDA tensor required")
    require(t.dim() == 2, f"{name}: expected 2 dims, got {tuple(t.shape)}")
    require(t.dtype == dtype, f"{name}: expected {dtype}, got {t.dtype}")
    require(t.shape[0] == rows, f"{name}: expected {rows} rows, got {t.shape[0]}")
    if cols is not None:
        require(t.shape[1] == cols, f"{name}: expected {cols} columns, got {t.shape[1]}")
    if t.shape[1] > 0 and t.shape[0] > 1 and not row_stride_ok:
        require(t.stride(1) == 1 and t.stride(0) == t.shape[1], f"{name}: must be contiguous")
    elif t.shape[1] > 0:
        require(t.stride(1) == 1, f"{name}: last dim must be contiguous")


def _check_1d(t, name, rows, dtype=torch.int32):
    require(isinstance(t, torch.Tensor) and t.is_cuda, f"{name}: CUDA tensor required")
    require(t.dim() == 1 and t.shape[0] == rows, f"{name}: expected shape ({rows},), got {tuple(t.shape)}")
    require(t.dtype == dtype, f"{name}: expected {dtype}, got {t.dtype}")
    require(t.is_contiguous() or rows <= 1, f"{name}: must be contiguous")


def _selected(selected, rows):
    require(selected.dtype in (torch.int32, torch.int64), "selected: int32 or int64 required")
    _check_2d(selected, "selected", rows, selected.dtype)
    return 1 if selected.dtype == torch.int64 else 0


class V1QueryModule:
    """The object returned by :func:`module` (reference: DS/query_fused.py:4-10)."""

    @staticmethod
    def route(scores, lens, takes, selected, pages, rt, ft, tail_rows, capacity, fill_table):
        """fused.route (VQ:155-180): page max of 8 centres + stable top pages (+ fine table)."""
        B = scores.shape[0] if scores.dim() == 2 else -1
        _check_2d(scores, "scores", B, torch.float32, row_stride_ok=True)
        _check_1d(lens, "lens", B)
        _check_1d(takes, "takes", B)
        sel64 = _selected(selected, B)
        _check_2d(rt, "rt", B, torch.int32, cols=int(pages))
        _check_2d(ft, "ft", B, torch.int32)
        _check_1d(tail_rows, "tail_rows", B)
        _lib.same_device(scores, lens, takes, selected, rt, ft, tail_rows)
        _lib.call("v1x_route", ptr(scores), scores.stride(0) if B > 0 else scores.shape[1],
                  scores.shape[1], ptr(lens), ptr(takes), ptr(selected), sel64, selected.shape[1],
                  int(pages), ptr(rt), ptr(ft), ft.shape[1], ptr(tail_rows), int(capacity),
                  int(bool(fill_table)), B, _lib.stream_of(scores), device=scores.device)

    @staticmethod
    def route_pages(page_scores, lens, takes, selected, pages, rt, ft, tail_rows, capacity, fill_table):
        """Extension: fused.route over per-page scores (max of each page's 8 centres)."""
        B = page_scores.shape[0] if page_scores.dim() == 2 else -1
        _check_2d(page_scores, "page_scores", B, torch.float32, row_stride_ok=True)
        _check_1d(lens, "lens", B)
        _check_1d(takes, "takes", B)
        sel64 = _selected(selected, B)
        _check_2d(rt, "rt", B, torch.int32, cols=int(pages))
        _check_2d(ft, "ft", B, torch.int32)
        _check_1d(tail_rows, "tail_rows", B)
        require(page_scores.shape[1] >= int(pages), "page_scores: need >= pages columns")
        _lib.same_device(page_scores, lens, takes, selected, rt, ft, tail_rows)
        _lib.call("v1x_route_pages", ptr(page_scores), page_scores.stride(0) if B > 1 else page_scores.shape[1],
                  ptr(lens), ptr(takes), ptr(selected), sel64, selected.shape[1], int(pages), ptr(rt), ptr(ft),
                  ft.shape[1], ptr(tail_rows), int(capacity), int(bool(fill_table)), B,
                  _lib.stream_of(page_scores), device=page_scores.device)

    @staticmethod
    def topk(scores, fine_lens, members, rt, nt, selected, lens, takes, physical, logical, raw,
             window, mask, expanded, physical_output, bucket_from_rank, fine_table, direct_fine):
        """fused.topk (VQ:181-220): mask + Top-T + raw->logical->physical (+ x4 expansion)."""
        B = scores.shape[0] if scores.dim() == 2 else -1
        _check_2d(scores, "scores", B, torch.float32, row_stride_ok=True)
        _check_1d(fine_lens, "fine_lens", B)
        require(members.dim() == 2 and members.shape[1] == 64 and members.dtype == torch.int32
                and members.is_contiguous(), "members: expected contiguous int32 [N, 64]")
        P = rt.shape[1] if rt.dim() == 2 else -1
        _check_2d(rt, "rt", B, torch.int32, cols=P)
        _check_2d(nt, "nt", B, torch.int32, cols=P)
        sel64 = _selected(selected, B)
        _check_1d(lens, "lens", B)
        _check_1d(takes, "takes", B)
        T = physical.shape[1] if physical.dim() == 2 else -1
        for name, t in (("physical", physical), ("logical", logical), ("raw", raw)):
            _check_2d(t, name, B, torch.int32, cols=T)
        require(expanded.dim() == 2 and expanded.shape[0] == B and expanded.dtype == torch.int32,
                "expanded: expected int32 [B, 0 or 4*topk+64]")
        es = expanded.shape[1]
        if es:
            _check_2d(expanded, "expanded", B, torch.int32)
        _check_2d(fine_table, "fine_table", B, torch.int32)
        _lib.same_device(scores, fine_lens, members, rt, nt, selected, lens, takes, physical,
                         logical, raw, fine_table)
        _lib.call("v1x_topk", ptr(scores), scores.stride(0) if B > 0 else scores.shape[1],
                  scores.shape[1], ptr(fine_lens), ptr(members), members.shape[0], ptr(rt), ptr(nt),
                  P, ptr(selected), sel64, selected.shape[1], ptr(lens), ptr(takes), ptr(physical),
                  ptr(logical), ptr(raw), T, int(window), int(bool(mask)),
                  ptr(expanded) if es else None, es, int(bool(physical_output)),
                  int(bool(bucket_from_rank)), ptr(fine_table), fine_table.shape[1],
                  int(bool(direct_fine)), B, _lib.stream_of(scores), device=scores.device)


@functools.lru_cache(maxsize=None)
def module() -> V1QueryModule:
    """Return the route/topk operator module (loads libv1x.so on first use)."""
    _lib.lib()
    return V1QueryModule()
