"""Drop-in for ``v1_native/kernels.py``: the slot gather ``_gather_slots``
(:62-77) and ``GatherWorkspace`` (:80-111), backed by the sm_100a copy kernel
of libv1x.so, and ``mask_scores`` (:47-59).

Extension: the head dimension D is not fixed to 128 (the MLA latent is 576
bf16 values), and ``v_pool`` may be None for a single-output gather when K and
V are the same latent.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr, require
from .kernels import _Op


def _gather_impl(grid, K, V, REQ, IDS, KG, VG, ROWS, TOP, HEAD, KS0, KS1, KS2, VS0=0, VS1=0, VS2=0,
                 IS0=None, BLOCK=None, D=None):
    dim = int(D) if D is not None else K.shape[-1]
    require(K.element_size() in (1, 2, 4), "_gather_slots: element size 1, 2 or 4")
    require(V is None or V.element_size() == K.element_size(), "K and V element sizes differ")
    require(REQ is None or REQ.dtype == torch.int32, "REQ: int32 slot map")
    require(IDS.dtype == torch.int32, "IDS: int32")
    is0 = int(IS0) if IS0 is not None else IDS.stride(0)
    _lib.call("v1x_gather_slots", ptr(K), ptr(V), ptr(REQ), ptr(IDS), ptr(KG), ptr(VG), int(ROWS),
              int(TOP), int(HEAD), int(KS0), int(KS1), int(KS2), int(VS0), int(VS1), int(VS2), is0, dim,
              K.element_size(), _lib.stream_of(K), device=K.device)


_gather_slots = _Op(_gather_impl)
_gather_slots.__doc__ = "KG[t] = K[REQ[IDS[t]], HEAD] (zeros for negative ids); NA/kernels.py:62-77."


def mask_scores(scores, table, mapping, positions, dedup_cols=0, fixed_start=0):
    """NA/kernels.py:47-59: in place, column c of row r becomes -inf when its
    logical token l = mapping[table[r, c // 64], c % 64] is < 0, > positions[r],
    or (c < dedup_cols and (l < 64 or l >= fixed_start)); a page outside the
    mapping reads as l = -1."""
    require(scores.dtype == torch.float32 and scores.dim() == 2 and scores.stride(1) == 1, "scores: float32 rows")
    require(table.dtype == torch.int32 and table.dim() == 2 and table.stride(1) == 1, "table: int32 [rows, -1]")
    require(mapping.dtype == torch.int32 and mapping.is_contiguous(), "mapping: int32 [pages, 64]")
    require(positions.dtype == torch.int32 and positions.numel() >= scores.shape[0], "positions: int32 [rows]")
    _lib.call("v1x_mask_scores", ptr(scores), scores.stride(0), scores.shape[1], ptr(table), table.stride(0),
              ptr(mapping), mapping.numel() // 64, ptr(positions), int(dedup_cols), int(fixed_start), scores.shape[0],
              _lib.stream_of(scores), device=scores.device)


class GatherWorkspace:
    """Backend-owned reusable gather output (reference NA/kernels.py:80-111).

    ``gather`` returns views [rows, top, 1, D] of buffers allocated once and
    reused (stable addresses) until ``clear()``; raises ValueError if a call
    has more rows than the workspace.
    """

    def __init__(self, rows, device, dtype, dim: int = 128, top: int = 2048):
        self.rows, self.device, self.dtype = rows, device, dtype
        self.dim, self.top = dim, top
        self.k = self.v = None

    def release_request(self, slot):
        """Shared scratch has no request-owned contents."""

    def clear(self):
        self.k = self.v = None

    def ensure_allocated(self, need_v: bool = True):
        if self.k is None:
            self.k = torch.empty((self.rows, self.top, 1, self.dim), device=self.device, dtype=self.dtype)
        if need_v and self.v is None:
            self.v = torch.empty_like(self.k)

    def gather(self, k_pool, v_pool, request_slots, ids, head):
        rows = len(ids)
        if rows > self.rows:
            raise ValueError("Gather workspace microbatch exceeded")
        require(k_pool.dim() == 3 and k_pool.shape[-1] == self.dim, f"k_pool: [slots, heads, {self.dim}]")
        self.ensure_allocated(v_pool is not None)
        k = self.k[:rows]
        v = self.v[:rows] if v_pool is not None else None
        vs = v_pool.stride() if v_pool is not None else (0, 0, 0)
        _gather_impl((1,), k_pool, v_pool, request_slots, ids, k, v, rows, self.top, head,
                     *k_pool.stride(), *vs, ids.stride(0), D=self.dim)
        return (k, v) if v_pool is not None else k
