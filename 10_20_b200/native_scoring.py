"""Drop-in for the v1_native backend's signed-score selection: ``Scorer``
(NA/scoring.py:25-99), its shared-page variant ``select`` / ``select_tensors``
(NA/shared_scoring.py:9-62) and ``quantize`` (NA/grouping.py:41-44), composed
from libv1x.so's operators:

- q packing (quantise the four query heads, fold the softmax scale into the
  head weights; padded to the 32 heads of the reference's scorer, or kept at
  four for the grouped scorer): ``v1x_pack_q``;
- signed FP8 logits (the no-ReLU DeepGEMM fork the reference loads): by
  default the grouped tensor-core scorer (``scoring.paged_logits_grouped``,
  ``scoring.mqa_logits_grouped`` for the ``dsa`` mode: 32 query rows x 4 heads
  per MMA operand, with the validity mask and ``mask_scores`` in the same pass);
  with ``Scorer.impl`` "tensor_core" or "simt" the per-row scorers
  (``scoring.fp8_paged_mqa_logits`` / ``fp8_mqa_logits``, ``relu=False``) and a
  separate ``gather.mask_scores``;
- page route: ``native_route`` (route.py's tie order);
- the mapped Top-2048: ``topk2048_mapped``; the ``dsa`` mode's plain
  Top-2048: ``topk2048``.

The backend's host state (its arenas, ``state`` / ``arena`` objects) is the
caller's, duck-typed as in the reference: ``state.pages``, ``state.centers``,
``state.valid``, ``state.fine``, ``state.mapping`` (flat [heads, pages * 64]),
``state.flat_k`` / ``state.flat_scale`` for ``dsa``; the shared variant reads
``state.arena`` (``centers``, ``valid``, ``fine``, ``mapping``, ``identity``,
``record()``), ``state.table``, ``state.wait()``, ``state.full_bucket_append``
and ``state.fixed_start``.  Query graphs (the reference's
``SGLANG_V1_*QUERY_GRAPH`` options) need the shared arenas' graph pools, which
the caller supplies as ``state.query_graph_pool`` exactly as in the reference.
"""
from __future__ import annotations

import os

import torch

from . import _lib
from ._lib import ptr, require
from . import scoring
from .gather import mask_scores
from .native_route import extension, rank_pages
from .topk2048 import topk2048
from .topk2048_mapped import mapped_top2048

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def query_graph_enabled(decode: bool = False) -> bool:
    """NA/config.py:16-19."""
    return (os.environ.get("SGLANG_V1_INDEX_GRAPHS", "0") == "1"
            or os.environ.get("SGLANG_V1_QUERY_GRAPH", "0") == "1"
            or (decode and os.environ.get("SGLANG_V1_DECODE_QUERY_GRAPH", "0") == "1"))


def pack_q(q, scale, out_heads: int = 32, out=None):
    """(q8 e4m3 [rows, out_heads, 128], weights float32 [rows, out_heads]) of q
    [rows, qheads, 128] (float32 / bf16 / fp16, unit inner stride): per (row,
    head) the power-of-two scale >= max(max|q|, 1e-4) / 448, q8 = q / scale,
    weight = scale * softmax scale / qheads; heads >= qheads are zero
    (NA/scoring.py:66-71, qwen_gqa_probe_kernels.py:15-20).  ``out`` = (q8,
    weights) buffers with at least as many rows to write into."""
    require(q.dim() == 3 and q.shape[2] == 128 and q.stride(2) == 1 and q.dtype in _DTYPES,
            "q: [rows, heads, 128] float32 / bfloat16 / float16 with unit inner stride")
    rows, qheads = q.shape[0], q.shape[1]
    require(qheads <= out_heads, "more query heads than output heads")
    if out is None:
        q8 = torch.empty((rows, out_heads, 128), dtype=torch.float8_e4m3fn, device=q.device)
        w = torch.empty((rows, out_heads), dtype=torch.float32, device=q.device)
    else:
        q8, w = out
        require(q8.dim() == 3 and q8.shape[1:] == (out_heads, 128) and q8.is_contiguous()
                and q8.dtype in (torch.float8_e4m3fn, torch.uint8) and q8.shape[0] >= rows,
                "q8: contiguous e4m3 [>= rows, out_heads, 128]")
        require(w.shape == (q8.shape[0], out_heads) and w.dtype == torch.float32 and w.is_contiguous(),
                "weights: contiguous float32 [q8 rows, out_heads]")
    require(q.is_cuda, "pack_q: q must be a CUDA tensor")
    _lib.same_device(q, q8, w)
    _lib.call("v1x_pack_q", ptr(q), _DTYPES[q.dtype], q.stride(0), q.stride(1), rows, q8.shape[0], qheads,
              out_heads, float(scale) / qheads, ptr(q8), ptr(w), _lib.stream_of(q), device=q.device)
    return q8, w


def quantize(x):
    """NA/grouping.py:41-44: (x / scale as e4m3, scale) with scale the power of
    two >= max(max|x|, 1e-4) / 448 over the last axis (128 wide)."""
    require(x.shape[-1] == 128, "quantize: last axis of 128")
    lead = x.shape[:-1]
    flat = x.reshape(-1, 1, 128)
    q8, w = pack_q(flat, 1.0, out_heads=1)
    return q8.reshape(*lead, 128), w.reshape(lead)


GROUP_ROWS = 32   # query rows per tensor-core operand of the grouped scorer


class _Packed:
    """A chunk's packed queries: ``grouped`` = four heads per row, rows padded to
    GROUP_ROWS (the grouped scorer); else the reference's 32-head layout."""

    def __init__(self, q8, weights, rows, grouped):
        self.q8, self.weights, self.rows, self.grouped = q8, weights, rows, grouped


class Scorer:
    """NA/scoring.py:25-99 on libv1x.so (sm_100a; the reference requires SM90 and
    its no-ReLU DeepGEMM fork).  ``impl`` (extension) picks the paged scorer:
    "auto" -- the grouped tensor-core scorer, 32 query rows x 4 heads per MMA
    operand, so that a key tile is read once per 32 rows (same logits as the
    per-row scorer); "tensor_core" -- the per-row tensor-core scorer over the 32
    padded heads, as the reference's DeepGEMM call; "simt" -- the fixed fp32
    evaluation order."""

    def __init__(self, config, device):
        self.config = config
        self.sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.query_graph = query_graph_enabled()
        self.decode_query_graph = query_graph_enabled(decode=True)
        self.impl = "auto"

    def select_decode(self, q, state, head, prefix, offset, total, fixed, scale):
        if self.decode_query_graph and self._graph_eligible(state):
            return self._select_graph(q, state, head, prefix, offset, total, fixed, scale)
        return self.select_eager(q, state, head, prefix, offset, total, fixed, scale)

    def _graph_eligible(self, state):
        return (self.config.mode == "v1" and self.config.share_active_pages
                and getattr(state, "full_bucket_append", False) and state.pages > 0)

    def _select_graph(self, q, state, head, prefix, offset, total, fixed, scale):
        if getattr(state, "query_graph_pool", None) is None:
            raise RuntimeError("Query graph pool was not initialized with the backend")
        return state.query_graph_pool.select(self, q, state, head, prefix, offset, total, fixed, scale)

    def paged(self, q8, weights, cache, table, count):
        """Signed paged logits [rows, count] of q8 [rows, 32, 128] over `cache`
        (packed pages [n, 64, 1, 132]) through `table` (NA/scoring.py:48-53)."""
        lengths = torch.full((len(q8), 1), count, device=q8.device, dtype=torch.int32)
        return scoring.fp8_paged_mqa_logits(q8, cache, weights, lengths, table, None, count,
                                            clean_logits=False, relu=False, impl=self.impl)

    def _pack(self, q, scale):
        rows = q.shape[0]
        if self.impl != "auto":
            q8, w = pack_q(q, scale)
            return _Packed(q8, w, rows, False)
        R = -(-rows // GROUP_ROWS) * GROUP_ROWS
        q8 = torch.empty((R, 4, 128), dtype=torch.float8_e4m3fn, device=q.device)
        w = torch.empty((R, 4), dtype=torch.float32, device=q.device)
        pack_q(q, scale, out_heads=4, out=(q8, w))
        return _Packed(q8, w, rows, True)

    def _logits(self, qp, cache, pages, keys, row_tables=None, key_valid=None, mask=None):
        """Logits of the packed rows over `cache`: without row tables [rows, keys]
        of the keys of `pages` (one table shared by the rows; -inf where
        `key_valid` is False); with row tables [rows, 64 * P] of each row's own
        pages, every one of them in `pages`, masked by ``gather.mask_scores(out,
        row_tables, *mask)`` when `mask` = (mapping, positions) is given."""
        if qp.grouped:
            width = row_tables.shape[1] * 64 if row_tables is not None else keys
            out = torch.empty((qp.rows, width), dtype=torch.float32, device=qp.q8.device)
            return scoring.paged_logits_grouped(qp.q8, qp.weights, cache, pages, keys, out, row_tables, GROUP_ROWS,
                                                relu=False, rows=qp.rows, key_valid=key_valid, mask=mask)
        if row_tables is not None:
            out = self.paged(qp.q8, qp.weights, cache, row_tables, row_tables.shape[1] * 64)
            if mask is not None:
                mask_scores(out, row_tables, *mask)
            return out
        out = self.paged(qp.q8, qp.weights, cache, pages[None].expand(qp.rows, -1).contiguous(), keys)
        if key_valid is not None:
            out[:, :keys].masked_fill_(~key_valid[:keys].bool()[None], -torch.inf)
        return out

    def select(self, q, state, head, prefix, offset, total, fixed, scale):
        if self.query_graph and self._graph_eligible(state):
            return self._select_graph(q, state, head, prefix, offset, total, fixed, scale)
        return self.select_eager(q, state, head, prefix, offset, total, fixed, scale)

    def select_eager(self, q, state, head, prefix, offset, total, fixed, scale):
        if self.config.share_active_pages:
            return select(self, q, state, head, prefix, offset, total, fixed, scale)
        rows, qheads, dim = q.shape
        if dim != 128 or qheads != 4:
            raise ValueError("This backend preserves Qwen's four-Q-head routing group")
        positions = torch.arange(prefix + offset, prefix + offset + rows, device=q.device, dtype=torch.int32)
        if self.config.mode == "dsa":
            kv = (state.flat_k[head, :total], state.flat_scale[head, :total])
            qp = self._pack(q, scale)
            if qp.grouped:
                scores = scoring.mqa_logits_grouped(qp.q8, qp.weights, kv, torch.zeros_like(positions),
                                                    positions + 1, rows=rows, group_rows=GROUP_ROWS, relu=False)
            else:
                scores = scoring.fp8_mqa_logits(qp.q8, kv, qp.weights, torch.zeros_like(positions), positions + 1,
                                                True, relu=False)
            return topk2048(scores, need_values=False)[1].int()
        qp = self._pack(q, scale)
        pages = state.pages
        centers = pages * 8
        center_pages = (centers + 63) // 64
        ct = torch.arange(center_pages, device=q.device, dtype=torch.int32)
        coarse = self._logits(qp, state.centers[head], ct, centers, key_valid=state.valid[head, :centers])
        coarse = coarse[:, :centers]
        take = self.config.budget(pages)
        table = torch.empty((rows, take + len(fixed)), device=q.device, dtype=torch.int32)
        table[:, take:] = fixed[None]
        if take == pages:
            table[:, :take] = torch.arange(pages, device=q.device, dtype=torch.int32)
        else:
            _route_into(coarse, table, pages, take)
        # the fine pages any row can name: the route's ids (below the smallest
        # power of two >= max(pages, 128): its blocked layout's padding ids
        # appear when -inf pages reach the take) and the fixed pages
        n = 128
        while n < pages:
            n *= 2
        span = min(n if pages <= 4096 else pages, state.fine[head].numel() // 8448)
        used = torch.cat((torch.arange(span, device=q.device, dtype=torch.int32), fixed.to(torch.int32)))
        scores = self._logits(qp, state.fine[head], used, used.numel() * 64, table,
                              mask=(state.mapping[head], positions))
        # logical original token positions (not physical slots, no x4 expansion)
        return mapped_top2048(scores, table, state.mapping[head])


def _route_into(coarse, table, pages, take):
    """The reference's route choice (NA/scoring.py:92-95): the route extension
    for 32 < pages <= 4096; fewer pages take the same ranking (the reference
    uses an unsorted torch top-k there, same set up to ties); more than 4096
    pages the torch top-k as in the reference."""
    if 32 < pages <= 4096:
        extension(64, 4).route(coarse, table, pages, take)
    elif pages <= 32:
        table[:, :take] = rank_pages(coarse, pages, take)
    else:
        rows = coarse.shape[0]
        table[:, :take] = coarse.reshape(rows, pages, 8).amax(-1).topk(take, sorted=False).indices.int()


def select(scorer, q, state, head, prefix, offset, total, fixed, scale):
    """NA/shared_scoring.py:9-27: the selection over shared physical index pages."""
    arena = state.arena
    state.wait()
    fixed.record_stream(torch.cuda.current_stream(q.device))
    rows, qheads, dim = q.shape
    if (qheads, dim) != (4, 128):
        raise ValueError("Expected four Q heads of dimension 128")
    qp = scorer._pack(q, scale)
    positions = torch.arange(prefix + offset, prefix + offset + rows, device=q.device, dtype=torch.int32)
    ids = _select_packed(scorer, qp, arena, head, state.table[head], fixed[head], positions,
                         state.full_bucket_append, state.fixed_start)
    arena.record()
    return ids


def select_tensors(scorer, q8, weights, arena, head, page_ids, fixed_ids, positions, full_bucket_append,
                   fixed_start, decode_meta=None):
    """NA/shared_scoring.py:30-62: query kernels only (stream dependencies and
    the page lifecycle stay with the caller); returns physical reordered
    storage ids through ``arena.identity``."""
    if decode_meta is not None:
        raise ValueError("decode_meta masks belong to the shared arenas' decode query graph, "
                         "which this library does not provide")
    return _select_packed(scorer, _Packed(q8, weights, len(q8), False), arena, head, page_ids, fixed_ids, positions,
                          full_bucket_append, fixed_start)


def _select_packed(scorer, qp, arena, head, page_ids, fixed_ids, positions, full_bucket_append, fixed_start):
    rows = qp.rows
    dev = qp.q8.device
    pages, take = page_ids.numel(), scorer.config.budget(page_ids.numel())
    selected = torch.empty((rows, take), device=dev, dtype=torch.int32)
    if take == pages:
        selected[:] = torch.arange(pages, device=dev, dtype=torch.int32)
    else:
        coarse = scorer._logits(qp, arena.centers[head], page_ids.to(torch.int32).contiguous(), pages * 64)
        coarse = coarse.reshape(rows, pages, 64)[:, :, :8].contiguous()
        valid = arena.valid[head, page_ids.long()]
        coarse.masked_fill_(~valid[None], -torch.inf)
        coarse = coarse.reshape(rows, pages * 8)
        _route_into(coarse, selected, pages, take)
    # a padding id of the route's blocked layout (>= pages, reached only when -inf
    # pages enter the take) would index past page_ids: it names the last page
    table = torch.cat((page_ids[selected.long().clamp_(max=pages - 1)], fixed_ids[None].expand(rows, -1)),
                      1).contiguous()
    used = torch.cat((page_ids, fixed_ids)).to(torch.int32).contiguous()
    scores = scorer._logits(qp, arena.fine[head], used, used.numel() * 64, table)
    mask_scores(scores, table, arena.mapping[head], positions,
                take * 64 if full_bucket_append else 0, fixed_start if full_bucket_append else 0)
    return mapped_top2048(scores, table, arena.identity)
