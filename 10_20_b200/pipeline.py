"""The query-side selection step on one GPU, as one capture-stable object.

`SelectionStep` runs, for a batch of query rows, the reference's optimised
query sequence (sglang/srt/layers/attention/v1_deepseek/runtime.py:417-636,
DeepGEMM ReLU path with fused route and fused topk) on libv1x.so kernels:

  1. query metadata with the fixed page budget  (BudgetMetadata)        :364-368
     and the sink/tail staging of step 4
  2. FP8 centre logits of every built page's 8 centres                  :434-444
     (centre counts derived from the token lengths in the scorer)
  3. fused.route: page max-of-8 + stable top pages                      :446-448
  4. fine_table_shared + stage_tail_shared                              :478-509
  5. FP8 fine logits over the fine page table                           :538-548
  6. fused.topk: boundary mask + Top-2048 + raw->logical->physical      :589-599
  7. _gather_slots of the selected latent K/V rows (qwen_gqa_probe_backend.py:202)

All buffers are allocated once; `run()` only launches kernels on the current
stream (no host synchronisation), so the whole step can be captured in a CUDA
graph with `capture()`.  Rows <= 512 take the same fused top-k: its outputs
equal the reference's non-fused topk_transform + output_ids path.

By default (`fused=True`) steps 1 and 3-6 are one launch per batch,
v1x_select_fused: each row's metadata, route, fine scoring (sink and tail keys
read from the native pages, so nothing is staged), boundary mask, Top-2048 and
mapping in one CTA, the fine logits kept on chip.  The step is then three
launches: centre scoring, selection, gather.  `fused=False` runs the
operator-by-operator sequence above (the reference-shaped ops, also used by
the parity tests as a second opinion).
"""
from __future__ import annotations

import torch

from . import _lib
from . import kernels as K
from . import query_fused, scoring
from .gather import _gather_impl
from .sharding import row_bytes


class SelectionStep:
    """One query step over a batch of rows (see the module docstring).

    All kernels run in order on the caller's current stream, the latency-bound
    selection kernels at high launch priority and the gather at the default, so
    that independent batches stepped on separate streams overlap: one batch's
    gather fills the GPU while the next batch is selected.
    """

    def __init__(self, case, gather: bool = True, gather_v: bool = False, fused_route_pages: bool = True,
                 keep_logits: bool = False, ratio=None, expand: bool = False, budget=None,
                 fused: bool = True, score_ctas: int = 0):
        """ratio=None: the fixed page budget take = min(pages, budget) (the
        reference's BudgetMetadata; budget an int32 device tensor of one element,
        by default holding case.take, which bounds it); ratio=(num, den): the
        reference's default take rule min(pages, max(ceil(pages*num/den),
        ceil(topk/64))).  expand: also write the x4 expanded logical positions
        ([B, 4*topk+64], -1 padded).  score_ctas > 0 caps the centre scorer's
        grid (for small batches stepped many at a time)."""
        c = self.case = case
        d = c.lens.device
        B = c.B
        self.ratio = (1, 2) if ratio is None else (int(ratio[0]), int(ratio[1]))
        if ratio is None:
            self.budget = torch.tensor([c.take], dtype=torch.int32, device=d) if budget is None else budget
        else:
            self.budget = None
        self.fine_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.takes = torch.zeros(B, dtype=torch.int32, device=d)
        self.dg_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.center_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.tail_rows = torch.zeros(B, dtype=torch.int32, device=d)
        self.center_logits = torch.empty((B, c.P * 8), dtype=torch.float32, device=d)
        self.page_scores = torch.empty((B, c.P), dtype=torch.float32, device=d)
        self.selected = torch.empty((B, c.take), dtype=torch.int32, device=d)
        self.width = c.width
        # Columns top-k reads: with the fixed page budget a row holds at most
        # take*64 + sink + max(window, 1024) candidates (the tail spans at most a
        # window, or the unbuilt remainder of the last bucket); the ratio rule
        # can take more pages, so it reads the whole row.
        span = c.take * 64 + 64 + max(c.window, 1024)
        self.topk_cols = min(self.width, (span + 3) // 4 * 4) if ratio is None else self.width
        self.fine_table = torch.zeros((B, self.width // 64), dtype=torch.int32, device=d)
        self.scores = torch.empty((B, self.width), dtype=torch.float32, device=d)
        self.physical = torch.empty((B, c.topk), dtype=torch.int32, device=d)
        self.logical = torch.empty_like(self.physical)
        self.raw = torch.empty_like(self.physical)
        self.no_expansion = torch.empty_strided((B, 0), (0, 1), device=d, dtype=torch.int32)
        self.expanded = (torch.empty((B, c.topk * 4 + 64), dtype=torch.int32, device=d) if expand
                         else self.no_expansion)
        self.gather = gather and c.latent is not None
        self.gather_v = gather_v
        if self.gather:
            D = c.latent.shape[-1]
            self.kv = torch.empty((B, c.topk, 1, D), dtype=c.latent.dtype, device=d)
            self.kv2 = torch.empty_like(self.kv) if gather_v else None
        self.fused = query_fused.module()
        self.graph = None
        # fused_route_pages: page maxima from the scoring epilogue + route_pages with
        # the fine-table write (the reference's query_route_table_fusion); equal
        # outputs to route(center_logits) + fine_table_shared.
        self.fused_route_pages = fused_route_pages
        self.keep_logits = keep_logits or not fused_route_pages
        # one-launch selection (route + fine scoring + top-k per row); the fine
        # logits reach HBM only when they are kept for checks
        self.fused_select = fused and fused_route_pages and (c.H == 1 or c.H % 32 == 0)
        self.fine_scores_kept = keep_logits or not self.fused_select
        if self.fused_select and not self.fine_scores_kept:
            self.scores = None
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        self.score_ctas = int(score_ctas)

    # -- the step ------------------------------------------------------------
    def _centres(self, rs):
        c = self.case
        if self.fused_route_pages:
            # centre scoring emits each page's max-of-8 directly; route reads P floats
            # per row and writes the fine page table itself (fill_table)
            scoring.fp8_paged_mqa_logits(c.q8[rs], c.centers, c.w[rs], c.lens[rs], c.center_table[rs], None,
                                         c.P * 8, page_max=self.page_scores[rs], logits=self.keep_logits,
                                         out=self.center_logits[rs] if self.keep_logits else None,
                                         clean_logits=False, lens_kind="centres", max_ctas=self.score_ctas)
        else:
            scoring.fp8_paged_mqa_logits(c.q8[rs], c.centers, c.w[rs], c.lens[rs], c.center_table[rs], None,
                                         c.P * 8, out=self.center_logits[rs], lens_kind="centres",
                                         max_ctas=self.score_ctas)

    def _route(self, rs):
        c = self.case
        n = rs.stop - rs.start
        if self.fused_route_pages:
            self.fused.route_pages(self.page_scores[rs], c.lens[rs], self.takes[rs], self.selected[rs], c.P,
                                   c.reordered_table[rs], self.fine_table[rs], self.tail_rows[rs], c.capacity,
                                   True)
        else:
            self.fused.route(self.center_logits[rs], c.lens[rs], self.takes[rs], self.selected[rs], c.P,
                             c.reordered_table[rs], self.fine_table[rs], self.tail_rows[rs], c.capacity, False)
            K.fine_table_shared[(n,)](c.reordered_table[rs], self.selected[rs], self.takes[rs], c.lens[rs],
                                      self.fine_table[rs], self.tail_rows[rs], c.capacity, c.P, c.take,
                                      self.width // 64, 68)

    def _fine(self, rs):
        c = self.case
        scoring.fp8_paged_mqa_logits(c.q8[rs], c.fine, c.w[rs], self.dg_lens[rs], self.fine_table[rs], None,
                                     self.width, out=self.scores[rs], clean_logits=False)

    def _topk(self, rs):
        c = self.case
        self.fused.topk(self.scores[rs, :self.topk_cols], self.fine_lens[rs], c.members, c.reordered_table[rs],
                        c.native_table[rs], self.selected[rs], c.lens[rs], self.takes[rs], self.physical[rs],
                        self.logical[rs], self.raw[rs], c.window, True, self.expanded[rs], True, True,
                        self.fine_table[rs], False)

    def _select(self):
        """v1x_select_fused over the whole batch (see the module docstring)."""
        c = self.case
        p = _lib.ptr
        num, den = (0, 0) if self.budget is not None else self.ratio
        scores = self.scores if self.fine_scores_kept else None
        _lib.call("v1x_select_fused", p(c.q8), p(c.w), c.H, p(c.lens), p(self.budget), num, den,
                  p(c.native_table), p(c.reordered_table), c.P, p(self.page_scores), self.page_scores.stride(0),
                  p(c.fine), c.fine.shape[0], p(c.members), c.members.shape[0], p(c.native), c.native.shape[0],
                  c.capacity, c.topk, c.window, self.selected.shape[1], self.fine_table.shape[1], p(self.fine_lens),
                  p(self.takes), p(self.dg_lens), p(self.center_lens), p(self.tail_rows), p(self.selected),
                  p(self.fine_table), p(self.physical), p(self.logical), p(self.raw),
                  p(self.expanded) if self.expanded.shape[1] else None, self.expanded.shape[1], p(scores),
                  scores.stride(0) if scores is not None else 0, c.B, p(self.status),
                  torch.cuda.current_stream(c.lens.device).cuda_stream, device=c.lens.device)

    def _gather(self, rs):
        c = self.case
        lat = c.latent
        n = rs.stop - rs.start
        _gather_impl((1,), lat, lat if self.gather_v else None, None, self.physical[rs], self.kv[rs],
                     self.kv2[rs] if self.gather_v else None, n, c.topk, 0, *lat.stride(),
                     *(lat.stride() if self.gather_v else (0, 0, 0)), self.physical.stride(0))

    def run(self, marks=None):
        """Launch the step on the current stream.  marks: a list that receives
        (stage name, CUDA event recorded after the stage) -- a per-stage time
        split for diagnostics (not for graph capture)."""
        c = self.case
        B = c.B
        rs = slice(0, B)

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        mark("start")
        if self.fused_select:
            self._centres(rs)
            mark("centre_scores")
            self._select()
            mark("select")
            if self.gather:
                self._gather(rs)
                mark("gather")
            return
        # query metadata with the fixed page budget + sink/tail staging, one launch
        K.query_prepare(c.lens, c.native_table, self.fine_lens, self.takes, self.dg_lens, self.center_lens,
                        self.tail_rows, c.P, c.topk, self.ratio[0], self.ratio[1], 64, c.window, c.native,
                        c.native.view(torch.float32), c.fine, c.fine.view(torch.float32), c.capacity, 68,
                        budget=self.budget)
        mark("prepare")
        self._centres(rs)
        mark("centre_scores")
        self._route(rs)
        mark("route")
        self._fine(rs)
        mark("fine_scores")
        self._topk(rs)
        mark("topk")
        if self.gather:
            self._gather(rs)
            mark("gather")

    def capture(self, warmup: int = 2):
        s = torch.cuda.Stream(device=self.case.lens.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.run()
        s.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self.run()
        s.synchronize()
        return self.graph

    def replay(self):
        if self.graph is None:
            self.run()
        else:
            self.graph.replay()

    # -- accounting ----------------------------------------------------------
    def launches(self) -> int:
        """Kernels one run() launches (centre scoring + selection, or the five
        operators; + the gather)."""
        return (2 if self.fused_select else 5) + (1 if self.gather else 0)

    def algorithmic_bytes(self) -> dict:
        """Compulsory bytes of one step, each input byte once, each output once
        (the per-request sum of `sharding.row_bytes`)."""
        c = self.case
        row = c.latent.shape[-1] * c.latent.element_size() if self.gather else 0
        total = {}
        for n in c.lens.tolist():
            for k, v in row_bytes(n, c.H, c.take, c.window, c.topk, row, 2 if self.gather_v else 1,
                                  staging=not self.fused_select).items():
                total[k] = total.get(k, 0) + v
        return total
