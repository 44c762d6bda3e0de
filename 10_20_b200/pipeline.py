"""The query-side selection step on one GPU, as one capture-stable object.

`SelectionStep` runs, for a batch of query rows, the reference's optimised
query sequence (sglang/srt/layers/attention/v1_deepseek/runtime.py:417-636,
DeepGEMM ReLU path with fused route and fused topk) on libv1x.so kernels:

  1. query metadata with the fixed page budget  (BudgetMetadata)        :364-368
     (side stream, with step 4's staging)
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
"""
from __future__ import annotations

import torch

from . import kernels as K
from . import query_fused, scoring
from .gather import _gather_impl


class SelectionStep:
    def __init__(self, case, gather: bool = True, gather_v: bool = False, fused_route_pages: bool = True,
                 keep_logits: bool = False):
        c = self.case = case
        d = c.lens.device
        B = c.B
        self.budget = torch.tensor([c.take], dtype=torch.int32, device=d)
        self.fine_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.takes = torch.zeros(B, dtype=torch.int32, device=d)
        self.dg_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.center_lens = torch.zeros(B, dtype=torch.int32, device=d)
        self.tail_rows = torch.zeros(B, dtype=torch.int32, device=d)
        self.center_logits = torch.empty((B, c.P * 8), dtype=torch.float32, device=d)
        self.page_scores = torch.empty((B, c.P), dtype=torch.float32, device=d)
        self.selected = torch.empty((B, c.take), dtype=torch.int32, device=d)
        self.width = c.width
        self.fine_table = torch.zeros((B, self.width // 64), dtype=torch.int32, device=d)
        self.scores = torch.empty((B, self.width), dtype=torch.float32, device=d)
        self.physical = torch.empty((B, c.topk), dtype=torch.int32, device=d)
        self.logical = torch.empty_like(self.physical)
        self.raw = torch.empty_like(self.physical)
        self.no_expansion = torch.empty_strided((B, 0), (0, 1), device=d, dtype=torch.int32)
        self.gather = gather and c.latent is not None
        self.gather_v = gather_v
        if self.gather:
            D = c.latent.shape[-1]
            self.kv = torch.empty((B, c.topk, 1, D), dtype=c.latent.dtype, device=d)
            self.kv2 = torch.empty_like(self.kv) if gather_v else None
        self.fused = query_fused.module()
        self.meta = K.BudgetMetadata(self.budget)
        self.graph = None
        # fused_route_pages: page maxima from the scoring epilogue + route_pages with
        # the fine-table write (the reference's query_route_table_fusion); equal
        # outputs to route(center_logits) + fine_table_shared.
        self.fused_route_pages = fused_route_pages
        self.keep_logits = keep_logits or not fused_route_pages
        # the sink/tail staging depends only on the metadata: it runs on a side
        # stream, concurrently with centre scoring and routing
        self.side = torch.cuda.Stream(device=d)

    # -- the step ------------------------------------------------------------
    def run(self):
        c = self.case
        B = c.B
        main = torch.cuda.current_stream(c.lens.device)
        # metadata and the sink/tail staging run on a side stream, concurrently
        # with centre scoring, which derives each row's centre count from the
        # token length itself (lens_kind="centres")
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            self.meta[(B,)](c.lens, c.native_table, self.fine_lens, self.takes, self.dg_lens,
                            self.center_lens, self.tail_rows, c.P, c.topk, 1, 2, 64, c.window)
            K.stage_tail_shared[(-(-B // 32) if B > 512 else B, 68)](
                c.native, c.native.view(torch.float32), c.native_table, c.lens, c.fine,
                c.fine.view(torch.float32), self.tail_rows, c.capacity, c.P, 68, 64, c.window,
                ROWS=B, GROUP=32 if B > 512 else 1)
        if self.fused_route_pages:
            # centre scoring emits each page's max-of-8 directly; route reads P floats
            # per row and writes the fine page table itself (fill_table)
            scoring.fp8_paged_mqa_logits(c.q8, c.centers, c.w, c.lens, c.center_table, None,
                                         c.P * 8, page_max=self.page_scores, logits=self.keep_logits,
                                         out=self.center_logits if self.keep_logits else None,
                                         clean_logits=False, lens_kind="centres")
            main.wait_stream(self.side)
            self.fused.route_pages(self.page_scores, c.lens, self.takes, self.selected, c.P,
                                   c.reordered_table, self.fine_table, self.tail_rows, c.capacity, True)
        else:
            scoring.fp8_paged_mqa_logits(c.q8, c.centers, c.w, c.lens, c.center_table, None,
                                         c.P * 8, out=self.center_logits, lens_kind="centres")
            main.wait_stream(self.side)
            self.fused.route(self.center_logits, c.lens, self.takes, self.selected, c.P,
                             c.reordered_table, self.fine_table, self.tail_rows, c.capacity, False)
            K.fine_table_shared[(B,)](c.reordered_table, self.selected, self.takes, c.lens,
                                      self.fine_table, self.tail_rows, c.capacity, c.P, c.take,
                                      self.width // 64, 68)
        scoring.fp8_paged_mqa_logits(c.q8, c.fine, c.w, self.dg_lens, self.fine_table, None,
                                     self.width, out=self.scores, clean_logits=False)
        self.fused.topk(self.scores, self.fine_lens, c.members, c.reordered_table, c.native_table,
                        self.selected, c.lens, self.takes, self.physical, self.logical, self.raw,
                        c.window, True, self.no_expansion, True, True, self.fine_table, False)
        if self.gather:
            lat = c.latent
            _gather_impl((1,), lat, lat if self.gather_v else None, None, self.physical, self.kv,
                         self.kv2, B, c.topk, 0, *lat.stride(),
                         *(lat.stride() if self.gather_v else (0, 0, 0)), self.physical.stride(0))

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
    def algorithmic_bytes(self) -> dict:
        """Compulsory bytes of one step, each input byte once, each output once."""
        c = self.case
        lens = c.lens.tolist()
        B, H = c.B, c.H
        pages = [max(n - 1, 0) // 1024 * 16 for n in lens]
        take = [min(p, c.take) for p in pages]
        sink = [min(64, n) for n in lens]
        tail = [max(s, min(max(n - 1, 0) // 1024 * 1024, max(s, n - c.window))) for n, s in zip(lens, sink)]
        count = [s + n - t for n, s, t in zip(lens, sink, tail)]
        fine = [tk * 64 + cnt for tk, cnt in zip(take, count)]
        q = B * H * (128 + 4)
        centres = sum(p * 8 for p in pages) * 132
        staging = sum(count) * 132 * 2
        fine_b = sum(fine) * 132 + sum(tk * 64 * 4 for tk in take)
        out = B * c.topk * 4 * 3
        gather = 0
        if self.gather:
            row = c.latent.shape[-1] * c.latent.element_size()
            gather = B * c.topk * row * (2 + (1 if self.gather_v else 0))
        return dict(q=q, centres=centres, staging=staging, fine=fine_b, topk_out=out, gather=gather,
                    total=q + centres + staging + fine_b + out + gather)
