"""Drop-in for the reference's ``Indexer`` library API
(sglang/srt/layers/attention/v1_deepseek/runtime.py:693-937): one layer's native
cache + V1 page arena, ``prepare`` / ``query`` / ``release_request`` / ``clear``
/ ``close``, calls serialised by a lock.

``query`` mirrors :828-907: input validation, the per-owner ``prepare`` to each
request's largest visible length, then per chunk of at most ``q_buckets[-1]``
rows a per-bucket ``Query`` (:281-678) that stages the rows into capture-stable
buffers (zeroing the padding rows, copying each owner's page tables), runs the
selection step (optionally as a captured CUDA graph) and returns clones of the
physical slot ids -- or of the x4 expanded logical positions when
``Config.expand_output`` -- plus the logical ids when ``return_logical``.

``prepare`` builds every new bucket from the native cache through the
request's native page table (Build.compute, :170-270): the index build of
index_build.py for all new buckets of the call in one launch, then the
fingerprint / match / allocate / publish of all of them through the batched
page lifecycle (``PageArena.prepare_many``; the arena state equals that of the
reference's per-bucket sequence).  The optional ``bucket_source(owner, bucket)
-> (tmp, mapping, centers)`` replaces the index build with supplied bucket
contents (see lifecycle.PageArena).
"""
from __future__ import annotations

import threading
from array import array

import torch

from . import _lib
from . import kernels as K
from ._lib import ptr
from .config import Config
from .index_build import BucketBuilder
from .lifecycle import PageArena
from .pipeline import SelectionStep
from .synth import QueryCase


class _Query:
    """Capture-stable buffers of one query bucket of `rows` rows (:281-313, :643-678)."""

    def __init__(self, owner: "Indexer", rows: int):
        c, d = owner.config, owner.device
        self.owner, self.rows = owner, rows
        a = owner.arena
        self.case = QueryCase(
            B=rows, H=c.heads, P=c.pages, take=c.take, window=c.window, topk=c.topk,
            lens=torch.zeros(rows, dtype=torch.int32, device=d),
            q8=torch.zeros((rows, c.heads, 128), dtype=torch.float8_e4m3fn, device=d),
            w=torch.zeros((rows, c.heads), dtype=torch.float32, device=d),
            native=owner.native, fine=a.fine, centers=a.centers, members=a.members,
            native_table=torch.zeros((rows, c.pages), dtype=torch.int32, device=d),
            reordered_table=torch.zeros((rows, c.pages), dtype=torch.int32, device=d),
            center_table=torch.zeros((rows, c.pages // 8), dtype=torch.int32, device=d),
            capacity=a.capacity)
        ratio = c.ratio
        # The reference's fixed-budget hook: a caller that replaces the metadata
        # op with BudgetMetadata(budget) (as qwen_gqa_probe_backend.py:48 does)
        # gets take = min(pages, budget) instead of the ratio rule.
        budget = getattr(K.query_metadata, "budget", None)
        if budget is not None:
            self.step = SelectionStep(self.case, gather=False, budget=budget, expand=c.expand_output)
        else:
            self.step = SelectionStep(self.case, gather=False, ratio=(ratio.numerator, ratio.denominator),
                                      expand=c.expand_output)
        self.graph = None
        self.graphs = c.graphs
        self.filled = 0        # rows [filled, rows) of the staged inputs are known to be zero
        self.device = d
        # the staging call's fixed arguments: the arena's request tables and the
        # bucket's capture-stable inputs
        self.stage_args = (ptr(a.state_tables), ptr(a.state_centers), a.state_tables.shape[0], ptr(self.case.q8),
                           ptr(self.case.w), ptr(self.case.lens), ptr(self.case.native_table),
                           ptr(self.case.reordered_table), ptr(self.case.center_table))
        self.views: dict[int, tuple] = {}   # n -> the outputs' first n rows

    def _execute(self):
        if not self.graphs:
            self.step.run()
            return
        if self.graph is None:
            self.step.run()     # the first call runs eagerly, then the step is captured
            s = torch.cuda.Stream(device=self.owner.device)
            s.wait_stream(torch.cuda.current_stream(self.owner.device))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self.step.run()
            torch.cuda.current_stream(self.owner.device).wait_stream(s)
            self.graph = g
            return
        self.graph.replay()

    def run(self, q, w, native_tables, lengths, rows, return_logical=False):
        """Stage n rows (``rows``: each row's arena row id), run the step and
        return clones of the outputs' first n rows (:643-678).  The staging --
        inputs, zeroed padding rows and the requests' table rows -- is one
        launch (v1x_query_stage)."""
        n = q.shape[0]
        c = self.owner.config
        ids = array("i", rows)
        stream = torch.cuda.current_stream(self.device)
        _lib.call("v1x_query_stage", q.data_ptr(), w.data_ptr(), lengths.data_ptr(), native_tables.data_ptr(),
                  native_tables.shape[1], ids.buffer_info()[0], *self.stage_args, c.heads, c.pages, n, self.filled,
                  stream.cuda_stream, device=self.device)
        self.filled = n
        self._execute()
        views = self.views.get(n)
        if views is None:
            out = self.step.expanded if c.expand_output else self.step.physical
            views = self.views[n] = (out[:n], self.step.logical[:n])
        result = views[0].clone()
        if return_logical:
            result = (result, views[1].clone())
        for t in (q, w, native_tables, lengths):     # read on this stream (:676-677)
            t.record_stream(stream)
        return result


class Indexer:
    """One layer's native cache + V1 arena (reference Indexer, :693-937)."""

    def __init__(self, native_cache, config: Config = Config(), bucket_source=None):
        if (
            native_cache.dtype != torch.uint8
            or not native_cache.is_cuda
            or not native_cache.is_contiguous()
            or native_cache.ndim not in (2, 4)
            or native_cache.numel() % 8448
            or (native_cache.ndim == 2 and native_cache.shape[1] != 8448)
            or (native_cache.ndim == 4 and native_cache.shape[1:] != (64, 1, 132))
        ):
            raise ValueError("Expected native contiguous FP8 page64 packed byte cache")
        if config.reservation > config.budget_bytes:
            raise ValueError(f"V1 reservation {config.reservation} exceeds budget {config.budget_bytes}")
        self.config = config
        self.native = native_cache.view(-1, 8448)
        self.device = native_cache.device
        self.capacity = config.pages * config.max_requests
        self.arena = PageArena(self.capacity, config.pages, self.device, max_requests=config.max_requests,
                               graphs=config.graphs, staging_rows=config.q_buckets[-1])
        self.bucket_source = bucket_source
        self.builder = BucketBuilder(self.device, max(config.pages // 16, 1)) if bucket_source is None else None
        self.queries: dict[int, _Query] = {}
        self.lock = threading.RLock()
        self.closed = False

    @property
    def states(self):
        return self.arena.states

    def _begin(self):
        if self.closed:
            raise RuntimeError("Indexer is closed")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("V1 index subgraphs must execute outside full-model capture")

    def _prepare(self, owner, native_table, length):
        if not 0 <= length <= self.config.max_context:
            raise ValueError("Index context capacity exceeded")
        if (native_table.dtype != torch.int32 or native_table.device != self.device or native_table.ndim != 1
                or native_table.numel() < -(-length // 64) or not native_table.is_contiguous()):
            raise ValueError("Invalid compact native page table")
        # The request's new buckets go through the batched page lifecycle
        # (v1x_prepare_buckets, up to 64 buckets per call), with the arena
        # state of the reference's per-bucket Build sequence.
        if self.bucket_source is not None:
            def batch_source(pairs):
                parts = [self.bucket_source(o, b) for o, b in pairs]
                return tuple(torch.stack([p[i] for p in parts]) for i in range(3))
        else:
            def batch_source(pairs):
                # consecutive new buckets of one request: their native pages are
                # one slice of its table, built in one launch
                buckets = [b for _, b in pairs]
                b0, n = buckets[0], len(buckets)
                source = native_table[b0 * 16:(b0 + n) * 16].view(n, 16)
                tmp, centers, mapping, _ = self.builder.build(self.native, source, [b * 1024 for b in buckets],
                                                              self.arena.status)
                return tmp, mapping, centers
        self.arena.prepare_many([(owner, length)], batch_source)
        return self.arena.states[owner]

    def _ready_rows(self, owners, cpu):
        """The arena rows of the owners when no row needs a prepare -- every
        owner known, no row shorter than its request's indexed length and no
        newly complete bucket -- recording each row's length as the request's;
        None otherwise (the full prepare path then runs, with the same result)."""
        rows, done = [], []
        for st, x in zip(map(self.arena.states.get, owners), cpu):
            if st is None or x < st.length or x >> 10 != len(st.leases):
                for st0, old in reversed(done):     # undo: the prepare path decides
                    st0.length = old
                return None
            done.append((st, st.length))
            st.length = x
            rows.append(st.row)
        return rows

    def _bucket(self, n):
        """The query bucket of the smallest configured size >= n (:881-884)."""
        rows = next(r for r in self.config.q_buckets if r >= n)
        qb = self.queries.get(rows)
        if qb is None:
            qb = self.queries[rows] = _Query(self, rows)
        return qb

    @torch.inference_mode()
    def prepare(self, owner, native_table, length):
        with self.lock:
            self._begin()
            return self._prepare(owner, native_table, length)

    @torch.inference_mode()
    def query(self, q, weights, native_tables, lengths, owners, lengths_cpu, return_logical=False):
        n = len(q)
        c = self.config
        if (
            q.shape != (n, c.heads, 128) or q.dtype != torch.float8_e4m3fn or not q.is_contiguous()
            or weights.shape != (n, c.heads) or weights.dtype != torch.float32 or not weights.is_contiguous()
            or native_tables.ndim != 2 or native_tables.shape[0] != n or native_tables.shape[1] > c.pages
            or native_tables.dtype != torch.int32 or not native_tables.is_contiguous()
            or lengths.numel() != n or lengths.dtype != torch.int32 or not lengths.is_contiguous()
            or len(owners) != n or len(lengths_cpu) != n
            or any(t.device != self.device for t in (q, weights, native_tables, lengths))
        ):
            raise ValueError("Unsupported V1 FP8/page64 query inputs")
        cpu = [int(x) for x in lengths_cpu]
        if cpu and (min(cpu) < 0 or max(cpu) > min(c.max_context, native_tables.shape[1] * 64)):
            raise ValueError("Query lengths exceed page-table/context capacity")
        with self.lock:
            self._begin()
            if not n:
                empty = torch.empty((0, c.topk * 4 + 64 if c.expand_output else c.topk), device=self.device,
                                    dtype=torch.int32)
                return (empty, torch.empty((0, c.topk), device=self.device, dtype=torch.int32)) \
                    if return_logical else empty
            rows = self._ready_rows(owners, cpu)
            if rows is None:
                # build each request to its largest visible length before querying
                longest = {}              # owner -> (length, row) of its longest row (ties: first row)
                for i, (key, x) in enumerate(zip(owners, cpu)):
                    if x > longest.get(key, (-1, 0))[0]:
                        longest[key] = (x, i)
                for key, (x, i) in longest.items():
                    self._prepare(key, native_tables[i], x)
                if self.arena.pending_check:      # new buckets: read the status word (a sync)
                    self.arena.check()
                states = self.states
                rows = [states[x].row for x in owners]
            step = c.q_buckets[-1]
            if n <= step:                     # one bucket: the caller's tensors as they are
                return self._bucket(n).run(q, weights, native_tables, lengths, rows, return_logical)
            outputs = []
            for start in range(0, n, step):
                end = min(n, start + step)
                outputs.append(self._bucket(end - start).run(q[start:end], weights[start:end],
                                                             native_tables[start:end],
                                                             lengths.reshape(-1)[start:end], rows[start:end],
                                                             return_logical))
            if len(outputs) == 1:
                return outputs[0]
            if return_logical:
                return tuple(torch.cat([x[i] for x in outputs]) for i in (0, 1))
            return torch.cat(outputs)

    @torch.inference_mode()
    def release_request(self, owner):
        with self.lock:
            self._begin()
            self.arena.release(owner)

    @torch.inference_mode()
    def clear(self):
        with self.lock:
            if self.closed:
                return
            for key in list(self.states):
                self.arena.release(key)
            torch.cuda.synchronize(self.device)
            self.queries.clear()

    def close(self):
        self.clear()
        self.closed = True
