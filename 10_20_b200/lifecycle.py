"""Host driver of the V1 page arena: the request-level page lifecycle.

Mirrors the page part of the reference's ``Indexer``
(sglang/srt/layers/attention/v1_deepseek/runtime.py):

  State            :681-690   a request's reordered page table, centre table,
                              leases and indexed length
  arena tensors    :718-745   fine pool, centre pool, members, refcounts, free
                              stack + count, hashes, lease tables, centre pages,
                              host stack of free leases
  _release         :771-780   release every lease of a request (kernel + host)
  _prepare         :806-825   index each newly complete 1K bucket of a request
  Build.compute    :230-270   per bucket: fingerprint -> match_pages ->
                              allocate -> publish

One bucket is 1024 tokens = 16 pages of 64.  A bucket's reordered pages,
members and centres come from ``bucket_source(owner, bucket) -> (tmp, mapping,
centers)``: tmp uint8 [16, 8448] packed pages, mapping int32 [16, 64] logical
token positions, centers uint8 [2, 8448] the bucket's 128 packed centres.  The
Indexer's source is the index build of index_build.py over the native cache
(Build.compute's initialize / grouping / assemble); ``batch(owner, buckets)``,
when given, is called once with all new buckets of a prepare first, so that
source can build them in one launch.

With ``graphs=True`` (the reference's ``Config.graphs``) the four kernels of a
bucket run as one captured CUDA graph over fixed input buffers, as the
reference's ``Build`` execution does; the bucket's inputs are copied into
those buffers first.  Every launch is asynchronous: an exhausted arena is
recorded in the device status word (the reference traps) and raised by
``check()``.

``prepare_many`` (an extension) prepares several requests at once: all their
new buckets, in the same canonical order, go through ``v1x_prepare_buckets``
(up to 64 buckets per call, five launches per call), which also writes the
requests' page-table rows.  The arena afterwards equals that of ``prepare``
called for each request in turn.  Request tables live as rows of one arena
tensor, so a batch updates them without per-request copies.  ``release_many``
releases several requests in one launch (``v1x_release_many``), with the arena
state of ``release`` called for each in turn.
"""
from __future__ import annotations

import itertools

import numpy as np
import torch

from . import _lib
from . import kernels as K

PAGE_BYTES = 8448
BATCH_BUCKETS = 64      # buckets per v1x_prepare_buckets call
PREPARE_WORK_INTS = 4 + 4 * 4096 + 1024 + 64 * 5   # V1X_PREPARE_WORK_INTS


class HostStaging:
    """Host -> device copies of small integer arrays without a host wait.

    A copy from pageable host memory may wait for the stream (the driver stages
    it), which would serialise the driver's host loop with the GPU; the values go
    through a ring of pinned buffers instead, each rewritten only after the copy
    that last read it has completed (an event per slot)."""

    def __init__(self, length: int, device, dtype=torch.int32, slots: int = 8):
        self.device = torch.device(device)
        self.buf = torch.empty((slots, length), dtype=dtype).pin_memory()
        self.host = self.buf.numpy()
        self.events = [None] * slots
        self.k = 0

    def copy(self, values, dst):
        """dst[:len(values)] = values (dst a contiguous device tensor), enqueued
        on the current stream."""
        n = len(values)
        k = self.k
        self.k = (k + 1) % len(self.events)
        ev = self.events[k]
        if ev is not None:
            ev.synchronize()
        else:
            ev = self.events[k] = torch.cuda.Event()
        self.host[k, :n] = values
        dst.view(-1)[:n].copy_(self.buf[k, :n], non_blocking=True)
        ev.record(torch.cuda.current_stream(self.device))
        return dst


class State:
    """A request's index state (reference State, DS/runtime.py:681-690): its
    leases, indexed length and arena row; ``table`` / ``center_table`` are that
    row of the arena's request tables (views made on first use)."""

    __slots__ = ("arena", "row", "leases", "length", "_views")

    def __init__(self, arena: "PageArena", row: int):
        self.arena, self.row = arena, row
        self.leases: list[int] = []
        self.length = 0
        self._views = None

    def _view(self, i):
        if self._views is None:
            self._views = (self.arena.state_tables[self.row], self.arena.state_centers[self.row])
        return self._views[i]

    @property
    def table(self):
        return self._view(0)

    @property
    def center_table(self):
        return self._view(1)


class PageArena:
    def __init__(self, capacity: int, pages: int, device, max_requests: int | None = None,
                 graphs: bool = False, staging_rows: int = 0):
        """capacity: arena pages; pages: per-request page-table capacity
        (Config.pages, max_context / 64); max_requests: live request limit;
        staging_rows: query rows whose 68 sink/tail staging pages follow the arena
        in the fine pool (the reference's q_buckets[-1] * 68, :729)."""
        if capacity <= 0 or capacity % 16 or pages <= 0 or pages % 16:
            raise ValueError("capacity and pages must be positive multiples of 16")
        d = self.device = torch.device(device)
        self.capacity, self.pages = capacity, pages
        self.max_requests = max_requests if max_requests is not None else max(capacity // pages, 1)
        self.max_leases = capacity // 16
        self.fine = torch.zeros((capacity + staging_rows * 68, PAGE_BYTES), dtype=torch.uint8, device=d)
        self.centers = torch.zeros((-(-capacity // 8), PAGE_BYTES), dtype=torch.uint8, device=d)
        self.members = torch.full((capacity, 64), -1, dtype=torch.int32, device=d)
        self.refs = torch.zeros(capacity, dtype=torch.int32, device=d)
        self.free = torch.arange(capacity, dtype=torch.int32, device=d)
        self.free_count = torch.full((), capacity, dtype=torch.int32, device=d)
        self.hashes = torch.zeros((capacity, 2), dtype=torch.int64, device=d)
        self.tables = torch.full((self.max_leases, 16), -1, dtype=torch.int32, device=d)
        self.center_pages = torch.arange(self.max_leases * 2, dtype=torch.int32, device=d).view(-1, 2)
        self.free_leases = list(range(self.max_leases - 1, -1, -1))
        self.states: dict = {}
        # per-bucket work buffers (the reference's Build tensors)
        self.tmp = torch.zeros((16, PAGE_BYTES), dtype=torch.uint8, device=d)
        self.mapping = torch.zeros((16, 64), dtype=torch.int32, device=d)
        self.bucket_centers = torch.zeros((2, PAGE_BYTES), dtype=torch.uint8, device=d)
        self.hash = torch.zeros((16, 2), dtype=torch.int64, device=d)
        self.matches = torch.zeros(16, dtype=torch.int32, device=d)
        self.new = torch.zeros(16, dtype=torch.bool, device=d)
        self.meta = torch.zeros(3, dtype=torch.int32, device=d)
        with torch.inference_mode(False):   # check() resets it in place from any mode
            self.status = torch.zeros(1, dtype=torch.int32, device=d)
        self.graphs = graphs
        self._graph = None
        # request tables: one row per live request (State.table / center_table are views)
        self.state_tables = torch.zeros((self.max_requests, pages), dtype=torch.int32, device=d)
        self.state_centers = torch.zeros((self.max_requests, pages // 8), dtype=torch.int32, device=d)
        self.free_rows = list(range(self.max_requests - 1, -1, -1))
        self.kernel_launches = 0   # kernels this driver has launched (reported by the bench)
        self.buckets_indexed = 0   # buckets launched for indexing (aborted ones included)
        # (owner, first bucket, leases, ...) of every run of consecutive buckets
        # of one request launched since the last check(), in launch order: an
        # exhaustion aborts a suffix of the buckets
        self.unchecked: list = []
        self._prepare_args = None
        self._source_key = self._source_val = None
        # batched prepare: meta records and per-page scratch of one call
        self.batch_hash = torch.zeros((BATCH_BUCKETS * 16, 2), dtype=torch.int64, device=d)
        self.batch_match = torch.zeros(BATCH_BUCKETS * 16, dtype=torch.int32, device=d)
        self.batch_new = torch.zeros(BATCH_BUCKETS * 16, dtype=torch.uint8, device=d)
        self.batch_work = torch.zeros(PREPARE_WORK_INTS, dtype=torch.int32, device=d)
        # release_many's leases, offsets and the released requests' table rows
        self.release_idx = torch.zeros(self.max_leases + 2 * self.max_requests + 1, dtype=torch.int32, device=d)
        self.staging = HostStaging(self.release_idx.numel(), d) if d.type == "cuda" else None

    # -- one bucket ------------------------------------------------------------
    def _kernels(self, tmp, mapping, centers):
        self.kernel_launches += 6   # fingerprint, match (3), allocate, publish
        K.fingerprint[(16,)](tmp, mapping, self.meta, self.hash)
        K.match_pages[(16,)](tmp, mapping, self.hash, self.meta, self.fine, self.members, self.hashes,
                             self.refs, self.matches, self.capacity)
        K.allocate[(1,)](self.meta, self.matches, self.free, self.free_count, self.refs, self.tables, self.new,
                         status=self.status, check=False)
        K.publish[(16,)](tmp, centers, centers.view(torch.float32), mapping, self.hash, self.meta, self.tables,
                         self.new, self.fine, self.centers, self.centers.view(torch.float32), self.members,
                         self.hashes)

    def _bucket(self, tmp, mapping, centers, start: int, lease: int):
        self.meta.copy_(torch.tensor([start, lease, 1], dtype=torch.int32), non_blocking=True)
        if not self.graphs:
            self._kernels(tmp, mapping, centers)
            return
        self.tmp.copy_(tmp, non_blocking=True)
        self.mapping.copy_(mapping, non_blocking=True)
        self.bucket_centers.copy_(centers, non_blocking=True)
        if self._graph is None:
            # capture on a side stream once the first bucket's inputs are in place;
            # the first bucket itself runs eagerly (capture does not execute)
            self._kernels(self.tmp, self.mapping, self.bucket_centers)
            s = torch.cuda.Stream(device=self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._kernels(self.tmp, self.mapping, self.bucket_centers)
            torch.cuda.current_stream(self.device).wait_stream(s)
            self._graph = g
            return
        self._graph.replay()

    # -- requests ---------------------------------------------------------------
    def prepare(self, owner, length: int, bucket_source, batch=None):
        """Index every newly complete bucket of `owner` up to `length` tokens
        (reference Indexer._prepare, DS/runtime.py:806-825)."""
        if not 0 <= length <= self.pages * 64:
            raise ValueError("Index context capacity exceeded")
        state = self.states.get(owner)
        if state is not None and length < state.length:
            self.release(owner)
            state = None
        if state is None:
            if len(self.states) >= self.max_requests:
                raise ValueError("V1 request capacity exceeded")
            state = self._new_state(owner)
        complete = length // 1024
        new = range(len(state.leases), complete)
        # the buckets that will get a lease (the loop raises at the first one
        # that does not, as the reference does, keeping those already built)
        ready = list(new)[:len(self.free_leases)]
        if batch is not None and ready:
            batch(owner, ready)
        for bucket in new:
            if not self.free_leases:
                raise RuntimeError("V1 bucket records exhausted")
            lease = self.free_leases.pop()
            tmp, mapping, centers = bucket_source(owner, bucket)
            self._bucket(tmp, mapping, centers, bucket * 1024, lease)
            self.unchecked.append((owner, bucket, [lease]))
            self.buckets_indexed += 1
            state.leases.append(lease)
            state.table[bucket * 16:(bucket + 1) * 16].copy_(self.tables[lease])
            state.center_table[bucket * 2:(bucket + 1) * 2].copy_(self.center_pages[lease])
        state.length = length
        return state

    def release(self, owner):
        """Drop every lease of `owner` (reference Indexer._release, :771-780)."""
        state = self.states.pop(owner, None)
        if state:
            for lease in state.leases:
                K.release[(1,)](self.tables[lease], self.refs, self.free, self.free_count)
                self.free_leases.append(lease)
                self.kernel_launches += 1
            self._free_row(state.row)

    def _free_row(self, row):
        # request table rows are zeroed when freed (they start zeroed), so a new
        # request's State needs no launch
        self.state_tables[row].zero_()
        self.state_centers[row].zero_()
        self.free_rows.append(row)

    def release_many(self, owners):
        """``release(owner)`` for every owner in order, in one launch
        (v1x_release_many); unknown owners are skipped as release skips them."""
        states = [(o, self.states.pop(o)) for o in owners if o in self.states]
        if not states:
            return
        leases = [lease for _, st in states for lease in st.leases]
        offsets = [0]
        for _, st in states:
            offsets.append(offsets[-1] + len(st.leases))
        rows = [st.row for _, st in states]
        idx = self.staging.copy(leases + offsets + rows, self.release_idx)
        _lib.call("v1x_release_many", _lib.ptr(self.tables), _lib.ptr(idx), _lib.ptr(idx[len(leases):]),
                  len(states), _lib.ptr(self.refs), _lib.ptr(self.free), _lib.ptr(self.free_count),
                  torch.cuda.current_stream(self.device).cuda_stream, device=self.device)
        # the released requests' table rows, zeroed in one pass each
        r0 = len(leases) + len(offsets)
        row_ids = idx[r0:r0 + len(rows)].long()
        self.state_tables.index_fill_(0, row_ids, 0)
        self.state_centers.index_fill_(0, row_ids, 0)
        self.kernel_launches += 1
        for _, st in states:
            self.free_leases.extend(st.leases)
        self.free_rows.extend(rows)

    def _new_state(self, owner):
        row = self.free_rows.pop()     # zeroed when it was freed (or never used)
        state = self.states[owner] = State(self, row)
        return state

    # -- several requests at once (extension) ----------------------------------
    def prepare_many(self, requests, batch_source):
        """``prepare(owner, length)`` for every (owner, length) of `requests`, in
        order, with all new buckets indexed by batched calls.  batch_source(pairs)
        -> (tmp uint8 [n, 16, 8448], mapping int32 [n, 16, 64], centers uint8
        [n, 2, 8448]) for the (owner, bucket) pairs in order, or -> (tmp, mapping,
        centers, ids): pools of bucket contents and, per pair, the index of its
        entry (read in place, nothing is copied).  Errors are those of
        ``prepare``, raised at the same request (buckets before it are indexed)."""
        runs = []        # (owner, first bucket, leases, state row) to index, in order
        states, free = self.states, self.free_leases
        limit = self.pages * 64
        try:
            for owner, length in requests:
                if not 0 <= length <= limit:
                    raise ValueError("Index context capacity exceeded")
                state = states.get(owner)
                if state is None or length < state.length:
                    if state is not None:
                        self._flush(runs, batch_source)
                        self.release(owner)
                    if len(states) >= self.max_requests:
                        raise ValueError("V1 request capacity exceeded")
                    state = self._new_state(owner)
                have = len(state.leases)
                n = (length >> 10) - have
                if n > 0:
                    # leases are popped from the end of the free list, one per bucket
                    k = min(n, len(free))
                    if k:
                        got = free[-k:]
                        del free[-k:]
                        got.reverse()
                        state.leases += got
                        run = (owner, have, got, state.row)
                        runs.append(run)
                        self.unchecked.append(run)
                    if k < n:
                        raise RuntimeError("V1 bucket records exhausted")
                state.length = length
        except BaseException:
            # as prepare() does, the buckets granted before the error are indexed
            self._flush(runs, batch_source)
            raise
        self._flush(runs, batch_source)

    def _flush(self, runs, batch_source):
        """Index the buckets of `runs` (emptied first, so none is indexed twice),
        64 per call."""
        if not runs:
            return
        todo = runs[:]
        runs.clear()
        cnt = np.fromiter((len(r[2]) for r in todo), dtype=np.int64, count=len(todo))
        total = int(cnt.sum())
        self.buckets_indexed += total
        pairs = [(o, b0 + i) for o, b0, leases, _ in todo for i in range(len(leases))]
        # meta records (start token, lease, 1, state row), then per chunk the source ids
        meta = np.empty((total, 4), dtype=np.int32)
        first = np.repeat(np.fromiter((r[1] for r in todo), dtype=np.int64, count=len(todo)) - (np.cumsum(cnt) - cnt),
                          cnt)
        meta[:, 0] = (first + np.arange(total)) * 1024
        meta[:, 1] = np.fromiter(itertools.chain.from_iterable(r[2] for r in todo), dtype=np.int32, count=total)
        meta[:, 2] = 1
        meta[:, 3] = np.repeat(np.fromiter((r[3] for r in todo), dtype=np.int32, count=len(todo)), cnt)
        mp = meta.ctypes.data          # host records: they travel in the launch parameters
        stream = torch.cuda.current_stream(self.device).cuda_stream
        for s in range(0, total, BATCH_BUCKETS):
            e = min(s + BATCH_BUCKETS, total)
            got = batch_source(pairs[s:e])
            if len(got) == 4:   # pools + the pairs' entries
                ids = np.asarray(got[3], dtype=np.int32)
                src, nsrc = ids.ctypes.data, got[0].shape[0]
            else:
                src, nsrc = None, 0
            self.kernel_launches += 5
            _lib.call("v1x_prepare_buckets", *self._source_ptrs(got), mp + 16 * s, src, nsrc, e - s,
                      *self._arena_args(), stream, device=self.device)

    def _source_ptrs(self, got):
        """(tmp, centre bytes, centre floats, mapping) pointers of a batch
        source's tensors; a pool source hands over the same tensors every call,
        so their pointers are kept."""
        key = self._source_key
        if key is not None and got[0] is key[0] and got[1] is key[1] and got[2] is key[2]:
            return self._source_val
        tmp, mapping, centers = (x.contiguous() for x in got[:3])
        val = (_lib.ptr(tmp), _lib.ptr(centers), _lib.ptr(centers.view(torch.float32)), _lib.ptr(mapping))
        if len(got) == 4:
            self._source_key, self._source_val = (got[0], got[1], got[2]), val
        return val

    def _arena_args(self):
        """v1x_prepare_buckets' arguments after `buckets` up to `status`: the
        arena's own buffers, which never move, converted once."""
        if self._prepare_args is None:
            p = _lib.ptr
            self._prepare_args = (
                p(self.batch_hash), p(self.batch_match), p(self.batch_new), p(self.fine), p(self.centers),
                p(self.centers.view(torch.float32)), p(self.members), p(self.hashes), p(self.refs), p(self.free),
                p(self.free_count), p(self.tables), p(self.center_pages), p(self.state_tables),
                self.state_tables.stride(0), p(self.state_centers), self.state_centers.stride(0), self.capacity,
                p(self.batch_work), p(self.status))
        return self._prepare_args

    @property
    def pending_check(self) -> bool:
        """True when buckets were launched since the last check()."""
        return bool(self.unchecked)

    def check(self):
        """Raise ArenaExhausted if an allocation found too few free pages (the
        reference's device_assert; it synchronises with the device).  The
        exhausted bucket and every bucket launched after it until this check
        changed nothing in the arena (the status word is sticky) and wrote -1 to
        their lease table rows; their leases are taken back from their requests
        here, each request keeps the buckets before its first aborted one (its
        indexed length ends there), and those buckets' page-table entries return
        to 0 -- so the host state again describes the arena, and a later
        release or prepare of the request sees only its allocated buckets."""
        unchecked, self.unchecked = self.unchecked, []
        code = int(self.status.item())
        if code:
            if code == _lib.V1X_STATUS_ARENA_EXHAUSTED:
                self._take_back_aborted(unchecked)
            self.status.zero_()
            if code == _lib.V1X_STATUS_ARENA_EXHAUSTED:
                raise K.ArenaExhausted("V1 DeepSeek page arena exhausted")
            raise RuntimeError(f"v1x device status {code}")

    def _take_back_aborted(self, launched):
        """Undo the host bookkeeping of the aborted suffix of `launched` (runs
        (owner, first bucket, leases, ...) in launch order)."""
        flat = [(run[0], run[1] + i, lease) for run in launched for i, lease in enumerate(run[2])]
        if not flat:
            return
        rows = self.tables[torch.tensor([lease for _, _, lease in flat], device=self.device)].cpu()
        aborted = (rows < 0).all(dim=1).tolist()
        first = next((i for i, a in enumerate(aborted) if a), len(flat))
        for owner, bucket, lease in reversed(flat[first:]):
            state = self.states.get(owner)
            if state is None or lease not in state.leases:
                continue            # released since: the lease went back already
            state.leases.remove(lease)
            self.free_leases.append(lease)
            state.table[bucket * 16:(bucket + 1) * 16].zero_()
            state.center_table[bucket * 2:(bucket + 1) * 2].zero_()
            state.length = min(state.length, bucket * 1024)
