"""CPU port of the whole query-side selection step, composed from the oracle.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (never imported by the product).
It follows the reference's optimised query sequence
(sglang/srt/layers/attention/v1_deepseek/runtime.py:417-636 with the fixed page
budget of bench_v1_dynamic_budget_metadata.py) row by row:
metadata -> centre logits -> route -> fine table -> sink/tail staging -> fine
logits -> fused top-k -> latent gather.  Scoring uses the BLAS form of the
reference formula (float64 matmul), so the timed CPU baseline uses every core
BLAS is given.
"""
from __future__ import annotations

import numpy as np

from . import v1x_oracle as O


def to_numpy_case(case, rows=None):
    """Copy the needed parts of a synth.QueryCase (any device) to numpy."""
    import torch

    rows = list(range(case.B)) if rows is None else list(rows)
    idx = torch.as_tensor(rows, dtype=torch.long, device=case.lens.device)
    g = lambda t: t.index_select(0, idx).cpu().numpy()
    return dict(rows=rows, lens=g(case.lens), q8=g(case.q8.view(torch.uint8)), w=g(case.w),
                nt=g(case.native_table), rt=g(case.reordered_table), ct=g(case.center_table),
                native=case.native.cpu().numpy(), fine=case.fine.cpu().numpy(),
                centers=case.centers.cpu().numpy(), members=case.members.cpu().numpy(),
                latent=None if case.latent is None else case.latent.view(torch.int16).cpu().numpy(),
                P=case.P, take=case.take, window=case.window, topk=case.topk, capacity=case.capacity)


def run_rows(c, rows=None):
    """Run the full step for the given row indices of a numpy case; returns per-row outputs."""
    rows = range(len(c["lens"])) if rows is None else rows
    out = []
    P, take_cfg, window, T, cap = c["P"], c["take"], c["window"], c["topk"], c["capacity"]
    width = -(-(take_cfg * 64 + 64 + 4096) // 256) * 256
    for r in rows:
        n = int(c["lens"][r])
        lens = np.array([n], np.int32)
        nt = c["nt"][r:r + 1]
        fl, tk, dg, cl, _ = O.query_metadata(lens, nt, P, T, 1, 2, 64, window, budget=take_cfg)
        tr = np.array([0], np.int32)       # the row owns its staging pages (private tail)
        clog = O.score_paged(c["q8"][r:r + 1], c["w"][r:r + 1], c["centers"], c["ct"][r:r + 1], cl,
                             P * 8, exact=False)
        sel, _ = O.route(clog, lens, tk, take_cfg, P, c["rt"][r:r + 1],
                         np.zeros((1, width // 64), np.int32), tr, cap, False)
        ft = O.fine_table_shared(c["rt"][r:r + 1], sel, tk, (1, width // 64), tr, cap, P, take_cfg, 68)
        # sink + tail tokens come straight from the native pages (what staging copies)
        sink, tail = (int(x) for x in O.bounds(n, 64, window))
        ids = np.concatenate([np.arange(sink), np.arange(tail, n)])
        k_sel, s_sel = O.page_keys(c["fine"], ft[0], int(tk[0]) * 64)
        k_nat, s_nat = O.page_keys(c["native"], nt[0], n)
        keys = np.concatenate([k_sel, k_nat[ids]])
        sc = np.concatenate([s_sel, s_nat[ids]])
        scores = np.full((1, width), -np.inf, np.float32)
        scores[0, :keys.shape[0]] = O.score_row(c["q8"][r], c["w"][r], keys, sc, exact=False)
        e = O.topk(scores, fl, c["members"], c["rt"][r:r + 1], nt, sel, lens, tk, window, True, T,
                   fine_table=ft, direct_fine=False)
        kv = None
        if c["latent"] is not None:
            kv, _ = O.gather_slots(c["latent"], None, None, e["physical"], 1, T, 0)
        out.append(dict(selected=sel[0], physical=e["physical"][0], kv=kv))
    return out


# --------------------------------------------------------------------------
# page lifecycle driver (DS/runtime.py:681-825, Build.compute page part :230-270)
# --------------------------------------------------------------------------

class ArenaPort:
    """numpy restatement of the request-level page lifecycle that
    10_20_b200/lifecycle.PageArena drives on the GPU: per request a page table,
    centre table and lease list; per newly complete bucket fingerprint ->
    match_pages -> allocate -> publish; release returns every lease."""

    def __init__(self, capacity, pages, max_requests=None):
        self.capacity, self.pages = capacity, pages
        self.max_requests = max_requests if max_requests is not None else max(capacity // pages, 1)
        self.max_leases = capacity // 16
        self.fine = np.zeros((capacity, O.PAGE_BYTES), np.uint8)
        self.centers = np.zeros((-(-capacity // 8), O.PAGE_BYTES), np.uint8)
        self.members = np.full((capacity, 64), -1, np.int32)
        self.refs = np.zeros(capacity, np.int32)
        self.free = np.arange(capacity, dtype=np.int32)
        self.count = capacity
        self.hashes = np.zeros((capacity, 2), np.int64)
        self.tables = np.full((self.max_leases, 16), -1, np.int32)
        self.center_pages = np.arange(self.max_leases * 2, dtype=np.int32).reshape(-1, 2)
        self.free_leases = list(range(self.max_leases - 1, -1, -1))
        self.states = {}

    def _bucket(self, tmp, mapping, centers, start, lease):
        meta = np.array([start, lease, 1], np.int32)
        h = O.fingerprint(tmp, mapping)
        match = O.match_pages(tmp, mapping, h, self.fine, self.members, self.hashes, self.refs, self.capacity)
        try:
            self.count, new = O.allocate(meta, match, self.free, self.count, self.refs, self.tables)
        except O.ArenaExhausted:
            # the arena is unchanged; the lease's table row reads "no page" (the
            # CUDA allocate's contract: a later release of the lease is a no-op)
            self.tables[lease] = -1
            raise
        O.publish(tmp, centers, mapping, h, meta, self.tables, new, self.fine, self.centers, self.members,
                  self.hashes)

    def prepare(self, owner, length, bucket_source):
        st = self.states.get(owner)
        if st is not None and length < st["length"]:
            self.release(owner)
            st = None
        if st is None:
            if len(self.states) >= self.max_requests:
                raise ValueError("V1 request capacity exceeded")
            st = self.states[owner] = dict(table=np.zeros(self.pages, np.int32),
                                           center_table=np.zeros(self.pages // 8, np.int32), leases=[],
                                           length=0)
        for bucket in range(len(st["leases"]), length // 1024):
            lease = self.free_leases.pop()
            tmp, mapping, centers = bucket_source(owner, bucket)
            self._bucket(tmp, mapping, centers, bucket * 1024, lease)
            st["leases"].append(lease)
            st["table"][bucket * 16:(bucket + 1) * 16] = self.tables[lease]
            st["center_table"][bucket * 2:(bucket + 1) * 2] = self.center_pages[lease]
        st["length"] = length
        return st

    def release(self, owner):
        st = self.states.pop(owner, None)
        if st:
            for lease in st["leases"]:
                self.count = O.release(self.tables[lease], self.refs, self.free, self.count)
                self.free_leases.append(lease)


# --------------------------------------------------------------------------
# batched lifecycle (the algorithm of v1x_prepare_buckets / v1x_release_many),
# restated to check that it gives the per-bucket sequence's arena state
# --------------------------------------------------------------------------

COLLISION = -2


def _same_page(bytes_a, bytes_b, members_a, members_b):
    return np.array_equal(bytes_a, bytes_b) and np.array_equal(members_a, members_b)


def prepare_buckets_batched(arena, tmp, centers, mapping, meta):
    """The batched prepare on an ArenaPort's arrays: tmp u8 [nb, 16, 8448],
    centers u8 [nb, 2, 8448], mapping i32 [nb, 16, 64], meta i32 [nb, 3] =
    (token start, lease, active).  Steps: fingerprints; each page's lowest
    match among the pages live at the START of the call; each page's lowest
    equal-fingerprint page in an earlier bucket, kept if its bytes and members
    are equal, else marked as a collision; then bucket by bucket the allocate
    decision -- no live match: the slot of the earliest equal page (or, after a
    collision, of an equal page published earlier in the call); fresh pages pop
    the free stack -- and the first bucket that finds the stack too short stops
    the call (it and the later buckets change nothing); finally publish.
    Returns (new flags [nb*16] with 2 = not allocated, exhausted: bool)."""
    nb = tmp.shape[0]
    nq = nb * 16
    tp = tmp.reshape(nq, O.PAGE_BYTES)
    mp = mapping.reshape(nq, 64)
    active = np.repeat(np.asarray(meta)[:, 2] != 0, 16)
    h = O.fingerprint(tp, mp)
    live = arena.refs[:arena.capacity] > 0          # snapshot at the start of the call
    match = np.full(nq, -1, np.int64)
    for q in np.nonzero(active)[0]:
        cand = np.nonzero(live & (arena.hashes[:, 0] == h[q, 0]) & (arena.hashes[:, 1] == h[q, 1]))[0]
        for j in cand:
            if _same_page(arena.fine[j], tp[q], arena.members[j], mp[q]):
                match[q] = j
                break
    first = {}
    for q in np.nonzero(active)[0]:
        b0 = q // 16 * 16
        earlier = [p for p in range(b0) if active[p] and h[p, 0] == h[q, 0] and h[p, 1] == h[q, 1]]
        if earlier:
            p = earlier[0]
            first[q] = p if _same_page(tp[p], tp[q], mp[p], mp[q]) else COLLISION
    dst = np.full(nq, -1, np.int64)
    new = np.zeros(nq, np.uint8)
    fresh_so_far = []
    exhausted = False
    for b in range(nb):
        if meta[b][2] == 0:
            continue
        qs = list(range(b * 16, b * 16 + 16))
        if exhausted:
            new[qs] = 2
            arena.tables[int(meta[b][1])] = -1
            continue
        m = []
        for q in qs:
            mq = match[q]
            if mq < 0 and q in first:
                if first[q] != COLLISION:
                    mq = dst[first[q]]
                else:
                    for p in fresh_so_far:
                        if (h[p] == h[q]).all() and _same_page(tp[p], tp[q], mp[p], mp[q]):
                            mq = dst[p]
                            break
            m.append(mq)
        fresh = [x < 0 for x in m]
        needed = sum(fresh)
        if arena.count < needed:
            exhausted = True
            new[qs] = 2
            arena.tables[int(meta[b][1])] = -1
            continue
        rank = 0
        lease = int(meta[b][1])
        for i, q in enumerate(qs):
            if fresh[i]:
                d = int(arena.free[arena.count - 1 - rank])
                rank += 1
                fresh_so_far.append(q)
            else:
                d = int(m[i])
            arena.refs[d] += 1
            arena.tables[lease, i] = d
            dst[q] = d
            new[q] = 1 if fresh[i] else 0
        arena.count -= needed
    for b in range(nb):
        if meta[b][2] != 0 and new[b * 16] != 2:
            O.publish(tmp[b], centers[b], mapping[b], h[b * 16:(b + 1) * 16], meta[b], arena.tables,
                      new[b * 16:(b + 1) * 16].astype(bool), arena.fine, arena.centers, arena.members, arena.hashes)
    return new, exhausted


def release_many(arena, requests_leases):
    """The batched release on an ArenaPort's arrays: requests one after another;
    within a request every lease's pages are decremented at once and the pages
    that reach zero are pushed in (lease, lane) order.  Equals the per-lease
    release sequence when a request's pages are distinct (asserted)."""
    for leases in requests_leases:
        pages = [int(arena.tables[lease, i]) for lease in leases for i in range(16)
                 if arena.tables[lease, i] >= 0]          # -1: an aborted lease
        assert len(set(pages)) == len(pages), "a request's pages must be distinct"
        dead = []
        for page in pages:
            arena.refs[page] -= 1
            if arena.refs[page] == 0:
                dead.append(page)
        arena.free[arena.count:arena.count + len(dead)] = dead
        arena.count += len(dead)
