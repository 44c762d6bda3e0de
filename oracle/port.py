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
        self.count, new = O.allocate(meta, match, self.free, self.count, self.refs, self.tables)
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
