"""numpy restatement of the reference's V1 query-side selection path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this file;
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
use it as the checker / the timed CPU port.

Every function cites the reference file and lines whose behaviour it
restates.  Paths are relative to the reference checkout root:

  DS  = sglang/srt/layers/attention/v1_deepseek
  NA  = sglang/srt/layers/attention/v1_native
  VQ  = sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh
  TKI = sglang/kernels/jit/include/sgl_kernel/deepseek_v4/topk_impl.cuh

Packed page format (DS/kernels.py:1-3, DS/README.txt:8-10): one 64-token
page is 8448 bytes = 64 x 128 FP8 e4m3 key bytes (token-major) followed by
64 fp32 scales; viewed as float32 the scale of token j sits at word 2048 + j.

Pinning: the golden fixtures under ``tests/golden/`` were produced by running
the reference's own Triton kernels (DS/kernels.py, NA/kernels.py,
NA/fused_grouping.py) in the Triton CPU interpreter, and by running the torch
reference math of DS/example_v1_query_single_head.py on CPU; the CPU test
suite checks every function below against them.

Two documented contract choices (the reference leaves them open):
  * Top-2048 exact ties at the selection boundary are broken by the lower
    candidate index (the reference resolves ties beyond 128 coarse-bin
    candidates by shared-memory atomic order, TKI:400-401).  Outputs are
    emitted in ascending raw-index order (the reference leaves the order
    unspecified, DS/example_v1_query_single_head.py:66).
  * Where the reference would read outside a row (route's fine-table write
    for a page id >= pages, VQ:47), the restatement writes -1.
"""
from __future__ import annotations

import numpy as np

PAGE_BYTES = 8448
K_BYTES = 8192
SCALE_WORD = 2048          # float32 index of the first scale within a page
PAGE_WORDS = PAGE_BYTES // 4
NEG_INF = np.float32(-np.inf)


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def _e4m3_table() -> np.ndarray:
    """Decode table for OCP FP8 e4m3 ("fn": no inf, S.1111.111 is NaN)."""
    t = np.zeros(256, np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 15 and m == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * m * 2.0 ** -9
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = _e4m3_table()


def e4m3_to_f32(u8: np.ndarray) -> np.ndarray:
    return E4M3[np.asarray(u8, np.uint8)]


def ctrunc_div(a, b):
    """C integer division (truncates toward zero), as CUDA's int '/'."""
    a = np.asarray(a, np.int64)
    q = np.abs(a) // b
    return np.where(a < 0, -q, q)


def cdiv(a, b):
    return -(-a // b)


def bounds(n, sink_cfg, window):
    """sink / tail of a row of visible length n.

    DS/kernels.py:242-243 (query_lengths), :543-544 (stage_tail_shared),
    VQ:69-70 (fused topk).
    """
    n = np.asarray(n, np.int64)
    sink = np.minimum(sink_cfg, n)
    built = np.maximum(n - 1, 0) // 1024 * 1024
    tail = np.maximum(sink, np.minimum(built, np.maximum(sink, n - window)))
    return sink, tail


def twiddle_key(values: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 key of float32 values, -0.0 folded onto +0.0.

    This is CUB's radix twiddle (flip all bits of negatives, set the sign bit
    of non-negatives) together with CUB's rule that -0.0 and +0.0 are equal
    radix keys (cub/block/radix_rank_sort_operations.cuh,
    BaseDigitExtractor::ProcessFloatMinusZero), which VQ:42 inherits through
    BlockRadixSort.  The Top-2048 selection uses the same key: the
    reference's fp32 boundary comparisons (TKI:586-595) also treat -0 == +0.
    """
    bits = np.ascontiguousarray(values, np.float32).view(np.uint32)
    key = np.where(bits & np.uint32(0x80000000), ~bits, bits | np.uint32(0x80000000))
    return np.where(key == np.uint32(0x7FFFFFFF), np.uint32(0x80000000), key).astype(np.uint32)


def select_topk(values: np.ndarray, topk: int) -> np.ndarray:
    """Top-`topk` candidate indices of one row, ascending index order.

    Selected set = the `topk` largest by (value desc, index asc); if the row
    holds <= topk candidates, indices [0, L) then -1 (VQ:109-111).
    """
    L = values.shape[0]
    out = np.full(topk, -1, np.int32)
    if L <= topk:
        out[:L] = np.arange(L, dtype=np.int32)
        return out
    key = twiddle_key(values).astype(np.uint64)
    comp = ((np.uint64(0xFFFFFFFF) - key) << np.uint64(32)) | np.arange(L, dtype=np.uint64)
    part = np.argpartition(comp, topk - 1)[:topk]
    out[:] = np.sort(part).astype(np.int32)
    return out


# --------------------------------------------------------------------------
# per-row metadata
# --------------------------------------------------------------------------

def query_metadata(lens, nt_flat, NP, TOPK, NUM, DEN, SINK, WINDOW, budget=None):
    """DS/kernels.py:568-591 (query_metadata).

    With ``budget`` the take rule is the benchmark's fixed page budget
    ``take = min(pages, budget)`` (bench_v1_dynamic_budget_metadata.py:5-27).
    Returns (fine_lens, takes, dg_lens, center_lens, tail_rows), int32.
    """
    lens = np.asarray(lens, np.int64)
    nt_flat = np.asarray(nt_flat, np.int64).reshape(-1)
    B = lens.shape[0]
    pages = np.maximum(lens - 1, 0) // 1024 * 16
    if budget is None:
        take = np.minimum(pages, np.maximum((pages * NUM + DEN - 1) // DEN, cdiv(TOPK, 64)))
    else:
        take = np.minimum(pages, int(budget))
    sink, tail = bounds(lens, SINK, WINDOW)
    fine = take * 64 + sink + lens - tail
    tail_rows = np.empty(B, np.int64)
    i = np.arange(128)
    for r in range(B):
        n = lens[r]
        page = np.where(i == 0, 0, tail[r] // 64 + i - 1)
        valid = (n > 0) & ((i == 0) | (page < (n + 63) // 64)) & (page < NP)
        mine = np.where(valid, nt_flat[np.where(valid, r * NP + page, 0)], -1)
        first = np.where(valid, nt_flat[np.where(valid, page, 0)], -1)
        share = (n == lens[0]) and bool(np.all(mine == first))
        tail_rows[r] = 0 if share else r
    i32 = lambda x: np.asarray(x, np.int64).astype(np.int32)
    return (i32(fine), i32(take), i32(np.maximum(fine, 1)), i32(np.maximum(pages * 8, 1)),
            i32(tail_rows))


def query_lengths(lens, TOPK, NUM, DEN, SINK, WINDOW):
    """DS/kernels.py:224-245 (query_lengths). Returns (fine_lens, takes)."""
    lens = np.asarray(lens, np.int64)
    pages = np.maximum(lens - 1, 0) // 1024 * 16
    take = np.minimum(pages, np.maximum((pages * NUM + DEN - 1) // DEN, cdiv(TOPK, 64)))
    sink, tail = bounds(lens, SINK, WINDOW)
    return ((take * 64 + sink + lens - tail).astype(np.int32), take.astype(np.int32))


# --------------------------------------------------------------------------
# fused.route  (VQ:7-49, host checks VQ:155-180)
# --------------------------------------------------------------------------

_ROUTE_SHAPES = ((128, 64, 2), (256, 64, 4), (512, 64, 8), (1024, 128, 8),
                 (2048, 128, 16), (4096, 128, 32))


def route_geometry(pages: int):
    """(THREADS, ITEMS) the reference picks for `pages` (VQ:175-177)."""
    for lim, t, it in _ROUTE_SHAPES:
        if pages <= lim:
            return t, it
    raise ValueError("pages > 4096")


def route(scores, lens, takes, K, pages, rt, ft, tail_rows, capacity, fill_table,
          selected_dtype=np.int32):
    """fused.route: per-page max of 8 centres, then a stable descending page sort.

    VQ:11-22   fine-table tail fill and the take >= active identity branch
    VQ:26-41   page score = fmaxf over its 8 centres (p < active), else -inf;
               thread t item i holds blocked rank t*I+i, i.e. page
               p = rank / BASE + (rank % BASE) * 128, BASE = T*I/128
    VQ:42      BlockRadixSort descending -> stable: ties keep blocked rank
    VQ:43-48   selected[row, rank] for rank < K; ft[row, rank] for rank < take
    Returns (selected [B,K], ft (copy, modified)).
    """
    scores = np.asarray(scores, np.float32)
    B = scores.shape[0]
    L = scores.shape[1]
    rt = np.asarray(rt).reshape(B, pages)
    ft = np.array(ft, np.int32, copy=True)
    fine_pages = ft.shape[1]
    T, I = route_geometry(pages)
    n_items = T * I
    base = n_items // 128
    sel = np.empty((B, K), selected_dtype)
    rank = np.arange(n_items)
    p_of_rank = rank // base + (rank % base) * 128
    for r in range(B):
        n = int(lens[r])
        take = int(takes[r])
        active = max(n - 1, 0) // 1024 * 16
        if fill_table:
            j = np.arange(max(take, 0), fine_pages)
            ft[r, j] = capacity + int(tail_rows[r]) * 68 + np.minimum(j - take, 67)
        if take >= active:
            sel[r, :] = np.arange(K)
            if fill_table:
                m = min(take, K)
                ft[r, :m] = rt[r, :m]
            continue
        act = min(active, L // 8)
        vals = np.full(n_items, NEG_INF, np.float32)
        valid = p_of_rank < act
        pv = p_of_rank[valid]
        cen = scores[r, : act * 8].reshape(act, 8)
        vals[valid] = np.fmax.reduce(cen, axis=1)[pv]
        key = twiddle_key(vals).astype(np.int64)
        order = np.lexsort((rank, 0xFFFFFFFF - key))      # key desc, blocked rank asc
        ids = p_of_rank[order]
        sel[r, :] = ids[:K]
        if fill_table:
            m = max(min(take, fine_pages), 0)
            got = ids[:m]
            ft[r, :m] = np.where(got < pages, rt[r, np.minimum(got, pages - 1)], -1)
    return sel, ft


# --------------------------------------------------------------------------
# fused.topk  (VQ:62-153) and the non-fused pieces it replaces
# --------------------------------------------------------------------------

def topk(scores, fine_lens, members, rt, nt, selected, lens, takes, window, mask,
         topk_n, expansion_stride=0, physical_output=True, bucket_from_rank=True,
         fine_table=None, direct_fine=False):
    """fused.topk.

    VQ:71-107  in-place -inf mask of boundary-bucket members (rows r < take)
    VQ:108-119 Top-`topk_n` over scores[row, :fine_lens[row]]
    VQ:121-148 raw -> logical -> physical mapping, optional x4 expansion
    Returns dict(scores=masked copy, logical, physical, raw, expanded);
    physical/raw are None when physical_output is False, expanded None when
    expansion_stride == 0.
    """
    s = np.array(scores, np.float32, copy=True)
    B, cols = s.shape
    members = np.asarray(members, np.int64).reshape(-1)
    pages = np.asarray(rt).shape[1]
    rt = np.asarray(rt, np.int64)
    nt = np.asarray(nt, np.int64)
    selected = np.asarray(selected, np.int64)
    if fine_table is not None:
        fine_table = np.asarray(fine_table, np.int64)
    logical_o = np.empty((B, topk_n), np.int32)
    physical_o = np.empty((B, topk_n), np.int32) if physical_output else None
    raw_o = np.empty((B, topk_n), np.int32) if physical_output else None
    expanded = np.empty((B, expansion_stride), np.int32) if expansion_stride else None
    offs = np.arange(64)
    for r in range(B):
        n = int(lens[r])
        take = int(takes[r])
        sink, tail = (int(x) for x in bounds(n, 64, window))
        if mask:
            for rr in range(max(take, 0)):
                rank = int(selected[r, rr])
                if bucket_from_rank:
                    bucket = (rank // 16) * 1024
                else:
                    bucket = int(ctrunc_div(members[int(rt[r, rank]) * 64], 1024)) * 1024
                if bucket < sink or bucket + 1024 > tail:
                    page = int(rt[r, rank])
                    lg = members[page * 64 + offs]
                    bad = (lg < sink) | (lg >= tail)
                    col = rr * 64 + offs
                    ok = bad & (col < cols)
                    s[r, col[ok]] = NEG_INF
        L = min(int(fine_lens[r]), cols)
        raw = select_topk(s[r, :max(L, 0)], topk_n)
        lg = np.full(topk_n, -1, np.int64)
        ph = np.full(topk_n, -1, np.int64)
        ok = (raw >= 0) & (raw < L)
        okv = ok.copy()
        okv[ok] = s[r, raw[ok]] != NEG_INF
        for t in np.nonzero(okv)[0]:
            x = int(raw[t])
            if x < take * 64:
                if direct_fine:
                    page = int(fine_table[r, x // 64])
                else:
                    page = int(rt[r, int(selected[r, x // 64])])
                logical = int(members[page * 64 + x % 64])
            else:
                off = x - take * 64
                logical = off if off < sink else tail + off - sink
            if 0 <= logical < n:
                lg[t] = logical
                ph[t] = nt[r, logical // 64] * 64 + logical % 64
        logical_o[r] = lg
        if physical_output:
            physical_o[r] = ph
            raw_o[r] = raw
        if expansion_stride:
            e = np.full(expansion_stride, -1, np.int64)
            base4 = lg[:, None] * 4 + np.arange(4)[None, :]
            e[: 4 * topk_n] = np.where(lg[:, None] < 0, -1, base4).reshape(-1)
            expanded[r] = e
    return dict(scores=s, logical=logical_o, physical=physical_o, raw=raw_o, expanded=expanded)


def mask_fine(scores, selected, rt, members, lens, takes, MAXP, TAKE, STRIDE, WIDTH, SINK,
              WINDOW):
    """DS/kernels.py:444-472 (mask_fine), returns the modified copy."""
    s = np.array(scores, np.float32, copy=True).reshape(-1)
    selected = np.asarray(selected, np.int64).reshape(-1)
    rt = np.asarray(rt, np.int64).reshape(-1)
    members = np.asarray(members, np.int64).reshape(-1)
    B = len(lens)
    j = np.arange(WIDTH)
    for r in range(B):
        n = int(lens[r])
        take = int(takes[r])
        sink, tail = (int(x) for x in bounds(n, SINK, WINDOW))
        count = take * 64 + sink + n - tail
        fine = j < take * 64
        rank = np.where(fine, selected[np.where(fine, r * TAKE + j // 64, 0)], 0)
        page = np.where(fine, rt[r * MAXP + rank], 0)
        logical = np.where(fine, members[page * 64 + j % 64], -1)
        good = (j < count) & (~fine | ((logical >= sink) & (logical < tail)))
        row = s[r * STRIDE: r * STRIDE + WIDTH]
        s[r * STRIDE: r * STRIDE + WIDTH] = np.where(good, row, NEG_INF)
    return s.reshape(np.asarray(scores).shape)


def reduce_centers(logits, lens, MAXP, STRIDE):
    """DS/kernels.py:475-486 (reduce_centers): [B, MAXP] page maxima."""
    logits = np.asarray(logits, np.float32).reshape(-1)
    B = len(lens)
    out = np.empty((B, MAXP), np.float32)
    p = np.arange(MAXP)
    for r in range(B):
        pages = max(int(lens[r]) - 1, 0) // 1024 * 16
        idx = r * STRIDE + p[:, None] * 8 + np.arange(8)[None, :]
        v = np.where((p < pages)[:, None], logits[np.where((p < pages)[:, None], idx, 0)], NEG_INF)
        out[r] = v.max(axis=1)
    return out


def output_ids(raw, scores, members, rt, nt, selected, lens, takes, MAXP, NP, TAKE, WIDTH,
               TOPK, SINK, WINDOW, map_physical=True, direct_fine=False, ft=None, FP=0):
    """DS/kernels.py:323-376 (output_ids): non-fused raw -> logical/physical map."""
    raw = np.asarray(raw, np.int64).reshape(-1)
    scores = np.asarray(scores, np.float32).reshape(-1)
    members = np.asarray(members, np.int64).reshape(-1)
    rt = np.asarray(rt, np.int64).reshape(-1)
    nt = np.asarray(nt, np.int64).reshape(-1)
    selected = np.asarray(selected, np.int64).reshape(-1)
    B = len(lens)
    out = np.empty((B, TOPK), np.int32)
    logical_o = np.empty((B, TOPK), np.int32)
    for r in range(B):
        rw = raw[r * TOPK:(r + 1) * TOPK]
        take = int(takes[r])
        n = int(lens[r])
        sink, tail = (int(x) for x in bounds(n, SINK, WINDOW))
        valid = (rw >= 0) & (rw < WIDTH)
        inb = valid & (rw < take * 64)
        if direct_fine:
            ftf = np.asarray(ft, np.int64).reshape(-1)
            page = np.where(inb, ftf[np.where(inb, r * FP + rw // 64, 0)], 0)
        else:
            rank = np.where(inb, selected[np.where(inb, r * TAKE + rw // 64, 0)], 0)
            page = np.where(inb, rt[r * MAXP + rank], 0)
        member = np.where(inb, members[np.where(inb, page * 64 + rw % 64, 0)], -1)
        off = rw - take * 64
        logical = np.where(rw < take * 64, member, np.where(off < sink, off, tail + off - sink))
        sc = np.where(valid, scores[np.where(valid, r * WIDTH + rw, 0)], NEG_INF)
        valid = valid & (sc != NEG_INF) & (logical >= 0) & (logical < n)
        if map_physical:
            ph = np.where(valid, nt[np.where(valid, r * NP + logical // 64, 0)] * 64 + logical % 64, -1)
            out[r] = ph
        logical_o[r] = np.where(valid, logical, -1)
    return out, logical_o


def expand_logical(logical, TOPK, STRIDE):
    """DS/kernels.py:594-600 (expand_logical)."""
    logical = np.asarray(logical, np.int64).reshape(len(logical), TOPK)
    B = logical.shape[0]
    out = np.full((B, STRIDE), -1, np.int32)
    j = np.arange(STRIDE)
    for r in range(B):
        lg = np.where(j < TOPK * 4, logical[r, np.minimum(j // 4, TOPK - 1)], -1)
        out[r] = np.where((j < TOPK * 4) & (lg >= 0), lg * 4 + j % 4, -1)
    return out


def fine_table_shared(rt, selected, takes, ft_shape, tail_rows, CAP, MAXP, TAKE, SCRATCH):
    """DS/kernels.py:488-514 (fine_table_shared). ft_shape = (B, FP)."""
    B, FP = ft_shape
    rt = np.asarray(rt, np.int64).reshape(-1)
    selected = np.asarray(selected, np.int64).reshape(-1)
    ft = np.empty((B, FP), np.int64)
    j = np.arange(FP)
    for r in range(B):
        take = int(takes[r])
        inb = j < take
        rank = np.where(inb, selected[np.where(inb, r * TAKE + j, 0)], 0)
        page = np.where(inb, rt[r * MAXP + rank], 0)
        pad = CAP + int(tail_rows[r]) * SCRATCH + np.minimum(np.maximum(j - take, 0), SCRATCH - 1)
        ft[r] = np.where(inb, page, pad)
    return ft.astype(np.int32)


def stage_tail_shared(native_u8, nt_flat, lens, fine_u8, tail_rows, CAP, NP, SCRATCH, SINK,
                      WINDOW, ROWS, GROUP, grid0, grid1):
    """DS/kernels.py:518-564 (stage_tail_shared); returns the modified fine pool copy.

    For each program (group, p) and each owner row (tail_rows[r] == r) of
    the group: copy candidate slots i in [p*64, p*64+64) -- logical
    i < sink ? i : tail + i - sink -- from the native page into staging page
    CAP + r*SCRATCH + p; masked slots (i >= count) get zero bytes / scale.
    """
    native_u8 = np.asarray(native_u8, np.uint8)
    nat_f = native_u8.view(np.float32).reshape(-1, PAGE_WORDS)
    fine = np.array(fine_u8, np.uint8, copy=True)
    fin_f = fine.view(np.float32).reshape(-1, PAGE_WORDS)
    nt_flat = np.asarray(nt_flat, np.int64).reshape(-1)
    lens = np.asarray(lens, np.int64)
    tail_rows = np.asarray(tail_rows, np.int64)
    for g in range(grid0):
        rows = g * GROUP + np.arange(GROUP)
        valid = rows < ROWS if ROWS > 0 else np.ones(GROUP, bool)
        for row in rows[valid]:
            if tail_rows[row] != row:
                continue
            n = int(lens[row])
            sink, tail = (int(x) for x in bounds(n, SINK, WINDOW))
            count = sink + n - tail
            for p in range(grid1):
                if not (p * 64 < count or p == 0):
                    continue
                i = p * 64 + np.arange(64)
                inb = i < count
                logical = np.where(i < sink, i, tail + i - sink)
                page = np.where(inb, nt_flat[np.where(inb, row * NP + logical // 64, 0)], 0)
                dst = CAP + row * SCRATCH + p
                vals = native_u8[page[:, None], (logical % 64)[:, None] * 128 + np.arange(128)[None, :]]
                vals = np.where(inb[:, None], vals, 0).astype(np.uint8)
                fine[dst, :K_BYTES] = vals.reshape(-1)
                sc = np.where(inb, nat_f[page, SCALE_WORD + logical % 64], np.float32(0))
                fin_f[dst, SCALE_WORD:SCALE_WORD + 64] = sc
    return fine


# --------------------------------------------------------------------------
# _sort  (NA/fused_grouping.py:64-76)
# --------------------------------------------------------------------------

def sort_segments(P, S, flag, N, groups, heads, O=None):
    """Stable descending sort of each N-record segment by score.

    Segment (g, h) covers flat positions h*4096 + g*N + [0, N).  Scores equal
    to zero become +0 (:69); the 64-bit key is (ordered score << 32) |
    (0xFFFFFFFF - i) sorted descending (:70-74), i.e. score desc, position
    asc.  O[...+i] = P[...+pos_i] (:75-76).  FLAG >= 0 makes it a no-op.
    """
    P = np.asarray(P, np.int32).reshape(-1)
    S = np.asarray(S, np.float32).reshape(-1)
    O = np.array(O if O is not None else np.zeros_like(P), np.int32, copy=True).reshape(-1)
    if int(np.asarray(flag).reshape(-1)[0]) >= 0:
        return O
    i = np.arange(N, dtype=np.int64)
    for h in range(heads):
        for g in range(groups):
            b = h * 4096 + g * N
            seg = S[b:b + N]
            seg = np.where(seg == 0, np.float32(0), seg).astype(np.float32)
            bits = seg.view(np.uint32).astype(np.int64)
            ordered = np.where(bits & 0x80000000, bits ^ 0xFFFFFFFF, bits ^ 0x80000000)
            order = np.lexsort((i, 0xFFFFFFFF - ordered))
            O[b:b + N] = P[b + order]
    return O


# --------------------------------------------------------------------------
# index build of one 1024-token bucket: initialize -> grouping -> assemble
# (DS/runtime.py:170-233, Build.compute's first three stages)
# --------------------------------------------------------------------------
BUILD_LEVELS = (1024, 512, 256, 128, 64, 32, 16)


def sum128(p):
    """tl.sum over a last axis of 128 float32 values as the Triton interpreter
    evaluates it (np.sum, numpy's pairwise float32 summation for n = 128):
    eight strided accumulators r_j = p[j] + p[8+j] + ... + p[120+j] in that
    order, then ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))."""
    p = np.asarray(p, np.float32)
    r = p[..., 0:8].copy()
    for i in range(1, 16):
        r = r + p[..., 8 * i:8 * i + 8]
    return ((r[..., 0] + r[..., 1]) + (r[..., 2] + r[..., 3])) + ((r[..., 4] + r[..., 5]) + (r[..., 6] + r[..., 7]))


_E4M3_POS = E4M3[:0x7F].astype(np.float64)   # codes 0x00..0x7E: 0 .. 448 ascending


def e4m3_from_f32(x):
    """float32 -> OCP e4m3fn bytes: round to nearest, ties to the even code,
    saturating at +-448 (the conversion `.to(float8e4nv)` of values that
    already lie within +-448); -0 -> 0x80, NaN -> 0x7F."""
    x = np.asarray(x, np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    hi = np.clip(np.searchsorted(_E4M3_POS, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dhi, dlo = _E4M3_POS[hi] - a, a - _E4M3_POS[lo]
    code = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(lo % 2 == 0, lo, hi)))
    code = np.where(_E4M3_POS[hi] == a, hi, code).astype(np.uint8)
    code = code | (np.signbit(x).astype(np.uint8) << 7)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def pow2_ceil(v):
    """Smallest power of two >= v (v > 0, float32), exactly.  The reference
    writes exp2(ceil(log2(v))) (DS/kernels.py:48-50); with a correctly rounded
    log2 the two agree except for v a few ulps above a power of two, where the
    floating-point log2 rounds down onto the integer."""
    v = np.asarray(v, np.float32)
    bits = v.view(np.uint32)
    exact = (bits & 0x007FFFFF) == 0
    up = ((bits >> 23) + 1).astype(np.uint32) << 23
    return np.where(exact, v, up.view(np.float32)).astype(np.float32)


def build_initialize(native_u8, table):
    """DS/kernels.py:9-29 (initialize).  Token i in [0, 1024) of the bucket:
    page = TABLE[i // 64]; x = e4m3(K[page, i % 64]) * scale (fp32 multiply);
    unit = x / max(sqrt(sum(x*x)), 1e-12).  Returns (unit f32 [1024, 128],
    perm i32 [1024] = 0..1023).  FLAG = -1 when active (:12-13)."""
    native_u8 = np.asarray(native_u8, np.uint8).reshape(-1, PAGE_BYTES)
    table = np.asarray(table, np.int64).reshape(-1)
    i = np.arange(1024)
    page = table[i // 64]
    kb = native_u8[page[:, None], (i % 64)[:, None] * 128 + np.arange(128)[None, :]]
    scale = native_u8.view(np.float32).reshape(-1, PAGE_WORDS)[page, SCALE_WORD + i % 64]
    x = (e4m3_to_f32(kb) * scale[:, None].astype(np.float32)).astype(np.float32)
    norm = np.sqrt(sum128(x * x)).astype(np.float32)
    unit = (x / np.maximum(norm, np.float32(1e-12))[:, None]).astype(np.float32)
    return unit, i.astype(np.int32)


def group_init(k_f32, req, start, heads):
    """NA/fused_grouping.py:27-37 (_init): for the 4096 positions i of head h,
    x = float(K[REQ[START + i], h]) and U[h, i] = x / max(sqrt(sum(x*x)), 1e-12);
    P[h, i] = START + i.  k_f32: [slots, heads, 128] float32 values of K."""
    k = np.asarray(k_f32, np.float32)
    slots = np.asarray(req, np.int64)[start:start + 4096]
    x = np.transpose(k[slots], (1, 0, 2))           # [heads, 4096, 128]
    norm = np.sqrt(sum128(x * x)).astype(np.float32)
    unit = (x / np.maximum(norm, np.float32(1e-12))[..., None]).astype(np.float32)
    P = np.tile(np.arange(4096, dtype=np.int32) + np.int32(start), (heads, 1))
    return unit, P


def group_levels(unit, P, start, levels, count, heads):
    """The level loop of FusedGroups.run / Build.compute over `count` positions
    per head (NA/fused_grouping.py:103-111): three _dots, two _anchor and one
    _sort per level n."""
    P = np.asarray(P, np.int32).reshape(-1).copy()
    A = np.zeros(heads * 512, np.int32)
    S = np.zeros(heads * 4096 if heads > 1 else count, np.float32)
    for n in levels:
        for mode in (0, 1, 2):
            S = group_dots(unit, P, A, S, n, start, mode, count=count, heads=heads)
            if mode < 2:
                A = group_anchor(P, A, S, n, mode, count=count, heads=heads)
        P = sort_segments(P, S, -1, n, count // n, heads, O=np.zeros_like(P))
    return P


def group_dots(unit, P, A, S, N, start, mode, count=1024, heads=1):
    """NA/fused_grouping.py:39-54 (_dots).  Position i of head h (flat index
    h*4096 + i, i < count): ids = P[.] - START; the anchor is the group's first
    member P[h*4096 + (i//N)*N] (MODE 0) or A[h*256 + i//N, MODE-1] (MODE 1, 2),
    minus START; value = sum(U[h, ids] * U[h, anchor]); MODE 2 subtracts the
    previous S.  U rows are [heads, stride, 128] with stride = 4096 for heads > 1
    (the 4K FusedGroups layout) and the compact bucket otherwise."""
    P = np.asarray(P, np.int64).reshape(-1)
    A = np.asarray(A, np.int64).reshape(-1)
    S = np.array(S, np.float32, copy=True).reshape(-1)
    U = np.asarray(unit, np.float32).reshape(heads, -1, 128)
    i = np.arange(count)
    for h in range(heads):
        f = h * 4096 + i
        ids = P[f] - start
        if mode == 0:
            anc = P[h * 4096 + (i // N) * N] - start
        else:
            anc = A[(h * 256 + i // N) * 2 + (mode - 1)] - start
        value = sum128(U[h, ids] * U[h, anc])
        S[f] = (value - S[f]).astype(np.float32) if mode == 2 else value
    return S


def group_anchor(P, A, S, N, slot, count=1024, heads=1):
    """NA/fused_grouping.py:56-63 (_anchor): for every group of N positions the
    position of the minimum score, leftmost on ties -> A[h*256+group, SLOT] =
    P[...+pos]."""
    P = np.asarray(P, np.int32).reshape(-1)
    S = np.asarray(S, np.float32).reshape(-1)
    A = np.array(A, np.int32, copy=True).reshape(-1)
    for h in range(heads):
        for g in range(count // N):
            b = h * 4096 + g * N
            A[(h * 256 + g) * 2 + slot] = P[b + int(np.argmin(S[b:b + N]))]
    return A


def group_bucket(unit, start=0, levels=BUILD_LEVELS):
    """The grouping loop of Build.compute (DS/runtime.py:183-215): for each
    level n, per group of n positions: MODE 0 dots against the first member,
    the farthest member b (anchor slot 0), MODE 1 dots against b, the farthest
    member a from b (slot 1), MODE 2 margin = dot(x, a) - dot(x, b), then the
    stable descending sort of the margins; the next level halves the groups.
    Returns the final member permutation (int32 [1024], offset by START)."""
    P = np.arange(1024, dtype=np.int32) + start
    A = np.zeros(2 * 256, np.int32)
    S = np.zeros(1024, np.float32)
    for n in levels:
        for mode in (0, 1, 2):
            S = group_dots(unit, P, A, S, n, start, mode)
            if mode < 2:
                A = group_anchor(P, A, S, n, mode)
        P = sort_segments(P, S, -1, n, 1024 // n, 1, O=np.zeros_like(P))
    return P


def build_assemble(native_u8, table, start, ids):
    """DS/kernels.py:32-54 (assemble), 16 pages x 8 groups of 8 members.
    Member i of page p: src = IDS[p*64 + i]; its K bytes and scale (native page
    TABLE[src // 64], row src % 64) are copied to TMP[p, i]; MAP[p, i] = START +
    src.  Each group's centre: mean = (sum over the 8 members, in order, of
    e4m3(K) * scale) / 8; cs = pow2_ceil(max(max|mean|, 1e-4) / 448); centre c =
    p*8 + g is written as e4m3(mean / cs) at CENTERS[c // 64, c % 64] with scale
    cs.  Returns (tmp u8 [16, 8448], centers u8 [2, 8448], mapping i32 [16, 64])."""
    native_u8 = np.asarray(native_u8, np.uint8).reshape(-1, PAGE_BYTES)
    table = np.asarray(table, np.int64).reshape(-1)
    src = np.asarray(ids, np.int64).reshape(16, 64)
    page = table[src // 64]
    kb = native_u8[page[..., None], (src % 64)[..., None] * 128 + np.arange(128)]
    scale = native_u8.view(np.float32).reshape(-1, PAGE_WORDS)[page, SCALE_WORD + src % 64]
    tmp = np.zeros((16, PAGE_BYTES), np.uint8)
    tmp[:, :K_BYTES] = kb.reshape(16, K_BYTES)
    tmp.view(np.float32)[:, SCALE_WORD:] = scale
    mapping = (start + src).astype(np.int32)
    x = (e4m3_to_f32(kb) * scale[..., None].astype(np.float32)).astype(np.float32).reshape(16, 8, 8, 128)
    acc = x[:, :, 0].copy()
    for j in range(1, 8):
        acc = acc + x[:, :, j]
    mean = (acc / np.float32(8.0)).astype(np.float32).reshape(128, 128)
    vmax = np.maximum(np.abs(mean).max(-1), np.float32(1e-4)).astype(np.float32)
    cs = pow2_ceil((vmax / np.float32(448.0)).astype(np.float32))
    centers = np.zeros((2, PAGE_BYTES), np.uint8)
    centers[:, :K_BYTES] = e4m3_from_f32(mean / cs[:, None]).reshape(2, K_BYTES)
    centers.view(np.float32)[:, SCALE_WORD:] = cs.reshape(2, 64)
    return tmp, centers, mapping


def build_bucket(native_u8, table, start):
    """initialize -> grouping -> assemble of one bucket (DS/runtime.py:170-233)."""
    unit, _ = build_initialize(native_u8, table)
    perm = group_bucket(unit)
    return build_assemble(native_u8, table, start, perm)


def group_offsets(keys_sorted_desc: np.ndarray, key_range: int) -> np.ndarray:
    """Exclusive descending-key offsets of one sorted segment (an extension:
    the reference emits only the permutation).  offs[j] = number of records
    whose key > key_range - 1 - j, j in [0, key_range]."""
    k = np.asarray(keys_sorted_desc, np.int64)
    counts = np.bincount(k, minlength=key_range)[::-1]
    return np.concatenate(([0], np.cumsum(counts))).astype(np.int32)


# --------------------------------------------------------------------------
# page lifecycle  (DS/kernels.py:57-179)
# --------------------------------------------------------------------------

def fingerprint(tmp, mapping, active=True):
    """DS/kernels.py:57-69: two int64 (wrapping) sums over bytes and members."""
    x = np.asarray(tmp, np.uint8).reshape(-1, PAGE_BYTES).astype(np.int64)
    m = np.asarray(mapping, np.int64).reshape(-1, 64)
    i = np.arange(PAGE_BYTES, dtype=np.int64)
    j = np.arange(64, dtype=np.int64)
    with np.errstate(over="ignore"):
        a = (x * (i + 1)).sum(1) + (m * 104729).sum(1)
        b = (x * ((i + 7) * 1000003)).sum(1) + (m * (j + 1) * 65537).sum(1)
    return np.stack([a, b], 1).astype(np.int64)


def match_pages(tmp, mapping, hsh, fine, members, hashes, refs, cap):
    """DS/kernels.py:72-113: lowest live page j with equal hashes, bytes and members."""
    tmp = np.asarray(tmp, np.uint8).reshape(-1, PAGE_BYTES)
    mapping = np.asarray(mapping, np.int32).reshape(-1, 64)
    fine = np.asarray(fine, np.uint8).reshape(-1, PAGE_BYTES)
    members = np.asarray(members, np.int32).reshape(-1, 64)
    hashes = np.asarray(hashes, np.int64).reshape(-1, 2)
    refs = np.asarray(refs, np.int32).reshape(-1)
    out = np.full(tmp.shape[0], -1, np.int32)
    hsh = np.asarray(hsh, np.int64).reshape(-1, 2)
    live = np.nonzero(refs[:cap] > 0)[0]              # ascending page ids
    h = hashes[live]
    # candidates of every tmp page at once: live pages with both hashes equal
    hit = (h[:, None, 0] == hsh[None, :, 0]) & (h[:, None, 1] == hsh[None, :, 1])
    for p in range(tmp.shape[0]):
        for j in live[hit[:, p]]:
            if np.array_equal(fine[j], tmp[p]) and np.array_equal(members[j], mapping[p]):
                out[p] = j
                break
    return out


class ArenaExhausted(RuntimeError):
    pass


def allocate(meta, match, free, count, refs, tables):
    """DS/kernels.py:116-131.  Mutates free/refs/tables in place, returns
    (new_count, new_flags).  Raises ArenaExhausted where the reference's
    device_assert (:125) would fire; state is then untouched."""
    meta = np.asarray(meta).reshape(-1)
    match = np.asarray(match, np.int64).reshape(16)
    fresh = match < 0
    rank = np.cumsum(fresh) - 1
    needed = int(fresh.sum())
    count = int(count)
    if count < needed:
        raise ArenaExhausted("V1 page arena exhausted")
    dst = match.copy()
    dst[fresh] = np.asarray(free)[count - 1 - rank[fresh]]
    for d in dst:
        refs[d] += 1
    tables.reshape(-1)[int(meta[1]) * 16 + np.arange(16)] = dst
    return count - needed, fresh.copy()


def publish(tmp, tc_u8, mapping, hsh, meta, tables, new, fine, centers_u8, members, hashes):
    """DS/kernels.py:134-167: fresh pages' bytes/members/hashes to their slots,
    then always the bucket's 128 centres (+ scales) to centre slots
    lease*128 + c.  Mutates fine/centers/members/hashes in place."""
    lease = int(np.asarray(meta).reshape(-1)[1])
    tab = np.asarray(tables).reshape(-1)
    tmp = np.asarray(tmp, np.uint8).reshape(-1, PAGE_BYTES)
    tc = np.asarray(tc_u8, np.uint8).reshape(-1, PAGE_BYTES)
    tcf = tc.view(np.float32).reshape(-1, PAGE_WORDS)
    cf = centers_u8.view(np.float32).reshape(-1, PAGE_WORDS)
    for p in range(16):
        if new[p]:
            d = int(tab[lease * 16 + p])
            fine[d] = tmp[p]
            members[d] = np.asarray(mapping).reshape(-1, 64)[p]
            hashes[d] = np.asarray(hsh).reshape(-1, 2)[p]
        for g in range(8):
            sc = p * 8 + g
            dc = lease * 128 + sc
            centers_u8[dc // 64, (dc % 64) * 128:(dc % 64) * 128 + 128] = \
                tc[sc // 64, (sc % 64) * 128:(sc % 64) * 128 + 128]
            cf[dc // 64, SCALE_WORD + dc % 64] = tcf[sc // 64, SCALE_WORD + sc % 64]


def release(table, refs, free, count):
    """DS/kernels.py:170-179: decrement refs; pages that hit zero are pushed
    to the free stack in lane order.  Returns the new count.  An entry of -1
    (a lease whose allocation aborted; the reference would have trapped before)
    is skipped, as the CUDA release does."""
    count = int(count)
    dead = []
    for page in np.asarray(table).reshape(-1)[:16]:
        if page < 0:
            continue
        old = int(refs[page])
        refs[page] = old - 1
        if old == 1:
            dead.append(int(page))
    for k, page in enumerate(dead):
        free[count + k] = page
    return count + len(dead)


# --------------------------------------------------------------------------
# FP8 paged scoring (DeepGEMM fp8_paged_mqa_logits semantics)
# --------------------------------------------------------------------------

def page_keys(pool_u8, table_row, length):
    """Decode the first `length` tokens of a paged row: (keys f32 [L,128], scales [L])."""
    pool_u8 = np.asarray(pool_u8, np.uint8).reshape(-1, PAGE_BYTES)
    j = np.arange(length)
    pages = np.asarray(table_row, np.int64)[j // 64]
    kb = pool_u8[pages[:, None], (j % 64)[:, None] * 128 + np.arange(128)[None, :]]
    sc = pool_u8.view(np.float32).reshape(-1, PAGE_WORDS)[pages, SCALE_WORD + j % 64]
    return e4m3_to_f32(kb), sc.astype(np.float32)


def score_row(q_u8, w, keys, scales, relu=True, exact=True):
    """score[j] = sum_h w[h] * relu(q[h] . k[j]) * scale[j].

    Formula: DS/kernels.py:310-313 (fine), :210-213 (coarse), pinned against
    DeepGEMM at experiments/fine_pool_shared_20261021/test_and_bench.py:37-41.
    exact=True fixes the fp32 evaluation order the SIMT CUDA scorer uses:
    per head, eight partial sums p_g over dims 16g..16g+15, each accumulated
    in fp32 from 0 in dim order (every e4m3 x e4m3 product is exact in fp32),
    combined as ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)); relu(x) = x if x > 0
    else +0; then heads 0..H-1 accumulated as acc += w[h] * relu(dot) with
    separately rounded multiply and add; then one multiply by the scale.
    exact=False uses a float64 BLAS product (for large cases / timing).
    """
    q = e4m3_to_f32(np.asarray(q_u8, np.uint8)).reshape(-1, 128)
    H = q.shape[0]
    w = np.asarray(w, np.float32).reshape(H)
    if not exact:
        d = keys.astype(np.float64) @ q.astype(np.float64).T
        if relu:
            d = np.maximum(d, 0)
        return ((d @ w.astype(np.float64)) * scales).astype(np.float32)
    qp = q.reshape(H, 1, 8, 16)
    kp = np.asarray(keys, np.float32).reshape(1, -1, 8, 16)
    p = np.zeros((H, keys.shape[0], 8), np.float32)
    for d in range(16):
        p = p + qp[..., d] * kp[..., d]
    p = p[..., 0::2] + p[..., 1::2]
    p = p[..., 0::2] + p[..., 1::2]
    dot = p[..., 0] + p[..., 1]
    if relu:
        dot = np.where(dot > 0, dot, np.float32(0)).astype(np.float32)
    acc = np.zeros(keys.shape[0], np.float32)
    for h in range(H):
        acc = acc + (w[h] * dot[h]).astype(np.float32)
    return (acc * scales).astype(np.float32)


def score_paged(q_u8, w, pool_u8, table, lens, max_len, relu=True, exact=True):
    """[B, max_len] logits; columns >= lens[b] are -inf."""
    B = len(lens)
    out = np.full((B, max_len), NEG_INF, np.float32)
    for b in range(B):
        n = min(int(lens[b]), max_len)
        if n <= 0:
            continue
        keys, sc = page_keys(pool_u8, table[b], n)
        out[b, :n] = score_row(q_u8[b], w[b], keys, sc, relu, exact)
    return out


# --------------------------------------------------------------------------
# _gather_slots  (NA/kernels.py:62-77)
# --------------------------------------------------------------------------

def gather_slots(K, V, REQ, IDS, rows, top, head):
    """KG[t] = K[REQ[IDS[t]], head, :] for IDS >= 0, zero rows otherwise.

    K, V: [slots, heads, D] arrays (any dtype, compared bytewise); REQ the
    logical -> physical slot map (None = identity); IDS [rows, >=top].
    Returns (KG, VG) of shape [rows*top, D] (VG None when V is None).
    """
    ids = np.asarray(IDS, np.int64)[:rows, :top].reshape(-1)
    valid = ids >= 0
    safe = np.where(valid, ids, 0)
    phys = safe if REQ is None else np.asarray(REQ, np.int64)[safe]
    kg = np.where(valid[:, None], K[phys, head], 0).astype(K.dtype)
    vg = None if V is None else np.where(valid[:, None], V[phys, head], 0).astype(V.dtype)
    return kg, vg


# --------------------------------------------------------------------------
# published-end shared-tail variant (one request's chunk of query rows)
#   EXP/tail_union_lab_20261021/union.py:10-40        bounds, stage_union
#   EXP/fine_pool_shared_20261021/kernels.py:8-76     tables, normalize, map_topk
#   EXP/fine_pool_shared_20261021/route_shared.cu:12-54  route_physical
# EXP = experiments
# --------------------------------------------------------------------------

def shared_bounds(n, end, sink, window):
    """(s, t, c) of a row of n visible tokens given the published index end
    (union.py:10-14): sink = min(n, S); tail = max(s, min(min(max(end, 0), n),
    max(s, n - W))); count = s + n - tail."""
    s = min(n, sink)
    t = max(s, min(min(max(end, 0), n), max(s, n - window)))
    return s, t, s + n - t


def stage_union(src_u8, nt, lens, end, dst_pages, sink, window, dst=None):
    """union.py:16-40.  The chunk's union of sink pages [0, sp) and tail pages
    [tp, ep) of the ONE page table `nt` (sp = ceil(min(last, S) / 64), tp =
    max(sp, tail(first) // 64), ep = ceil(last / 64)), copied page by page into
    dst[u] (u < total = sp + max(ep - tp, 0)); meta[r] = (s, t, c) per row; desc
    = (sp, tp, ep, total).  dst pages at and past `total` keep their contents."""
    src = np.asarray(src_u8, np.uint8).reshape(-1, PAGE_BYTES)
    nt = np.asarray(nt, np.int64).reshape(-1)
    lens = [int(x) for x in np.asarray(lens).reshape(-1)]
    first, last = lens[0], lens[-1]
    _, tail, _ = shared_bounds(first, end, sink, window)
    sp = (min(last, sink) + 63) // 64
    tp = max(sp, tail // 64)
    ep = (last + 63) // 64
    total = sp + max(ep - tp, 0)
    out = np.zeros((dst_pages, PAGE_BYTES), np.uint8) if dst is None else np.array(dst, np.uint8, copy=True)
    for u in range(min(total, dst_pages)):
        lp = u if u < sp else tp + u - sp
        out[u] = src[nt[lp]]
    meta = np.array([shared_bounds(n, end, sink, window) for n in lens], np.int32).reshape(-1, 3)
    desc = np.array([sp, tp, ep, total], np.int32)
    return out, meta, desc


def shared_tables(lens, end, takes, selected, desc, cap, max_take, scratch, fp, sink, window, shared):
    """kernels.py:13-41 (tables).  Row r, column j < FP: the first `take`
    columns are the selected pages; then the staged pages -- shared: the
    chunk's union pages (sink page k -> CAP + k, tail page -> CAP + desc.sp +
    tp_r - desc.tp + k - sp_r), else the row's own scratch pages CAP + r*SCRATCH
    + k -- and 0 past them.  dglens = max(take*64 + span, 1) with span the
    scored tail span (page-aligned in shared mode); clens = take*64 + count."""
    R = len(lens)
    ft = np.zeros((R, fp), np.int32)
    dg = np.zeros(R, np.int32)
    cl = np.zeros(R, np.int32)
    selected = np.asarray(selected, np.int64).reshape(R, -1)
    gsp, gtp = int(desc[0]), int(desc[1])
    for r in range(R):
        n, take = int(lens[r]), int(takes[r])
        s, t, c = shared_bounds(n, end, sink, window)
        if shared:
            sp = (s + 63) // 64
            tp = max(sp, t // 64)
            ep = (n + 63) // 64
            pages = sp + max(ep - tp, 0)
            span = sp * 64 + n - tp * 64 if ep > tp else n
        else:
            pages = (c + 63) // 64
            span = c
        for j in range(fp):
            k = j - take
            if j < take:
                page = int(selected[r, j]) if j < max_take else 0
            elif 0 <= k < pages:
                if shared:
                    page = cap + k if k < sp else cap + gsp + tp - gtp + k - sp
                else:
                    page = cap + r * scratch + k
            else:
                page = 0
            ft[r, j] = page
        dg[r] = max(take * 64 + span, 1)
        cl[r] = take * 64 + c
    return ft, dg, cl


def shared_normalize(raw, lens, end, takes, selected, members, max_take, width, sink, window, shared):
    """kernels.py:43-63 (normalize): the canonical compact candidate order
    [selected pages' members | sink | tail] with the masks applied before
    Top-K: a selected member outside [s, t) or at/after n or the published end
    -> -inf; candidates past the count -> -inf.  Shared mode reads a tail
    candidate from its page-aligned slot in the union layout."""
    raw = np.asarray(raw, np.float32)
    R = len(lens)
    members = np.asarray(members, np.int64).reshape(-1)
    selected = np.asarray(selected, np.int64).reshape(R, -1)
    out = np.full((R, width), NEG_INF, np.float32)
    j = np.arange(width)
    for r in range(R):
        n, take = int(lens[r]), int(takes[r])
        s, t, c = shared_bounds(n, end, sink, window)
        hist = take * 64
        fine = j < hist
        x = j - hist
        col = j // 64
        page = np.where(fine & (col < max_take), selected[r, np.minimum(col, max_take - 1)] if max_take else 0, 0)
        ok = (page >= 0) & (page * 64 < len(members))
        member = np.where(fine & ok, members[np.where(ok, page * 64 + j % 64, 0)], -1)
        logical = np.where(x < s, x, t + x - s)
        if shared:
            sp = (s + 63) // 64
            tp = max(sp, t // 64)
            slot = np.where(logical < sp * 64, logical, sp * 64 + logical - tp * 64)
            source = np.where(fine, j, hist + slot)
        else:
            source = j
        valid = np.where(fine, (member >= s) & (member < t) & (member < n) & (member < end), (x >= 0) & (x < c))
        valid &= source < raw.shape[1]     # a column past the raw row reads as masked
        out[r, valid] = raw[r, source[valid]]
    return out


def shared_map_topk(ids, values, lens, end, takes, selected, members, nt, max_take, sink, window):
    """kernels.py:65-76 (map_topk): Top-K candidate rank -> logical position
    (a selected page's member, or the sink/tail position) -> physical slot
    through the request's page table; -inf picks and positions outside [0, n)
    -> -1."""
    ids = np.asarray(ids, np.int64)
    values = np.asarray(values, np.float32)
    R, top = ids.shape
    members = np.asarray(members, np.int64).reshape(-1)
    nt = np.asarray(nt, np.int64).reshape(-1)
    selected = np.asarray(selected, np.int64).reshape(R, -1)
    logical = np.full((R, top), -1, np.int32)
    slots = np.full((R, top), -1, np.int32)
    for r in range(R):
        n, take = int(lens[r]), int(takes[r])
        s, t, c = shared_bounds(n, end, sink, window)
        rank = ids[r].astype(np.int32).astype(np.int64)
        fine = (rank >= 0) & (rank < take * 64)
        col = np.where(fine, rank // 64, 0)
        page = np.where(fine & (col < max_take), selected[r, np.clip(col, 0, max(max_take - 1, 0))], 0)
        ok = (page >= 0) & (page * 64 < len(members))
        member = np.where(fine & ok, members[np.where(ok, page * 64 + rank % 64, 0)], -1)
        x = rank - take * 64
        lg = np.where(fine, member, np.where(x < s, x, t + x - s))
        valid = (values[r] != NEG_INF) & (lg >= 0) & (lg < n) & (lg // 64 < len(nt))
        phys = np.where(valid, nt[np.clip(lg // 64, 0, len(nt) - 1)] * 64 + lg % 64, -1)
        logical[r] = np.where(valid, lg, -1)
        slots[r] = phys
    return logical, slots


def route_physical(scores, published, budgets, rt, take_stride):
    """route_shared.cu:12-54.  active = clamp(published, 0, pages); take =
    min(max(budget, 0), active, take_stride).  take == 0 or take == active:
    selected[i] = rt[i] for i < take.  Otherwise the page score is the max of
    its 8 centres (an all -inf active page becomes -FLT_MAX, so it still
    precedes padding), padding slots -inf, a stable descending radix sort over
    the blocked layout of 128 threads x ITEMS (ITEMS the smallest power of two
    with 128*ITEMS >= pages; ties keep blocked rank (p % 128)*ITEMS + p // 128,
    -0 == +0) and selected[rank] = rt[page] for rank < take.  Padding entries
    are 0.  Returns (selected int32 [R, take_stride], takes int32 [R])."""
    scores = np.asarray(scores, np.float32)
    rt = np.asarray(rt, np.int64)
    R, pages = rt.shape
    items = 1
    while items * 128 < pages:
        items *= 2
    n_items = 128 * items
    rank = np.arange(n_items)
    p_of_rank = rank // items + (rank % items) * 128
    sel = np.zeros((R, take_stride), np.int32)
    takes = np.zeros(R, np.int32)
    for r in range(R):
        active = min(max(int(published[r]), 0), pages)
        take = min(min(max(int(budgets[r]), 0), active), take_stride)
        takes[r] = take
        if take == 0 or take == active:
            sel[r, :take] = rt[r, :take]
            continue
        vals = np.full(n_items, NEG_INF, np.float32)
        valid = p_of_rank < active
        m = np.fmax.reduce(scores[r, :active * 8].reshape(active, 8), axis=1)
        m = np.where(m == NEG_INF, np.float32(-np.finfo(np.float32).max), m).astype(np.float32)
        vals[valid] = m[p_of_rank[valid]]
        key = twiddle_key(vals).astype(np.int64)
        order = np.lexsort((rank, 0xFFFFFFFF - key))
        sel[r, :take] = rt[r, p_of_rank[order][:take]]
    return sel, takes


# --------------------------------------------------------------------------
# v1_native (signed-score Qwen) operators
# --------------------------------------------------------------------------

def topk_transform(scores, seq_lens, page_table, page_size, topk, original_ids=None):
    """TopK-v2's transform as the v1_native backend calls it
    (NA/deps/topk2048.py:15-32 with an identity page table,
    NA/deps/topk2048_mapped_20261012.py:13-21 with original ids).

    Per row b: raw = select_topk(scores[b, :seq_lens[b]], topk) -- the topk
    largest by (value desc, index asc) in ascending index order, or [0, L) then
    -1 when L <= topk (the trivial transform, topk_v2.cuh:139-144); out = -1
    for raw < 0, else idx = page_table[b, raw >> bits] << bits | raw & mask
    (page_to_indices, topk_impl.cuh:162-165), through original_ids[idx] when
    given (transform_output, :187-190).  page_table rows may all be one row
    (stride 0 in the reference).  Returns (out, raw) int32 [B, topk].
    """
    s = np.asarray(scores, np.float32)
    B, cols = s.shape
    pt = np.asarray(page_table, np.int64)
    if pt.ndim == 1:
        pt = np.broadcast_to(pt, (B, pt.shape[0]))
    bits = int(page_size).bit_length() - 1
    out = np.full((B, topk), -1, np.int32)
    raw = np.full((B, topk), -1, np.int32)
    for b in range(B):
        L = min(int(seq_lens[b]), cols)
        r = select_topk(s[b, :max(L, 0)], topk)
        raw[b] = r
        ok = r >= 0
        idx = (pt[b, r[ok] >> bits] << bits) | (r[ok] & ((1 << bits) - 1))
        out[b, ok] = idx if original_ids is None else np.asarray(original_ids, np.int64)[idx]
    return out, raw


def mask_scores(scores, table, mapping, positions, dedup_cols=0, fixed_start=0):
    """NA/kernels.py:47-59: column c of row r becomes -inf when its logical token
    l = mapping[table[r, c // 64], c % 64] is < 0, > positions[r], or (c <
    dedup_cols and (l < 64 or l >= fixed_start)).  A table entry outside the
    mapping reads as l = -1 (the reference reads past the mapping there).
    Returns a masked copy."""
    s = np.array(scores, np.float32, copy=True)
    B, W = s.shape
    table = np.asarray(table, np.int64)
    mapping = np.asarray(mapping, np.int64)
    cols = np.arange(W)
    for r in range(B):
        pg = table[r, cols // 64]
        ok = (pg >= 0) & (pg < mapping.shape[0])
        lg = np.where(ok, mapping[np.where(ok, pg, 0), cols % 64], -1)
        bad = (lg < 0) | (lg > int(positions[r])) | ((cols < dedup_cols) & ((lg < 64) | (lg >= fixed_start)))
        s[r, bad] = NEG_INF
    return s


def page_route(scores, pages, take):
    """NA/deps/route.py:20-49 (the route extension, any THREADS it accepts).

    n = the smallest of 128, 256, ..., 4096 holding the pages; blocked rank
    r holds page p = r // (n / 128) + (r % (n / 128)) * 128, scored as the
    fmaxf of its 8 centres (p < pages) or -inf; a stable descending radix
    sort (CUB keys, -0 == +0) and the first `take` page ids per row.
    Returns (ids int32 [B, take], bitmap uint8 [B, pages]).
    """
    s = np.asarray(scores, np.float32)
    B = s.shape[0]
    n = 128
    while n < pages:
        n *= 2
    base = n // 128
    rank = np.arange(n)
    p_of_rank = rank // base + (rank % base) * 128
    ids = np.empty((B, take), np.int32)
    bitmap = np.zeros((B, pages), np.uint8)
    valid = p_of_rank < pages
    for r in range(B):
        vals = np.full(n, NEG_INF, np.float32)
        vals[valid] = np.fmax.reduce(s[r, :pages * 8].reshape(pages, 8), axis=1)[p_of_rank[valid]]
        key = twiddle_key(vals).astype(np.int64)
        order = np.lexsort((rank, 0xFFFFFFFF - key))
        ids[r] = p_of_rank[order[:take]]
        bitmap[r, ids[r][ids[r] < pages]] = 1
    return ids, bitmap


def pack_q(q, out_heads, w_mul, out_rows=None):
    """qwen_gqa_probe_kernels.py:15-20 (and NA/scoring.py:66-71 with
    NA/grouping.py:41-44): q float [rows, qheads, 128] -> (q8 uint8 e4m3
    [out_rows, out_heads, 128], w float32 [out_rows, out_heads]); scale = the
    power of two >= max(max|q|, 1e-4) / 448 (pow2_ceil), q8 = e4m3(q / scale),
    w = scale * w_mul for the live (row, head) entries, zeros elsewhere."""
    q = np.asarray(q, np.float32)
    rows, qheads, _ = q.shape
    out_rows = rows if out_rows is None else out_rows
    q8 = np.zeros((out_rows, out_heads, 128), np.uint8)
    w = np.zeros((out_rows, out_heads), np.float32)
    m = np.maximum(np.abs(q).max(-1), np.float32(1e-4)).astype(np.float32)
    scale = pow2_ceil((m / np.float32(448)).astype(np.float32))
    q8[:rows, :qheads] = e4m3_from_f32((q / scale[..., None]).astype(np.float32))
    w[:rows, :qheads] = (scale * np.float32(w_mul)).astype(np.float32)
    return q8, w


def mqa_logits(q_u8, w, k_u8, k_scale, starts, ends, relu=True, clean=True):
    """DeepGEMM fp8_mqa_logits (NA/scoring.py:75-77): [M, N] float32 with
    logits[i, j] = score_row over keys starts[i] <= j < ends[i], -inf elsewhere
    (clean) -- the same fixed fp32 evaluation order as score_row(exact=True)."""
    k = e4m3_to_f32(np.asarray(k_u8, np.uint8)).reshape(-1, 128)
    sc = np.asarray(k_scale, np.float32).reshape(-1)
    M, N = len(starts), k.shape[0]
    out = np.full((M, N), NEG_INF, np.float32)
    for i in range(M):
        lo, hi = max(int(starts[i]), 0), min(int(ends[i]), N)
        if hi > lo:
            out[i, lo:hi] = score_row(q_u8[i], w[i], k[lo:hi], sc[lo:hi], relu, True)
    return out
