"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run (CPU only, needs the reference checkout):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

The reference's own Triton kernels (DS/kernels.py, NA/kernels.py,
NA/fused_grouping.py, the shared-tail experiments, qwen_gqa_probe_kernels.py)
are loaded by file path, exactly as the reference's tests load them, and
executed on CPU tensors by the Triton interpreter (TRITON_INTERPRET=1); torch
helpers (NA/grouping.py quantize) run on CPU.  The fused CUDA route/topk cannot run here, so their
fixture is the torch reference math of DS/example_v1_query_single_head.py
evaluated on CPU.  Inputs are seeded; outputs are written as .npz next to this
script.  The test suite never runs this script; it only reads the .npz files.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def i32(x):
    return torch.tensor(x, dtype=torch.int32)


def save(name, **arrays):
    out = {k: (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)) for k, v in arrays.items()}
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print("wrote", name, sum(a.nbytes for a in out.values()), "bytes")


def fp8_pages(gen, pages, amp=1.0):
    """Random packed pages: e4m3 key bytes from N(0, amp) and positive scales."""
    k = (torch.randn((pages, 64, 128), generator=gen) * amp).to(torch.float8_e4m3fn)
    buf = torch.zeros((pages, 8448), dtype=torch.uint8)
    buf[:, :8192] = k.view(torch.uint8).reshape(pages, 8192)
    buf.view(torch.float32)[:, 2048:] = torch.rand((pages, 64), generator=gen) + 0.25
    return buf


# ---------------------------------------------------------------------------
def gen_sort(fg):
    gen = torch.Generator().manual_seed(1)
    flag = i32(-1)
    # (a) the reference's adversarial 16-member vector (NA/test_fused_grouping_small.py:88-99)
    values = [2., -1., 2., 0., -0., 3., -3., 1., 1., 2., -1., 0., 4., 4., -4., 0.]
    ids = [115, 102, 108, 101, 109, 103, 114, 100, 113, 104, 112, 105, 111, 106, 110, 107]
    perm = i32(ids)
    scores = torch.tensor(values)
    out16 = torch.full((16,), -99, dtype=torch.int32)
    fg._sort[(1, 1)](perm, out16, scores, flag, 16, num_warps=4)
    # (b) two heads, N=256 segments: heavy ties, +-0, +-inf, layout [heads, 4096]
    heads = 2
    s = torch.randint(-4, 5, (heads, 4096), generator=gen).float() * 0.5
    s[s == 0] = torch.where(torch.rand(int((s == 0).sum()), generator=gen) < 0.5, 0.0, -0.0)
    s.view(-1)[::97] = float("inf")
    s.view(-1)[::89] = float("-inf")
    p = torch.randperm(heads * 4096, generator=gen).to(torch.int32).reshape(heads, 4096)
    o256 = torch.full_like(p, -7)
    fg._sort[(4096 // 256, heads)](p, o256, s, flag, 256, num_warps=4)
    # (c) one head, N=4096: integer group keys in [0, 4096) with duplicate runs
    keys = torch.randint(0, 4096, (4096,), generator=gen)
    run = torch.rand(4096, generator=gen) < 0.3
    for i in range(1, 4096):
        if run[i]:
            keys[i] = keys[i - 1]
    s4 = keys.float()[None]
    p4 = torch.arange(4096, dtype=torch.int32)[None].contiguous()
    o4 = torch.full_like(p4, -7)
    fg._sort[(1, 1)](p4, o4, s4, flag, 4096, num_warps=8)
    save("sort", ids16=perm, values16=scores, out16=out16, s256=s, p256=p, o256=o256,
         s4096=s4, p4096=p4, o4096=o4)


# ---------------------------------------------------------------------------
def gen_gather(nk):
    gen = torch.Generator().manual_seed(2)
    # (a) the reference's small case (NA/test_gather_slots_small.py:26-43)
    x = torch.arange(8 * 2 * 128, dtype=torch.float32).reshape(8, 2, 128)
    k = x.to(torch.bfloat16)
    v = (-x - 16).to(torch.bfloat16)
    req = i32([5, 1, 7, 0, 6, 2])
    backing = i32([[0, 2, -1, 99], [4, 1, 4, 99]])
    ids = backing[:, :3]
    kp = torch.empty((8, 2, 256), dtype=torch.bfloat16)[:, :, ::2]
    kp.copy_(k)
    vp = torch.empty((8, 4, 128), dtype=torch.bfloat16)[:, ::2, :]
    vp.copy_(v)
    outs = {}
    for head in (0, 1):
        ok = torch.empty((2, 3, 1, 128), dtype=torch.bfloat16)
        ov = torch.empty_like(ok)
        nk._gather_slots[(1,)](kp, vp, req, ids, ok, ov, 2, 3, head, *kp.stride(), *vp.stride(),
                               ids.stride(0), 32, num_warps=4)
        outs[f"small_k{head}"] = ok.view(torch.int16)
        outs[f"small_v{head}"] = ov.view(torch.int16)
    # (b) random: 3 heads, 500 slots, 2 rows x 96 ids with -1 holes, padded row stride
    slots, heads = 200, 3
    kpool = torch.randn((slots, heads, 128), generator=gen).to(torch.bfloat16)
    vpool = torch.randn((slots, heads, 128), generator=gen).to(torch.bfloat16)
    req2 = torch.randperm(slots, generator=gen).to(torch.int32)
    ids2b = torch.randint(-1, slots, (2, 100), generator=gen).to(torch.int32)
    ids2 = ids2b[:, :96]
    ok = torch.empty((2, 96, 1, 128), dtype=torch.bfloat16)
    ov = torch.empty_like(ok)
    nk._gather_slots[(((2 * 96) + 31) // 32,)](kpool, vpool, req2, ids2, ok, ov, 2, 96, 2,
                                                *kpool.stride(), *vpool.stride(), ids2.stride(0),
                                                32, num_warps=4)
    save("gather", k=k.view(torch.int16), v=v.view(torch.int16), req=req, ids=ids,
         kpool=kpool.view(torch.int16), vpool=vpool.view(torch.int16), req2=req2, ids2=ids2b,
         rand_k=ok.view(torch.int16), rand_v=ov.view(torch.int16), **outs)


# ---------------------------------------------------------------------------
def gen_pages(dk):
    """Page lifecycle: the reference test's sequence plus a random 3-bucket run."""
    gen = torch.Generator().manual_seed(3)
    rec = {}
    # (a) DS/test_page_management_and_tail_small.py:14-57
    cap = 16
    tmp = torch.arange(16, dtype=torch.uint8)[:, None].expand(16, 8448).contiguous()
    mapping = torch.arange(1024, dtype=torch.int32).reshape(16, 64)
    meta = i32([0, 0, 1])
    hashes = torch.empty((16, 2), dtype=torch.int64)
    centers = torch.zeros((2, 8448), dtype=torch.uint8)
    centers[:, :8192] = 7
    centers.view(torch.float32)[:, 2048:] = 1.25
    fine = torch.zeros_like(tmp)
    members = torch.full_like(mapping, -1)
    live_hash = torch.zeros_like(hashes)
    refs = torch.zeros(cap, dtype=torch.int32)
    free = torch.arange(cap, dtype=torch.int32)
    count = i32(cap)
    tables = torch.full((2, 16), -1, dtype=torch.int32)
    new = torch.empty(16, dtype=torch.bool)
    match = torch.empty(16, dtype=torch.int32)
    center_pool = torch.zeros((4, 8448), dtype=torch.uint8)

    def lookup():
        dk.match_pages[(16,)](tmp, mapping, hashes, meta, fine, members, live_hash, refs, match,
                              cap, 16)

    def alloc_publish():
        dk.allocate[(1,)](meta, match, free, count, refs, tables, new)
        dk.publish[(16,)](tmp, centers, centers.view(torch.float32), mapping, hashes, meta, tables,
                          new, fine, center_pool, center_pool.view(torch.float32), members,
                          live_hash)

    dk.fingerprint[(16,)](tmp, mapping, meta, hashes)
    rec["t_hash"] = hashes.clone()
    lookup()
    rec["t_match0"] = match.clone()
    alloc_publish()
    rec["t_tables1"] = tables.clone()
    rec["t_count1"] = count.clone()
    rec["t_refs1"] = refs.clone()
    rec["t_new1"] = new.clone()
    tmp[0, 0] = 99
    lookup()
    rec["t_match_byte"] = match.clone()
    tmp[0, 0] = 0
    mapping[0, 0] = 9999
    lookup()
    rec["t_match_member"] = match.clone()
    mapping[0, 0] = 0
    meta[1] = 1
    lookup()
    rec["t_match2"] = match.clone()
    alloc_publish()
    rec["t_tables2"] = tables.clone()
    rec["t_refs2"] = refs.clone()
    rec["t_center_pool"] = center_pool.clone()
    dk.release[(1,)](tables[0], refs, free, count)
    rec["t_refs3"] = refs.clone()
    rec["t_count3"] = count.clone()
    dk.release[(1,)](tables[1], refs, free, count)
    rec["t_refs4"] = refs.clone()
    rec["t_count4"] = count.clone()
    rec["t_free4"] = free.clone()

    # (b) random run: CAP=48 arena, buckets A, B (shares 8 pages of A), C (collision)
    cap = 48
    fine = torch.zeros((cap, 8448), dtype=torch.uint8)
    members = torch.full((cap, 64), -1, dtype=torch.int32)
    live = torch.zeros((cap, 2), dtype=torch.int64)
    refs = torch.zeros(cap, dtype=torch.int32)
    free = torch.randperm(cap, generator=gen).to(torch.int32)
    count = i32(cap)
    tables = torch.full((4, 16), -1, dtype=torch.int32)
    center_pool = torch.zeros((8, 8448), dtype=torch.uint8)
    rec["r_free0"] = free.clone()
    buckets = []
    a_tmp = torch.randint(0, 256, (16, 8448), generator=gen, dtype=torch.uint8)
    a_tmp.view(torch.float32)[:, 2048:] = torch.rand((16, 64), generator=gen)
    a_map = torch.randperm(1024, generator=gen).to(torch.int32).reshape(16, 64)
    b_tmp = torch.randint(0, 256, (16, 8448), generator=gen, dtype=torch.uint8)
    b_map = torch.randperm(1024, generator=gen).to(torch.int32).reshape(16, 64) + 1024
    b_tmp[::2] = a_tmp[::2]
    b_map[::2] = a_map[::2]
    c_tmp = torch.randint(0, 256, (16, 8448), generator=gen, dtype=torch.uint8)
    c_map = torch.randperm(1024, generator=gen).to(torch.int32).reshape(16, 64) + 2048
    for lease, (t, m) in enumerate(((a_tmp, a_map), (b_tmp, b_map), (c_tmp, c_map))):
        tc = torch.randint(0, 256, (2, 8448), generator=gen, dtype=torch.uint8)
        meta = i32([lease * 1024, lease, 1])
        h = torch.empty((16, 2), dtype=torch.int64)
        dk.fingerprint[(16,)](t, m, meta, h)
        if lease == 2:
            # forge a collision: a live page (A's page 1) advertises C page 3's hash
            live[tables[0, 1].long()] = h[3]
        mt = torch.empty(16, dtype=torch.int32)
        dk.match_pages[(16,)](t, m, h, meta, fine, members, live, refs, mt, cap, 64)
        nw = torch.empty(16, dtype=torch.bool)
        dk.allocate[(1,)](meta, mt, free, count, refs, tables, nw)
        dk.publish[(16,)](t, tc, tc.view(torch.float32), m, h, meta, tables, nw, fine,
                          center_pool, center_pool.view(torch.float32), members, live)
        buckets.append(dict(tmp=t.clone(), map=m.clone(), tc=tc, hash=h, match=mt, new=nw))
        rec[f"r_tables{lease}"] = tables.clone()
        rec[f"r_refs{lease}"] = refs.clone()
        rec[f"r_count{lease}"] = count.clone()
        rec[f"r_free{lease}"] = free.clone()
    for lease in (1, 0):
        dk.release[(1,)](tables[lease], refs, free, count)
        rec[f"r_rel_refs{lease}"] = refs.clone()
        rec[f"r_rel_count{lease}"] = count.clone()
        rec[f"r_rel_free{lease}"] = free.clone()
    for lease, b in enumerate(buckets):
        for key, val in b.items():
            rec[f"r_b{lease}_{key}"] = val
    rec["r_fine"] = fine
    rec["r_members"] = members
    rec["r_live"] = live
    rec["r_center_pool"] = center_pool
    save("pages", **rec)


# ---------------------------------------------------------------------------
def gen_tail_and_meta(dk):
    gen = torch.Generator().manual_seed(4)
    rec = {}
    # (a) DS/test_page_management_and_tail_small.py:59-88
    rows, np_, cap, scratch = 4, 18, 1, 3
    native = torch.zeros((np_, 8448), dtype=torch.uint8)
    for page in range(np_):
        native[page, :8192].view(torch.float8_e4m3fn).fill_(page + 1)
        native.view(torch.float32)[page, 2048:] = torch.arange(64) + 1
    nt = torch.arange(np_ - 1, -1, -1, dtype=torch.int32)[None].expand(rows, -1).contiguous()
    lens = i32([1100, 1100, 1101, 1101])
    owners = i32([0, 0, 2, 2])
    out = torch.full((cap + rows * scratch, 8448), 255, dtype=torch.uint8)
    dk.stage_tail_shared[(1, scratch)](native.view(torch.float8_e4m3fn), native.view(torch.float32),
                                       nt, lens, out.view(torch.float8_e4m3fn),
                                       out.view(torch.float32), owners, cap, np_, scratch, 64, 64,
                                       ROWS=rows, GROUP=4, num_warps=4)
    rt = torch.zeros((rows, np_), dtype=torch.int32)
    selected = torch.zeros((rows, 1), dtype=torch.int32)
    takes = i32([0] * rows)
    ft = torch.empty((rows, scratch), dtype=torch.int32)
    dk.fine_table_shared[(rows,)](rt, selected, takes, lens, ft, owners, cap, np_, 1, scratch,
                                  scratch, 4)
    rec.update(t_native=native, t_nt=nt, t_lens=lens, t_owners=owners, t_out=out, t_ft=ft)

    # (b) query_metadata on rows with shared and private tails, window 64 and 2048
    B, NP = 12, 96
    base = torch.randperm(NP, generator=gen).to(torch.int32)
    nt = base[None].repeat(B, 1)
    lens = torch.full((B,), 4097, dtype=torch.int32)
    lens[3] = 5000
    lens[5] = 1023
    lens[6] = 0
    lens[7] = 1
    nt[8, 70] = (nt[8, 70] + 1) % NP          # differs inside row 8's tail pages
    nt[9, 0] = (nt[9, 0] + 1) % NP            # differs at page 0 (the sink)
    nt[10, 90] = (nt[10, 90] + 1) % NP        # differs beyond the tail: still shared
    for window in (64, 2048):
        outs = [torch.empty(B, dtype=torch.int32) for _ in range(5)]
        dk.query_metadata[(B,)](lens, nt, *outs, NP, 2048, 1, 2, 64, window)
        rec[f"m_out{window}"] = torch.stack(outs)
    rec.update(m_lens=lens, m_nt=nt)

    # (c) stage_tail_shared, 40 rows, GROUP=32, 68 staging pages, mixed owners
    B, NP, CAP = 34, 40, 5
    nat_pages = 48
    native = fp8_pages(gen, nat_pages)
    nt = torch.stack([torch.randperm(nat_pages, generator=gen)[:NP] for _ in range(B)]).to(torch.int32)
    lens = torch.randint(1, NP * 64, (B,), generator=gen).to(torch.int32)
    lens[:6] = lens[0]
    nt[:6] = nt[0]
    owners = torch.zeros(B, dtype=torch.int32)
    for r in (7, 15, 31, 32, 33):
        owners[r] = r
    lens[31] = 2049
    lens[32] = 64
    out = torch.full((CAP + B * 68, 8448), 255, dtype=torch.uint8)
    for window in (64, 2048):
        o = out.clone()
        dk.stage_tail_shared[((B + 31) // 32, 68)](native.view(torch.float8_e4m3fn),
                                                   native.view(torch.float32), nt, lens,
                                                   o.view(torch.float8_e4m3fn),
                                                   o.view(torch.float32), owners, CAP, NP, 68, 64,
                                                   window, ROWS=B, GROUP=32, num_warps=4)
        rec[f"s_out{window}"] = o
    rec.update(s_native=native, s_nt=nt, s_lens=lens, s_owners=owners)

    # (d) fine_table_shared on random selections
    B, MAXP, TAKE, FP = 6, 64, 12, 20
    rt = torch.randint(0, 1000, (B, MAXP), generator=gen).to(torch.int32)
    sel = torch.randint(0, MAXP, (B, TAKE), generator=gen).to(torch.int32)
    takes = i32([0, 3, 12, 7, 12, 1])
    lens = i32([5000] * B)
    trows = i32([0, 1, 0, 3, 4, 4])
    ft = torch.empty((B, FP), dtype=torch.int32)
    dk.fine_table_shared[(B,)](rt, sel, takes, lens, ft, trows, 777, MAXP, TAKE, FP, 68, 32)
    rec.update(f_rt=rt, f_sel=sel, f_takes=takes, f_trows=trows, f_ft=ft)
    save("tail_meta", **rec)


# ---------------------------------------------------------------------------
def gen_select_maps(dk):
    """mask_fine, output_ids, reduce_centers, expand_logical on random rows."""
    gen = torch.Generator().manual_seed(5)
    B, MAXP, NP, TAKE, TOPK, SINK, WINDOW = 5, 96, 96, 8, 256, 64, 64
    lens = i32([4097, 5000, 2100, 1025, 6000])
    cap = 64
    members = torch.full((cap, 64), -1, dtype=torch.int32)
    # buckets of 16 pages whose members stay inside their own 1K bucket
    for page in range(cap):
        bucket = page // 16
        members[page] = bucket * 1024 + torch.randperm(1024, generator=gen)[:64].to(torch.int32)
    rt = torch.stack([torch.randperm(cap, generator=gen) for _ in range(B)]).to(torch.int32)
    rt = torch.cat([rt, torch.zeros((B, MAXP - cap), dtype=torch.int32)], 1).contiguous()
    nt = torch.stack([torch.randperm(NP, generator=gen) for _ in range(B)]).to(torch.int32)
    selected = torch.stack([torch.randperm(16 * 4, generator=gen)[:TAKE] for _ in range(B)]).to(torch.int32)
    takes = i32([8, 8, 8, 5, 8])
    WIDTH = 768
    scores = torch.randn((B, WIDTH), generator=gen)
    scores[:, ::37] = float("-inf")
    masked = scores.clone()
    dk.mask_fine[(B, (WIDTH + 255) // 256)](masked, selected, rt, members, lens, takes, MAXP, TAKE,
                                            WIDTH, WIDTH, SINK, WINDOW)
    raw = torch.stack([torch.randperm(WIDTH + 40, generator=gen)[:TOPK] for _ in range(B)]).to(torch.int32)
    raw[:, ::9] = -1
    out = torch.empty((B, TOPK), dtype=torch.int32)
    logical = torch.empty_like(out)
    dk.output_ids[(B, (TOPK + 255) // 256)](raw, masked, members, rt, nt, selected, lens, takes,
                                            out, logical, rt, MAXP, NP, TAKE, WIDTH, TOPK, SINK,
                                            WINDOW)
    logits = torch.randn((B, MAXP * 8 + 16), generator=gen)
    coarse = torch.empty((B, MAXP))
    dk.reduce_centers[(B, (MAXP + 31) // 32)](logits, lens, coarse, MAXP, logits.stride(0))
    stride = TOPK * 4 + 64
    exp = torch.empty((B, stride), dtype=torch.int32)
    dk.expand_logical[(B,)](logical, exp, TOPK, stride, 2048)
    save("select_maps", lens=lens, members=members, rt=rt, nt=nt, selected=selected, takes=takes,
         scores=scores, masked=masked, raw=raw, out=out, logical=logical, logits=logits,
         coarse=coarse, expanded=exp)


# ---------------------------------------------------------------------------
def gen_scores(dk):
    """Reference FP8 score formula via the reference's coarse/fine Triton kernels."""
    gen = torch.Generator().manual_seed(6)
    B, H, MAXP, NP = 2, 16, 64, 24
    lens = i32([1100, 1500])
    q = (torch.randn((B, H, 128), generator=gen) * 2).to(torch.float8_e4m3fn)
    w = torch.rand((B, H), generator=gen)
    centers = fp8_pages(gen, 8)
    ctable = torch.randint(0, 8, (B, MAXP // 8), generator=gen).to(torch.int32)
    coarse = torch.empty((B, MAXP))
    dk.coarse[(B, MAXP // 8)](q, w, centers.view(torch.float8_e4m3fn), centers.view(torch.float32),
                              ctable, lens, coarse, MAXP, H, True, num_warps=4)
    fine_pool = fp8_pages(gen, 32)
    native = fp8_pages(gen, NP)
    members = torch.full((32, 64), -1, dtype=torch.int32)
    for page in range(32):
        members[page] = (page // 16) * 1024 + torch.randperm(1024, generator=gen)[:64].to(torch.int32)
    rt = torch.stack([torch.randperm(32, generator=gen) for _ in range(B)]).to(torch.int32)
    rt = torch.cat([rt, torch.zeros((B, 32), dtype=torch.int32)], 1).contiguous()
    nt = torch.stack([torch.randperm(NP, generator=gen) for _ in range(B)]).to(torch.int32)
    TAKE, WIDTH = 4, 512
    selected = torch.stack([torch.randperm(32, generator=gen)[:TAKE] for _ in range(B)]).to(torch.int32)
    takes = i32([4, 3])
    assert int(nt.shape[1]) * 64 >= int(lens.max())
    fine = torch.empty((B, WIDTH))
    dk.fine[(B, WIDTH // 64)](q, w, fine_pool.view(torch.float8_e4m3fn), fine_pool.view(torch.float32),
                              native.view(torch.float8_e4m3fn), native.view(torch.float32), members,
                              rt, nt, selected, lens, takes, fine, 64, NP, TAKE, WIDTH, 64, 64, H,
                              True, num_warps=4)
    save("scores", lens=lens, q=q.view(torch.uint8), w=w, centers=centers, ctable=ctable,
         coarse=coarse, fine_pool=fine_pool, native=native, members=members, rt=rt, nt=nt,
         selected=selected, takes=takes, fine=fine)


# ---------------------------------------------------------------------------
def gen_route_topk_example():
    """Torch reference math of DS/example_v1_query_single_head.py:8-74 on CPU.

    All 1024 query rows of that example are identical, so one row is stored.
    """
    B, P, CAP, TAKE, N, TOP, WINDOW = 1, 128, 128, 40, 4097, 2048, 64
    gen = torch.Generator().manual_seed(19)
    native_pages = torch.randperm(P, generator=gen).to(torch.int32)
    reorder_pages = torch.randperm(CAP, generator=gen).to(torch.int32)
    k = torch.zeros((N, 128))
    k[:, 0] = torch.arange(N) / 8192
    q = torch.zeros((B, 128))
    q[:, 0] = 1
    logical_order = torch.arange(4096, dtype=torch.int32).view(4, 1024).flip(1).reshape(64, 64)
    members = torch.full((CAP, 64), -1, dtype=torch.int32)
    members[reorder_pages[:64].long()] = logical_order
    reordered_k = k[logical_order.long()]
    centers = reordered_k.reshape(64, 8, 8, 128).mean(2)
    scores = torch.full((B, P * 8), float("-inf"))
    scores[:, :64 * 8] = q @ centers.reshape(-1, 128).T
    reference_pages = scores[:, :512].view(B, 64, 8).amax(-1).topk(TAKE, dim=-1).indices
    rt = reorder_pages[None]
    ft_sel = rt.gather(1, reference_pages)
    sink = 64
    tail = max(sink, min((N - 1) // 1024 * 1024, max(sink, N - WINDOW)))
    chosen = members[ft_sel.long()].reshape(B, -1)
    fixed = torch.cat((torch.arange(sink), torch.arange(tail, N))).to(torch.int32)
    candidate_ids = torch.cat((chosen, fixed[None]), dim=1)
    fine_scores = (q @ k[candidate_ids[0].long()].T).contiguous()
    valid = torch.ones_like(candidate_ids, dtype=torch.bool)
    valid[:, :TAKE * 64] = (chosen >= sink) & (chosen < tail)
    reference_scores = fine_scores.masked_fill(~valid, float("-inf"))
    expected_raw = reference_scores.topk(TOP, dim=-1).indices
    expected_logical = candidate_ids.gather(1, expected_raw)
    expected_physical = native_pages[None].gather(1, (expected_logical // 64).long()) * 64 + expected_logical % 64
    save("route_topk_example", native_pages=native_pages, reorder_pages=reorder_pages,
         members=members, scores=scores, selected=reference_pages, ft_sel=ft_sel,
         fine_scores=fine_scores, masked=reference_scores, raw_sorted=expected_raw.sort(1).values,
         logical_sorted=expected_logical.sort(1).values,
         physical_sorted=expected_physical.sort(1).values, candidate_ids=candidate_ids)


def gen_build(dk, fg):
    """Index build of one bucket (DS/runtime.py:170-233 Build.compute's
    initialize, grouping levels and assemble), run on the reference's kernels.
    Bucket 0: random keys.  Bucket 1: duplicated tokens (exact dot ties), all-zero
    tokens (unit vectors of zero) and one page of a single repeated token."""
    gen = torch.Generator().manual_seed(11)
    native = fp8_pages(gen, 40)
    # adversarial pages 20..35: duplicates, zero tokens, a constant page
    adv = native[20:36].clone()
    kb = adv[:, :8192].view(16, 64, 128)
    sc = adv.view(torch.float32)[:, 2048:]
    for _ in range(120):
        a, b = torch.randint(0, 16 * 64, (2,), generator=gen).tolist()
        kb[b // 64, b % 64] = kb[a // 64, a % 64]
        sc[b // 64, b % 64] = sc[a // 64, a % 64]
    for t in torch.randint(0, 16 * 64, (40,), generator=gen).tolist():
        kb[t // 64, t % 64] = 0
    kb[5] = kb[5, 0]
    sc[5] = sc[5, 0]
    native[20:36] = adv
    tables = torch.stack([torch.randperm(20, generator=gen)[:16], 20 + torch.randperm(16, generator=gen)]).int()
    starts = torch.tensor([4096, 65536], dtype=torch.int32)
    out = dict(native=native, tables=tables, starts=starts)
    fp8 = native.view(torch.float8_e4m3fn)
    f32 = native.view(torch.float32)
    for b in range(2):
        source = tables[b].clone()
        meta = torch.tensor([int(starts[b]), 0, 1], dtype=torch.int32)
        unit = torch.empty((1024, 128))
        perm = [torch.empty(1024, dtype=torch.int32) for _ in range(2)]
        anchor = torch.empty((64, 2), dtype=torch.int32)
        scores = torch.empty(1024)
        flag = torch.zeros((), dtype=torch.int32)
        dk.initialize[(64,)](fp8, f32, source, meta, unit, perm[0], flag, num_warps=4)
        cur = 0
        for n in (1024, 512, 256, 128, 64, 32, 16):
            for mode in (0, 1, 2):
                fg._dots[(64, 1)](unit, perm[cur], anchor, scores, flag, n, 0, mode, num_warps=4,
                                  enable_fp_fusion=False)
                if mode < 2:
                    fg._anchor[(1024 // n, 1)](perm[cur], anchor, scores, flag, n, mode, num_warps=4)
            fg._sort[(1024 // n, 1)](perm[cur], perm[1 - cur], scores, flag, n, num_warps=4)
            cur = 1 - cur
        tmp = torch.zeros((16, 8448), dtype=torch.uint8)
        centers = torch.zeros((2, 8448), dtype=torch.uint8)
        mapping = torch.zeros((16, 64), dtype=torch.int32)
        dk.assemble[(16, 8)](fp8, f32, source, meta, perm[cur], tmp.view(torch.float8_e4m3fn),
                             tmp.view(torch.float32), centers.view(torch.float8_e4m3fn), centers.view(torch.float32),
                             mapping, num_warps=4)
        out.update({f"unit{b}": unit, f"perm{b}": perm[cur].clone(), f"tmp{b}": tmp, f"centers{b}": centers,
                    f"mapping{b}": mapping, f"flag{b}": flag.reshape(1)})
    save("build", **out)


def gen_shared(un, sk):
    """Published-end shared-tail variant (experiments/tail_union_lab_20261021/
    union.py, experiments/fine_pool_shared_20261021/kernels.py) on small chunks:
    an on-time end, a lagging unaligned end, zero window, and empty rows."""
    import triton
    gen = torch.Generator().manual_seed(12)
    out = {}
    cases = [(4096, 8, 17, 64, 4096), (4096 + 100, 16, 64, 128, 3000), (2051, 6, 65, 0, 1025), (0, 4, 65, 0, 0)]
    for ci, (h, R, S, W, end) in enumerate(cases):
        np_pages = max(1, -(-(h + R) // 64)) + 3
        src = fp8_pages(gen, np_pages)
        nt = torch.randperm(np_pages, generator=gen).to(torch.int32)
        lens = torch.arange(h + 1, h + R + 1, dtype=torch.int32) if h else torch.zeros(R, dtype=torch.int32)
        iend = torch.tensor([end], dtype=torch.int32)
        cap_pages = np_pages + 2
        dst = torch.full((cap_pages, 8448), 165, dtype=torch.uint8)
        meta = torch.zeros((R, 3), dtype=torch.int32)
        desc = torch.zeros(4, dtype=torch.int32)
        un.launch(src, nt, lens, iend, dst, meta, desc, S, W, block=256)
        pre = f"c{ci}_"
        out.update({pre + "case": torch.tensor([h, R, S, W, end, cap_pages]), pre + "src": src, pre + "nt": nt,
                    pre + "dst": dst, pre + "meta": meta, pre + "desc": desc})
        # tables / normalize / map_topk over this chunk
        CAP, MAXTAKE, SCRATCH = 48, 5, 3
        FP = 16
        takes = torch.randint(0, MAXTAKE + 1, (R,), generator=gen).to(torch.int32)
        selected = torch.randint(0, CAP, (R, MAXTAKE), generator=gen).to(torch.int32)
        members = torch.randint(-2, h + R + 2, (CAP, 64), generator=gen).to(torch.int32)
        # width as the reference's fixture sizes it: every row's history plus its
        # page-aligned tail span fits (experiments/fine_pool_shared_20261021/experiment.py:41-42)
        n_last = h + R if h else 0
        s_last = min(n_last, S)
        t_last = max(s_last, min(min(max(end, 0), n_last), max(s_last, n_last - W)))
        WIDTH = -(-(MAXTAKE * 64 + s_last + n_last - t_last + 128) // 256) * 256
        STRIDE = WIDTH + 32
        raw = torch.randn((R, STRIDE), generator=gen)
        TOP = 96
        ids = torch.randint(0, WIDTH, (R, TOP), generator=gen).to(torch.int64)
        values = torch.randn((R, TOP), generator=gen)
        values[torch.rand((R, TOP), generator=gen) < 0.1] = float("-inf")
        out.update({pre + "width": torch.tensor(WIDTH), pre + "takes": takes, pre + "selected": selected,
                    pre + "members": members, pre + "raw": raw,
                    pre + "ids": ids, pre + "values": values})
        for shared in (0, 1):
            ft = torch.full((R, FP), -9, dtype=torch.int32)
            dg = torch.zeros(R, dtype=torch.int32)
            cl = torch.zeros(R, dtype=torch.int32)
            sk.tables[(R,)](lens, iend, takes, selected, desc, ft, dg, cl, CAP, MAXTAKE, SCRATCH, FP, S, W,
                            triton.next_power_of_2(FP), shared, num_warps=4)
            norm = torch.zeros((R, WIDTH))
            sk.normalize[(R, -(-WIDTH // 256))](raw, lens, iend, takes, selected, members, norm, MAXTAKE, WIDTH,
                                               STRIDE, S, W, 256, shared, num_warps=4)
            out.update({pre + f"ft{shared}": ft, pre + f"dg{shared}": dg, pre + f"cl{shared}": cl,
                        pre + f"norm{shared}": norm})
        logical = torch.zeros((R, TOP), dtype=torch.int32)
        slots = torch.zeros((R, TOP), dtype=torch.int32)
        sk.map_topk[(R,)](ids, values, lens, iend, takes, selected, members, nt, logical, slots, MAXTAKE, TOP, S, W,
                          triton.next_power_of_2(TOP), num_warps=4)
        out.update({pre + "logical": logical, pre + "slots": slots})
    save("shared_tail", **out)


def gen_signed(nk, pk, gr):
    """The signed-score path's Triton ops and torch math: NA/kernels.py
    mask_scores (:40-59), the probe's pack_q (qwen_gqa_probe_kernels.py:14-20)
    and NA/grouping.py quantize (:41-44)."""
    gen = torch.Generator().manual_seed(23)
    out = {}
    rows, width, pages = 6, 1100, 40
    for i, (dedup, fixed) in enumerate(((0, 0), (256, 2000))):
        scores = torch.randn((rows, width + 4), generator=gen)[:, :width]   # row stride 1104
        table = torch.randint(0, pages, (rows, (width + 63) // 64), generator=gen, dtype=torch.int32)
        mapping = torch.randint(-5, 3000, (pages * 64,), generator=gen, dtype=torch.int32)
        positions = torch.randint(0, 3000, (rows,), generator=gen, dtype=torch.int32)
        pre = f"mask{i}_"
        out.update({pre + "scores_in": scores.clone(), pre + "table": table, pre + "mapping": mapping,
                    pre + "positions": positions, pre + "dedup": i32([dedup, fixed])})
        nk.mask_scores(scores, table, mapping, positions, dedup, fixed)
        out[pre + "scores_out"] = scores.contiguous()
    q = torch.randn((5, 8, 128), generator=gen) * torch.logspace(-5, 2, 5)[:, None, None]
    q[2] = 0
    q = q.to(torch.bfloat16)
    qh = q[:, 4:8]                                  # the probe packs a 4-head group of a wider q
    q8 = torch.zeros((7, 32, 128), dtype=torch.float8_e4m3fn)
    w = torch.zeros((7, 32), dtype=torch.float32)
    pk.pack_q[(7, 32)](qh, q8, w, 5, qh.stride(0), qh.stride(1), 0.0883883)
    qq, qs = gr.quantize(q)
    out.update(q=q.view(torch.int16), pack_q8=q8.view(torch.uint8), pack_w=w,
               quant_q8=qq.view(torch.uint8), quant_scale=qs)
    save("signed", **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    root = Path(args.reference) / "sglang/srt/layers/attention"
    dk = load("ref_ds_kernels", root / "v1_deepseek/kernels.py")
    nk = load("ref_na_kernels", root / "v1_native/kernels.py")
    fg = load("ref_fused_grouping", root / "v1_native/fused_grouping.py")
    jobs = dict(sort=lambda: gen_sort(fg), gather=lambda: gen_gather(nk),
                pages=lambda: gen_pages(dk), tail_meta=lambda: gen_tail_and_meta(dk),
                select_maps=lambda: gen_select_maps(dk), scores=lambda: gen_scores(dk),
                route_topk=gen_route_topk_example, build=lambda: gen_build(dk, fg),
                shared_tail=lambda: gen_shared(load("ref_union", Path(args.reference) /
                                                    "experiments/tail_union_lab_20261021/union.py"),
                                               load("ref_shared_kernels", Path(args.reference) /
                                                    "experiments/fine_pool_shared_20261021/kernels.py")),
                signed=lambda: gen_signed(nk, load("ref_probe_kernels", Path(args.reference) /
                                                   "qwen_gqa_probe_kernels.py"),
                                          load("ref_grouping", root / "v1_native/grouping.py")))
    for name, job in jobs.items():
        if args.only and name not in args.only.split(","):
            continue
        job()


if __name__ == "__main__":
    sys.exit(main())
