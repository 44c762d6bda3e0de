"""CPU: the numpy oracle reproduces the reference's own outputs (golden fixtures).

Fixtures come from tests/golden/make_golden.py, which ran the reference's
Triton kernels in the Triton interpreter and the torch math of
DS/example_v1_query_single_head.py on CPU.
"""
import numpy as np
import pytest
import torch

import oracle as O


def test_e4m3_table_matches_torch():
    allbytes = torch.arange(256, dtype=torch.uint8)
    ref = allbytes.view(torch.float8_e4m3fn).float().numpy()
    mine = O.e4m3_to_f32(allbytes.numpy())
    same = (ref == mine) | (np.isnan(ref) & np.isnan(mine))
    assert same.all()


def test_sort_golden(golden):
    g = golden("sort")
    out = O.sort_segments(g["ids16"], g["values16"], -1, 16, 1, 1)[:16]
    assert np.array_equal(out, g["out16"])
    vals = g["values16"].tolist()
    ids = g["ids16"].tolist()
    expected = [ids[i] for i in sorted(range(16), key=lambda i: (-vals[i], i))]
    assert out.tolist() == expected
    # FLAG >= 0 is a no-op
    assert np.array_equal(O.sort_segments(g["ids16"], g["values16"], 0, 16, 1, 1,
                                          O=np.full(16, -99, np.int32)), np.full(16, -99))
    o = O.sort_segments(g["p256"], g["s256"], -1, 256, 16, 2)
    assert np.array_equal(o, g["o256"].reshape(-1))
    o = O.sort_segments(g["p4096"], g["s4096"], -1, 4096, 1, 1)
    assert np.array_equal(o, g["o4096"].reshape(-1))


def test_gather_golden(golden):
    g = golden("gather")
    k = g["k"].reshape(8, 2, 128)
    v = g["v"].reshape(8, 2, 128)
    for head in (0, 1):
        kg, vg = O.gather_slots(k, v, g["req"], g["ids"], 2, 3, head)
        assert np.array_equal(kg, g[f"small_k{head}"].reshape(6, 128))
        assert np.array_equal(vg, g[f"small_v{head}"].reshape(6, 128))
    kg, vg = O.gather_slots(g["kpool"], g["vpool"], g["req2"], g["ids2"], 2, 96, 2)
    assert np.array_equal(kg, g["rand_k"].reshape(-1, 128))
    assert np.array_equal(vg, g["rand_v"].reshape(-1, 128))


def test_page_lifecycle_reference_sequence(golden):
    g = golden("pages")
    cap = 16
    tmp = np.repeat(np.arange(16, dtype=np.uint8)[:, None], 8448, 1)
    mapping = np.arange(1024, dtype=np.int32).reshape(16, 64)
    h = O.fingerprint(tmp, mapping)
    assert np.array_equal(h, g["t_hash"])
    fine = np.zeros_like(tmp)
    members = np.full_like(mapping, -1)
    live = np.zeros((16, 2), np.int64)
    refs = np.zeros(cap, np.int32)
    free = np.arange(cap, dtype=np.int32)
    tables = np.full((2, 16), -1, np.int32)
    centers = np.zeros((2, 8448), np.uint8)
    centers[:, :8192] = 7
    centers.view(np.float32)[:, 2048:] = 1.25
    cpool = np.zeros((4, 8448), np.uint8)
    m = O.match_pages(tmp, mapping, h, fine, members, live, refs, cap)
    assert np.array_equal(m, g["t_match0"])
    count, new = O.allocate([0, 0, 1], m, free, cap, refs, tables)
    O.publish(tmp, centers, mapping, h, [0, 0, 1], tables, new, fine, cpool, members, live)
    assert np.array_equal(tables, g["t_tables1"]) and count == int(g["t_count1"])
    assert np.array_equal(refs, g["t_refs1"]) and np.array_equal(new, g["t_new1"])
    assert tables[0].tolist() == list(range(15, -1, -1))
    t2 = tmp.copy()
    t2[0, 0] = 99
    assert np.array_equal(O.match_pages(t2, mapping, h, fine, members, live, refs, cap),
                          g["t_match_byte"])
    m2 = mapping.copy()
    m2[0, 0] = 9999
    assert np.array_equal(O.match_pages(tmp, m2, h, fine, members, live, refs, cap),
                          g["t_match_member"])
    m = O.match_pages(tmp, mapping, h, fine, members, live, refs, cap)
    assert np.array_equal(m, g["t_match2"])
    count, new = O.allocate([0, 1, 1], m, free, count, refs, tables)
    O.publish(tmp, centers, mapping, h, [0, 1, 1], tables, new, fine, cpool, members, live)
    assert np.array_equal(tables, g["t_tables2"]) and np.array_equal(refs, g["t_refs2"])
    assert np.array_equal(cpool, g["t_center_pool"])
    count = O.release(tables[0], refs, free, count)
    assert np.array_equal(refs, g["t_refs3"]) and count == int(g["t_count3"])
    count = O.release(tables[1], refs, free, count)
    assert np.array_equal(refs, g["t_refs4"]) and count == int(g["t_count4"])
    assert np.array_equal(free, g["t_free4"])


def test_page_lifecycle_random_with_sharing_and_collision(golden):
    g = golden("pages")
    cap = 48
    fine = np.zeros((cap, 8448), np.uint8)
    members = np.full((cap, 64), -1, np.int32)
    live = np.zeros((cap, 2), np.int64)
    refs = np.zeros(cap, np.int32)
    free = g["r_free0"].copy()
    count = cap
    tables = np.full((4, 16), -1, np.int32)
    cpool = np.zeros((8, 8448), np.uint8)
    for lease in range(3):
        t, m, tc = g[f"r_b{lease}_tmp"], g[f"r_b{lease}_map"], g[f"r_b{lease}_tc"]
        meta = [lease * 1024, lease, 1]
        h = O.fingerprint(t, m)
        assert np.array_equal(h, g[f"r_b{lease}_hash"])
        if lease == 2:
            live[tables[0, 1]] = h[3]
        mt = O.match_pages(t, m, h, fine, members, live, refs, cap)
        assert np.array_equal(mt, g[f"r_b{lease}_match"])
        count, new = O.allocate(meta, mt, free, count, refs, tables)
        assert np.array_equal(new, g[f"r_b{lease}_new"])
        O.publish(t, tc, m, h, meta, tables, new, fine, cpool, members, live)
        assert np.array_equal(tables, g[f"r_tables{lease}"])
        assert np.array_equal(refs, g[f"r_refs{lease}"])
        assert count == int(g[f"r_count{lease}"])
        assert np.array_equal(free, g[f"r_free{lease}"])
    assert (g["r_b1_match"][::2] >= 0).all()       # B shares A's even pages
    assert g["r_b2_match"][3] == -1                 # forged hash collision must miss
    for lease in (1, 0):
        count = O.release(tables[lease], refs, free, count)
        assert np.array_equal(refs, g[f"r_rel_refs{lease}"])
        assert count == int(g[f"r_rel_count{lease}"])
        assert np.array_equal(free, g[f"r_rel_free{lease}"])
    assert np.array_equal(fine, g["r_fine"]) and np.array_equal(members, g["r_members"])
    assert np.array_equal(live, g["r_live"]) and np.array_equal(cpool, g["r_center_pool"])


def test_allocate_exhaustion_leaves_state():
    free = np.arange(4, dtype=np.int32)
    refs = np.zeros(4, np.int32)
    tables = np.full((1, 16), -1, np.int32)
    with pytest.raises(O.ArenaExhausted):
        O.allocate([0, 0, 1], np.full(16, -1), free, 4, refs, tables)
    assert (refs == 0).all() and (tables == -1).all()


def test_stage_tail_and_fine_table_reference_case(golden):
    g = golden("tail_meta")
    out = np.full((1 + 4 * 3, 8448), 255, np.uint8)
    got = O.stage_tail_shared(g["t_native"], g["t_nt"], g["t_lens"], out, g["t_owners"], 1, 18, 3,
                              64, 64, 4, 4, 1, 3)
    assert np.array_equal(got, g["t_out"])
    ft = O.fine_table_shared(np.zeros((4, 18), np.int32), np.zeros((4, 1), np.int32),
                             [0, 0, 0, 0], (4, 3), g["t_owners"], 1, 18, 1, 3)
    assert np.array_equal(ft, g["t_ft"])
    assert ft.tolist() == [[1, 2, 3], [1, 2, 3], [7, 8, 9], [7, 8, 9]]


def test_stage_tail_random_groups(golden):
    g = golden("tail_meta")
    B = g["s_lens"].shape[0]
    out = np.full((5 + B * 68, 8448), 255, np.uint8)
    for window in (64, 2048):
        got = O.stage_tail_shared(g["s_native"], g["s_nt"], g["s_lens"], out, g["s_owners"], 5, 40,
                                  68, 64, window, B, 32, (B + 31) // 32, 68)
        assert np.array_equal(got, g[f"s_out{window}"])


def test_query_metadata_golden(golden):
    g = golden("tail_meta")
    for window in (64, 2048):
        outs = O.query_metadata(g["m_lens"], g["m_nt"], 96, 2048, 1, 2, 64, window)
        assert np.array_equal(np.stack(outs), g[f"m_out{window}"])


def test_fine_table_shared_golden(golden):
    g = golden("tail_meta")
    ft = O.fine_table_shared(g["f_rt"], g["f_sel"], g["f_takes"], (6, 20), g["f_trows"], 777, 64,
                             12, 68)
    assert np.array_equal(ft, g["f_ft"])


def test_mask_output_reduce_expand_golden(golden):
    g = golden("select_maps")
    B, MAXP, NP, TAKE, TOPK, WIDTH = 5, 96, 96, 8, 256, 768
    masked = O.mask_fine(g["scores"], g["selected"], g["rt"], g["members"], g["lens"], g["takes"],
                         MAXP, TAKE, WIDTH, WIDTH, 64, 64)
    assert np.array_equal(masked, g["masked"])
    out, logical = O.output_ids(g["raw"], g["masked"], g["members"], g["rt"], g["nt"],
                                g["selected"], g["lens"], g["takes"], MAXP, NP, TAKE, WIDTH, TOPK,
                                64, 64)
    assert np.array_equal(out, g["out"]) and np.array_equal(logical, g["logical"])
    coarse = O.reduce_centers(g["logits"], g["lens"], MAXP, g["logits"].shape[1])
    assert np.array_equal(coarse, g["coarse"])
    exp = O.expand_logical(g["logical"], TOPK, TOPK * 4 + 64)
    assert np.array_equal(exp, g["expanded"])


def test_fused_mask_equals_mask_fine(golden):
    """The fused in-kernel mask (VQ:71-107) and mask_fine agree below count."""
    g = golden("select_maps")
    B, WIDTH, TAKE = 5, 768, 8
    members = g["members"]
    sink, tail = O.bounds(g["lens"], 64, 64)
    fl = g["takes"].astype(np.int64) * 64 + sink + g["lens"] - tail
    for from_rank in (False,):
        r = O.topk(g["scores"], np.minimum(fl, WIDTH), members, g["rt"], g["nt"], g["selected"],
                   g["lens"], g["takes"], 64, True, 128, bucket_from_rank=from_rank)
        for row in range(B):
            n = min(int(fl[row]), WIDTH)
            assert np.array_equal(r["scores"][row, :n], g["masked"][row, :n])


def test_score_formula_golden(golden):
    """The oracle's FP8 score formula vs the reference's coarse/fine kernels."""
    g = golden("scores")
    B, H = 2, 16
    q = g["q"].reshape(B, H, 128)
    for exact in (True, False):
        # coarse: centre pages via centre table, page max of 8
        for r in range(B):
            pages = (int(g["lens"][r]) - 1) // 1024 * 16
            keys, sc = O.page_keys(g["centers"], g["ctable"][r], pages * 8)
            s = O.score_row(q[r], g["w"][r], keys, sc, exact=exact)
            pm = s.reshape(pages, 8).max(1)
            np.testing.assert_allclose(pm, g["coarse"][r, :pages], rtol=2e-5, atol=2e-5)
            assert np.isneginf(g["coarse"][r, pages:]).all()
        # fine: selected reordered pages + native sink/tail
        for r in range(B):
            n = int(g["lens"][r])
            take = int(g["takes"][r])
            sink, tail = (int(x) for x in O.bounds(n, 64, 64))
            count = take * 64 + sink + n - tail
            sel_pages = g["rt"][r, g["selected"][r, :take]]
            k1, s1 = O.page_keys(g["fine_pool"], np.repeat(sel_pages, 1), take * 64)
            ids = np.concatenate([np.arange(sink), np.arange(tail, n)])
            k2, s2 = O.page_keys(g["native"], g["nt"][r], n)
            keys = np.concatenate([k1, k2[ids]])
            sc = np.concatenate([s1, s2[ids]])
            s = O.score_row(q[r], g["w"][r], keys, sc, exact=exact)
            lg = g["members"][sel_pages].reshape(-1)
            keep = np.concatenate([(lg >= sink) & (lg < tail), np.ones(len(ids), bool)])
            s = np.where(keep, s, -np.inf)
            width = g["fine"].shape[1]
            m = min(count, width)
            np.testing.assert_allclose(g["fine"][r, :m], s[:m], rtol=2e-5, atol=2e-5)
            assert np.isneginf(g["fine"][r, m:]).all()


def test_route_topk_example(golden):
    """DS/example_v1_query_single_head.py: route pages, fine table, Top-2048 sets."""
    g = golden("route_topk_example")
    B, P, CAP, TAKE, N, TOP, WINDOW = 4, 128, 128, 40, 4097, 2048, 64
    scores = np.repeat(g["scores"], B, 0)
    lens = np.full(B, N, np.int32)
    takes = np.full(B, TAKE, np.int32)
    rt = np.repeat(g["reorder_pages"][None], B, 0)
    nt = np.repeat(g["native_pages"][None], B, 0)
    ft0 = np.full((B, TAKE + 68), -1, np.int32)
    sel, ft = O.route(scores, lens, takes, TAKE, P, rt, ft0, np.zeros(B, np.int32), CAP, True)
    assert np.array_equal(sel, np.repeat(g["selected"], B, 0))
    assert sel[0, :8].tolist() == [48, 49, 50, 51, 52, 53, 54, 55]
    assert np.array_equal(ft[:, :TAKE], np.repeat(g["ft_sel"], B, 0))
    assert np.array_equal(ft[:, TAKE:], np.repeat((CAP + np.arange(68))[None], B, 0))
    fine = np.repeat(g["fine_scores"], B, 0)
    fl = np.full(B, fine.shape[1], np.int32)
    for direct in (False, True):
        r = O.topk(fine, fl, g["members"], rt, nt, sel, lens, takes, WINDOW, True, TOP,
                   bucket_from_rank=True, fine_table=ft, direct_fine=direct)
        assert np.array_equal(r["scores"], np.repeat(g["masked"], B, 0))
        assert np.array_equal(np.sort(r["raw"], 1), np.repeat(g["raw_sorted"], B, 0))
        assert np.array_equal(np.sort(r["logical"], 1), np.repeat(g["logical_sorted"], B, 0))
        assert np.array_equal(np.sort(r["physical"], 1), np.repeat(g["physical_sorted"], B, 0))
        cid = np.repeat(g["candidate_ids"], B, 0)
        assert np.array_equal(r["logical"], np.take_along_axis(cid, r["raw"].astype(np.int64), 1))
        # bucket_from_rank=False reads bucket identity from members: same result
        r2 = O.topk(fine, fl, g["members"], rt, nt, sel, lens, takes, WINDOW, True, TOP,
                    bucket_from_rank=False, fine_table=ft, direct_fine=direct)
        assert np.array_equal(r2["raw"], r["raw"])


def test_route_blocked_rank_ties():
    """Equal page scores keep CUB's blocked-rank order (VQ:26-30, VQ:42)."""
    B, P = 1, 300               # T*I = 512, BASE = 4
    T, I = O.route_geometry(P)
    assert (T, I) == (64, 8)
    n = 1 + 1024 * (P // 16)
    active = (n - 1) // 1024 * 16
    scores = np.zeros((B, P * 8), np.float32)     # all pages tie at 0 (incl. -0.0)
    scores[0, 8:16] = -0.0
    sel, _ = O.route(scores, [n], [10], 10, P, np.zeros((B, P), np.int32),
                     np.zeros((B, 10), np.int32), [0], 1, False)
    base = T * I // 128
    ranks = sorted(range(active), key=lambda p: (p % 128) * base + p // 128)
    assert sel[0].tolist() == ranks[:10]


def test_topk_ties_lower_index():
    vals = np.array([1, 3, 3, 2, 3, 0, -0.0, 3], np.float32)
    assert O.select_topk(vals, 3).tolist() == [1, 2, 4]
    assert O.select_topk(vals, 5).tolist() == [1, 2, 3, 4, 7]
    assert O.select_topk(vals, 9).tolist() == list(range(8)) + [-1]
    v = np.zeros(6, np.float32)
    v[[1, 3]] = -0.0
    assert O.select_topk(v, 3).tolist() == [0, 1, 2]
