"""GPU: the published-end shared-tail variant against the oracle, bit-exact --
stage_union / tables / normalize / map_topk on the interpreter fixture's inputs
and on a 64K-history chunk, route_physical over every capacity branch, the
union staging replayed in one CUDA graph while the published end moves, and
the composed chain (stage -> tables -> FP8 scoring over the shared pool ->
normalize -> Top-K -> map) against the oracle's candidate reconstruction."""
import importlib

import numpy as np
import pytest
import torch

from oracle import v1x_oracle as O

pytestmark = pytest.mark.gpu

ST = importlib.import_module("10_20_b200.shared_tail")
S = importlib.import_module("10_20_b200.scoring")


def dev(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x))
    return (t.to(dtype) if dtype is not None else t).cuda()


@pytest.mark.parametrize("ci", range(4))
def test_golden_inputs(golden, ci, cuda_dev):
    g = golden("shared_tail")
    p = f"c{ci}_"
    h, R, Sk, W, end, cap = (int(x) for x in g[p + "case"])
    lens = dev(np.arange(h + 1, h + R + 1) if h else np.zeros(R), torch.int32)
    iend = torch.tensor([end], dtype=torch.int32, device="cuda")
    src = dev(g[p + "src"])
    dst = torch.full((cap, 8448), 165, dtype=torch.uint8, device="cuda")
    meta = torch.zeros((R, 3), dtype=torch.int32, device="cuda")
    desc = torch.zeros(4, dtype=torch.int32, device="cuda")
    ST.launch(src, dev(g[p + "nt"]), lens, iend, dst, meta, desc, Sk, W)
    assert np.array_equal(dst.cpu().numpy(), g[p + "dst"])
    assert np.array_equal(meta.cpu().numpy(), g[p + "meta"]) and np.array_equal(desc.cpu().numpy(), g[p + "desc"])
    width = int(g[p + "width"])
    takes, selected, members = dev(g[p + "takes"]), dev(g[p + "selected"]), dev(g[p + "members"])
    raw = dev(g[p + "raw"])
    for shared in (0, 1):
        ft = torch.full((R, 16), -9, dtype=torch.int32, device="cuda")
        dg = torch.zeros(R, dtype=torch.int32, device="cuda")
        cl = torch.zeros(R, dtype=torch.int32, device="cuda")
        ST.tables[(R,)](lens, iend, takes, selected, desc, ft, dg, cl, 48, 5, 3, 16, Sk, W, 16, shared)
        assert np.array_equal(ft.cpu().numpy(), g[p + f"ft{shared}"])
        assert np.array_equal(dg.cpu().numpy(), g[p + f"dg{shared}"]) and np.array_equal(cl.cpu().numpy(), g[p + f"cl{shared}"])
        norm = torch.zeros((R, width), device="cuda")
        ST.normalize[(R, -(-width // 256))](raw, lens, iend, takes, selected, members, norm, 5, width,
                                            raw.shape[1], Sk, W, 256, shared)
        assert np.array_equal(norm.cpu().numpy(), g[p + f"norm{shared}"])
    logical = torch.zeros((R, 96), dtype=torch.int32, device="cuda")
    slots = torch.zeros_like(logical)
    ST.map_topk[(R,)](dev(g[p + "ids"]), dev(g[p + "values"]), lens, iend, takes, selected, members,
                      dev(g[p + "nt"]), logical, slots, 5, 96, Sk, W, 128)
    assert np.array_equal(logical.cpu().numpy(), g[p + "logical"]) and np.array_equal(slots.cpu().numpy(), g[p + "slots"])


def _chunk(history, rows, seed):
    rng = np.random.default_rng(seed)
    npg = -(-(history + rows) // 64) + 2
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn((npg, 64, 128), generator=gen).to(torch.float8_e4m3fn)
    src = torch.zeros((npg, 8448), dtype=torch.uint8)
    src[:, :8192] = k.view(torch.uint8).reshape(npg, 8192)
    src.view(torch.float32)[:, 2048:] = torch.rand((npg, 64), generator=gen) * 0.25 + 0.05
    nt = rng.permutation(npg).astype(np.int32)
    lens = np.arange(history + 1, history + rows + 1, dtype=np.int32)
    return src.numpy(), nt, lens


@pytest.mark.parametrize("end", [65536, 61440, 61001])
def test_stage_union_64k_chunk(end, cuda_dev):
    src, nt, lens = _chunk(65536, 1024, 3)
    cap = 160
    d_src, d_nt, d_lens = dev(src), dev(nt), dev(lens)
    iend = torch.tensor([end], dtype=torch.int32, device="cuda")
    dst = torch.full((cap, 8448), 7, dtype=torch.uint8, device="cuda")
    meta = torch.zeros((1024, 3), dtype=torch.int32, device="cuda")
    desc = torch.zeros(4, dtype=torch.int32, device="cuda")
    stage = ST.PreparedStage(d_src, d_nt, d_lens, iend, dst, meta, desc, 64, 2048)
    stage()
    e_dst, e_meta, e_desc = O.stage_union(src, nt, lens, end, cap, 64, 2048, dst=np.full((cap, 8448), 7, np.uint8))
    assert np.array_equal(dst.cpu().numpy(), e_dst)
    assert np.array_equal(meta.cpu().numpy(), e_meta) and np.array_equal(desc.cpu().numpy(), e_desc)


def test_stage_union_graph_follows_published_end(cuda_dev):
    """One captured graph; the published end and the page table change between
    replays (the reference's same-graph regression)."""
    src, nt, lens = _chunk(65536, 4096, 4)
    cap = 200
    d_src, d_nt, d_lens = dev(src), dev(nt), dev(lens)
    iend = torch.tensor([65536], dtype=torch.int32, device="cuda")
    dst = torch.zeros((cap, 8448), dtype=torch.uint8, device="cuda")
    meta = torch.zeros((4096, 3), dtype=torch.int32, device="cuda")
    desc = torch.zeros(4, dtype=torch.int32, device="cuda")
    stage = ST.PreparedStage(d_src, d_nt, d_lens, iend, dst, meta, desc, 64, 2048)
    stage()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stage()
    for end in (65536, 61440, 61001, 65536):
        iend.fill_(end)
        nt = nt[::-1].copy()
        d_nt.copy_(torch.from_numpy(nt))
        g.replay()
        torch.cuda.synchronize()
        e_dst, e_meta, e_desc = O.stage_union(src, nt, lens, end, cap, 64, 2048)
        total = int(e_desc[3])
        assert np.array_equal(dst[:total].cpu().numpy(), e_dst[:total])
        assert np.array_equal(meta.cpu().numpy(), e_meta) and np.array_equal(desc.cpu().numpy(), e_desc)
    assert meta[-1].tolist() == [64, 65536, 4160]


@pytest.mark.parametrize("pages", [1, 17, 64, 129, 1024, 3904, 4096])
def test_route_physical_vs_oracle(pages, cuda_dev):
    rng = np.random.default_rng(pages)
    width = min(40, pages)
    scores = rng.standard_normal((8, pages * 8)).astype(np.float32)
    scores[1, ::5] = 0.0
    scores[1, 1::5] = -0.0
    scores[2, :] = np.round(scores[2] * 2) / 2        # many equal page maxima
    rt = np.stack([rng.permutation(pages) + 100 for _ in range(8)]).astype(np.int32)
    pub = np.array([pages, pages // 2, 0, pages, pages + 5, -1, pages, pages], np.int32)
    bud = np.array([40, 100, 4, 0, 1, 8, -1, pages], np.int32)
    for sc in (scores, np.full_like(scores, -np.inf)):
        sel = torch.full((8, width), -5, dtype=torch.int32, device="cuda")
        takes = torch.full((8,), -5, dtype=torch.int32, device="cuda")
        ST.route(dev(sc), dev(pub), dev(bud), dev(rt), sel, takes)
        e_sel, e_takes = O.route_physical(sc, pub, bud, rt, width)
        assert np.array_equal(takes.cpu().numpy(), e_takes)
        assert np.array_equal(sel.cpu().numpy(), e_sel)


def test_composed_chain_vs_oracle(cuda_dev):
    """stage_union -> tables -> FP8 scoring (SIMT, fixed order) over the single
    fine pool -> normalize -> Top-K -> map_topk.  Scores equal the oracle's
    scoring of the canonical candidates (selected members | sink | tail); the
    mapped slots follow the request's page table."""
    history, rows, sink, window, take, H = 8192, 64, 64, 512, 6, 4
    end = 7000
    src, nt, lens = _chunk(history, rows, 5)
    rng = np.random.default_rng(5)
    cap = 32                                           # reordered pages in the fine pool
    members = rng.permutation(history)[:cap * 64].reshape(cap, 64).astype(np.int32)
    fine = np.zeros((cap + 64, 8448), np.uint8)
    page, off = nt[members // 64], members % 64
    fine[:cap, :8192] = src[page[..., None], off[..., None] * 128 + np.arange(128)].reshape(cap, 8192)
    fine.view(np.float32)[:cap, 2048:] = src.view(np.float32)[page, 2048 + off]
    takes = np.full(rows, take, np.int32)
    selected = np.stack([rng.permutation(cap)[:take] for _ in range(rows)]).astype(np.int32)
    q = torch.randn((rows, H, 128)).to(torch.float8_e4m3fn)
    w = rng.random((rows, H)).astype(np.float32)
    c_max = O.shared_bounds(history + rows, end, sink, window)[2]
    width = -(-(take * 64 + c_max + 128) // 256) * 256
    fp = width // 64
    d = {k: dev(v) for k, v in dict(src=src, nt=nt, lens=lens, takes=takes, selected=selected,
                                    members=members).items()}
    d_fine = dev(fine)
    iend = torch.tensor([end], dtype=torch.int32, device="cuda")
    meta = torch.zeros((rows, 3), dtype=torch.int32, device="cuda")
    desc = torch.zeros(4, dtype=torch.int32, device="cuda")
    ST.PreparedStage(d["src"], d["nt"], d["lens"], iend, d_fine[cap:], meta, desc, sink, window)()
    ft = torch.zeros((rows, fp), dtype=torch.int32, device="cuda")
    dg = torch.zeros(rows, dtype=torch.int32, device="cuda")
    cl = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ST.tables[(rows,)](d["lens"], iend, d["takes"], d["selected"], desc, ft, dg, cl, cap, take, 0, fp, sink, window,
                       fp, True)
    raw = S.fp8_paged_mqa_logits(q.cuda(), d_fine, dev(w), dg, ft, None, width, impl="simt")
    out = torch.empty((rows, width), device="cuda")
    ST.normalize[(rows, width // 256)](raw, d["lens"], iend, d["takes"], d["selected"], d["members"], out, take,
                                       width, raw.stride(0), sink, window, 256, True)
    top = 512
    values, ids = torch.topk(out, top, dim=-1)
    logical = torch.empty((rows, top), dtype=torch.int32, device="cuda")
    slots = torch.empty_like(logical)
    ST.map_topk[(rows,)](ids, values, d["lens"], iend, d["takes"], d["selected"], d["members"], d["nt"], logical,
                         slots, take, top, sink, window, top)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    q8 = q.view(torch.uint8).numpy()
    for r in (0, rows // 2, rows - 1):
        n = int(lens[r])
        s, t, c = O.shared_bounds(n, end, sink, window)
        ids_tail = np.concatenate([np.arange(s), np.arange(t, n)])
        sel = selected[r]
        keys = np.concatenate([O.e4m3_to_f32(fine[sel, :8192].reshape(-1, 128)),
                               O.e4m3_to_f32(src[nt[ids_tail // 64][:, None], (ids_tail % 64)[:, None] * 128 + np.arange(128)])])
        scl = np.concatenate([fine.view(np.float32)[sel, 2048:].reshape(-1),
                              src.view(np.float32)[nt[ids_tail // 64], 2048 + ids_tail % 64]])
        ref = O.score_row(q8[r], w[r], keys, scl, exact=True)
        mem = members[sel].reshape(-1)
        keep = (mem >= s) & (mem < t) & (mem < n) & (mem < end)
        ref[:take * 64] = np.where(keep, ref[:take * 64], -np.inf)
        assert np.array_equal(got[r, :ref.size], ref), r
        assert np.isneginf(got[r, ref.size:]).all()
    e_lg, e_sl = O.shared_map_topk(ids.cpu().numpy(), values.cpu().numpy(), lens, end, takes, selected, members, nt,
                                   take, sink, window)
    assert np.array_equal(logical.cpu().numpy(), e_lg) and np.array_equal(slots.cpu().numpy(), e_sl)
