"""The signed-score (v1_native) path's operators against the oracle: TopK-v2's
transform (plain and through original ids), mask_scores and the page route
extension, called through their drop-in modules."""
import importlib
import math

import numpy as np
import pytest
import torch

from oracle import v1x_oracle as O

pytestmark = pytest.mark.gpu

pkg = importlib.import_module("10_20_b200")
topk2048 = importlib.import_module("10_20_b200.topk2048")
mapped = importlib.import_module("10_20_b200.topk2048_mapped")
gather = importlib.import_module("10_20_b200.gather")
native_route = importlib.import_module("10_20_b200.native_route")

DEV = "cuda:0"


def _scores(rng, rows, cols, levels=None):
    if levels:   # few distinct values: many ties at the boundary
        s = rng.integers(-levels, levels, (rows, cols)).astype(np.float32) * 0.25
    else:
        s = rng.standard_normal((rows, cols)).astype(np.float32)
    s[:, ::97] = -0.0
    return s


@pytest.mark.parametrize("page_size,levels", [(64, None), (64, 3), (1, 2), (16, None)])
def test_topk_transform_matches_oracle(page_size, levels):
    rng = np.random.default_rng(page_size + (levels or 0))
    rows, cols, K = 9, 5000, 2048
    s = _scores(rng, rows, cols, levels)
    lens = np.array([0, 1, 2047, 2048, 2049, 3000, 4999, 5000, 4096], np.int32)
    P = (cols + page_size - 1) // page_size
    table = np.stack([rng.permutation(P * 2)[:P] for _ in range(rows)]).astype(np.int32)
    st = torch.zeros((rows, cols + 12), dtype=torch.float32, device=DEV)   # row stride 5012 floats
    st[:, :cols] = torch.from_numpy(s).to(DEV)
    out = torch.full((rows, K), 7, dtype=torch.int32, device=DEV)
    raw = torch.full((rows, K), 7, dtype=torch.int32, device=DEV)
    topk2048.transform(st[:, :cols], torch.from_numpy(lens).to(DEV), torch.from_numpy(table).to(DEV), out,
                       page_size, raw)
    want_out, want_raw = O.topk_transform(s, lens, table, page_size, K)
    np.testing.assert_array_equal(raw.cpu().numpy(), want_raw)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)


def test_topk_transform_original_ids_and_shared_table():
    rng = np.random.default_rng(5)
    rows, cols, K = 6, 3 * 2048 + 4, 2048
    s = _scores(rng, rows, cols, 4)
    lens = np.array([cols, cols - 1, 2048, 100, 2049, cols], np.int32)
    P = (cols + 63) // 64
    one = rng.permutation(P).astype(np.int32)
    ids = rng.integers(-1, 1 << 30, P * 64).astype(np.int32)
    table = torch.from_numpy(one).to(DEV)[None].expand(rows, -1)      # row stride 0
    out = torch.empty((rows, K), dtype=torch.int32, device=DEV)
    raw = torch.empty_like(out)
    m = mapped.module()
    plan = torch.empty((rows + 1, 2), dtype=torch.int32, device=DEV)
    lt = torch.from_numpy(lens).to(DEV)
    m.topk_plan(lt, plan, 0)
    m.topk_transform(torch.from_numpy(s).to(DEV), lt, table, out, 64, plan, raw, torch.from_numpy(ids).to(DEV))
    want_out, want_raw = O.topk_transform(s, lens, one, 64, K, original_ids=ids)
    np.testing.assert_array_equal(raw.cpu().numpy(), want_raw)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)
    assert plan[0, 0].item() == rows and plan[1:, 1].cpu().tolist() == lens.tolist()


def test_topk_topk_below_2048_and_raw_optional():
    rng = np.random.default_rng(11)
    rows, cols, K = 4, 1500, 300
    s = _scores(rng, rows, cols, 2)
    lens = np.array([1500, 300, 299, 301], np.int32)
    table = np.arange((cols + 63) // 64, dtype=np.int32)[None].repeat(rows, 0)
    out = torch.empty((rows, K), dtype=torch.int32, device=DEV)
    topk2048.transform(torch.from_numpy(s).to(DEV), torch.from_numpy(lens).to(DEV), torch.from_numpy(table).to(DEV),
                       out, 64)
    want_out, _ = O.topk_transform(s, lens, table, 64, K)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)


def test_topk2048_and_mapped_wrappers():
    rng = np.random.default_rng(3)
    rows, cols = 5, 2048 * 3
    s = _scores(rng, rows, cols, 5)
    st = torch.from_numpy(s).to(DEV)
    values, idx = topk2048.topk2048(st)
    want = np.stack([O.select_topk(s[r], 2048) for r in range(rows)])
    np.testing.assert_array_equal(idx.cpu().numpy(), want)
    assert idx.dtype == torch.int64
    np.testing.assert_array_equal(values.cpu().numpy(), np.take_along_axis(s, want.astype(np.int64), 1))
    assert topk2048.topk2048(st, need_values=False)[0] is None
    # width == 2048: every candidate, in order
    _, idx2 = topk2048.topk2048(st[:, :2048].contiguous())
    assert (idx2.cpu() == torch.arange(2048)).all()

    P = cols // 64
    table = np.stack([rng.permutation(P) for _ in range(rows)]).astype(np.int32)
    ids = rng.integers(0, 1 << 20, P * 64).astype(np.int32)
    out, raw = mapped.mapped_top2048(st, torch.from_numpy(table).to(DEV), torch.from_numpy(ids).to(DEV), True)
    want_out, want_raw = O.topk_transform(s, np.full(rows, cols), table, 64, 2048, original_ids=ids)
    np.testing.assert_array_equal(raw.cpu().numpy(), want_raw)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)
    only = mapped.mapped_top2048(st, torch.from_numpy(table).to(DEV), torch.from_numpy(ids).to(DEV))
    assert torch.equal(only, out)


def test_topk_transform_rejects_bad_arguments():
    s = torch.zeros((2, 4096), device=DEV)
    lens = torch.full((2,), 4096, dtype=torch.int32, device=DEV)
    table = torch.zeros((2, 64), dtype=torch.int32, device=DEV)
    out = torch.empty((2, 2048), dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="power of 2"):
        topk2048.transform(s, lens, table, out, 48)
    with pytest.raises(ValueError, match="multiple of 4"):
        topk2048.transform(torch.zeros((2, 4099), device=DEV)[:, :4096], lens, table, out, 64)
    with pytest.raises(ValueError, match="topk"):
        topk2048.transform(s, lens, table, torch.empty((2, 4096), dtype=torch.int32, device=DEV), 64)
    with pytest.raises(ValueError, match="metadata"):
        topk2048.module().topk_transform(s, lens, table, out, 64, torch.empty((2, 2), dtype=torch.int32,
                                                                                 device=DEV))


@pytest.mark.parametrize("dedup", [0, 256])
def test_mask_scores_matches_oracle(dedup):
    rng = np.random.default_rng(17 + dedup)
    rows, width, pages = 7, 1100, 40
    s = rng.standard_normal((rows, width)).astype(np.float32)
    table = rng.integers(0, pages, (rows, (width + 63) // 64)).astype(np.int32)
    table[2, 3], table[4, 0] = pages + 3, -1        # outside the mapping: no token
    mapping = rng.integers(-5, 3000, (pages, 64)).astype(np.int32)
    positions = rng.integers(0, 3000, rows).astype(np.int32)
    fixed = 2000 if dedup else 0
    st = torch.zeros((rows, width + 4), dtype=torch.float32, device=DEV)
    st[:, :width] = torch.from_numpy(s).to(DEV)
    st[:, width:] = 5.0
    gather.mask_scores(st[:, :width], torch.from_numpy(table).to(DEV), torch.from_numpy(mapping).to(DEV),
                       torch.from_numpy(positions).to(DEV), dedup, fixed)
    want = O.mask_scores(s, table, mapping, positions, dedup, fixed)
    got = st.cpu().numpy()
    np.testing.assert_array_equal(got[:, :width], want)
    assert (got[:, width:] == 5.0).all()


@pytest.mark.parametrize("threads,pages,take", [(64, 33, 33), (64, 64, 20), (64, 100, 99), (64, 130, 130),
                                                (128, 65, 10), (256, 300, 255), (256, 1000, 7),
                                                (512, 2049, 2048), (512, 4096, 4096)])
def test_page_route_extension_matches_oracle(threads, pages, take):
    rng = np.random.default_rng(threads + pages + take)
    rows = 5
    s = rng.integers(-4, 4, (rows, pages * 8 + 24)).astype(np.float32)
    s[1, :] = -np.inf                       # one row of ties only (padding ids reach the ranking)
    s[2, : pages * 8 // 2] = -0.0
    ext = native_route.extension(threads, 4)
    st = torch.from_numpy(s).to(DEV)
    t = torch.full((rows, take + 3), -7, dtype=torch.int32, device=DEV)
    ext.route(st, t, pages, take)
    want, want_bm = O.page_route(s, pages, take)
    got = t.cpu().numpy()
    np.testing.assert_array_equal(got[:, :take], want)
    assert (got[:, take:] == -7).all()
    bm = torch.full((rows, pages), 9, dtype=torch.uint8, device=DEV)
    t2 = torch.zeros((rows, take), dtype=torch.int32, device=DEV)
    ext.route_mask(st, t2, pages, take, bm)
    np.testing.assert_array_equal(t2.cpu().numpy(), want)
    np.testing.assert_array_equal(bm.cpu().numpy(), want_bm)


def test_page_route_extension_rejects_bad_arguments():
    ext = native_route.extension(256, 4)
    s = torch.zeros((2, 8 * 200), device=DEV)
    t = torch.zeros((2, 200), dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        ext.route(s, t, 100, 10)          # pages <= threads / 2
    with pytest.raises(ValueError):
        ext.route(s, t, 200, 201)         # take > pages
    with pytest.raises(ValueError):
        ext.route(s[:, :8 * 199], t, 200, 10)
    with pytest.raises(ValueError):
        native_route.extension(96, 4)


# ---------------------------------------------------------------------------
# q packing, flat MQA logits and the composed Scorer
# ---------------------------------------------------------------------------

native_scoring = importlib.import_module("10_20_b200.native_scoring")
scoring = importlib.import_module("10_20_b200.scoring")
synth = importlib.import_module("10_20_b200.synth")


def _u8(t):
    return t.view(torch.uint8).cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_pack_q_matches_oracle(dtype):
    g = torch.Generator().manual_seed(7)
    q = (torch.randn((37, 6, 128), generator=g) * torch.logspace(-6, 3, 37)[:, None, None]).to(dtype)
    q[3] = 0                                   # all-zero rows take the 1e-4 floor
    q[5, :, 7] = 448.0 * 2 ** -3               # absmax / 448 an exact power of two
    qd = q.to(DEV)
    big = torch.empty((40, 7, 128), dtype=dtype, device=DEV)
    big[:, :6] = torch.zeros_like(big[:, :6])
    big[:37, :6] = qd
    view = big[:37, :6]                        # head stride 128, row stride 7 * 128
    q8, w = native_scoring.pack_q(view[:, :4], 0.0883883, out_heads=32)
    want_q8, want_w = O.pack_q(q[:, :4].float().numpy(), 32, np.float32(0.0883883 / 4))
    np.testing.assert_array_equal(_u8(q8), want_q8)
    np.testing.assert_array_equal(w.cpu().numpy(), want_w)
    qq, sc = native_scoring.quantize(qd)
    want_q8, want_w = O.pack_q(q.float().numpy().reshape(-1, 1, 128), 1, 1.0)
    np.testing.assert_array_equal(_u8(qq).reshape(-1, 128), want_q8.reshape(-1, 128))
    np.testing.assert_array_equal(sc.cpu().numpy().reshape(-1), want_w.reshape(-1))


@pytest.mark.parametrize("relu,heads", [(False, 32), (True, 4), (False, 1)])
def test_mqa_logits_matches_oracle(relu, heads):
    rng = np.random.default_rng(heads)
    M, N = 11, 3001
    q8 = O.e4m3_from_f32(rng.standard_normal((M, heads, 128)).astype(np.float32))
    w = rng.uniform(-1, 1, (M, heads)).astype(np.float32)
    k8 = O.e4m3_from_f32(rng.standard_normal((N, 128)).astype(np.float32))
    ks = rng.uniform(0.01, 2, N).astype(np.float32)
    starts = np.array([0, 0, 5, 100, 3000, 3001, 0, 17, 2999, 40, 0], np.int32)
    ends = np.array([1, 3001, 6, 99, 3001, 3001, 5000, 2048, 3000, 2500, 0], np.int32)
    t = lambda a: torch.from_numpy(a).to(DEV)
    out = scoring.fp8_mqa_logits(t(q8).view(torch.float8_e4m3fn), (t(k8).view(torch.float8_e4m3fn), t(ks)), t(w),
                                 t(starts), t(ends), clean_logits=True, relu=relu)
    want = O.mqa_logits(q8, w, k8, ks, starts, ends, relu=relu, clean=True)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    # clean_logits=False leaves the columns outside [ks, ke) untouched
    keep = torch.full((M, N + 3), 3.5, device=DEV)
    scoring.fp8_mqa_logits(t(q8).view(torch.float8_e4m3fn), (t(k8).view(torch.float8_e4m3fn), t(ks)), t(w),
                           t(starts), t(ends), clean_logits=False, relu=relu, out=keep)
    got = keep.cpu().numpy()
    live = np.isfinite(want)
    np.testing.assert_array_equal(got[:, :N][live], want[live])
    assert (got[:, :N][~live] == 3.5).all() and (got[:, N:] == 3.5).all()


class _Config:
    def __init__(self, mode, fraction, share=False):
        self.mode, self.fraction, self.share_active_pages = mode, fraction, share

    def budget(self, pages):
        return min(pages, math.ceil(pages * self.fraction))


class _State:
    pass


def _pool(rng, pages):
    """Packed pages [pages, 64, 1, 132] of random FP8 keys with random scales."""
    k8 = O.e4m3_from_f32(rng.standard_normal((pages, 64, 128)).astype(np.float32))
    sc = rng.uniform(0.01, 1, (pages, 64)).astype(np.float32)
    raw = np.concatenate([k8.reshape(pages, 8192), sc.view(np.uint8).reshape(pages, 256)], 1)
    return raw.reshape(pages, 64, 1, 132)


def _oracle_v1(q, scale, centers_u8, valid, fine_u8, mapping, fixed, pages, take, positions):
    rows = q.shape[0]
    q8, w = O.pack_q(q, 32, np.float32(scale / 4))
    C = pages * 8
    ct = np.arange((C + 63) // 64)[None].repeat(rows, 0)
    coarse = O.score_paged(q8, w, centers_u8, ct, [C] * rows, C, relu=False)
    coarse[:, ~valid[:C]] = -np.inf
    if take == pages:
        sel = np.arange(pages)[None].repeat(rows, 0)
    else:
        sel, _ = O.page_route(coarse, pages, take)
    table = np.concatenate([sel, np.asarray(fixed)[None].repeat(rows, 0)], 1).astype(np.int32)
    W = table.shape[1] * 64
    fine = O.score_paged(q8, w, fine_u8, table, [W] * rows, W, relu=False)
    fine = O.mask_scores(fine, table, mapping.reshape(-1, 64), positions)
    out, _ = O.topk_transform(fine, [W] * rows, table, 64, 2048, original_ids=mapping)
    return out


@pytest.mark.parametrize("pages,fraction", [(100, 0.3), (30, 0.5), (48, 1.0)])
def test_scorer_v1_matches_oracle(pages, fraction):
    rng = np.random.default_rng(pages)
    heads, rows, nfixed = 2, 6, 36 if pages == 30 else 4
    C = pages * 8
    cp = (C + 63) // 64
    fp = pages + nfixed
    st = _State()
    st.pages = pages
    centers = np.stack([_pool(rng, cp) for _ in range(heads)])
    fine = np.stack([_pool(rng, fp) for _ in range(heads)])
    valid = rng.random((heads, C)) > 0.1
    mapping = rng.integers(-1, 5000, (heads, fp * 64)).astype(np.int32)
    st.centers, st.fine = torch.from_numpy(centers).to(DEV), torch.from_numpy(fine).to(DEV)
    st.valid, st.mapping = torch.from_numpy(valid).to(DEV), torch.from_numpy(mapping).to(DEV)
    fixed = np.arange(pages, fp, dtype=np.int32)
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(pages)).to(torch.bfloat16)
    scorer = native_scoring.Scorer(_Config("v1", fraction), DEV)
    scorer.impl = "simt"
    take = scorer.config.budget(pages)
    prefix, offset = 4000, 3
    positions = np.arange(prefix + offset, prefix + offset + rows)
    for head in range(heads):
        got = scorer.select(q.to(DEV), st, head, prefix, offset, 0, torch.from_numpy(fixed).to(DEV), 0.0883883)
        want = _oracle_v1(q.float().numpy(), 0.0883883, centers[head], valid[head], fine[head], mapping[head],
                          fixed, pages, take, positions)
        np.testing.assert_array_equal(got.cpu().numpy(), want)
    # the tensor-core scorer (the default) selects the same tokens up to near-ties
    scorer.impl = "auto"
    got = scorer.select(q.to(DEV), st, 0, prefix, offset, 0, torch.from_numpy(fixed).to(DEV), 0.0883883).cpu()
    want = _oracle_v1(q.float().numpy(), 0.0883883, centers[0], valid[0], fine[0], mapping[0], fixed, pages, take,
                      positions)
    agree = np.mean([len(np.intersect1d(got[r].numpy(), want[r])) / len(np.unique(want[r])) for r in range(rows)])
    assert agree > 0.95


def test_scorer_dsa_matches_oracle():
    rng = np.random.default_rng(9)
    heads, rows, N = 2, 5, 4100
    st = _State()
    k8 = O.e4m3_from_f32(rng.standard_normal((heads, N, 128)).astype(np.float32))
    ks = rng.uniform(0.01, 1, (heads, N)).astype(np.float32)
    st.flat_k = torch.from_numpy(k8).to(DEV).view(torch.float8_e4m3fn)
    st.flat_scale = torch.from_numpy(ks).to(DEV)
    scorer = native_scoring.Scorer(_Config("dsa", 0.5), DEV)
    scorer.impl = "simt"
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    prefix, offset, total = 3000, 90, 3500
    got = scorer.select(q.to(DEV), st, 1, prefix, offset, total, None, 0.125)
    q8, w = O.pack_q(q.float().numpy(), 32, np.float32(0.125 / 4))
    pos = np.arange(prefix + offset, prefix + offset + rows)
    logits = O.mqa_logits(q8, w, k8[1, :total], ks[1, :total], np.zeros(rows), pos + 1, relu=False)
    want = np.stack([O.select_topk(logits[r], 2048) for r in range(rows)])
    assert got.dtype == torch.int32
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    # the tensor-core default selects the same tokens up to near-ties
    scorer.impl = "auto"
    got = scorer.select(q.to(DEV), st, 1, prefix, offset, total, None, 0.125).cpu().numpy()
    assert np.mean([len(np.intersect1d(got[r], want[r])) / 2048 for r in range(rows)]) > 0.99


@pytest.mark.parametrize("relu", [False, True])
def test_mqa_logits_grouped_equals_per_row_tensor_core(relu):
    rng = np.random.default_rng(61 + relu)
    rows, N = 45, 3001
    k8 = O.e4m3_from_f32(rng.standard_normal((N, 128)).astype(np.float32))
    ks = rng.uniform(0.01, 1, N).astype(np.float32)
    P = (N + 63) // 64
    raw = np.zeros((P, 8448), np.uint8)
    kk = np.zeros((P * 64, 128), np.uint8)
    kk[:N] = k8
    sc = np.zeros(P * 64, np.float32)
    sc[:N] = ks
    raw[:, :8192] = kk.reshape(P, 8192)
    raw[:, 8192:] = sc.view(np.uint8).reshape(P, 256)
    pool = torch.from_numpy(raw).to(DEV)
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    q8, w, q8c, wc = _packs(q, 0.07, 64)
    lens = torch.full((rows,), N, dtype=torch.int32, device=DEV)
    table = torch.arange(P, dtype=torch.int32, device=DEV)[None].expand(rows, -1).contiguous()
    want = scoring.fp8_paged_mqa_logits(q8, pool, w, lens, table, None, N, clean_logits=False, relu=relu,
                                        impl="tensor_core")
    lo = rng.integers(0, N, rows).astype(np.int32)
    hi = np.minimum(lo + rng.integers(0, 3 * N // 2, rows), N + 7).astype(np.int32)
    lo[0], hi[0] = 0, N
    lo[1], hi[1] = 10, 10
    kd = torch.from_numpy(k8).to(DEV).view(torch.float8_e4m3fn)
    got = scoring.mqa_logits_grouped(q8c, wc, (kd, torch.from_numpy(ks).to(DEV)), torch.from_numpy(lo).to(DEV),
                                     torch.from_numpy(hi).to(DEV), rows=rows, relu=relu)
    cols = torch.arange(N, device=DEV)[None]
    inside = (cols >= torch.from_numpy(lo).to(DEV)[:, None].long()) & (cols < torch.from_numpy(hi).to(DEV)[:, None].long())
    assert torch.equal(got, want.masked_fill(~inside, -torch.inf))
    ref = O.mqa_logits(_u8(q8), w.cpu().numpy(), k8, ks, lo, hi, relu=relu)
    fin = np.isfinite(ref)
    assert (np.isfinite(got.cpu().numpy()) == fin).all()
    np.testing.assert_allclose(got.cpu().numpy()[fin], ref[fin], rtol=1e-2, atol=1e-3 * np.abs(ref[fin]).max())


def test_shared_select_matches_oracle():
    rng = np.random.default_rng(21)
    heads, rows, phys, pages, nfixed = 2, 4, 150, 90, 6
    arena = _State()
    centers = np.stack([_pool(rng, phys) for _ in range(heads)])
    fine = np.stack([_pool(rng, phys) for _ in range(heads)])
    valid = rng.random((heads, phys, 8)) > 0.05
    mapping = rng.integers(-1, 9000, (heads, phys * 64)).astype(np.int32)
    arena.centers, arena.fine = torch.from_numpy(centers).to(DEV), torch.from_numpy(fine).to(DEV)
    arena.valid, arena.mapping = torch.from_numpy(valid).to(DEV), torch.from_numpy(mapping).to(DEV)
    arena.identity = torch.arange(phys * 64, dtype=torch.int32, device=DEV)
    arena.record = lambda: None
    st = _State()
    st.arena, st.wait = arena, (lambda: None)
    page_ids = np.stack([rng.permutation(phys)[:pages] for _ in range(heads)]).astype(np.int32)
    fixed = np.stack([rng.permutation(phys)[:nfixed] for _ in range(heads)]).astype(np.int32)
    st.table = torch.from_numpy(page_ids).to(DEV)
    st.full_bucket_append, st.fixed_start, st.pages = True, 6000, pages
    scorer = native_scoring.Scorer(_Config("v1", 0.3, share=True), DEV)
    scorer.impl = "simt"
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    prefix, offset = 7000, 0
    got = scorer.select(q.to(DEV), st, 1, prefix, offset, 0, torch.from_numpy(fixed).to(DEV), 0.1)
    take = scorer.config.budget(pages)
    q8, w = O.pack_q(q.float().numpy(), 32, np.float32(0.1 / 4))
    ids = page_ids[1]
    coarse = O.score_paged(q8, w, centers[1], ids[None].repeat(rows, 0), [pages * 64] * rows, pages * 64,
                           relu=False)
    coarse = coarse.reshape(rows, pages, 64)[:, :, :8].copy()
    coarse[:, ~valid[1][ids]] = -np.inf
    sel, _ = O.page_route(coarse.reshape(rows, -1), pages, take)
    table = np.concatenate([ids[sel], fixed[1][None].repeat(rows, 0)], 1).astype(np.int32)
    W = table.shape[1] * 64
    sc = O.score_paged(q8, w, fine[1], table, [W] * rows, W, relu=False)
    sc = O.mask_scores(sc, table, mapping[1].reshape(-1, 64), np.arange(prefix, prefix + rows), take * 64, 6000)
    want, _ = O.topk_transform(sc, [W] * rows, table, 64, 2048, original_ids=np.arange(phys * 64))
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_mask_scores_and_quantize_golden(golden):
    g = golden("signed")
    for i in range(2):
        pre = f"mask{i}_"
        dedup, fixed = g[pre + "dedup"].tolist()
        rows, width = g[pre + "scores_in"].shape
        buf = torch.zeros((rows, width + 4), device=DEV)
        buf[:, :width] = torch.from_numpy(g[pre + "scores_in"]).to(DEV)
        gather.mask_scores(buf[:, :width], torch.from_numpy(g[pre + "table"]).to(DEV),
                           torch.from_numpy(g[pre + "mapping"]).to(DEV), torch.from_numpy(g[pre + "positions"]).to(DEV),
                           dedup, fixed)
        np.testing.assert_array_equal(buf[:, :width].cpu().numpy(), g[pre + "scores_out"])
    q = torch.from_numpy(g["q"]).view(torch.bfloat16).to(DEV)
    qq, qs = native_scoring.quantize(q)
    np.testing.assert_array_equal(_u8(qq), g["quant_q8"])
    np.testing.assert_array_equal(qs.cpu().numpy(), g["quant_scale"])


@pytest.mark.parametrize("levels", [None, 40, 2])
def test_topk_transform_wide_rows(levels):
    """Rows wider than the shared-memory stage (the unstaged mode with its
    selection bitmap): distinct values, a crowded threshold bin, mass ties."""
    rng = np.random.default_rng(100 + (levels or 0))
    rows, cols, K = 5, 62532, 2048
    s = _scores(rng, rows, cols, levels)
    s[4] = -np.inf
    lens = np.array([cols, cols - 1000, 50000, 2049, cols], np.int32)
    P = (cols + 63) // 64
    table = np.stack([rng.permutation(P) for _ in range(rows)]).astype(np.int32)
    ids = rng.integers(-1, 1 << 30, P * 64).astype(np.int32)
    out = torch.empty((rows, K), dtype=torch.int32, device=DEV)
    raw = torch.empty_like(out)
    topk2048.transform(torch.from_numpy(s).to(DEV), torch.from_numpy(lens).to(DEV), torch.from_numpy(table).to(DEV),
                       out, 64, raw, torch.from_numpy(ids).to(DEV))
    want_out, want_raw = O.topk_transform(s, lens, table, 64, K, original_ids=ids)
    np.testing.assert_array_equal(raw.cpu().numpy(), want_raw)
    np.testing.assert_array_equal(out.cpu().numpy(), want_out)


def _packs(q, scale, rows_pad):
    """(32-head q8, w) and the grouped layout (4 heads, rows padded) of q."""
    q8, w = native_scoring.pack_q(q, scale)
    q8c = torch.empty((rows_pad, 4, 128), dtype=torch.float8_e4m3fn, device=DEV)
    wc = torch.empty((rows_pad, 4), dtype=torch.float32, device=DEV)
    native_scoring.pack_q(q, scale, out_heads=4, out=(q8c, wc))
    return q8, w, q8c, wc


@pytest.mark.parametrize("relu", [False, True])
def test_grouped_logits_equal_per_row_scorer(relu):
    rng = np.random.default_rng(31 + relu)
    rows, npool = 45, 300
    pool = torch.from_numpy(_pool(rng, npool)).to(DEV)
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    q8, w, q8c, wc = _packs(q, 0.09, 64)
    assert (q8c[rows:].view(torch.uint8) == 0).all() and (wc[rows:] == 0).all()
    shared = torch.from_numpy(rng.permutation(npool)[:200].astype(np.int32)).to(DEV)
    keys = 200 * 64 - 17
    got = torch.full((rows, keys + 5), 7.0, device=DEV)
    scoring.paged_logits_grouped(q8c, wc, pool, shared, keys, got, None, 32, relu=relu, rows=rows)
    lens = torch.full((rows,), keys, dtype=torch.int32, device=DEV)
    want = scoring.fp8_paged_mqa_logits(q8, pool, w, lens, shared[None].expand(rows, -1).contiguous(), None, keys,
                                        clean_logits=False, relu=relu, impl="tensor_core")
    assert torch.equal(got[:, :keys], want)
    assert (got[:, keys:] == 7.0).all()
    valid = torch.from_numpy(rng.random(keys + 3) > 0.2).to(DEV)
    scoring.paged_logits_grouped(q8c, wc, pool, shared, keys, got, None, 32, relu=relu, rows=rows, key_valid=valid)
    assert torch.equal(got[:, :keys], want.masked_fill(~valid[:keys][None], -torch.inf))
    # per-row tables over the shared pages, a repeated page and a page outside the pool
    sh = shared.cpu().numpy()
    rt = np.stack([rng.choice(sh, 30, replace=False) for _ in range(rows)]).astype(np.int32)
    rt[3, 7] = rt[3, 2]
    rt[9, 0] = npool + 5
    rtd = torch.from_numpy(rt).to(DEV)
    got = torch.full((rows, 30 * 64), 7.0, device=DEV)
    scoring.paged_logits_grouped(q8c, wc, pool, shared, 200 * 64, got, rtd, 32, relu=relu, rows=rows)
    ok = rt.copy()
    ok[9, 0] = sh[0]
    lens = torch.full((rows,), 30 * 64, dtype=torch.int32, device=DEV)
    want = scoring.fp8_paged_mqa_logits(q8, pool, w, lens, torch.from_numpy(ok).to(DEV), None, 30 * 64,
                                        clean_logits=False, relu=relu, impl="tensor_core")
    g, wnt = got.cpu(), want.cpu()
    assert (g[9, :64] == 0).all()
    g[9, :64] = wnt[9, :64]
    assert torch.equal(g, wnt)
    # mask_scores fused into the same pass
    mapping = torch.from_numpy(rng.integers(-3, 4000, npool * 64).astype(np.int32)).to(DEV)
    positions = torch.from_numpy(rng.integers(0, 4000, rows).astype(np.int32)).to(DEV)
    scoring.paged_logits_grouped(q8c, wc, pool, shared, 200 * 64, got, rtd, 32, relu=relu, rows=rows,
                                 mask=(mapping, positions))
    gather.mask_scores(want, rtd, mapping, positions)      # the page outside the pool: masked
    assert torch.equal(got, want)
    assert torch.isinf(want).any() and torch.isinf(want[9, :64]).all()


@pytest.mark.parametrize("share", [False, True])
def test_scorer_grouped_equals_per_row_tensor_core(share):
    rng = np.random.default_rng(41 + share)
    rows = 70
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(8)).to(torch.bfloat16).to(DEV)
    if not share:
        pages, nfixed = 100, 4
        C, fp = pages * 8, pages + nfixed
        st = _State()
        st.pages = pages
        st.centers = torch.from_numpy(_pool(rng, (C + 63) // 64)[None]).to(DEV)
        st.fine = torch.from_numpy(_pool(rng, fp)[None]).to(DEV)
        st.valid = torch.from_numpy(rng.random((1, C)) > 0.1).to(DEV)
        st.mapping = torch.from_numpy(rng.integers(-1, 5000, (1, fp * 64)).astype(np.int32)).to(DEV)
        fixed = torch.arange(pages, fp, dtype=torch.int32, device=DEV)
        cfg = _Config("v1", 0.3)
        args = (st, 0, 4000, 0, 0, fixed, 0.0883883)
    else:
        phys, pages, nfixed = 150, 90, 6
        arena = _State()
        arena.centers = torch.from_numpy(_pool(rng, phys)[None]).to(DEV)
        arena.fine = torch.from_numpy(_pool(rng, phys)[None]).to(DEV)
        arena.valid = torch.from_numpy(rng.random((1, phys, 8)) > 0.05).to(DEV)
        arena.mapping = torch.from_numpy(rng.integers(-1, 9000, (1, phys * 64)).astype(np.int32)).to(DEV)
        arena.identity = torch.arange(phys * 64, dtype=torch.int32, device=DEV)
        arena.record = lambda: None
        st = _State()
        st.arena, st.wait = arena, (lambda: None)
        st.table = torch.from_numpy(rng.permutation(phys)[None, :pages].astype(np.int32)).to(DEV)
        st.full_bucket_append, st.fixed_start, st.pages = True, 6000, pages
        fixed = torch.from_numpy(rng.permutation(phys)[None, :nfixed].astype(np.int32)).to(DEV)
        cfg = _Config("v1", 0.3, share=True)
        args = (st, 0, 7000, 0, 0, fixed, 0.1)
    scorer = native_scoring.Scorer(cfg, DEV)
    assert scorer.impl == "auto"
    got = scorer.select(q, *args)
    scorer.impl = "tensor_core"
    want = scorer.select(q, *args)
    assert torch.equal(got, want)


def test_select_tensors_public_api_matches_select():
    """select_tensors (NA/shared_scoring.py:30-62) with the caller's 32-head q8 /
    weights, against the shared select of the same query."""
    rng = np.random.default_rng(71)
    rows, phys, pages, nfixed = 6, 120, 70, 5
    arena = _State()
    arena.centers = torch.from_numpy(_pool(rng, phys)[None]).to(DEV)
    arena.fine = torch.from_numpy(_pool(rng, phys)[None]).to(DEV)
    arena.valid = torch.from_numpy(rng.random((1, phys, 8)) > 0.05).to(DEV)
    arena.mapping = torch.from_numpy(rng.integers(-1, 9000, (1, phys * 64)).astype(np.int32)).to(DEV)
    arena.identity = torch.arange(phys * 64, dtype=torch.int32, device=DEV)
    arena.record = lambda: None
    st = _State()
    st.arena, st.wait = arena, (lambda: None)
    page_ids = torch.from_numpy(rng.permutation(phys)[:pages].astype(np.int32)).to(DEV)
    fixed = torch.from_numpy(rng.permutation(phys)[None, :nfixed].astype(np.int32)).to(DEV)
    st.table = page_ids[None]
    st.full_bucket_append, st.fixed_start, st.pages = True, 6000, pages
    scorer = native_scoring.Scorer(_Config("v1", 0.4, share=True), DEV)
    scorer.impl = "tensor_core"
    q = torch.randn((rows, 4, 128), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(DEV)
    want = scorer.select(q, st, 0, 7000, 2, 0, fixed, 0.1)
    q8, w = native_scoring.pack_q(q, 0.1)
    positions = torch.arange(7002, 7002 + rows, dtype=torch.int32, device=DEV)
    got = native_scoring.select_tensors(scorer, q8, w, arena, 0, page_ids, fixed[0], positions, True, 6000)
    assert torch.equal(got, want)
    with pytest.raises(ValueError):
        native_scoring.select_tensors(scorer, q8, w, arena, 0, page_ids, fixed[0], positions, True, 6000,
                                      decode_meta=object())
