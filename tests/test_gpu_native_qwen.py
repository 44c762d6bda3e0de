"""The signed-score (v1_native) path's operators against the oracle: TopK-v2's
transform (plain and through original ids), mask_scores and the page route
extension, called through their drop-in modules."""
import importlib

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
