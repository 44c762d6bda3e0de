"""Known answers for the oracle's restatements of the signed-score path's
operators (TopK-v2 transform, mask_scores, the route extension)."""
import numpy as np
import pytest

from oracle import v1x_oracle as O


def test_topk_transform_small_known_answer():
    # page_size 2: raw r -> table[r >> 1] << 1 | r & 1
    s = np.array([[5, 1, 5, 9, 0, 5, 7, -1]], np.float32)
    table = np.array([[3, 0, 7, 1]], np.int32)
    out, raw = O.topk_transform(s, [8], table, 2, 4)
    # largest four by (value desc, index asc): 9@3, 7@6, 5@0, 5@2 -> ascending
    assert raw.tolist() == [[0, 2, 3, 6]]
    assert out.tolist() == [[6, 0, 1, 2]]
    ids = np.arange(16, dtype=np.int32) * 10
    out2, _ = O.topk_transform(s, [8], table[0], 2, 4, original_ids=ids)    # one shared table row
    assert out2.tolist() == [[60, 0, 10, 20]]


def test_topk_transform_trivial_rows():
    s = np.zeros((3, 10), np.float32)
    out, raw = O.topk_transform(s, [0, 3, 10], np.arange(10, dtype=np.int32)[None].repeat(3, 0), 1, 4)
    assert raw.tolist() == [[-1] * 4, [0, 1, 2, -1], [0, 1, 2, 3]]
    assert out.tolist() == raw.tolist()


def test_topk_transform_identity_table_is_select_topk():
    rng = np.random.default_rng(0)
    s = rng.integers(-3, 3, (4, 700)).astype(np.float32)
    table = np.arange(11, dtype=np.int32)[None].repeat(4, 0)
    out, raw = O.topk_transform(s, [700] * 4, table, 64, 256)
    for r in range(4):
        assert raw[r].tolist() == O.select_topk(s[r], 256).tolist()
    assert (out == raw).all()


def test_mask_scores_known_answer():
    s = np.ones((2, 128), np.float32)
    table = np.array([[1, 0], [0, 0]], np.int32)
    mapping = np.stack([np.arange(64), np.arange(64) + 100]).astype(np.int32)
    mapping[1, 5] = -1
    got = O.mask_scores(s, table, mapping, positions=[130, 40])
    # row 0: columns 0..63 read page 1 (logical 100..163; > 130 masked, col 5 invalid), 64.. page 0
    want0 = np.ones(128, np.float32)
    want0[31:64] = -np.inf
    want0[5] = -np.inf
    assert np.array_equal(got[0], want0)
    want1 = np.where(np.arange(128) % 64 > 40, -np.inf, 1).astype(np.float32)
    assert np.array_equal(got[1], want1)
    # dedup: the first 64 columns also drop logical < 64 and >= fixed_start
    got = O.mask_scores(s, table, mapping, positions=[1000, 1000], dedup_cols=64, fixed_start=120)
    assert np.isinf(got[0, 20:64]).all() and np.isinf(got[0, 5])
    assert not np.isinf(np.delete(got[0, :20], 5)).any() and not np.isinf(got[0, 64:]).any()
    assert np.isinf(got[1, :64]).all() and not np.isinf(got[1, 64:]).any()


def test_page_route_tie_order_two_per_thread():
    # 200 pages -> n = 256, two blocked ranks per 128: ties keep rank order
    # 0, 128, 1, 129, ... (page p at rank 2 * (p % 128) + p // 128)
    s = np.zeros((1, 200 * 8), np.float32)
    ids, bm = O.page_route(s, 200, 6)
    assert ids.tolist() == [[0, 128, 1, 129, 2, 130]]
    assert bm.sum() == 6 and bm[0, [0, 1, 2, 128, 129, 130]].all()
    s[0, 8 * 150 + 3] = 1.0
    s[0, 8 * 7] = -0.0
    ids, _ = O.page_route(s, 200, 3)
    assert ids.tolist() == [[150, 0, 128]]


def test_page_route_all_inf_reaches_padding_ids():
    s = np.full((1, 200 * 8), -np.inf, np.float32)
    ids, bm = O.page_route(s, 200, 200)
    assert (ids >= 200).sum() > 0          # blocked ranks of pages 200..255 interleave
    assert bm.sum() == (ids < 200).sum()


@pytest.mark.parametrize("pages,take", [(64, 10), (100, 99), (256, 256), (1000, 300), (4096, 2048)])
def test_page_route_equals_vq_route_ranking(pages, take):
    rng = np.random.default_rng(pages)
    s = rng.integers(-3, 3, (3, pages * 8)).astype(np.float32)
    ids, _ = O.page_route(s, pages, take)
    n = (pages + 15) // 16 * 1024 + 1
    sel, _ = O.route(s, np.full(3, n), np.full(3, min(take, pages - 1)), take, pages,
                     np.zeros((3, pages), np.int32), np.zeros((3, take), np.int32), np.zeros(3), 1, False)
    assert (ids == sel).all()


def test_pack_q_known_answer():
    q = np.zeros((2, 5, 128), np.float32)
    q[0, 0, :3] = [56.0, -28.0, 1.0]      # absmax / 448 = 1/8 exactly: scale 1/8
    q[0, 1, 0] = 57.0                      # just above: scale 1/4
    q[1, 2, 5] = 1e-9                      # below the 1e-4 floor: scale 2^-22
    q8, w = O.pack_q(q[:, :4], 8, np.float32(0.5), out_rows=3)
    assert q8.shape == (3, 8, 128) and w.shape == (3, 8)
    assert O.e4m3_to_f32(q8[0, 0, :3]).tolist() == [448.0, -224.0, 8.0]
    assert w[0, 0] == np.float32(0.125 * 0.5) and w[0, 1] == np.float32(0.25 * 0.5)
    assert O.e4m3_to_f32(q8[0, 1, :1]).tolist() == [224.0]     # 57 / 0.25 = 228 -> 224 (step 16)
    assert w[1, 2] == np.float32(2.0 ** -22 * 0.5)
    assert (q8[:, 4:] == 0).all() and (w[:, 4:] == 0).all() and (q8[2] == 0).all() and (w[2] == 0).all()


def test_mqa_logits_is_score_row_on_each_window():
    rng = np.random.default_rng(4)
    q8 = O.e4m3_from_f32(rng.standard_normal((3, 2, 128)).astype(np.float32))
    w = rng.standard_normal((3, 2)).astype(np.float32)
    k8 = O.e4m3_from_f32(rng.standard_normal((50, 128)).astype(np.float32))
    ks = rng.uniform(0.1, 1, 50).astype(np.float32)
    out = O.mqa_logits(q8, w, k8, ks, [0, 10, 30], [50, 20, 10], relu=False)
    k = O.e4m3_to_f32(k8)
    assert np.array_equal(out[0], O.score_row(q8[0], w[0], k, ks, relu=False))
    assert np.isinf(out[1, :10]).all() and np.isinf(out[1, 20:]).all()
    assert np.array_equal(out[1, 10:20], O.score_row(q8[1], w[1], k[10:20], ks[10:20], relu=False))
    assert np.isinf(out[2]).all()


def test_mask_scores_golden(golden):
    g = golden("signed")
    for i in range(2):
        pre = f"mask{i}_"
        dedup, fixed = g[pre + "dedup"].tolist()
        got = O.mask_scores(g[pre + "scores_in"], g[pre + "table"], g[pre + "mapping"].reshape(-1, 64),
                            g[pre + "positions"], dedup, fixed)
        assert np.array_equal(got, g[pre + "scores_out"])
        assert np.isinf(got).sum() > 0


def test_pack_q_and_quantize_golden(golden):
    from test_oracle_build import _interpreter_cast_defect
    g = golden("signed")
    q = g["q"].view(np.uint16).astype(np.uint32) << 16
    q = q.view(np.float32)                                   # bf16 -> f32
    q8, w = O.pack_q(q[:, 4:8], 32, np.float32(0.0883883 / 4), out_rows=7)
    assert np.array_equal(w, g["pack_w"])
    ref = g["pack_q8"]
    differ = q8 != ref
    # the interpreter's float8 cast (not round-to-nearest-even; the GPU's cvt.rn
    # is) is the only difference: its two known defects, and exact ties (bf16
    # inputs over a power-of-two scale often sit halfway between two e4m3
    # codes), which it rounds away from zero where RTNE keeps the even code
    x = q[:, 4:8]
    scale = O.pow2_ceil(np.maximum(np.abs(x).max(-1), np.float32(1e-4)) / np.float32(448))
    v = np.zeros((7, 32, 128), np.float64)
    v[:5, :4] = np.abs(x / scale[..., None])
    lo = O.e4m3_to_f32(q8 & 0x7F).astype(np.float64)
    hi = O.e4m3_to_f32((q8 & 0x7F) + 1).astype(np.float64)
    tie = (ref.astype(int) == q8.astype(int) + 1) & (q8 % 2 == 0) & (v == (lo + hi) / 2)
    assert (_interpreter_cast_defect(q8, ref) | tie)[differ].all()
    assert differ.mean() < 0.05
    # quantize is torch math on CPU (torch's e4m3 cast rounds to nearest even): exact
    q8, w = O.pack_q(q.reshape(-1, 1, 128), 1, 1.0)
    assert np.array_equal(q8.reshape(-1), g["quant_q8"].reshape(-1))
    assert np.array_equal(w.reshape(-1), g["quant_scale"].reshape(-1))


def test_mask_scores_page_outside_mapping_is_masked():
    s = np.ones((1, 128), np.float32)
    mapping = np.zeros((2, 64), np.int32)
    got = O.mask_scores(s, np.array([[5, -1]], np.int32), mapping, [10])
    assert np.isinf(got).all()


def test_route_extension_layout_equals_fused_route_for_every_accepted_shape():
    """NA/deps/route.py:71-76 picks n = the smallest of 128..4096 (and >= THREADS)
    holding the pages, BASE = n / 128; fused.route (VQ:175-177) picks THREADS x
    ITEMS by the page count alone.  For every (threads, pages) the extension
    accepts (pages > threads / 2) the two blocked layouts are the same, which
    is what lets the extension run on fused.route's ranking."""
    for threads in (64, 128, 256, 512):
        sizes = [n for n in (128, 256, 512, 1024, 2048, 4096) if n >= threads]
        for pages in range(threads // 2 + 1, 4097):
            n_ext = next(n for n in sizes if pages <= n)
            t, it = O.route_geometry(max(pages, 64))
            assert n_ext == t * it, (threads, pages)


def test_mqa_logits_equals_paged_scoring_of_the_same_keys():
    """The flat-key logits of the dsa mode equal the paged scorer's over the
    same keys packed into pages (identity table), inside each row's window."""
    rng = np.random.default_rng(8)
    N, rows = 200, 3
    k8 = O.e4m3_from_f32(rng.standard_normal((N, 128)).astype(np.float32))
    ks = rng.uniform(0.1, 1, N).astype(np.float32)
    q8 = O.e4m3_from_f32(rng.standard_normal((rows, 4, 128)).astype(np.float32))
    w = rng.standard_normal((rows, 4)).astype(np.float32)
    P = (N + 63) // 64
    pool = np.zeros((P, 8448), np.uint8)
    kk = np.zeros((P * 64, 128), np.uint8)
    kk[:N] = k8
    sc = np.zeros(P * 64, np.float32)
    sc[:N] = ks
    pool[:, :8192] = kk.reshape(P, 8192)
    pool[:, 8192:] = sc.view(np.uint8).reshape(P, 256)
    paged = O.score_paged(q8, w, pool, np.arange(P)[None].repeat(rows, 0), [N] * rows, N, relu=False)
    flat = O.mqa_logits(q8, w, k8, ks, [0, 50, 0], [N, 120, 1], relu=False)
    assert np.array_equal(flat[0], paged[0])
    assert np.array_equal(flat[1, 50:120], paged[1, 50:120]) and np.isinf(flat[1, :50]).all()
    assert flat[2, 0] == paged[2, 0] and np.isinf(flat[2, 1:]).all()
