"""CPU: the oracle's published-end shared-tail variant against the reference's
Triton kernels run in the interpreter (tests/golden/shared_tail.npz), the
known answers of the reference's README / regression test, and route_physical
against the properties its own test checks."""
import numpy as np
import pytest

from oracle import v1x_oracle as O


def _case(g, ci):
    p = f"c{ci}_"
    h, R, S, W, end, cap = (int(x) for x in g[p + "case"])
    lens = np.arange(h + 1, h + R + 1) if h else np.zeros(R, np.int64)
    return p, h, R, S, W, end, cap, lens


@pytest.mark.parametrize("ci", range(4))
def test_shared_tail_golden(golden, ci):
    g = golden("shared_tail")
    p, h, R, S, W, end, cap, lens = _case(g, ci)
    dst, meta, desc = O.stage_union(g[p + "src"], g[p + "nt"], lens, end, cap, S, W,
                                    dst=np.full((cap, 8448), 165, np.uint8))
    assert np.array_equal(dst, g[p + "dst"]) and np.array_equal(meta, g[p + "meta"])
    assert np.array_equal(desc, g[p + "desc"])
    width = int(g[p + "width"])
    for shared in (0, 1):
        ft, dg, cl = O.shared_tables(lens, end, g[p + "takes"], g[p + "selected"], desc, 48, 5, 3, 16, S, W, shared)
        assert np.array_equal(ft, g[p + f"ft{shared}"]) and np.array_equal(dg, g[p + f"dg{shared}"])
        assert np.array_equal(cl, g[p + f"cl{shared}"])
        norm = O.shared_normalize(g[p + "raw"], lens, end, g[p + "takes"], g[p + "selected"], g[p + "members"], 5,
                                  width, S, W, shared)
        assert np.array_equal(norm, g[p + f"norm{shared}"])
    lg, sl = O.shared_map_topk(g[p + "ids"], g[p + "values"], lens, end, g[p + "takes"], g[p + "selected"],
                               g[p + "members"], g[p + "nt"], 5, S, W)
    assert np.array_equal(lg, g[p + "logical"]) and np.array_equal(sl, g[p + "slots"])


def test_published_end_known_answers():
    """History 65536, 4096 rows, sink 64, window 2048, published end 65536: the
    last row keeps the unindexed token 65537 although it is outside its window
    (the bucket formula would start its tail at 67584)."""
    lens = np.arange(65537, 65537 + 4096)
    nt = np.arange(2000, dtype=np.int32)
    src = np.zeros((2000, 8448), np.uint8)
    _, meta, desc = O.stage_union(src, nt, lens, 65536, 100, 64, 2048)
    assert meta[-1].tolist() == [64, 65536, 4160] and desc.tolist() == [1, 992, 1088, 97]
    assert meta[0].tolist() == [64, 63489, 2112] and meta[2047].tolist() == [64, 65536, 2112]
    s, t, c = meta[-1]
    assert t <= 65537 < lens[-1]
    old_tail = max(64, min((69632 - 1) // 1024 * 1024, 69632 - 2048))
    assert old_tail == 67584
    # the candidate set is exactly sink | last window | [end, n)
    for n, (s, t, c) in zip(lens[::257], meta[::257]):
        got = set(range(s)) | set(range(t, n))
        want = set(range(min(n, 64))) | set(range(max(0, n - 2048), n)) | set(range(min(65536, n), n))
        assert got == want and c == len(got)


def _route_case(rng, rows, pages, width):
    scores = rng.standard_normal((rows, pages * 8)).astype(np.float32)
    rt = np.stack([rng.permutation(pages) + 100 for _ in range(rows)]).astype(np.int32)
    return scores, rt


@pytest.mark.parametrize("pages", [1, 17, 64, 129, 1024, 3904, 4096])
def test_route_physical_properties(pages):
    """The checks of experiments/fine_pool_shared_20261021/test_route_shared.py:5-25."""
    rng = np.random.default_rng(pages)
    width = min(40, pages)
    scores, rt = _route_case(rng, 8, pages, width)
    pub = np.array([pages, pages // 2, 0, pages, pages + 5, -1, pages, pages])
    bud = np.array([40, 100, 4, 0, 1, 8, -1, pages])
    for sc in (scores, np.full_like(scores, -np.inf)):
        sel, takes = O.route_physical(sc, pub, bud, rt, width)
        actual = np.minimum(np.maximum(bud, 0), np.clip(pub, 0, pages)).clip(max=width)
        assert np.array_equal(takes, actual)
        reduced = sc.reshape(8, pages, 8).max(-1)
        for r in range(8):
            k, a = int(actual[r]), int(np.clip(pub[r], 0, pages))
            if k:
                ids = sel[r, :k]
                pos = [int(np.nonzero(rt[r, :a] == x)[0][0]) for x in ids]
                assert len(set(ids.tolist())) == k
                got = np.sort(reduced[r, pos])[::-1]
                want = np.sort(reduced[r, :a])[::-1][:k]
                assert np.array_equal(got, want)
            assert (sel[r, k:] == 0).all()


def test_route_physical_tie_order():
    """Equal page scores keep the blocked rank (p % 128) * ITEMS + p // 128 of
    the 128-thread layout (ITEMS = 2 for 129..256 pages)."""
    pages = 200
    scores = np.zeros((1, pages * 8), np.float32)
    rt = np.arange(pages, dtype=np.int32)[None] + 1000
    sel, takes = O.route_physical(scores, [pages], [7], rt, 7)
    items = 2
    order = sorted(range(pages), key=lambda p: (p % 128) * items + p // 128)
    assert sel[0, :7].tolist() == [1000 + p for p in order[:7]]
    # -0 and +0 are one key; an all -inf published page precedes nothing else
    scores[0, 8:16] = -0.0
    sel2, _ = O.route_physical(scores, [pages], [7], rt, 7)
    assert np.array_equal(sel, sel2)
    scores[0, :] = 0
    scores[0, 3 * 8:4 * 8] = -np.inf
    sel3, _ = O.route_physical(scores, [4], [3], rt[:, :4].copy(), 3)
    assert 1003 not in sel3[0].tolist()
