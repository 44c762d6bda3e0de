"""GPU parity: _sort (NA/fused_grouping.py:64-76) and the page lifecycle
(DS/kernels.py:57-179) vs the oracle and the reference's golden vectors."""
import importlib

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

FG = importlib.import_module("10_20_b200.fused_grouping")
K = importlib.import_module("10_20_b200.kernels")


def dev(x):
    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def test_sort_golden(golden, cuda_dev):
    g = golden("sort")
    flag = torch.tensor(-1, dtype=torch.int32, device="cuda")
    out = torch.full((16,), -99, dtype=torch.int32, device="cuda")
    perm = dev(g["ids16"])
    FG._sort[(1, 1)](perm, out, dev(g["values16"]), flag, 16, num_warps=4)
    assert out.cpu().numpy().tolist() == g["out16"].tolist()
    assert perm.cpu().numpy().tolist() == g["ids16"].tolist()
    flag.fill_(0)
    out.fill_(-99)
    FG._sort[(1, 1)](perm, out, dev(g["values16"]), flag, 16)
    assert bool((out == -99).all())
    flag.fill_(-1)
    o = torch.full((2, 4096), -7, dtype=torch.int32, device="cuda")
    FG._sort[(16, 2)](dev(g["p256"]), o, dev(g["s256"]), flag, 256)
    assert np.array_equal(o.cpu().numpy(), g["o256"])
    o = torch.full((1, 4096), -7, dtype=torch.int32, device="cuda")
    FG._sort[(1, 1)](dev(g["p4096"]), o, dev(g["s4096"]), flag, 4096)
    assert np.array_equal(o.cpu().numpy(), g["o4096"])


@pytest.mark.parametrize("N", [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096])
def test_sort_random_sizes(N, cuda_dev):
    rng = np.random.default_rng(N)
    heads = 16
    S = rng.integers(-5, 6, size=(heads, 4096)).astype(np.float32) * 0.5
    S[S == 0] = np.where(rng.random(int((S == 0).sum())) < 0.5, 0.0, -0.0)
    S.reshape(-1)[::101] = np.inf
    S.reshape(-1)[::103] = -np.inf
    S.reshape(-1)[::107] = np.nan
    P = rng.permutation(heads * 4096).astype(np.int32).reshape(heads, 4096)
    flag = torch.tensor(-1, dtype=torch.int32, device="cuda")
    o = torch.full((heads, 4096), -7, dtype=torch.int32, device="cuda")
    FG._sort[(4096 // N, heads)](dev(P), o, dev(S), flag, N)
    assert np.array_equal(o.cpu().numpy().reshape(-1), O.sort_segments(P, S, -1, N, 4096 // N, heads))


@pytest.mark.parametrize("N,groups", [(16, 5), (64, 3), (256, 1), (1024, 2)])
def test_sort_partial_grid(N, groups, cuda_dev):
    """A grid of fewer groups than 4096 / N sorts only those segments; the rest
    of O is untouched.  Unaligned (offset) views take the same answers."""
    rng = np.random.default_rng(N + groups)
    heads = 3
    S = rng.integers(0, 7, size=(heads, 4096)).astype(np.float32)
    P = rng.permutation(heads * 4096).astype(np.int32).reshape(heads, 4096)
    flag = torch.tensor(-1, dtype=torch.int32, device="cuda")
    o = torch.full((heads, 4096), -7, dtype=torch.int32, device="cuda")
    FG._sort[(groups, heads)](dev(P), o, dev(S), flag, N)
    got = o.cpu().numpy()
    exp = np.full((heads, 4096), -7, np.int32)
    full = O.sort_segments(P, S, -1, N, groups, heads).reshape(heads, 4096)
    exp[:, :groups * N] = full[:, :groups * N]
    assert np.array_equal(got, exp)
    # 4-byte (not 16-byte) aligned views of the same data
    Sb = torch.zeros(heads * 4096 + 1, device="cuda")
    Sb[1:] = dev(S).reshape(-1)
    Pb = torch.zeros(heads * 4096 + 1, dtype=torch.int32, device="cuda")
    Pb[1:] = dev(P).reshape(-1)
    ob = torch.full((heads * 4096 + 1,), -7, dtype=torch.int32, device="cuda")
    FG._sort[(groups, heads)](Pb[1:].view(heads, 4096), ob[1:].view(heads, 4096), Sb[1:].view(heads, 4096), flag,
                              N)
    assert np.array_equal(ob[1:].view(heads, 4096).cpu().numpy(), exp)


def test_sort_baseline_records_and_offsets(cuda_dev):
    """65,536 records (16 x 4096) keyed by group ids with duplicate runs."""
    rng = np.random.default_rng(11)
    keys = rng.integers(0, 4096, size=(16, 4096))
    run = rng.random((16, 4096)) < 0.3
    for h in range(16):
        for i in range(1, 4096):
            if run[h, i]:
                keys[h, i] = keys[h, i - 1]
    S = keys.astype(np.float32)
    P = np.arange(16 * 4096, dtype=np.int32).reshape(16, 4096)
    flag = torch.tensor(-1, dtype=torch.int32, device="cuda")
    o = torch.empty((16, 4096), dtype=torch.int32, device="cuda")
    FG._sort[(1, 16)](dev(P), o, dev(S), flag, 4096)
    exp = O.sort_segments(P, S, -1, 4096, 1, 16).reshape(16, 4096)
    assert np.array_equal(o.cpu().numpy(), exp)
    offs = FG.group_offsets(dev(S), 4096, 16, 4096).cpu().numpy()
    for h in range(16):
        sk = keys[h][exp[h] - h * 4096]
        assert np.array_equal(offs[h], O.group_offsets(sk, 4096))


@pytest.mark.parametrize("N", [256, 1024, 4096])
@pytest.mark.parametrize("kind", ["groups", "mixed"])
def test_sort_grouped_equals_sort_then_offsets(N, kind, cuda_dev):
    """The fused sort + offsets launch == _sort followed by group_offsets."""
    rng = np.random.default_rng(N + len(kind))
    heads, K = 8, 3000
    if kind == "groups":
        S = rng.integers(0, K, size=(heads, 4096)).astype(np.float32)
        S[:, 1::3] = S[:, 0::3][:, : S[:, 1::3].shape[1]]          # duplicate runs
        S[0] = 7.0                                                  # one segment of equal keys
    else:   # non-integers, negatives, out-of-range keys, +-0, inf and NaN mixed in
        S = rng.integers(-50, K + 50, size=(heads, 4096)).astype(np.float32)
        S[:, ::5] += 0.5
        S.reshape(-1)[::97] = -0.0
        S.reshape(-1)[::89] = np.inf
        S.reshape(-1)[::83] = np.nan
    P = rng.permutation(heads * 4096).astype(np.int32).reshape(heads, 4096)
    flag = torch.tensor(-1, dtype=torch.int32, device="cuda")
    o1 = torch.empty((heads, 4096), dtype=torch.int32, device="cuda")
    o2 = torch.empty_like(o1)
    FG._sort[(4096 // N, heads)](dev(P), o1, dev(S), flag, N)
    offs1 = FG.group_offsets(dev(S), N, heads, K)
    offs2 = FG.sort_grouped(dev(P), o2, dev(S), flag, N, heads, K)
    assert torch.equal(o1, o2)
    assert torch.equal(offs1, offs2)
    assert np.array_equal(o1.cpu().numpy().reshape(-1), O.sort_segments(P, S, -1, N, 4096 // N, heads))


def _state(cap, free=None):
    return dict(fine=torch.zeros((cap, 8448), dtype=torch.uint8, device="cuda"),
                members=torch.full((cap, 64), -1, dtype=torch.int32, device="cuda"),
                live=torch.zeros((cap, 2), dtype=torch.int64, device="cuda"),
                refs=torch.zeros(cap, dtype=torch.int32, device="cuda"),
                free=(torch.arange(cap, dtype=torch.int32) if free is None else torch.as_tensor(free)).cuda(),
                count=torch.tensor(cap, dtype=torch.int32, device="cuda"))


def test_page_lifecycle_reference_sequence(golden, cuda_dev):
    g = golden("pages")
    cap = 16
    st = _state(cap)
    tmp = torch.arange(16, dtype=torch.uint8, device="cuda")[:, None].expand(16, 8448).contiguous()
    mapping = torch.arange(1024, dtype=torch.int32, device="cuda").reshape(16, 64)
    meta = torch.tensor([0, 0, 1], dtype=torch.int32, device="cuda")
    hashes = torch.empty((16, 2), dtype=torch.int64, device="cuda")
    centers = torch.zeros((2, 8448), dtype=torch.uint8, device="cuda")
    centers[:, :8192] = 7
    centers.view(torch.float32)[:, 2048:] = 1.25
    tables = torch.full((2, 16), -1, dtype=torch.int32, device="cuda")
    new = torch.empty(16, dtype=torch.bool, device="cuda")
    match = torch.empty(16, dtype=torch.int32, device="cuda")
    cpool = torch.zeros((4, 8448), dtype=torch.uint8, device="cuda")

    def lookup():
        K.match_pages[(16,)](tmp, mapping, hashes, meta, st["fine"], st["members"], st["live"],
                             st["refs"], match, cap, 16)

    def alloc_publish():
        K.allocate[(1,)](meta, match, st["free"], st["count"], st["refs"], tables, new, debug=True)
        K.publish[(16,)](tmp, centers, centers.view(torch.float32), mapping, hashes, meta, tables, new,
                         st["fine"], cpool, cpool.view(torch.float32), st["members"], st["live"])

    K.fingerprint[(16,)](tmp, mapping, meta, hashes)
    assert np.array_equal(hashes.cpu().numpy(), g["t_hash"])
    lookup()
    assert np.array_equal(match.cpu().numpy(), g["t_match0"])
    alloc_publish()
    assert tables[0].tolist() == list(range(15, -1, -1))
    assert np.array_equal(tables.cpu().numpy(), g["t_tables1"])
    assert st["count"].item() == 0 and bool(new.all()) and bool((st["refs"] == 1).all())
    assert torch.equal(st["fine"][tables[0].long()], tmp)
    assert torch.equal(cpool[:2], centers)
    tmp[0, 0] = 99
    lookup()
    assert match[0].item() == -1
    tmp[0, 0] = 0
    mapping[0, 0] = 9999
    lookup()
    assert match[0].item() == -1
    mapping[0, 0] = 0
    meta[1] = 1
    lookup()
    assert torch.equal(match, tables[0])
    alloc_publish()
    assert torch.equal(tables[1], tables[0]) and not bool(new.any())
    assert bool((st["refs"] == 2).all()) and torch.equal(cpool[2:], centers)
    assert np.array_equal(cpool.cpu().numpy(), g["t_center_pool"])
    K.release[(1,)](tables[0], st["refs"], st["free"], st["count"])
    assert st["count"].item() == 0 and bool((st["refs"] == 1).all())
    K.release[(1,)](tables[1], st["refs"], st["free"], st["count"])
    assert st["count"].item() == 16 and bool((st["refs"] == 0).all())
    assert np.array_equal(st["free"].cpu().numpy(), g["t_free4"])


def test_page_lifecycle_sharing_collision_golden(golden, cuda_dev):
    g = golden("pages")
    cap = 48
    st = _state(cap, g["r_free0"])
    tables = torch.full((4, 16), -1, dtype=torch.int32, device="cuda")
    cpool = torch.zeros((8, 8448), dtype=torch.uint8, device="cuda")
    for lease in range(3):
        t, m, tc = dev(g[f"r_b{lease}_tmp"]), dev(g[f"r_b{lease}_map"]), dev(g[f"r_b{lease}_tc"])
        meta = torch.tensor([lease * 1024, lease, 1], dtype=torch.int32, device="cuda")
        h = torch.empty((16, 2), dtype=torch.int64, device="cuda")
        K.fingerprint[(16,)](t, m, meta, h)
        assert np.array_equal(h.cpu().numpy(), g[f"r_b{lease}_hash"])
        if lease == 2:
            st["live"][tables[0, 1].long()] = h[3]
        mt = torch.empty(16, dtype=torch.int32, device="cuda")
        K.match_pages[(16,)](t, m, h, meta, st["fine"], st["members"], st["live"], st["refs"], mt, cap, 64)
        assert np.array_equal(mt.cpu().numpy(), g[f"r_b{lease}_match"])
        nw = torch.empty(16, dtype=torch.bool, device="cuda")
        K.allocate[(1,)](meta, mt, st["free"], st["count"], st["refs"], tables, nw)
        K.publish[(16,)](t, tc, tc.view(torch.float32), m, h, meta, tables, nw, st["fine"], cpool,
                         cpool.view(torch.float32), st["members"], st["live"])
        assert np.array_equal(tables.cpu().numpy(), g[f"r_tables{lease}"])
        assert np.array_equal(st["refs"].cpu().numpy(), g[f"r_refs{lease}"])
        assert np.array_equal(st["free"].cpu().numpy(), g[f"r_free{lease}"])
    for lease in (1, 0):
        K.release[(1,)](tables[lease], st["refs"], st["free"], st["count"])
        assert np.array_equal(st["refs"].cpu().numpy(), g[f"r_rel_refs{lease}"])
        assert st["count"].item() == int(g[f"r_rel_count{lease}"])
        assert np.array_equal(st["free"].cpu().numpy(), g[f"r_rel_free{lease}"])
    assert np.array_equal(st["fine"].cpu().numpy(), g["r_fine"])
    assert np.array_equal(st["members"].cpu().numpy(), g["r_members"])
    assert np.array_equal(st["live"].cpu().numpy(), g["r_live"])
    assert np.array_equal(cpool.cpu().numpy(), g["r_center_pool"])


def test_allocate_exhausted_reports_and_leaves_state(cuda_dev):
    cap = 8
    st = _state(cap)
    tables = torch.full((1, 16), -1, dtype=torch.int32, device="cuda")
    meta = torch.tensor([0, 0, 1], dtype=torch.int32, device="cuda")
    match = torch.full((16,), -1, dtype=torch.int32, device="cuda")
    new = torch.zeros(16, dtype=torch.bool, device="cuda")
    with pytest.raises(K.ArenaExhausted):
        K.allocate[(1,)](meta, match, st["free"], st["count"], st["refs"], tables, new)
    assert st["count"].item() == cap and bool((st["refs"] == 0).all()) and bool((tables == -1).all())
    K.check_status("cuda:0")  # status was reset by the raise
    meta[2] = 0                # inactive: no-op, no error
    K.allocate[(1,)](meta, match, st["free"], st["count"], st["refs"], tables, new)


def test_large_arena_lowest_match(cuda_dev):
    """CAP = 131,072: the whole-GPU sweep returns the lowest live exact match."""
    cap = 131072
    rng = np.random.default_rng(1)
    st = _state(cap)
    tmp = torch.as_tensor(rng.integers(0, 256, (16, 8448), dtype=np.uint8)).cuda()
    mapping = torch.as_tensor(rng.integers(0, 1 << 20, (16, 64)).astype(np.int32)).cuda()
    meta = torch.tensor([0, 0, 1], dtype=torch.int32, device="cuda")
    h = torch.empty((16, 2), dtype=torch.int64, device="cuda")
    K.fingerprint[(16,)](tmp, mapping, meta, h)
    # plant page 3 at slots 100000 (live) and 120000 (live), page 5 at 7 (dead) and 90000 (live),
    # page 9's hash at 500 with one differing byte (collision that must miss)
    for p, j, live in ((3, 120000, 1), (3, 100000, 1), (5, 7, 0), (5, 90000, 1), (9, 500, 1)):
        st["fine"][j] = tmp[p]
        st["members"][j] = mapping[p]
        st["live"][j] = h[p]
        st["refs"][j] = live
    st["fine"][500, 17] ^= 1
    match = torch.empty(16, dtype=torch.int32, device="cuda")
    K.match_pages[(16,)](tmp, mapping, h, meta, st["fine"], st["members"], st["live"], st["refs"], match,
                         cap, 131072)
    m = match.cpu().numpy()
    assert m[3] == 100000 and m[5] == 90000 and m[9] == -1
    assert (np.delete(m, [3, 5]) == -1).all()
