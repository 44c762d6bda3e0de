"""GPU parity: fused.route and fused.topk (sm_100a kernels) vs the CPU oracle.

Bit-exact: selected page ranks, fine page tables, raw/logical/physical slots,
expansion and the in-place mask.  Reference behaviour:
sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:7-220 and
DS/example_v1_query_single_head.py:8-74.
"""
import importlib

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

qf = importlib.import_module("10_20_b200.query_fused")


def dev(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def test_reference_example(golden, cuda_dev):
    g = golden("route_topk_example")
    B, P, CAP, TAKE, N, TOP, WINDOW = 1024, 128, 128, 40, 4097, 2048, 64
    mod = qf.module()
    scores = dev(np.repeat(g["scores"], B, 0))
    lens = torch.full((B,), N, dtype=torch.int32, device="cuda")
    takes = torch.full((B,), TAKE, dtype=torch.int32, device="cuda")
    selected = torch.full((B, TAKE), -1, dtype=torch.int32, device="cuda")
    ft = torch.full((B, TAKE + 68), -1, dtype=torch.int32, device="cuda")
    tail_rows = torch.zeros(B, dtype=torch.int32, device="cuda")
    rt = dev(np.repeat(g["reorder_pages"][None], B, 0))
    nt = dev(np.repeat(g["native_pages"][None], B, 0))
    mod.route(scores, lens, takes, selected, P, rt, ft, tail_rows, CAP, True)
    assert torch.equal(selected.cpu(), torch.as_tensor(np.repeat(g["selected"], B, 0)).int())
    assert selected[0, :8].tolist() == [48, 49, 50, 51, 52, 53, 54, 55]
    assert torch.equal(ft[:, :TAKE].cpu(), torch.as_tensor(np.repeat(g["ft_sel"], B, 0)))
    assert torch.equal(ft[:, TAKE:].cpu(), (CAP + torch.arange(68, dtype=torch.int32))[None].expand(B, -1))
    members = dev(g["members"])
    fine = np.repeat(g["fine_scores"], B, 0)
    fl = torch.full((B,), fine.shape[1], dtype=torch.int32, device="cuda")
    phys = torch.empty((B, TOP), dtype=torch.int32, device="cuda")
    logical = torch.empty_like(phys)
    raw = torch.empty_like(phys)
    noexp = torch.empty_strided((B, 0), (0, 1), device="cuda", dtype=torch.int32)
    for direct in (False, True):
        work = dev(fine)
        mod.topk(work, fl, members, rt, nt, selected, lens, takes, phys, logical, raw, WINDOW, True,
                 noexp, True, True, ft, direct)
        torch.cuda.synchronize()
        assert torch.equal(work.cpu(), torch.as_tensor(np.repeat(g["masked"], B, 0)))
        assert torch.equal(raw.sort(1).values.cpu().long(), torch.as_tensor(np.repeat(g["raw_sorted"], B, 0)))
        assert torch.equal(logical.sort(1).values.cpu(), torch.as_tensor(np.repeat(g["logical_sorted"], B, 0)).int())
        assert torch.equal(phys.sort(1).values.cpu(), torch.as_tensor(np.repeat(g["physical_sorted"], B, 0)).int())
        # ascending raw order, mapping per entry
        assert bool((raw[:, 1:] > raw[:, :-1]).all())
        cid = torch.as_tensor(np.repeat(g["candidate_ids"], B, 0)).cuda()
        assert torch.equal(logical, cid.gather(1, raw.long()))


def _route_case(rng, B, P, K, take_choices, tie_mode):
    pages_max = P
    lens = rng.integers(1, pages_max * 64 + 1, size=B).astype(np.int32)
    lens[0] = pages_max * 64
    lens[1] = 1
    if B > 2:
        lens[2] = 1025
    takes = rng.choice(take_choices, size=B).astype(np.int32)
    L = P * 8 + 8
    if tie_mode == "int":
        scores = rng.integers(-3, 4, size=(B, L)).astype(np.float32)
        scores[scores == 0] = np.where(rng.random(int((scores == 0).sum())) < 0.5, 0.0, -0.0)
    elif tie_mode == "neginf":
        scores = rng.standard_normal((B, L)).astype(np.float32)
        scores[:, ::3] = -np.inf
        scores[: B // 2, :] = -np.inf
    else:
        scores = rng.standard_normal((B, L)).astype(np.float32)
    rt = rng.integers(0, 100000, size=(B, P)).astype(np.int32)
    tail_rows = rng.integers(0, B, size=B).astype(np.int32)
    return lens, takes, scores, rt, tail_rows


@pytest.mark.parametrize("P", [64, 128, 200, 300, 700, 1500, 2048, 4096])
@pytest.mark.parametrize("tie_mode", ["float", "int", "neginf"])
def test_route_random(P, tie_mode, cuda_dev):
    rng = np.random.default_rng(P * 7 + len(tie_mode))
    B = 37
    K = min(P, 40)
    lens, takes, scores, rt, tail_rows = _route_case(rng, B, P, K, [0, 1, K // 2, K], tie_mode)
    for sel_dtype in (torch.int32, torch.int64):
        for fill in (True, False):
            ft0 = np.full((B, K + 68), -7, np.int32)
            sel = torch.full((B, K), -5, dtype=sel_dtype, device="cuda")
            ft = dev(ft0)
            qf.module().route(dev(scores), dev(lens), dev(takes), sel, P, dev(rt), ft, dev(tail_rows),
                              1000, fill)
            esel, eft = O.route(scores, lens, takes, K, P, rt, ft0, tail_rows, 1000, fill)
            assert np.array_equal(sel.cpu().numpy(), esel), (P, tie_mode, fill)
            assert np.array_equal(ft.cpu().numpy(), eft), (P, tie_mode, fill)


@pytest.mark.parametrize("P", [300, 1500, 2048, 4096])
@pytest.mark.parametrize("tie_mode", ["float", "int", "neginf"])
def test_route_many_winners(P, tie_mode, cuda_dev):
    """Takes of hundreds to thousands of pages: the winners are ordered through
    the histogram bins (or, with crowded bins, by the bitwise search and sort)."""
    rng = np.random.default_rng(P * 11 + len(tie_mode))
    B = 21
    K = P // 2 if P < 4096 else 3000
    lens, takes, scores, rt, tail_rows = _route_case(rng, B, P, K, [K // 3, K - 1, K], tie_mode)
    ft0 = np.full((B, K + 68), -7, np.int32)
    sel = torch.full((B, K), -5, dtype=torch.int32, device="cuda")
    ft = dev(ft0)
    qf.module().route(dev(scores), dev(lens), dev(takes), sel, P, dev(rt), ft, dev(tail_rows), 1000, True)
    esel, eft = O.route(scores, lens, takes, K, P, rt, ft0, tail_rows, 1000, True)
    assert np.array_equal(sel.cpu().numpy(), esel), (P, tie_mode)
    assert np.array_equal(ft.cpu().numpy(), eft), (P, tie_mode)


def test_route_strided_scores_and_checks(cuda_dev):
    rng = np.random.default_rng(5)
    B, P, K = 9, 256, 40
    lens, takes, scores, rt, tail_rows = _route_case(rng, B, P, K, [40], "float")
    big = torch.full((B, P * 8 + 64), float("nan"), device="cuda")
    big[:, : scores.shape[1]] = dev(scores)
    view = big[:, : P * 8 + 8]
    sel = torch.empty((B, K), dtype=torch.int32, device="cuda")
    ft = torch.empty((B, K + 68), dtype=torch.int32, device="cuda")
    qf.module().route(view, dev(lens), dev(takes), sel, P, dev(rt), ft, dev(tail_rows), 9, True)
    esel, eft = O.route(scores, lens, takes, K, P, rt, np.zeros((B, K + 68), np.int32), tail_rows, 9, True)
    assert np.array_equal(sel.cpu().numpy(), esel) and np.array_equal(ft.cpu().numpy(), eft)
    with pytest.raises(ValueError):  # pages below the reference's 64 minimum
        qf.module().route(view, dev(lens), dev(takes), sel, 32, dev(rt[:, :32]), ft, dev(tail_rows), 9, True)
    with pytest.raises(ValueError):  # score stride not a multiple of 4
        odd = torch.zeros((B, P * 8 + 9), device="cuda")[:, : P * 8 + 2]
        qf.module().route(odd[:, 1:], dev(lens), dev(takes), sel, P, dev(rt), ft, dev(tail_rows), 9, True)


def _topk_case(rng, B, L, T, take, P=96, cap=64, tie="float"):
    members = np.full((cap, 64), -1, np.int32)
    for page in range(cap):
        bucket = page % 6
        members[page] = bucket * 1024 + rng.permutation(1024)[:64]
    rt = np.stack([rng.permutation(cap) for _ in range(B)]).astype(np.int32)
    rt = np.concatenate([rt, np.zeros((B, P - cap), np.int32)], 1)
    nt = np.stack([rng.permutation(P) for _ in range(B)]).astype(np.int32)
    selected = np.stack([rng.permutation(cap)[:take] for _ in range(B)]).astype(np.int32)
    lens = rng.integers(1024, 6 * 1024, size=B).astype(np.int32)
    takes = np.full(B, take, np.int32)
    takes[0] = take // 2
    if tie == "zeros":
        scores = np.maximum(rng.standard_normal((B, L)), 0).astype(np.float32)
    elif tie == "coarse":
        scores = (rng.integers(0, 5, size=(B, L)) * 0.25).astype(np.float32)
    else:
        scores = rng.standard_normal((B, L)).astype(np.float32)
    fl = rng.integers(max(T - 100, 1), L + 1, size=B).astype(np.int32)
    fl[0] = L
    fl[1] = T
    fl[2] = T - 5
    ft = np.stack([rt[b, selected[b]] for b in range(B)]).astype(np.int32)
    ft = np.concatenate([ft, np.full((B, 4), 7, np.int32)], 1)
    return members, rt, nt, selected, lens, takes, scores, fl, ft


@pytest.mark.parametrize("L,T", [(2688, 2048), (3648, 2048), (700, 512), (6912, 2048), (9000, 2048),
                                 (20000, 1024), (46000, 2048)])
@pytest.mark.parametrize("tie", ["float", "zeros", "coarse"])
def test_topk_random(L, T, tie, cuda_dev):
    rng = np.random.default_rng(L + T + len(tie))
    B, take = 11, 12
    members, rt, nt, selected, lens, takes, scores, fl, ft = _topk_case(rng, B, L, T, take, tie=tie)
    for direct, from_rank, phys_out, mask in ((False, True, True, True), (True, False, True, True),
                                               (False, True, False, False)):
        es = T * 4 + 64 if not phys_out else 0
        work = dev(scores)
        phys = torch.full((B, T), -9, dtype=torch.int32, device="cuda")
        logical = torch.full_like(phys, -9)
        raw = torch.full_like(phys, -9)
        exp = torch.full((B, es), -9, dtype=torch.int32, device="cuda") if es else \
            torch.empty_strided((B, 0), (0, 1), device="cuda", dtype=torch.int32)
        qf.module().topk(work, dev(fl), dev(members), dev(rt), dev(nt), dev(selected), dev(lens),
                         dev(takes), phys, logical, raw, 64, mask, exp, phys_out, from_rank, dev(ft), direct)
        e = O.topk(scores, fl, members, rt, nt, selected, lens, takes, 64, mask, T, es, phys_out,
                   from_rank, ft, direct)
        assert np.array_equal(work.cpu().numpy(), e["scores"])
        assert np.array_equal(logical.cpu().numpy(), e["logical"])
        if phys_out:
            assert np.array_equal(raw.cpu().numpy(), e["raw"])
            assert np.array_equal(phys.cpu().numpy(), e["physical"])
        else:
            assert bool((phys == -9).all()) and bool((raw == -9).all())
        if es:
            assert np.array_equal(exp.cpu().numpy(), e["expanded"])


@pytest.mark.parametrize("L,cols,T", [(2688, 3648, 2048), (4096, 4096, 2048), (1500, 2000, 1024)])
@pytest.mark.parametrize("tie", ["float", "zeros"])
def test_topk_many_rows(L, cols, T, tie, cuda_dev):
    """More rows than two waves of SMs and rows of at most 4096 columns: the
    256-thread variant (four CTAs per SM) -- same results as the oracle,
    including strided score rows (a column slice of a wider buffer)."""
    rng = np.random.default_rng(L + cols + len(tie))
    B, take = 320, 12
    members, rt, nt, selected, lens, takes, scores, fl, ft = _topk_case(rng, B, L, T, take, tie=tie)
    wide = np.full((B, cols + 64), 7.0, np.float32)
    wide[:, :scores.shape[1]] = scores
    work = dev(wide)
    phys = torch.full((B, T), -9, dtype=torch.int32, device="cuda")
    logical, raw = torch.full_like(phys, -9), torch.full_like(phys, -9)
    noexp = torch.empty_strided((B, 0), (0, 1), device="cuda", dtype=torch.int32)
    qf.module().topk(work[:, :cols], dev(np.minimum(fl, cols).astype(np.int32)), dev(members), dev(rt), dev(nt),
                     dev(selected), dev(lens), dev(takes), phys, logical, raw, 64, True, noexp, True, True, dev(ft),
                     False)
    fl2 = np.minimum(fl, cols).astype(np.int32)
    e = O.topk(wide[:, :cols].copy(), fl2, members, rt, nt, selected, lens, takes, 64, True, T, 0, True, True, ft,
               False)
    assert np.array_equal(work[:, :cols].cpu().numpy(), e["scores"])
    assert np.array_equal(raw.cpu().numpy(), e["raw"])
    assert np.array_equal(logical.cpu().numpy(), e["logical"])
    assert np.array_equal(phys.cpu().numpy(), e["physical"])
    assert bool((work[:, cols:] == 7.0).all())


def test_topk_streaming_path_and_all_neginf(cuda_dev):
    """Rows wider than the shared-memory stage (60000 cols) and all -inf rows."""
    rng = np.random.default_rng(3)
    B, L, T, take = 4, 60000, 2048, 8
    members, rt, nt, selected, lens, takes, scores, fl, ft = _topk_case(rng, B, L, T, take)
    scores[1] = -np.inf
    scores[2, ::2] = 0.0
    work = dev(scores)
    phys = torch.empty((B, T), dtype=torch.int32, device="cuda")
    logical, raw = torch.empty_like(phys), torch.empty_like(phys)
    noexp = torch.empty_strided((B, 0), (0, 1), device="cuda", dtype=torch.int32)
    qf.module().topk(work, dev(fl), dev(members), dev(rt), dev(nt), dev(selected), dev(lens), dev(takes),
                     phys, logical, raw, 64, True, noexp, True, True, dev(ft), False)
    e = O.topk(scores, fl, members, rt, nt, selected, lens, takes, 64, True, T, 0, True, True, ft, False)
    assert np.array_equal(raw.cpu().numpy(), e["raw"])
    assert np.array_equal(logical.cpu().numpy(), e["logical"])
    assert np.array_equal(phys.cpu().numpy(), e["physical"])


def test_topk_argument_checks(cuda_dev):
    B, T = 2, 64
    z = lambda *s: torch.zeros(s, dtype=torch.int32, device="cuda")
    scores = torch.zeros((B, 128), device="cuda")
    noexp = torch.empty_strided((B, 0), (0, 1), device="cuda", dtype=torch.int32)
    args = [scores, z(B), z(4, 64), z(B, 8), z(B, 8), z(B, 2), z(B), z(B), z(B, T), z(B, T), z(B, T)]
    with pytest.raises(ValueError):   # window above 4096
        qf.module().topk(*args, 5000, True, noexp, True, True, z(B, 2), False)
    with pytest.raises(ValueError):   # expansion stride not 4*topk+64
        qf.module().topk(*args, 64, True, z(B, 10), True, True, z(B, 2), False)
    with pytest.raises(ValueError):   # direct fine table narrower than the take stride
        qf.module().topk(*args, 64, True, noexp, True, True, z(B, 1), True)
