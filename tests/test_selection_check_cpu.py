"""The row checker used at the benchmark configurations (oracle/selection_check.py),
tested on CPU: a step whose outputs come from the oracle itself passes with no
differences, and each planted mistake -- made in the oracle's outputs, on the
CPU -- is caught by the bar it breaks."""
import importlib
import types

import numpy as np
import pytest
import torch

import oracle as O
from oracle import selection_check as SC

synth = importlib.import_module("10_20_b200.synth")


def oracle_step(case):
    """A stand-in for SelectionStep whose buffers hold the oracle's results."""
    lens = case.lens.numpy()
    nt = case.native_table.numpy()
    rt = case.reordered_table.numpy()
    B, P, T, take_cfg = case.B, case.P, case.topk, case.take
    width = case.width
    fl, tk, dg, cl, tr = O.query_metadata(lens, nt, P, T, 1, 2, 64, case.window, budget=take_cfg)
    q8 = case.q8.view(torch.uint8).numpy()
    w = case.w.numpy()
    clog = O.score_paged(q8, w, case.centers.numpy(), case.center_table.numpy(), cl, P * 8, exact=False)
    for r in range(B):
        clog[r, int(cl[r]):] = -np.inf
    sel, _ = O.route(clog, lens, tk, take_cfg, P, rt, np.zeros((B, width // 64), np.int32), tr, case.capacity,
                     False)
    ft = O.fine_table_shared(rt, sel, tk, (B, width // 64), tr, case.capacity, P, take_cfg, 68)
    scores = np.full((B, width), -np.inf, np.float32)
    fine = case.fine.numpy()
    native = case.native.numpy()
    for r in range(B):
        n = int(lens[r])
        sink, tail = (int(x) for x in O.bounds(n, 64, case.window))
        ids = np.concatenate([np.arange(sink), np.arange(tail, n)])
        k_sel, s_sel = O.page_keys(fine, ft[r], int(tk[r]) * 64)
        k_nat, s_nat = O.page_keys(native, nt[r], n)
        keys = np.concatenate([k_sel, k_nat[ids]])
        sc = np.concatenate([s_sel, s_nat[ids]])
        if keys.shape[0]:
            scores[r, :keys.shape[0]] = O.score_row(q8[r], w[r], keys, sc, exact=False)
    e = O.topk(scores, fl, case.members.numpy(), rt, nt, sel, lens, tk, case.window, True, T, fine_table=ft)
    lat = case.latent.view(torch.int16).numpy()
    kg, _ = O.gather_slots(lat, None, None, e["physical"], B, T, 0)
    t = torch.from_numpy
    return types.SimpleNamespace(
        width=width, topk_cols=width, keep_logits=True, gather=True, fine_scores_kept=True,
        fine_lens=t(fl), takes=t(tk), dg_lens=t(dg), center_lens=t(cl), tail_rows=t(tr),
        center_logits=t(clog), selected=t(sel), fine_table=t(ft), scores=t(e["scores"]),
        physical=t(e["physical"]), logical=t(e["logical"]), raw=t(e["raw"]),
        kv=t(kg).view(torch.bfloat16).reshape(B, T, 1, -1))


@pytest.fixture(scope="module")
def small():
    case = synth.make_query_case(4, 4, [20000, 30000, 4097, 70], P=512, take=40, window=64, topk=2048, seed=5,
                                 device="cpu", latent_dim=64)
    return case, oracle_step(case)


def test_oracle_outputs_pass(small):
    case, step = small
    rep = SC.check_rows(step, case, range(case.B))
    assert rep["ok"], rep
    assert rep["route_pages_differing"] == 0 and rep["slots_differing_given_device_route"] == 0
    assert rep["slots_differing_end_to_end"] == 0


@pytest.mark.parametrize("mistake", ["physical", "selected", "metadata", "gather", "score"])
def test_planted_mistakes_are_caught(small, mistake):
    case, step = small
    s = types.SimpleNamespace(**vars(step))
    if mistake == "physical":
        s.physical = step.physical.clone()
        s.physical[1, 7] += 1
        key = "topk_exact_given_device_scores"
    elif mistake == "selected":
        s.selected = step.selected.clone()
        s.selected[0, [0, 1]] = s.selected[0, [1, 0]]
        key = "route_exact_given_device_scores"
    elif mistake == "metadata":
        s.takes = step.takes.clone()
        s.takes[3] += 1
        key = "metadata_exact"
    elif mistake == "gather":
        s.kv = step.kv.clone()
        s.kv[0, 5, 0, 3] += 1
        key = "gather_exact"
    else:
        s.scores = step.scores.clone()
        col = int(torch.nonzero(torch.isfinite(s.scores[1]))[0])
        s.scores[1, col] *= 1.5
        key = "fine_scores_within_tol"
    rep = SC.check_rows(s, case, range(case.B))
    assert rep[key] is False and rep["ok"] is False


def test_near_tie_flip_is_within_band(small):
    """A slot swapped across the selection threshold between two oracle scores
    that are equal within the tolerance counts as a difference inside the band;
    a swap with a far-below-threshold slot does not."""
    case, step = small
    r = 1
    lens = case.lens.numpy()
    sc = step.scores[r].numpy()
    raw = step.raw[r].numpy()
    phys = step.physical[r].numpy()
    chosen = set(raw[raw >= 0].tolist())
    L = int(step.fine_lens[r])
    fin = [c for c in range(L) if np.isfinite(sc[c])]
    thr = min(sc[c] for c in chosen if np.isfinite(sc[c]))
    out = sorted((c for c in fin if c not in chosen), key=lambda c: -sc[c])
    assert out and lens[r] > 2048

    def swap_to(col):
        s = types.SimpleNamespace(**vars(step))
        s.physical = step.physical.clone()
        worst = min((c for c in chosen if np.isfinite(sc[c])), key=lambda c: sc[c])
        t = int(np.nonzero(raw == worst)[0][0])
        nt = case.native_table.numpy()[r]
        sink, tail = (int(x) for x in O.bounds(int(lens[r]), 64, case.window))
        take = int(step.takes[r])
        if col < take * 64:
            page = int(case.reordered_table[r, int(step.selected[r, col // 64])])
            lg = int(case.members[page, col % 64])
        else:
            off = col - take * 64
            lg = off if off < sink else tail + off - sink
        s.physical[r, t] = int(nt[lg // 64]) * 64 + lg % 64
        s.fine_scores_kept = False          # check the slots by the oracle's scores alone
        return SC.check_rows(s, case, [r], latent_check=False)

    near = out[0]                            # the best unselected slot: just below the threshold
    rep = swap_to(near)
    assert rep["slots_differing_given_device_route"] == 1
    assert rep["slot_differences_within_band"] == bool(abs(sc[near] - thr) <= SC._band(sc[:L], thr))
    far = out[-1]                            # the worst finite slot
    rep = swap_to(far)
    assert rep["slots_differing_given_device_route"] == 1 and rep["slot_differences_within_band"] is False
    assert phys is not None
