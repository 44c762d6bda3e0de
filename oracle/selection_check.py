"""Row-level parity check of a GPU selection step against the oracle.

TEST INFRASTRUCTURE ONLY: used by ``tests/`` and by ``bench.py``'s parity spot
check, never by the product.

``check_rows(step, case, rows)`` takes a ``SelectionStep`` that has run on a
``synth.QueryCase`` and compares sampled rows with the numpy restatement of the
reference's optimised query sequence (sglang/srt/layers/attention/v1_deepseek/
runtime.py:417-636 with the fixed budget of bench_v1_dynamic_budget_metadata.py:
5-28).  Only the pages a sampled row touches are copied to the host, so the
check runs at the benchmark's full sizes (a 131,072-token row reads ~30 MB).

Bars:
  * query metadata (fine_lens, takes, dg_lens, center_lens, tail_rows) of every
    row: exact (DS/kernels.py:568-591);
  * centre and fine logits: within 1e-2 relative of the fp64 restatement of the
    FP8 dequant math (DS/kernels.py:310-313) for every score of at least 1/10 of
    its row's largest |score|, within 1e-3 x that maximum below it (a score near
    zero is a cancelling sum: fp32 rounding is bounded by the terms' magnitudes,
    not by the result);
  * route (VQ:7-49), fine table (DS/kernels.py:488-514), Top-2048 raw / logical /
    physical (VQ:62-153) and gathered latent bytes (NA/kernels.py:62-77):
    bit-exact GIVEN THE DEVICE'S OWN SCORES (when the step kept them);
  * selection agreement: the route and the Top-2048 recomputed from the
    oracle's scores; every page or slot where they differ from the GPU's must
    sit within the score tolerance band of the oracle's selection threshold
    (a near-tie that the 1e-2 score bar allows to flip).  The counts of such
    differences are reported.
"""
from __future__ import annotations

import numpy as np

from . import v1x_oracle as O

RTOL = 1e-2
FLOOR = 1e-3


def _scores_close(got, exp):
    """Per-element score bar on finite entries (see the module docstring)."""
    fin = np.isfinite(exp)
    if not np.array_equal(np.isfinite(got), fin):
        return False
    if not fin.any():
        return True
    e, g = exp[fin].astype(np.float64), got[fin].astype(np.float64)
    bound = np.maximum(RTOL * np.abs(e), FLOOR * np.abs(e).max())
    return bool(np.all(np.abs(g - e) <= bound))


def _band(values, thr):
    """Tolerance band around a selection threshold, from the row's magnitudes."""
    fin = values[np.isfinite(values)]
    top = float(np.abs(fin).max()) if fin.size else 0.0
    return max(RTOL * abs(float(thr)), FLOOR * top)


def _pool_rows(pool, ids):
    """pool[ids] copied to the host (ids a 1-D int array of page ids)."""
    import torch

    if len(ids) == 0:
        return np.zeros((0, O.PAGE_BYTES), np.uint8)
    idx = torch.as_tensor(np.asarray(ids, np.int64), device=pool.device)
    return pool.index_select(0, idx).cpu().numpy()


def _decode_tokens(pages_u8, logical):
    """Keys f32 [L,128] and scales [L] of logical positions whose page p = l // 64
    is row p of pages_u8 (a row's pages in table order)."""
    logical = np.asarray(logical, np.int64)
    pg, sl = logical // 64, logical % 64
    kb = pages_u8[pg[:, None], sl[:, None] * 128 + np.arange(128)[None, :]]
    sc = pages_u8.view(np.float32).reshape(-1, O.PAGE_WORDS)[pg, O.SCALE_WORD + sl]
    return O.e4m3_to_f32(kb), sc.astype(np.float32)


def check_rows(step, case, rows, latent_check=True):
    """Compare sampled rows of a finished step with the oracle; returns a dict of
    figures and booleans (``ok`` = every bar met)."""
    import torch

    if case.lens.is_cuda:
        torch.cuda.synchronize(case.lens.device)
    B, P, T = case.B, case.P, case.topk
    take_cfg, window, cap = case.take, case.window, case.capacity
    lens = case.lens.cpu().numpy()
    nt_all = case.native_table.cpu().numpy()
    rep = dict(rows=[int(r) for r in rows])

    # ---- metadata of every row: exact ------------------------------------------------
    fl, tk, dg, cl, tr = O.query_metadata(lens, nt_all, P, T, 1, 2, 64, window, budget=take_cfg)
    meta_ok = True
    for name, exp in (("fine_lens", fl), ("takes", tk), ("dg_lens", dg), ("center_lens", cl),
                      ("tail_rows", tr)):
        t = getattr(step, name, None)
        if t is not None:
            meta_ok &= bool(np.array_equal(t.cpu().numpy(), exp))
    rep["metadata_exact"] = meta_ok

    members = case.members.cpu().numpy()
    width = step.width
    has_clog = getattr(step, "keep_logits", False) and getattr(step, "center_logits", None) is not None
    has_fine = getattr(step, "fine_scores_kept", True) and getattr(step, "scores", None) is not None
    ok = dict(centre=True, fine=True, route=True, table=True, topk=True, gather=True, route_band=True,
              slot_band=True)
    route_diff = slot_diff = e2e_diff = 0
    gathered = []
    for r in rows:
        r = int(r)
        n = int(lens[r])
        take = int(tk[r])
        nb = max(n - 1, 0) // 1024
        rt_r = case.reordered_table[r].cpu().numpy()
        ct_r = case.center_table[r].cpu().numpy()
        nt_r = nt_all[r]
        q8 = case.q8[r].view(torch.uint8).cpu().numpy()
        w = case.w[r].cpu().numpy()
        # ---- centre logits: oracle over the row's centre pages ----------------
        ncen = int(cl[r]) if nb > 0 else 0
        cpages = _pool_rows(case.centers, ct_r[:2 * nb])
        clog_o = np.full(P * 8, -np.inf, np.float32)
        if nb > 0:
            kc, sc = _decode_tokens(cpages, np.arange(ncen))
            clog_o[:ncen] = O.score_row(q8, w, kc, sc, exact=False)
        if has_clog:
            clog_d = step.center_logits[r].cpu().numpy()
            d = np.full(P * 8, -np.inf, np.float32)
            d[:ncen] = clog_d[:ncen]
            ok["centre"] &= _scores_close(d[:ncen], clog_o[:ncen])
            clog_for_route = d
        else:
            pm = step.page_scores[r].cpu().numpy()
            clog_for_route = np.repeat(pm[:P], 8).astype(np.float32)
        # ---- route given the device scores: exact --------------------------------
        z = np.zeros((1, width // 64), np.int32)
        sel_exp, _ = O.route(clog_for_route[None], lens[r:r + 1], tk[r:r + 1], take_cfg, P, rt_r[None], z,
                             tr[r:r + 1], cap, False)
        sel_d = step.selected[r].cpu().numpy()
        ok["route"] &= bool(np.array_equal(sel_d, sel_exp[0]))
        # ---- route agreement from the oracle's own logits -------------------------
        sel_o, _ = O.route(clog_o[None], lens[r:r + 1], tk[r:r + 1], take_cfg, P, rt_r[None], z, tr[r:r + 1], cap,
                           False)
        sel_o = sel_o[0]
        active = nb * 16
        if take < active:
            page_o = np.fmax.reduce(clog_o[:active * 8].reshape(active, 8), axis=1)
            a, b = set(sel_d[:take].tolist()), set(sel_o[:take].tolist())
            differ = sorted(a ^ b)
            route_diff += len(differ) // 2
            if differ:
                thr = page_o[sel_o[take - 1]]
                band = _band(page_o, thr)
                ok["route_band"] &= bool(all(abs(float(page_o[p]) - float(thr)) <= band for p in differ))
        # ---- fine table ------------------------------------------------------------
        ft_exp = O.fine_table_shared(rt_r[None], sel_d[None], tk[r:r + 1], (1, width // 64), tr[r:r + 1], cap, P,
                                     take_cfg, 68)
        ft_d = getattr(step, "fine_table", None)
        if ft_d is not None:
            ok["table"] &= bool(np.array_equal(ft_d[r].cpu().numpy(), ft_exp[0]))
        # ---- fine logits of the device's candidates: oracle -------------------------
        sink, tail = (int(x) for x in O.bounds(n, 64, window))
        tail_ids = np.concatenate([np.arange(sink), np.arange(tail, n)]).astype(np.int64)

        def fine_scores(sel):
            out = np.full(width, -np.inf, np.float32)
            if take + tail_ids.size == 0:
                return out
            fpages = _pool_rows(case.fine, rt_r[sel[:take]]) if take else np.zeros((0, O.PAGE_BYTES), np.uint8)
            ks, ss = _decode_tokens(fpages, np.arange(take * 64))
            npg = np.unique(tail_ids // 64)
            npages = _pool_rows(case.native, nt_r[npg])
            kt, st = _decode_tokens(npages, np.searchsorted(npg, tail_ids // 64) * 64 + tail_ids % 64)
            keys = np.concatenate([ks, kt])
            sc = np.concatenate([ss, st])
            out[:keys.shape[0]] = O.score_row(q8, w, keys, sc, exact=False)
            return out

        fine_o = fine_scores(sel_d)
        L = int(fl[r])
        cols = getattr(step, "topk_cols", width)
        if has_fine:
            fine_d = step.scores[r].cpu().numpy()
            # the step's top-k masks boundary members to -inf in place: compare
            # the unmasked oracle only where the device kept a finite score
            m = np.isfinite(fine_d[:L])
            ok["fine"] &= _scores_close(fine_d[:L][m], fine_o[:L][m])
            sd = np.full((1, cols), -np.inf, np.float32)
            sd[0, :min(L, cols)] = fine_d[:min(L, cols)]
            e = O.topk(sd, fl[r:r + 1], members, rt_r[None], nt_r[None], sel_d[None], lens[r:r + 1], tk[r:r + 1],
                       window, True, T, fine_table=ft_exp, direct_fine=False)
            for name in ("physical", "logical", "raw"):
                ok["topk"] &= bool(np.array_equal(getattr(step, name)[r].cpu().numpy(), e[name][0]))
        # ---- selection agreement from the oracle's scores ---------------------------
        so = np.full((1, cols), -np.inf, np.float32)
        so[0, :min(L, cols)] = fine_o[:min(L, cols)]
        eo = O.topk(so, fl[r:r + 1], members, rt_r[None], nt_r[None], sel_d[None], lens[r:r + 1], tk[r:r + 1],
                    window, True, T, fine_table=ft_exp, direct_fine=False)
        phys_d = step.physical[r].cpu().numpy()
        a = set(phys_d[phys_d >= 0].tolist())
        b = set(eo["physical"][0][eo["physical"][0] >= 0].tolist())
        differ = a ^ b
        slot_diff += len(a - b)
        if differ:
            masked = eo["scores"][0][:min(L, cols)]
            raw_o = eo["raw"][0]
            thr = masked[raw_o[raw_o >= 0]].min()
            band = _band(masked, thr)
            # the oracle's score of each differing slot: map physical -> raw column
            col_of = {}
            for col in range(min(L, cols)):
                if col < take * 64:
                    lg = int(members[int(rt_r[sel_d[col // 64]]), col % 64])
                else:
                    off = col - take * 64
                    lg = off if off < sink else tail + off - sink
                if 0 <= lg < n:
                    col_of[int(nt_r[lg // 64]) * 64 + lg % 64] = col
            ok["slot_band"] &= bool(all(p in col_of and abs(float(masked[col_of[p]]) - float(thr)) <= band
                                        for p in differ))
        # ---- end to end from the oracle's own route ----------------------------------
        if not np.array_equal(sel_o[:take], sel_d[:take]):
            ft_o = O.fine_table_shared(rt_r[None], sel_o[None], tk[r:r + 1], (1, width // 64), tr[r:r + 1], cap, P,
                                       take_cfg, 68)
            fo2 = fine_scores(sel_o)
            so2 = np.full((1, cols), -np.inf, np.float32)
            so2[0, :min(L, cols)] = fo2[:min(L, cols)]
            eo = O.topk(so2, fl[r:r + 1], members, rt_r[None], nt_r[None], sel_o[None], lens[r:r + 1],
                        tk[r:r + 1], window, True, T, fine_table=ft_o, direct_fine=False)
        b = set(eo["physical"][0][eo["physical"][0] >= 0].tolist())
        e2e_diff += len(a - b)
        gathered.append((r, phys_d))
    # ---- gathered latent bytes: exact -----------------------------------------------
    if latent_check and getattr(step, "gather", False) and case.latent is not None:
        D = case.latent.shape[-1]
        for r, phys in gathered:
            used = np.unique(phys[phys >= 0])
            pool = _pool_rows(case.latent.view(torch.int16).reshape(-1, D), used)
            ids = np.where(phys >= 0, np.searchsorted(used, phys), -1)
            exp_k, _ = O.gather_slots(pool[:, None, :], None, None, ids[None], 1, T, 0)
            got = step.kv[r].view(torch.int16).reshape(-1, D).cpu().numpy()
            ok["gather"] &= bool(np.array_equal(got, exp_k))
    rep.update({
        "centre_scores_within_tol": ok["centre"] if has_clog else None,
        "fine_scores_within_tol": ok["fine"] if has_fine else None,
        "route_exact_given_device_scores": ok["route"],
        "fine_table_exact": ok["table"],
        "topk_exact_given_device_scores": ok["topk"] if has_fine else None,
        "gather_exact": ok["gather"],
        "route_pages_differing": route_diff,
        "route_differences_within_band": ok["route_band"],
        "slots_differing_given_device_route": slot_diff,
        "slot_differences_within_band": ok["slot_band"],
        "slots_differing_end_to_end": e2e_diff,
        "slots_checked": len(rows) * T,
    })
    rep["ok"] = bool(meta_ok and all(ok.values()))
    return rep
