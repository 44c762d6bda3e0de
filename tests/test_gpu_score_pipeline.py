"""GPU parity: FP8 paged scoring (DeepGEMM fp8_paged_mqa_logits contract) and
the composed selection step vs the oracle.

Tolerances: the few-head SIMT scorer follows the oracle's fixed fp32 order and
must match it exactly; the tensor-core scorer (many heads) must be within
rtol = 1e-2 of the fp64 reference math (the north-star score tolerance) for
every score of at least 1/10 of its row's largest |score|, and within
1e-3 x that largest |score| below it.  Why the floor: a score near zero is a
sum whose head terms cancel (w_h * relu(q_h . k) with q_h . k itself a signed
128-term sum), and the rounding error of any fp32 summation order is bounded by
eps x the sum of the terms' magnitudes, not by |result|; the reference's own
DeepGEMM and Triton restatement sum in different orders and differ there too.
Every score of at least 1/10 of the row maximum meets the pure relative bar.
Selection parity is bit-exact given the device scores; how often the score
tolerance changes the selected set is measured separately (selection
agreement, test_gpu_full_configs.py).
"""
import importlib

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

S = importlib.import_module("10_20_b200.scoring")
synth = importlib.import_module("10_20_b200.synth")
pipeline = importlib.import_module("10_20_b200.pipeline")

RTOL = 1e-2


def dev(x):
    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def close(got, exp):
    fin = np.isfinite(exp)
    assert np.array_equal(np.isfinite(got), fin)
    for r in range(exp.shape[0]):
        e, g = exp[r][fin[r]], got[r][fin[r]]
        if e.size == 0:
            continue
        # 1e-2 relative, with the floor 1e-3 x row max only below 1/10 of it
        bound = np.maximum(RTOL * np.abs(e), 1e-3 * np.abs(e).max())
        assert np.all(np.abs(g - e) <= bound), r


def test_score_golden_formula(golden, cuda_dev):
    """Centre logits: the reference coarse kernel's page maxima (H=16)."""
    g = golden("scores")
    B, H, MAXP = 2, 16, 64
    lens = torch.as_tensor([(int(n) - 1) // 1024 * 128 for n in g["lens"]], dtype=torch.int32).cuda()
    out = S.fp8_paged_mqa_logits(dev(g["q"]).view(torch.float8_e4m3fn), dev(g["centers"]), dev(g["w"]),
                                 lens, dev(g["ctable"]), None, MAXP * 8)
    pm = out.view(B, MAXP, 8).amax(-1).cpu().numpy()
    np.testing.assert_allclose(pm, g["coarse"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("H", [1, 2, 16, 32, 64])
def test_score_simt_exact_vs_oracle(H, cuda_dev):
    rng = np.random.default_rng(H)
    B, NP = 3, 40
    pool = np.zeros((NP, 8448), np.uint8)
    kb = torch.randn((NP, 64, 128), generator=torch.Generator().manual_seed(H)).to(torch.float8_e4m3fn)
    pool[:, :8192] = kb.view(torch.uint8).reshape(NP, 8192).numpy()
    pool.view(np.float32)[:, 2048:] = rng.random((NP, 64)).astype(np.float32) + 0.1
    q = torch.randn((B, H, 128), generator=torch.Generator().manual_seed(7 + H)).to(torch.float8_e4m3fn)
    q8 = q.view(torch.uint8).numpy()
    w = rng.random((B, H)).astype(np.float32)
    table = np.stack([rng.permutation(NP)[:20] for _ in range(B)]).astype(np.int32)
    lens = np.array([1280, 1, 700], np.int32)
    out = S.fp8_paged_mqa_logits(q.cuda(), dev(pool), dev(w), dev(lens), dev(table), None, 1300,
                                 impl="simt").cpu().numpy()
    exp = O.score_paged(q8, w, pool, table, lens, 1300, exact=True)
    assert np.array_equal(out, exp), np.abs(out - exp).max()
    close(out, O.score_paged(q8, w, pool, table, lens, 1300, exact=False))


def test_score_auto_single_head_beyond_tensor_core_rows(cuda_dev):
    """Automatic dispatch takes the tensor cores for one head only up to 8192
    rows; a larger batch runs on the SIMT scorer (bit-identical to impl="simt"
    and to the oracle's exact mode) instead of failing."""
    rng = np.random.default_rng(5)
    B, NP = 8193, 12
    pool = np.zeros((NP, 8448), np.uint8)
    kb = torch.randn((NP, 64, 128), generator=torch.Generator().manual_seed(5)).to(torch.float8_e4m3fn)
    pool[:, :8192] = kb.view(torch.uint8).reshape(NP, 8192).numpy()
    pool.view(np.float32)[:, 2048:] = rng.random((NP, 64)).astype(np.float32) + 0.1
    q = torch.randn((B, 1, 128), generator=torch.Generator().manual_seed(6)).to(torch.float8_e4m3fn)
    w = rng.random((B, 1)).astype(np.float32)
    table = rng.integers(0, NP, size=(B, 2)).astype(np.int32)
    lens = rng.integers(0, 129, size=B).astype(np.int32)
    args = (q.cuda(), dev(pool), dev(w), dev(lens), dev(table), None, 128)
    auto = S.fp8_paged_mqa_logits(*args).cpu().numpy()
    simt = S.fp8_paged_mqa_logits(*args, impl="simt").cpu().numpy()
    assert np.array_equal(auto, simt)
    rows = [0, 1, 4096, 8191, 8192]
    exp = O.score_paged(q.view(torch.uint8).numpy()[rows], w[rows], pool, table[rows], lens[rows], 128, exact=True)
    assert np.array_equal(auto[rows], exp)


def test_score_tensor_core_rejects_unsupported_heads(cuda_dev):
    q = torch.zeros((2, 256, 128), dtype=torch.float8_e4m3fn, device="cuda")
    pool = torch.zeros((4, 8448), dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception):
        S.fp8_paged_mqa_logits(q, pool, torch.zeros((2, 256), device="cuda"),
                               torch.ones(2, dtype=torch.int32, device="cuda"),
                               torch.zeros((2, 1), dtype=torch.int32, device="cuda"), None, 64,
                               impl="tensor_core")


@pytest.mark.parametrize("H", [1, 32, 64, 96, 128])
@pytest.mark.parametrize("relu", [True, False])
def test_score_tensor_core_vs_oracle(H, relu, cuda_dev):
    """tcgen05 scorer: ragged rows (empty, one key, partial tiles, longer than
    max_len), many rows over many CTAs, non-multiple-of-128 max_len."""
    rng = np.random.default_rng(H + relu)
    B, NP = 70, 300
    pool = np.zeros((NP, 8448), np.uint8)
    kb = torch.randn((NP, 64, 128), generator=torch.Generator().manual_seed(H)).to(torch.float8_e4m3fn)
    pool[:, :8192] = kb.view(torch.uint8).reshape(NP, 8192).numpy()
    pool.view(np.float32)[:, 2048:] = rng.random((NP, 64)).astype(np.float32) + 0.1
    q = torch.randn((B, H, 128), generator=torch.Generator().manual_seed(9 + H)).to(torch.float8_e4m3fn)
    q8 = q.view(torch.uint8).numpy()
    w = rng.random((B, H)).astype(np.float32)
    table = np.stack([rng.permutation(NP)[:40] for _ in range(B)]).astype(np.int32)
    lens = rng.integers(0, 2600, size=B).astype(np.int32)
    lens[:6] = [0, 1, 127, 128, 129, 2560]
    max_len = 2500
    out = torch.full((B, 2600), 7.0, device="cuda")
    S.fp8_paged_mqa_logits(q.cuda(), dev(pool), dev(w), dev(lens), dev(table), None, max_len,
                           relu=relu, out=out, impl="tensor_core")
    got = out.cpu().numpy()
    exp = O.score_paged(q8, w, pool, table, np.minimum(lens, max_len), max_len, relu=relu, exact=False)
    if relu:
        close(got[:, :max_len], exp)
    else:   # signed scores: absolute tolerance relative to the row scale
        fin = np.isfinite(exp)
        assert np.array_equal(np.isfinite(got[:, :max_len]), fin)
        for r in range(B):
            if fin[r].any():
                e = exp[r][fin[r]]
                assert np.abs(got[r, :max_len][fin[r]] - e).max() <= 1e-2 * np.abs(e).max()
    assert (got[:, max_len:] == 7.0).all()          # columns past max_len untouched
    # clean_logits=False leaves the padding alone
    out.fill_(7.0)
    S.fp8_paged_mqa_logits(q.cuda(), dev(pool), dev(w), dev(lens), dev(table), None, max_len,
                           relu=relu, out=out, impl="tensor_core", clean_logits=False)
    got2 = out.cpu().numpy()
    for r in range(B):
        n = min(int(lens[r]), max_len)
        assert (got2[r, n:] == 7.0).all()
        assert np.array_equal(got2[r, :n], got[r, :n])


def _small_case(B=24, H=64, seed=5, latent=576):
    lens = synth.decode_lens(B, 2048, 20000, seed)
    lens[0] = 4097
    lens[1] = 3073
    return synth.make_query_case(B, H, lens, P=512, take=12, window=64, topk=2048, seed=seed,
                                 device="cuda", latent_dim=latent)


def test_selection_step_end_to_end(cuda_dev):
    """Every stage of the operator sequence vs the oracle: metadata exact,
    centre/fine scores within tolerance, route/top-k/gather bit-exact given the
    device scores.  (The one-launch selection is compared with this sequence in
    test_gpu_select_fused.py.)"""
    case = _small_case()
    step = pipeline.SelectionStep(case, gather=True, keep_logits=True, fused=False)
    step.run()
    torch.cuda.synchronize()
    c = case
    lens = c.lens.cpu().numpy()
    nt = c.native_table.cpu().numpy()
    fl, tk, dg, cl, tr = O.query_metadata(lens, nt, c.P, 2048, 1, 2, 64, c.window, budget=c.take)
    assert np.array_equal(step.fine_lens.cpu().numpy(), fl)
    assert np.array_equal(step.takes.cpu().numpy(), tk)
    assert np.array_equal(step.tail_rows.cpu().numpy(), tr)
    q8 = c.q8.view(torch.uint8).cpu().numpy()
    w = c.w.cpu().numpy()
    centers = c.centers.cpu().numpy()
    ctab = c.center_table.cpu().numpy()
    clog = step.center_logits.cpu().numpy()
    ccols = np.arange(clog.shape[1])[None, :]
    clog = np.where(ccols < cl[:, None], clog, -np.inf).astype(np.float32)  # unwritten past center_lens
    close(clog, O.score_paged(q8, w, centers, ctab, cl, c.P * 8, exact=False))
    rt = c.reordered_table.cpu().numpy()
    sel, ft = O.route(clog, lens, tk, c.take, c.P, rt, np.zeros((c.B, step.width // 64), np.int32), tr,
                      c.capacity, False)
    assert np.array_equal(step.selected.cpu().numpy(), sel)
    ft = O.fine_table_shared(rt, sel, tk, (c.B, step.width // 64), tr, c.capacity, c.P, c.take, 68)
    assert np.array_equal(step.fine_table.cpu().numpy(), ft)
    fine_pool = c.fine.cpu().numpy()
    fine_exp = O.score_paged(q8, w, fine_pool, ft, dg, step.width, exact=False)
    got_scores = step.scores.cpu().numpy()   # masked in place by the top-k
    cols = np.arange(got_scores.shape[1])[None, :]
    got_scores = np.where(cols < fl[:, None], got_scores, -np.inf).astype(np.float32)  # past fine_lens: unwritten
    members = c.members.cpu().numpy()
    e = O.topk(got_scores, fl, members, rt, nt, sel, lens, tk, c.window, True, 2048,
               fine_table=ft, direct_fine=False)
    assert np.array_equal(e["scores"], got_scores)          # mask is idempotent
    assert np.array_equal(step.raw.cpu().numpy(), e["raw"])
    assert np.array_equal(step.logical.cpu().numpy(), e["logical"])
    assert np.array_equal(step.physical.cpu().numpy(), e["physical"])
    fin = np.isfinite(got_scores)
    close(np.where(fin, got_scores, -np.inf), np.where(fin, fine_exp, -np.inf))
    # page maxima from the scoring epilogue == max of the centre logits of each page
    pm = step.page_scores.cpu().numpy()
    for r in range(c.B):
        np_ = int(cl[r]) // 8
        assert np.array_equal(pm[r, :np_], clog[r, :np_ * 8].reshape(np_, 8).max(1))
    lat = c.latent.view(torch.int16).cpu().numpy()
    kg, _ = O.gather_slots(lat, None, None, step.physical.cpu().numpy(), c.B, 2048, 0)
    assert np.array_equal(step.kv.view(torch.int16).reshape(-1, lat.shape[-1]).cpu().numpy(), kg)


def test_selection_step_graph_replay(cuda_dev):
    case = _small_case(B=8, seed=9, latent=0)
    step = pipeline.SelectionStep(case, gather=False)
    step.run()
    ref = step.physical.clone()
    step.capture()
    step.physical.fill_(-3)
    step.replay()
    torch.cuda.synchronize()
    assert torch.equal(step.physical, ref)


@pytest.mark.parametrize("ctas", [1, 16, 37])
def test_selection_step_score_ctas_cap(ctas, cuda_dev):
    """A capped centre-scorer grid (each CTA takes a longer tile range) gives the
    same selection as the default grid."""
    case = _small_case(B=8, seed=13, latent=0)
    ref = pipeline.SelectionStep(case, gather=False, keep_logits=True)
    ref.run()
    step = pipeline.SelectionStep(case, gather=False, keep_logits=True, score_ctas=ctas)
    step.run()
    torch.cuda.synchronize()
    assert torch.equal(step.page_scores, ref.page_scores)
    assert torch.equal(step.physical, ref.physical) and torch.equal(step.logical, ref.logical)


@pytest.mark.parametrize("impl,H", [("simt", 1), ("simt", 16), ("tensor_core", 1), ("tensor_core", 64)])
def test_page_max_and_route_pages(impl, H, cuda_dev):
    """Scoring page maxima + route_pages == route over the centre logits (bit-exact)."""
    rng = np.random.default_rng(H)
    B, P, NP = 33, 256, 400
    pool = np.zeros((NP, 8448), np.uint8)
    kb = torch.randn((NP, 64, 128), generator=torch.Generator().manual_seed(1)).to(torch.float8_e4m3fn)
    pool[:, :8192] = kb.view(torch.uint8).reshape(NP, 8192).numpy()
    pool.view(np.float32)[:, 2048:] = rng.random((NP, 64)).astype(np.float32) + 0.1
    q = torch.randn((B, H, 128), generator=torch.Generator().manual_seed(2)).to(torch.float8_e4m3fn).cuda()
    w = dev(rng.random((B, H)).astype(np.float32))
    ctable = dev(rng.integers(0, NP, size=(B, P // 8)).astype(np.int32))
    lens = rng.integers(1, P * 64, size=B).astype(np.int32)
    lens[:3] = [1, 1025, P * 64]
    clen = dev(np.maximum((np.maximum(lens - 1, 0) // 1024) * 128, 1).astype(np.int32))
    logits = torch.empty((B, P * 8), device="cuda")
    pm = torch.full((B, P), 5.0, device="cuda")
    S.fp8_paged_mqa_logits(q, dev(pool), w, clen, ctable, None, P * 8, out=logits, page_max=pm, impl=impl)
    lg = logits.cpu().numpy()
    pmn = pm.cpu().numpy()
    assert np.array_equal(pmn, lg.reshape(B, P, 8).max(2))
    # lens_kind="centres" on the token lengths == the derived centre lengths
    logits2 = torch.empty_like(logits)
    pm2 = torch.full_like(pm, 5.0)
    S.fp8_paged_mqa_logits(q, dev(pool), w, dev(lens), ctable, None, P * 8, out=logits2, page_max=pm2,
                           impl=impl, lens_kind="centres")
    assert torch.equal(logits, logits2) and torch.equal(pm, pm2)
    qf = importlib.import_module("10_20_b200.query_fused")
    takes = dev(rng.integers(0, 40, size=B).astype(np.int32))
    rt = dev(rng.integers(0, 10000, size=(B, P)).astype(np.int32))
    trows = dev(rng.integers(0, B, size=B).astype(np.int32))
    sel_a = torch.empty((B, 40), dtype=torch.int32, device="cuda")
    sel_b = torch.empty_like(sel_a)
    ft_a = torch.full((B, 40 + 68), -3, dtype=torch.int32, device="cuda")
    ft_b = ft_a.clone()
    qf.module().route(logits, dev(lens), takes, sel_a, P, rt, ft_a, trows, 77, True)
    qf.module().route_pages(pm, dev(lens), takes, sel_b, P, rt, ft_b, trows, 77, True)
    assert torch.equal(sel_a, sel_b) and torch.equal(ft_a, ft_b)
