"""GPU parity: per-row query metadata, fine tables, shared tail staging, the
non-fused mask/mapping ops (DS/kernels.py) and _gather_slots (NA/kernels.py)."""
import importlib

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

K = importlib.import_module("10_20_b200.kernels")
G = importlib.import_module("10_20_b200.gather")


def dev(x):
    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def test_query_metadata_golden_and_budget(golden, cuda_dev):
    g = golden("tail_meta")
    lens, nt = dev(g["m_lens"]), dev(g["m_nt"])
    B = lens.shape[0]
    for window in (64, 2048):
        outs = [torch.empty(B, dtype=torch.int32, device="cuda") for _ in range(5)]
        K.query_metadata[(B,)](lens, nt, *outs, 96, 2048, 1, 2, 64, window)
        assert np.array_equal(torch.stack(outs).cpu().numpy(), g[f"m_out{window}"])
        budget = torch.tensor([40], dtype=torch.int32, device="cuda")
        K.BudgetMetadata(budget)[(B,)](lens, nt, *outs, 96, 2048, 1, 2, 64, window)
        exp = O.query_metadata(g["m_lens"], g["m_nt"], 96, 2048, 1, 2, 64, window, budget=40)
        assert np.array_equal(torch.stack(outs).cpu().numpy(), np.stack(exp))
    fl = torch.empty(B, dtype=torch.int32, device="cuda")
    tk = torch.empty(B, dtype=torch.int32, device="cuda")
    K.query_lengths[(B,)](lens, fl, tk, 40, 2048, 1, 2, 64, 64)
    efl, etk = O.query_lengths(g["m_lens"], 2048, 1, 2, 64, 64)
    assert np.array_equal(fl.cpu().numpy(), efl) and np.array_equal(tk.cpu().numpy(), etk)


def test_stage_tail_shared_golden(golden, cuda_dev):
    g = golden("tail_meta")
    out = torch.full((1 + 4 * 3, 8448), 255, dtype=torch.uint8, device="cuda")
    nat = dev(g["t_native"])
    K.stage_tail_shared[(1, 3)](nat.view(torch.float8_e4m3fn), nat.view(torch.float32), dev(g["t_nt"]),
                                dev(g["t_lens"]), out.view(torch.float8_e4m3fn), out.view(torch.float32),
                                dev(g["t_owners"]), 1, 18, 3, 64, 64, ROWS=4, GROUP=4, num_warps=4)
    assert np.array_equal(out.cpu().numpy(), g["t_out"])
    B = g["s_lens"].shape[0]
    nat = dev(g["s_native"])
    for window in (64, 2048):
        out = torch.full((5 + B * 68, 8448), 255, dtype=torch.uint8, device="cuda")
        K.stage_tail_shared[((B + 31) // 32, 68)](nat, nat.view(torch.float32), dev(g["s_nt"]),
                                                  dev(g["s_lens"]), out, out.view(torch.float32),
                                                  dev(g["s_owners"]), 5, 40, 68, 64, window, ROWS=B,
                                                  GROUP=32)
        assert np.array_equal(out.cpu().numpy(), g[f"s_out{window}"])


def test_fine_table_shared_golden(golden, cuda_dev):
    g = golden("tail_meta")
    ft = torch.empty((4, 3), dtype=torch.int32, device="cuda")
    z = torch.zeros((4, 18), dtype=torch.int32, device="cuda")
    K.fine_table_shared[(4,)](z, torch.zeros((4, 1), dtype=torch.int32, device="cuda"),
                              torch.zeros(4, dtype=torch.int32, device="cuda"), dev(g["t_lens"]), ft,
                              dev(g["t_owners"]), 1, 18, 1, 3, 3, 4)
    assert ft.tolist() == [[1, 2, 3], [1, 2, 3], [7, 8, 9], [7, 8, 9]]
    ft = torch.empty((6, 20), dtype=torch.int32, device="cuda")
    for sel in (dev(g["f_sel"]), dev(g["f_sel"]).long()):
        K.fine_table_shared[(6,)](dev(g["f_rt"]), sel, dev(g["f_takes"]), dev(g["f_takes"]), ft,
                                  dev(g["f_trows"]), 777, 64, 12, 20, 68, 32)
        assert np.array_equal(ft.cpu().numpy(), g["f_ft"])


def test_mask_output_reduce_expand_golden(golden, cuda_dev):
    g = golden("select_maps")
    B, MAXP, NP, TAKE, TOPK, WIDTH = 5, 96, 96, 8, 256, 768
    s = dev(g["scores"])
    K.mask_fine[(B, 3)](s, dev(g["selected"]), dev(g["rt"]), dev(g["members"]), dev(g["lens"]),
                        dev(g["takes"]), MAXP, TAKE, WIDTH, WIDTH, 64, 64)
    assert np.array_equal(s.cpu().numpy(), g["masked"])
    out = torch.empty((B, TOPK), dtype=torch.int32, device="cuda")
    logical = torch.empty_like(out)
    K.output_ids[(B, 1)](dev(g["raw"]), dev(g["masked"]), dev(g["members"]), dev(g["rt"]), dev(g["nt"]),
                         dev(g["selected"]), dev(g["lens"]), dev(g["takes"]), out, logical, dev(g["rt"]),
                         MAXP, NP, TAKE, WIDTH, TOPK, 64, 64)
    assert np.array_equal(out.cpu().numpy(), g["out"])
    assert np.array_equal(logical.cpu().numpy(), g["logical"])
    coarse = torch.empty((B, MAXP), device="cuda")
    K.reduce_centers[(B, 3)](dev(g["logits"]), dev(g["lens"]), coarse, MAXP, g["logits"].shape[1])
    assert np.array_equal(coarse.cpu().numpy(), g["coarse"])
    exp = torch.empty((B, TOPK * 4 + 64), dtype=torch.int32, device="cuda")
    K.expand_logical[(B,)](dev(g["logical"]), exp, TOPK, TOPK * 4 + 64, 2048)
    assert np.array_equal(exp.cpu().numpy(), g["expanded"])


def test_gather_golden(golden, cuda_dev):
    g = golden("gather")
    k = dev(g["k"]).view(torch.bfloat16).reshape(8, 2, 128)
    v = dev(g["v"]).view(torch.bfloat16).reshape(8, 2, 128)
    kp = torch.empty((8, 2, 256), dtype=torch.bfloat16, device="cuda")[:, :, ::2]
    kp.copy_(k)
    vp = torch.empty((8, 4, 128), dtype=torch.bfloat16, device="cuda")[:, ::2, :]
    vp.copy_(v)
    before = kp.clone(), vp.clone()
    backing = torch.tensor([[0, 2, -1, 99], [4, 1, 4, 99]], dtype=torch.int32, device="cuda")
    ids = backing[:, :3]
    for head in (0, 1):
        ok = torch.empty((2, 3, 1, 128), dtype=torch.bfloat16, device="cuda")
        ov = torch.empty_like(ok)
        G._gather_slots[(1,)](kp, vp, dev(g["req"]), ids, ok, ov, 2, 3, head, *kp.stride(), *vp.stride(),
                              ids.stride(0), 32, num_warps=4)
        assert np.array_equal(ok.view(torch.int16).cpu().numpy(), g[f"small_k{head}"])
        assert np.array_equal(ov.view(torch.int16).cpu().numpy(), g[f"small_v{head}"])
    assert torch.equal(kp, before[0]) and torch.equal(vp, before[1])
    kpool = dev(g["kpool"]).view(torch.bfloat16)
    vpool = dev(g["vpool"]).view(torch.bfloat16)
    ids2 = dev(g["ids2"])[:, :96]
    ok = torch.empty((2, 96, 1, 128), dtype=torch.bfloat16, device="cuda")
    ov = torch.empty_like(ok)
    G._gather_slots[(6,)](kpool, vpool, dev(g["req2"]), ids2, ok, ov, 2, 96, 2, *kpool.stride(),
                          *vpool.stride(), ids2.stride(0), 32)
    assert np.array_equal(ok.view(torch.int16).cpu().numpy(), g["rand_k"])
    assert np.array_equal(ov.view(torch.int16).cpu().numpy(), g["rand_v"])


def test_gather_workspace_reuse(cuda_dev):
    x = torch.arange(8 * 2 * 128, dtype=torch.float32, device="cuda").reshape(8, 2, 128)
    k, v = x.to(torch.bfloat16), (-x - 16).to(torch.bfloat16)
    req = torch.tensor([5, 1, 7, 0, 6, 2], dtype=torch.int32, device="cuda")
    ids = (torch.arange(4096, device="cuda") % 6).to(torch.int32).reshape(2, 2048)
    work = G.GatherWorkspace(2, "cuda:0", torch.bfloat16)
    a, b = work.gather(k, v, req, ids, 0)
    ea, eb = O.gather_slots(k.view(torch.int16).cpu().numpy(), v.view(torch.int16).cpu().numpy(),
                            req.cpu().numpy(), ids.cpu().numpy(), 2, 2048, 0)
    assert np.array_equal(a.view(torch.int16).reshape(-1, 128).cpu().numpy(), ea)
    assert np.array_equal(b.view(torch.int16).reshape(-1, 128).cpu().numpy(), eb)
    addr = (a.data_ptr(), b.data_ptr())
    changed = ids.flip(1).contiguous()
    a, b = work.gather(k, v, req, changed, 1)
    assert addr == (a.data_ptr(), b.data_ptr())
    ea, eb = O.gather_slots(k.view(torch.int16).cpu().numpy(), v.view(torch.int16).cpu().numpy(),
                            req.cpu().numpy(), changed.cpu().numpy(), 2, 2048, 1)
    assert np.array_equal(a.view(torch.int16).reshape(-1, 128).cpu().numpy(), ea)
    with pytest.raises(ValueError):
        work.gather(k, v, req, torch.zeros((3, 2048), dtype=torch.int32, device="cuda"), 0)
    work.clear()
    assert work.k is None and work.v is None


@pytest.mark.parametrize("D,strided", [(576, False), (128, True), (64, False), (100, False)])
def test_gather_latent_random(D, strided, cuda_dev):
    """MLA latent D=576 (extension), strided pools (scalar path) and odd D."""
    rng = np.random.default_rng(D)
    slots, rows, top = 5000, 3, 2048
    pool = torch.randn((slots, 2, D * (2 if strided else 1)), dtype=torch.bfloat16, device="cuda")
    kp = pool[:, :, ::2] if strided else pool
    ids = torch.as_tensor(rng.integers(-1, slots, size=(rows, top)).astype(np.int32)).cuda()
    ws = G.GatherWorkspace(rows, "cuda:0", torch.bfloat16, dim=D)
    for call in range(4):   # the workspace is reused for 4 back-to-back calls
        idc = ids.roll(call * 17, 1).contiguous()
        out = ws.gather(kp, None, None, idc, 1)
        e, _ = O.gather_slots(kp.contiguous().view(torch.int16).cpu().numpy(), None, None,
                              idc.cpu().numpy(), rows, top, 1)
        assert np.array_equal(out.view(torch.int16).reshape(-1, D).cpu().numpy(), e)


def test_query_prepare_equals_metadata_then_staging(cuda_dev):
    """The fused metadata + staging launch == query_metadata + stage_tail_shared."""
    synth = importlib.import_module("10_20_b200.synth")
    rng = np.random.default_rng(17)
    B, P = 9, 256
    lens = rng.integers(100, P * 64, size=B).tolist()
    lens[1] = lens[0]
    lens[2], lens[3] = 0, 40
    case = synth.make_query_case(B, 4, lens, P=P, take=8, window=64, topk=512, seed=3, device="cuda")
    case.native_table[1] = case.native_table[0]      # row 1 shares row 0's tail pages
    budget = torch.tensor([8], dtype=torch.int32, device="cuda")
    outs = []
    for fused in (False, True):
        meta = [torch.full((B,), -7, dtype=torch.int32, device="cuda") for _ in range(5)]
        fine = case.fine.clone()
        fine[case.capacity:] = 255
        if fused:
            K.query_prepare(case.lens, case.native_table, *meta, P, 512, 1, 2, 64, 64, case.native,
                            case.native.view(torch.float32), fine, fine.view(torch.float32), case.capacity, 68,
                            budget=budget)
        else:
            K.BudgetMetadata(budget)[(B,)](case.lens, case.native_table, *meta, P, 512, 1, 2, 64, 64)
            K.stage_tail_shared[(B, 68)](case.native, case.native.view(torch.float32), case.native_table,
                                         case.lens, fine, fine.view(torch.float32), meta[4], case.capacity,
                                         P, 68, 64, 64, ROWS=B, GROUP=1)
        outs.append((torch.stack(meta).cpu().numpy(), fine[case.capacity:].cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert outs[0][0][4][1] == 0                       # the shared row points at row 0
    assert np.array_equal(outs[0][1], outs[1][1])


def test_gather_latent_bulk_path_edges(cuda_dev):
    """The single-output 576-wide path: a slot map (REQ), strided id rows, a
    last row group of fewer than four rows, and negative ids."""
    rng = np.random.default_rng(23)
    slots, rows, top = 3000, 5, 1027
    pool = torch.randn((slots, 1, 576), dtype=torch.bfloat16, device="cuda")
    req = torch.as_tensor(rng.permutation(slots).astype(np.int32)).cuda()
    ids_full = torch.as_tensor(rng.integers(-1, slots, size=(rows, top + 5)).astype(np.int32)).cuda()
    ids = ids_full[:, :top]                      # row stride top + 5
    out = torch.full((rows, top, 1, 576), 7.0, dtype=torch.bfloat16, device="cuda")
    G._gather_impl((1,), pool, None, req, ids, out, None, rows, top, 0, *pool.stride(), IS0=ids_full.stride(0))
    torch.cuda.synchronize()
    e, _ = O.gather_slots(pool.view(torch.int16).cpu().numpy(), None, req.cpu().numpy(),
                          ids.contiguous().cpu().numpy(), rows, top, 0)
    assert np.array_equal(out.view(torch.int16).reshape(-1, 576).cpu().numpy(), e)
