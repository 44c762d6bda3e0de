"""The one-launch selection (v1x_select_fused: metadata + route + fine FP8
scoring + boundary mask + Top-T + mapping per row) against the operator
sequence it replaces (query_prepare -> scorer page maxima -> route_pages ->
fine scorer -> fused top-k, each oracle-tested on its own), bit-exact on every
output: the fine logits are computed by the same tensor-core instruction
sequence and summation order, so they -- and everything selected from them --
must agree exactly.  The sampled rows are also checked against the oracle."""
import importlib

import numpy as np
import pytest
import torch

from oracle import selection_check as SC

pytestmark = pytest.mark.gpu

synth = importlib.import_module("10_20_b200.synth")
pipeline = importlib.import_module("10_20_b200.pipeline")

OUTPUTS = ("fine_lens", "takes", "dg_lens", "center_lens", "tail_rows", "selected", "fine_table", "physical",
           "logical", "raw")


def _compare(fused, ref):
    for name in OUTPUTS:
        assert torch.equal(getattr(fused, name), getattr(ref, name)), name
    if fused.expanded.shape[1]:
        assert torch.equal(fused.expanded, ref.expanded)
    if fused.gather:
        assert torch.equal(fused.kv.view(torch.int16), ref.kv.view(torch.int16))
    if fused.fine_scores_kept:
        fl = ref.fine_lens.cpu().numpy()
        a, b = fused.scores.cpu().numpy(), ref.scores.cpu().numpy()
        for r in range(len(fl)):
            assert np.array_equal(a[r, :fl[r]], b[r, :fl[r]]), r


def _run_pair(case, **kw):
    fused = pipeline.SelectionStep(case, fused=True, **kw)
    ref = pipeline.SelectionStep(case, fused=False, **kw)
    assert fused.fused_select and not ref.fused_select
    ref.run()
    fused.run()
    torch.cuda.synchronize()
    assert int(fused.status.item()) == 0
    return fused, ref


@pytest.mark.parametrize("H,P,take,window,topk", [
    (64, 512, 12, 64, 2048),       # decode-like, short tables
    (64, 2048, 40, 64, 2048),      # the decode geometry
    (32, 192, 48, 64, 512),        # the Indexer test geometry
    (1, 128, 40, 64, 2048),        # the single-head geometry
    (64, 1024, 40, 2048, 2048),    # a wide window: many tail pages
    (64, 4096, 40, 0, 2048),       # the largest route table, no window
])
def test_fused_equals_operator_sequence(H, P, take, window, topk, cuda_dev):
    rng = np.random.default_rng(H * 7 + P)
    B = 24
    lens = [int(x) for x in rng.integers(1, P * 64 + 1, size=B)]
    lens[:6] = [1, 63, 64, 1025, 4097, P * 64]            # edges: no page, partial sink, no built page, ...
    case = synth.make_query_case(B, H, lens, P=P, take=take, window=window, topk=topk, seed=P + H, device="cuda",
                                 latent_dim=64)
    fused, ref = _run_pair(case, gather=True, keep_logits=True)
    _compare(fused, ref)
    rep = SC.check_rows(fused, case, [0, 3, 4, 5, 6, B - 1])
    assert rep["ok"], rep
    # the production form (no kept logits) gives the same outputs
    prod = pipeline.SelectionStep(case, gather=True)
    prod.run()
    torch.cuda.synchronize()
    for name in OUTPUTS:
        assert torch.equal(getattr(prod, name), getattr(ref, name)), name


def test_fused_ratio_rule_expansion_and_shared_tails(cuda_dev):
    """The ratio take rule, the x4 expansion, and rows that share row 0's tail
    (same length and native pages: tail_rows = 0, the fine table points at row
    0's staging pages)."""
    B, H, P = 16, 32, 256
    lens = [9000] * 4 + [int(x) for x in np.random.default_rng(3).integers(2000, P * 64, size=B - 4)]
    case = synth.make_query_case(B, H, lens, P=P, take=32, window=64, topk=512, seed=4, device="cuda")
    for r in (1, 2, 3):                                    # rows 1-3: row 0's pages and length
        case.native_table[r].copy_(case.native_table[0])
        case.reordered_table[r].copy_(case.reordered_table[0])
        case.center_table[r].copy_(case.center_table[0])
    fused, ref = _run_pair(case, gather=False, keep_logits=True, ratio=(1, 8), expand=True)
    _compare(fused, ref)
    assert fused.tail_rows[:4].tolist() == [0, 0, 0, 0]


def test_fused_graph_replay_and_budget_word(cuda_dev):
    """Captured in a CUDA graph; the budget is read on the device at every replay."""
    B, H, P = 8, 64, 512
    lens = synth.decode_lens(B, 8000, P * 64, 2)
    case = synth.make_query_case(B, H, lens, P=P, take=24, window=64, topk=2048, seed=2, device="cuda")
    step = pipeline.SelectionStep(case, gather=False)
    step.capture()
    step.replay()
    torch.cuda.synchronize()
    ref = pipeline.SelectionStep(case, gather=False, fused=False)
    ref.run()
    torch.cuda.synchronize()
    for name in OUTPUTS:
        assert torch.equal(getattr(step, name), getattr(ref, name)), name
    step.budget.fill_(10)
    ref.budget.fill_(10)
    step.replay()
    ref.run()
    torch.cuda.synchronize()
    assert int(step.takes.max()) == 10
    for name in OUTPUTS:
        assert torch.equal(getattr(step, name), getattr(ref, name)), name


def test_fused_rejects_bad_arguments(cuda_dev):
    """Host-side checks run before anything is launched (all pointers NULL)."""
    _lib = importlib.import_module("10_20_b200._lib")
    types = _lib.SIGNATURES["v1x_select_fused"]

    def args(**ints):   # NULL pointers, integer arguments by position
        a = [None if t is _lib.P else 0 for t in types]
        for i, v in ints.items():
            a[int(i[1:])] = v
        return a
    good = dict(a2=64, a5=1, a6=2, a9=2048, a11=2048, a13=1, a15=1, a17=1, a19=2048, a20=64, a21=40, a22=108,
                a37=1)
    for bad in (dict(a2=48), dict(a19=4096), dict(a20=8192), dict(a9=32), dict(a21=0), dict(a22=8)):
        with pytest.raises(ValueError):
            _lib.call("v1x_select_fused", *args(**{**good, **bad}))
