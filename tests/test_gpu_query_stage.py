"""v1x_query_stage: the one-launch row staging of a query bucket (the copies of
the reference's Query.run, DS/runtime.py:643-666), against the same copies made
with torch ops -- live rows, zeroed padding rows, narrow native tables,
unaligned views, more rows than one launch carries, and rejected row ids."""
import importlib
from array import array

import pytest
import torch

pytestmark = pytest.mark.gpu

_lib = importlib.import_module("10_20_b200._lib")


def _stage(q, w, lens, nt, rows, st, sc, outs, heads, pages, filled):
    ids = array("i", rows)
    _lib.call("v1x_query_stage", q.data_ptr(), w.data_ptr(), lens.data_ptr(), nt.data_ptr(), nt.shape[1],
              ids.buffer_info()[0], st.data_ptr(), sc.data_ptr(), st.shape[0], *[o.data_ptr() for o in outs],
              heads, pages, q.shape[0], filled, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("cap,n,filled,width,offset", [
    (16, 12, 0, 192, 0),        # full-width tables
    (16, 5, 12, 77, 0),         # a shorter call after a longer one; odd width (4-byte path)
    (600, 533, 600, 192, 1),    # three launches of row ids; inputs at odd element offsets
    (4, 0, 3, 192, 0),          # nothing live: every row zeroed
])
def test_query_stage_matches_torch_copies(cap, n, filled, width, offset, cuda_dev):
    torch.manual_seed(cap + n)
    H, P, R = 32, 192, 40
    g = lambda *s: torch.randint(-2**31, 2**31 - 1, s, dtype=torch.int32, device="cuda")
    # inputs as views at an element offset into larger buffers
    qbase = torch.randint(0, 256, (n * H * 128 + offset,), dtype=torch.uint8, device="cuda")
    q = qbase[offset:].view(n, H, 128)
    w = torch.randn(n * H + offset, device="cuda")[offset:].view(n, H)
    lens = g(n + offset)[offset:]
    nt = g(n * width + offset)[offset:].view(n, width)
    st, sc = g(R, P), g(R, P // 8)
    rows = [int(x) for x in torch.randint(0, R, (n,))]
    outs = [torch.randint(0, 256, (cap, H * 128), dtype=torch.uint8, device="cuda"), torch.randn(cap, H, device="cuda"),
            g(cap), g(cap, P), g(cap, P), g(cap, P // 8)]
    before = [o.clone() for o in outs]
    _stage(q, w, lens, nt, rows, st, sc, outs, H, P, filled)
    torch.cuda.synchronize()
    top = max(n, filled)
    exp = [o.clone() for o in before]
    for o in exp:
        o[n:top].zero_()
    exp[0][:n] = q.reshape(n, H * 128)
    exp[1][:n] = w
    exp[2][:n] = lens
    exp[3][:n, :width] = nt
    exp[3][:n, width:] = 0
    ridx = torch.tensor(rows, dtype=torch.long, device="cuda")
    exp[4][:n] = st[ridx]
    exp[5][:n] = sc[ridx]
    for a, b in zip(outs, exp):
        assert torch.equal(a.view(torch.uint8) if a.dtype == torch.float32 else a,
                           b.view(torch.uint8) if b.dtype == torch.float32 else b)


def test_query_stage_rejects_bad_rows(cuda_dev):
    H, P, R = 32, 64, 4
    q = torch.zeros(2, H, 128, dtype=torch.uint8, device="cuda")
    w = torch.zeros(2, H, device="cuda")
    lens = torch.zeros(2, dtype=torch.int32, device="cuda")
    nt = torch.zeros(2, P, dtype=torch.int32, device="cuda")
    st, sc = torch.zeros(R, P, dtype=torch.int32, device="cuda"), torch.zeros(R, P // 8, dtype=torch.int32,
                                                                               device="cuda")
    outs = [torch.zeros_like(q).view(2, -1), torch.zeros_like(w), torch.zeros_like(lens), torch.zeros_like(nt),
            torch.zeros_like(nt), torch.zeros(2, P // 8, dtype=torch.int32, device="cuda")]
    for rows in ([0, R], [-1, 0]):
        with pytest.raises(ValueError):
            _stage(q, w, lens, nt, rows, st, sc, outs, H, P, 0)
    with pytest.raises(ValueError):      # native tables wider than the page count
        _stage(q, w, lens, torch.zeros(2, P + 8, dtype=torch.int32, device="cuda"), [0, 1], st, sc, outs, H, P, 0)
