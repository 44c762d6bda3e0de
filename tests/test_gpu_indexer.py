"""The Indexer library surface (reference Indexer.prepare/query/release_request,
DS/runtime.py:693-937): built over the index-build output of a synthetic case,
its query returns the same slot ids as the selection step run on that case."""
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

synth = importlib.import_module("10_20_b200.synth")
pipeline = importlib.import_module("10_20_b200.pipeline")
indexer_mod = importlib.import_module("10_20_b200.indexer")
Config = importlib.import_module("10_20_b200.config").Config


def _setup(graphs, expand=False):
    B, H, P = 12, 32, 192
    cfg = Config(max_context=P * 64, heads=H, max_requests=B, topk=512, page_fraction=0.25, window=64,
                 q_buckets=(1, 4, 16), graphs=graphs, expand_output=expand)
    lens = synth.decode_lens(B, 3000, P * 64, 5)
    case = synth.make_query_case(B, H, lens, P=P, take=cfg.take, window=64, topk=512, seed=9, device="cuda")

    def source(owner, bucket):     # the synthetic index build of request `owner`
        pages = case.reordered_table[owner, bucket * 16:(bucket + 1) * 16].long()
        cpages = case.center_table[owner, bucket * 2:(bucket + 1) * 2].long()
        return case.fine[pages], case.members[pages], case.centers[cpages]

    ix = indexer_mod.Indexer(case.native, cfg, bucket_source=source)
    ratio = cfg.ratio
    ref = pipeline.SelectionStep(case, gather=False, ratio=(ratio.numerator, ratio.denominator), expand=expand)
    ref.run()
    torch.cuda.synchronize()
    return B, case, ix, ref, lens


@pytest.mark.parametrize("graphs", [False, True])
def test_indexer_query_matches_selection_step(graphs, cuda_dev):
    B, case, ix, ref, lens = _setup(graphs)
    owners = list(range(B))
    for _ in range(2):         # second call: buckets already built, query graph replayed
        phys, logical = ix.query(case.q8, case.w, case.native_table, case.lens, owners, lens, return_logical=True)
        assert torch.equal(phys, ref.physical) and torch.equal(logical, ref.logical)
    # rows split over two buckets (16 + 4 rows) give the same answer per row
    idx = list(range(B)) + list(range(8))
    q2 = ix.query(case.q8[idx], case.w[idx], case.native_table[idx].contiguous(), case.lens[idx].contiguous(),
                  [owners[i] for i in idx], [lens[i] for i in idx])
    assert torch.equal(q2, ref.physical[idx])
    assert ix.query(case.q8[:0], case.w[:0], case.native_table[:0], case.lens[:0], [], []).shape == (0, 512)
    ix.release_request(3)
    assert 3 not in ix.states
    ix.close()
    with pytest.raises(RuntimeError):
        ix.query(case.q8, case.w, case.native_table, case.lens, owners, lens)


def test_indexer_expanded_output_and_checks(cuda_dev):
    B, case, ix, ref, lens = _setup(False, expand=True)
    out = ix.query(case.q8, case.w, case.native_table, case.lens, list(range(B)), lens)
    assert out.shape == (B, 512 * 4 + 64) and torch.equal(out, ref.expanded)
    with pytest.raises(ValueError):      # weights of the wrong width
        ix.query(case.q8, case.w[:, :16].contiguous(), case.native_table, case.lens, list(range(B)), lens)
    with pytest.raises(ValueError):      # a length past its page table
        bad = list(lens)
        bad[0] = 192 * 64 + 1
        ix.query(case.q8, case.w, case.native_table, case.lens, list(range(B)), bad)


def test_indexer_padding_narrow_tables_and_repeated_owners(cuda_dev):
    """A shorter call after a longer one on the same bucket (its padding rows are
    zeroed again), native tables narrower than the configured page count, and
    one request on several rows with different lengths (each row masks to its
    own length; the request is built to the longest)."""
    B, case, ix, ref, lens = _setup(True)
    owners = list(range(B))
    assert torch.equal(ix.query(case.q8, case.w, case.native_table, case.lens, owners, lens), ref.physical)
    part = ix.query(case.q8[:5], case.w[:5], case.native_table[:5], case.lens[:5], owners[:5], lens[:5])
    assert torch.equal(part, ref.physical[:5])
    width = max(-(-x // 64) for x in lens)
    narrow = case.native_table[:, :width].contiguous()
    assert torch.equal(ix.query(case.q8, case.w, narrow, case.lens, owners, lens), ref.physical)
    # request r on two rows, the second 5 tokens shorter (same complete buckets)
    r = next(i for i in range(B) if lens[i] % 1024 >= 8 and i != 1)
    idx = [1, r, r]
    rl = [lens[1], lens[r], lens[r] - 5]
    out = ix.query(case.q8[idx], case.w[idx], case.native_table[idx].contiguous(),
                   torch.tensor(rl, dtype=torch.int32, device="cuda"), [owners[i] for i in idx], rl)
    assert torch.equal(out[:2], ref.physical[[1, r]])
    assert ix.states[r].length == lens[r]
    alone = ix.query(case.q8[[r]], case.w[[r]], case.native_table[[r]].contiguous(),
                     torch.tensor([lens[r] - 5], dtype=torch.int32, device="cuda"), [r], [lens[r] - 5])
    assert torch.equal(out[2:], alone)
    ix.close()
