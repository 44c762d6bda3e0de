"""GPU: the C4Adapter end to end over a fake backend whose native Index-K
cache is a synthetic case (DS/adapter.py:104-157): its outputs equal an
Indexer driven directly with the same owners and compressed lengths; the
layer budget and the native-address check hold."""
import importlib
from types import SimpleNamespace as NS

import pytest
import torch

pytestmark = pytest.mark.gpu

synth = importlib.import_module("10_20_b200.synth")
adapter = importlib.import_module("10_20_b200.adapter")
indexer_mod = importlib.import_module("10_20_b200.indexer")
Config = importlib.import_module("10_20_b200.config").Config


def test_adapter_decode_matches_indexer(cuda_dev):
    B, H, P = 6, 32, 128
    cfg = Config(max_context=P * 64, heads=H, max_requests=8, topk=512, page_fraction=0.25, window=64,
                 q_buckets=(1, 4, 8))
    lens = synth.decode_lens(B, 2100, P * 64, 8)
    case = synth.make_query_case(B, H, lens, P=P, take=cfg.take, window=64, topk=512, seed=4, device="cuda")
    native = {"buf": case.native}
    gens = [0] * 16
    gens[2] = 5
    pool = NS(req_generation=gens, add_native_index_listener=lambda a: None)
    be = NS(req_to_token_pool=pool,
            token_to_kv_pool=NS(get_index_k_with_scale_buffer=lambda layer_id: native["buf"]))
    a = adapter.C4Adapter(be, cfg, cfg.reservation)
    slots = [0, 2, 4, 6, 8, 10]
    batch = NS(native_req_pool_indices_cpu=slots, forward_mode=NS(is_decode=lambda: True, is_extend=lambda: False),
               seq_lens_cpu=torch.tensor([4 * n + 3 for n in lens]))
    meta = NS(page_table=case.native_table, c4_seq_lens=case.lens, c4_page_size=64)
    c4 = NS(layer_id=3, use_fp4_indexer=False)
    out = torch.empty((B, 512), dtype=torch.int32, device="cuda")
    raw = torch.empty_like(out)
    a.query(c4, batch, case.q8, case.w, meta, out, raw)
    owners = [(s, gens[s]) for s in slots]
    ref = indexer_mod.Indexer(case.native, cfg)
    phys, logical = ref.query(case.q8, case.w, case.native_table, case.lens, owners, lens, return_logical=True)
    assert torch.equal(out, phys) and torch.equal(raw, logical)
    out2 = torch.empty_like(out)
    a.query(c4, batch, case.q8, case.w, meta, out2)          # second call: buckets already built
    assert torch.equal(out2, phys)
    assert sorted(a.layers[3].states) == sorted(owners)
    a.release_request(2)
    assert (2, 5) not in a.layers[3].states
    with pytest.raises(ValueError, match="exceeds total_budget_bytes"):
        a.query(NS(layer_id=4, use_fp4_indexer=False), batch, case.q8, case.w, meta, out)
    native["buf"] = case.native.clone()
    with pytest.raises(RuntimeError, match="changed address"):
        a.query(c4, batch, case.q8, case.w, meta, out)
    a.clear()
    assert a.layers == {}
