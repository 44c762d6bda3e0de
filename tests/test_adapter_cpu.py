"""CPU: the C4Adapter's configuration checks and row ownership
(DS/adapter.py:24-102, 145-157) against fake backend objects."""
import importlib
import json
from types import SimpleNamespace as NS

import pytest
import torch

adapter = importlib.import_module("10_20_b200.adapter")
Config = importlib.import_module("10_20_b200.config").Config


def _backend(heads=32, topk=512, layers=2, max_context_len=4 * 8192, **args):
    server = dict(disable_cuda_graph=True, disable_prefill_cuda_graph=True, tp_size=1, pp_size=1,
                  speculative_algorithm=None, enable_prefill_context_parallel=False,
                  enable_dsa_prefill_context_parallel=False)
    server.update(args)
    listeners = []
    pool = NS(req_generation=[0] * 16, add_native_index_listener=listeners.append, listeners=listeners)
    mapping = [NS(compress_ratio=4)] * layers + [NS(compress_ratio=128), None]
    return NS(model_runner=NS(model_config=NS(hf_text_config=NS(index_n_heads=heads)),
                              server_args=NS(**server)),
              enable_deepseek_v4_fp4_indexer=False, hisparse_coordinator=None, c4_topk=topk,
              token_to_kv_pool=NS(layer_mapping=mapping), max_context_len=max_context_len,
              device=torch.device("cpu"), req_to_token_pool=pool)


def _env(monkeypatch, **fields):
    cfg = dict(max_context=8192, topk=512, page_fraction=0.25, window=64, max_requests=4, q_buckets=[1, 4])
    cfg.update(fields)
    monkeypatch.setenv("SGLANG_V1_DEEPSEEK_CONFIG", json.dumps(cfg))
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None: (1 << 40, 1 << 40))


def test_from_environment_accepts_and_registers(monkeypatch):
    monkeypatch.delenv("SGLANG_V1_DEEPSEEK_CONFIG", raising=False)
    assert adapter.C4Adapter.from_environment(_backend()) is None
    be = _backend()
    reservation = Config(max_context=8192, heads=32, topk=512, page_fraction=0.25, window=64, max_requests=4,
                         q_buckets=(1, 4)).reservation
    _env(monkeypatch, total_budget_bytes=2 * reservation)
    a = adapter.C4Adapter.from_environment(be)
    assert a.config.heads == 32 and a.config.q_buckets == (1, 4) and a.total_budget_bytes == 2 * reservation
    assert be.req_to_token_pool.listeners == [a]


@pytest.mark.parametrize("case, message", [
    (dict(backend=dict(heads=64), env=dict(heads=32)), "heads must match"),
    (dict(backend=dict(disable_cuda_graph=False)), "--disable-cuda-graph"),
    (dict(backend=dict(tp_size=2)), "single-GPU FP8"),
    (dict(backend=dict(speculative_algorithm="eagle")), "single-GPU FP8"),
    (dict(backend=dict(topk=1024)), "topk must match"),
    (dict(budget=1), "below all-layer reservation"),
    (dict(backend=dict(max_context_len=4 * 8192 + 1)), "context / 4"),
])
def test_from_environment_refusals(monkeypatch, case, message):
    be = _backend(**case.get("backend", {}))
    _env(monkeypatch, total_budget_bytes=case.get("budget", 1 << 40), **case.get("env", {}))
    with pytest.raises(ValueError, match=message):
        adapter.C4Adapter.from_environment(be)


def test_from_environment_free_memory(monkeypatch):
    _env(monkeypatch, total_budget_bytes=1 << 40)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda device=None: (1, 1 << 40))
    with pytest.raises(ValueError, match="Insufficient free GPU memory"):
        adapter.C4Adapter.from_environment(_backend())


def _mode(decode):
    return NS(is_decode=lambda: decode, is_extend=lambda: not decode)


def test_row_metadata_decode_and_extend():
    be = _backend()
    be.req_to_token_pool.req_generation[3] = 7
    a = adapter.C4Adapter(be, Config(max_context=8192, topk=512, max_requests=4, q_buckets=(1, 4)), 1 << 40)
    dec = NS(native_req_pool_indices_cpu=[3, 5], forward_mode=_mode(True), seq_lens_cpu=torch.tensor([4097, 2]))
    assert a.row_metadata(dec, 2) == ([(3, 7), (5, 0)], [1024, 0])
    ext = NS(native_req_pool_indices_cpu=[3, 1], forward_mode=_mode(False), extend_prefix_lens_cpu=[6, 0],
             extend_seq_lens_cpu=[3, 2])
    assert a.row_metadata(ext, 5) == ([(3, 7)] * 3 + [(1, 0)] * 2, [1, 2, 2, 0, 0])
    with pytest.raises(ValueError, match="unpadded"):
        a.row_metadata(ext, 6)
    idle = NS(native_req_pool_indices_cpu=[1], forward_mode=NS(is_decode=lambda: False, is_extend=lambda: False))
    with pytest.raises(ValueError, match="speculative/idle"):
        a.row_metadata(idle, 1)
    with pytest.raises(ValueError, match="CPU request slots"):
        a.row_metadata(NS(native_req_pool_indices_cpu=None), 1)


def test_release_request_drops_every_generation():
    be = _backend()
    a = adapter.C4Adapter(be, Config(max_context=8192, topk=512, max_requests=4, q_buckets=(1, 4)), 1 << 40)
    released = []
    layer = NS(states={(2, 0): 1, (2, 1): 1, (3, 0): 1}, release_request=released.append, close=lambda: None)
    a.layers = {5: layer}
    a.release_request(2)
    assert released == [(2, 0), (2, 1)]
    a.clear()
    assert a.layers == {}
