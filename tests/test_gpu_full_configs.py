"""GPU parity at the benchmark configurations themselves, at full size.

* d5, the decode batch: 128 requests, contexts U[32K, 128K] from the benchmark's
  seed, 64 index heads, page table of 2048 pages, fixed page budget 40, window
  64, Top-2048, gather of the 576-wide bf16 latent -- the whole step through
  ``SelectionStep`` (the reference's sequence: runtime.py:417-636 with the fixed
  budget of bench_v1_dynamic_budget_metadata.py:5-28).
* d1, the single-head batch: 1024 rows of 4097 tokens, one head (tensor-core
  scorer, MMA width 16), 2688 candidates per row, through ``SelectionStep``.
* d3, the page lifecycle: a 131,072-page arena, 256 requests with chains of
  1-128 buckets (16-2048 pages), half sharing a prefix, 8 rounds; the GPU arena
  (per-bucket driver and batched driver) against the CPU port after every round.

Rows are checked by ``oracle/selection_check.py``: metadata of every row exact;
scores within the 1e-2 bar; route, fine table, Top-2048 and gathered bytes
bit-exact given the device's own scores; and the selection agreement -- the
route and Top-2048 recomputed from the oracle's scores may differ from the GPU's
only by pages / slots inside the tolerance band of the selection threshold.
"""
import importlib
import json
import os

import numpy as np
import pytest
import torch

from oracle import selection_check as SC

pytestmark = pytest.mark.gpu

synth = importlib.import_module("10_20_b200.synth")
pipeline = importlib.import_module("10_20_b200.pipeline")
lifecycle = importlib.import_module("10_20_b200.lifecycle")
port = importlib.import_module("oracle.port")


def _sample(lens, k, seed):
    """k rows: the shortest, the longest and k-2 more drawn from the seed."""
    order = np.argsort(lens, kind="stable")
    rng = np.random.default_rng(seed)
    rest = [int(x) for x in rng.permutation(len(lens)) if x not in (order[0], order[-1])]
    return sorted({int(order[0]), int(order[-1]), *rest[:k - 2]})


def _record(name, rep):
    """Append the figures to $V1X_PARITY_LOG (JSON lines) when it is set."""
    path = os.environ.get("V1X_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": name, **rep}) + "\n")


def _assert_report(rep):
    for key in ("metadata_exact", "route_exact_given_device_scores", "fine_table_exact", "gather_exact",
                "route_differences_within_band", "slot_differences_within_band"):
        assert rep[key] is True, (key, rep)
    for key in ("centre_scores_within_tol", "fine_scores_within_tol", "topk_exact_given_device_scores"):
        assert rep[key] in (True, None), (key, rep)
    assert rep["ok"], rep


@pytest.fixture(scope="module")
def d5():
    lens = synth.decode_lens(128, 32768, 131072, 1000)      # the benchmark's context lengths
    case = synth.make_query_case(128, 64, lens, P=2048, take=40, window=64, topk=2048, seed=1000,
                                 device="cuda", latent_dim=576)
    yield case, lens
    del case
    torch.cuda.empty_cache()


def test_d5_decode_batch_full_size(d5):
    case, lens = d5
    step = pipeline.SelectionStep(case, gather=True, keep_logits=True)
    step.run()
    rows = _sample(np.asarray(lens), 8, 5)
    rep = SC.check_rows(step, case, rows)
    _record("d5 decode, 128 requests, kept logits", rep)
    _assert_report(rep)
    assert rep["centre_scores_within_tol"] is True and rep["fine_scores_within_tol"] is True
    assert rep["topk_exact_given_device_scores"] is True


def test_d5_production_step_equals_checked_step(d5):
    """The benchmark's step (page maxima only, captured in a CUDA graph) gives the
    same route, Top-2048 and gathered bytes as the step whose logits were kept
    and checked above, on every row."""
    case, lens = d5
    checked = pipeline.SelectionStep(case, gather=True, keep_logits=True)
    checked.run()
    prod = pipeline.SelectionStep(case, gather=True)
    prod.capture()
    prod.replay()
    torch.cuda.synchronize()
    for name in ("selected", "physical", "logical", "raw"):
        assert torch.equal(getattr(prod, name), getattr(checked, name)), name
    assert torch.equal(prod.kv.view(torch.int16), checked.kv.view(torch.int16))
    rep = SC.check_rows(prod, case, _sample(np.asarray(lens), 4, 9))
    _record("d5 decode, 128 requests, graph replay", rep)
    _assert_report(rep)


def test_d1_single_head_batch_full_size(cuda_dev):
    case = synth.make_query_case(1024, 1, [4097] * 1024, P=128, take=40, window=64, topk=2048, seed=19,
                                 device="cuda")
    step = pipeline.SelectionStep(case, gather=False, keep_logits=True)
    step.run()
    rows = _sample(np.full(1024, 4097), 16, 19)
    rep = SC.check_rows(step, case, rows, latent_check=False)
    _record("d1 single head, 1024 rows", rep)
    _assert_report(rep)
    assert rep["centre_scores_within_tol"] is True and rep["fine_scores_within_tol"] is True
    assert rep["topk_exact_given_device_scores"] is True


# ---------------------------------------------------------------------------
# d3: the page lifecycle at full size
# ---------------------------------------------------------------------------

def _page_digest(pool):
    """Per-page int64 digest of a packed pool (same arithmetic on GPU and host)."""
    if isinstance(pool, torch.Tensor):
        x = pool.view(torch.int64)
        w = torch.arange(1, x.shape[1] + 1, dtype=torch.int64, device=x.device)
        return (x * w).sum(1).cpu().numpy()
    x = pool.view(np.int64)
    w = np.arange(1, x.shape[1] + 1, dtype=np.int64)
    with np.errstate(over="ignore"):
        return (x * w).sum(1)


def _compare_arena(gpu, cpu, full=False):
    assert int(gpu.free_count.item()) == cpu.count
    for name in ("refs", "free", "tables", "members", "hashes"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(cpu, name)), name
    if full:
        assert np.array_equal(gpu.fine.cpu().numpy(), cpu.fine)
        assert np.array_equal(gpu.centers.cpu().numpy(), cpu.centers)
    else:
        assert np.array_equal(_page_digest(gpu.fine[:gpu.capacity]), _page_digest(cpu.fine))
        assert np.array_equal(_page_digest(gpu.centers), _page_digest(cpu.centers))
    assert sorted(gpu.states) == sorted(cpu.states)
    for owner, st in gpu.states.items():
        assert st.leases == cpu.states[owner]["leases"]
        assert np.array_equal(st.table.cpu().numpy(), cpu.states[owner]["table"])
        assert np.array_equal(st.center_table.cpu().numpy(), cpu.states[owner]["center_table"])


def test_d3_lifecycle_full_arena(cuda_dev):
    cap, pages, requests = 131072, 2048, 256
    wl = synth.LifecycleWorkload(requests, 128, 8, 31, cap // 16, share=0.5, grow=8)
    contents = wl.contents("cuda")
    host = tuple(x.cpu().numpy() for x in contents)
    cpu = port.ArenaPort(cap, pages, max_requests=requests)
    per_bucket = lifecycle.PageArena(cap, pages, "cuda", max_requests=requests, graphs=True)
    batched = lifecycle.PageArena(cap, pages, "cuda", max_requests=requests)
    src_gpu, bsrc, src_cpu = wl.source(contents), wl.pool_source(contents), wl.source(host)
    buckets = shared = 0
    for k, ops in enumerate(wl.ops):
        prep, rel = [], []
        for op in ops + [("end",)]:
            if op[0] != "prepare" and prep:
                batched.prepare_many(prep, bsrc)
                prep = []
            if op[0] != "release" and rel:
                batched.release_many(rel)
                rel = []
            if op[0] == "prepare":
                before = len(cpu.states[op[1]]["leases"]) if op[1] in cpu.states else 0
                cpu.prepare(op[1], op[2], src_cpu)
                buckets += len(cpu.states[op[1]]["leases"]) - before
                per_bucket.prepare(op[1], op[2], src_gpu)
                prep.append((op[1], op[2]))
            elif op[0] == "release":
                cpu.release(op[1])
                per_bucket.release(op[1])
                rel.append(op[1])
        per_bucket.check()
        batched.check()
        torch.cuda.synchronize()
        last = k == len(wl.ops) - 1
        _compare_arena(per_bucket, cpu, full=last)
        _compare_arena(batched, cpu, full=last)
        shared += int((cpu.refs > 1).sum())
    _record("d3 lifecycle, 131072 pages, 256 requests, 8 rounds",
            {"buckets": buckets, "shared_page_rounds": shared, "ok": True})
    assert buckets > 4000 and shared > 0
