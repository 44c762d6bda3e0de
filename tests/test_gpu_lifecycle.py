"""The request-level page lifecycle (reference Indexer._prepare/_release and the
page part of Build.compute) on the GPU against the CPU port, bit-exact after
every round: lease tables, request page tables, refcounts, the free stack and
its count, and the fine/centre pools, members and hashes."""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

synth = importlib.import_module("10_20_b200.synth")
lifecycle = importlib.import_module("10_20_b200.lifecycle")
port = importlib.import_module("oracle.port")


def _compare(gpu, cpu):
    assert gpu.free_leases == cpu.free_leases
    assert int(gpu.free_count.item()) == cpu.count
    for name in ("refs", "free", "tables", "members", "hashes"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(cpu, name)), name
    assert np.array_equal(gpu.fine.cpu().numpy(), cpu.fine)
    assert np.array_equal(gpu.centers.cpu().numpy(), cpu.centers)
    assert sorted(gpu.states) == sorted(cpu.states)
    for owner, st in gpu.states.items():
        assert st.leases == cpu.states[owner]["leases"]
        assert np.array_equal(st.table.cpu().numpy(), cpu.states[owner]["table"])
        assert np.array_equal(st.center_table.cpu().numpy(), cpu.states[owner]["center_table"])


@pytest.mark.parametrize("graphs", [False, True])
def test_lifecycle_rounds_match_cpu_port(graphs, cuda_dev):
    cap, pages = 1024, 128
    wl = synth.LifecycleWorkload(requests=10, max_buckets=6, rounds=4, seed=3, max_leases=cap // 16,
                                 share=0.6, grow=3)
    contents = wl.contents("cuda")
    host = tuple(x.cpu().numpy() for x in contents)
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=16, graphs=graphs)
    cpu = port.ArenaPort(cap, pages, max_requests=16)
    src_gpu, src_cpu = wl.source(contents), wl.source(host)
    hits = 0
    for ops in wl.ops:
        for op in ops:
            if op[0] == "prepare":
                gpu.prepare(op[1], op[2], src_gpu)
                cpu.prepare(op[1], op[2], src_cpu)
            else:
                gpu.release(op[1])
                cpu.release(op[1])
        gpu.check()
        torch.cuda.synchronize()
        _compare(gpu, cpu)
        hits += int((cpu.refs > 1).sum())
    assert hits > 0          # shared prefixes did share pages


def test_lifecycle_limits(cuda_dev):
    """Out of lease records the driver raises before launching anything (as the
    reference's _prepare does); lengths past the page table and too many
    requests are rejected; a shrinking length releases and rebuilds."""
    wl = synth.LifecycleWorkload(requests=2, max_buckets=3, rounds=1, seed=5, max_leases=64, share=0.0)
    contents = wl.contents("cuda")
    arena = lifecycle.PageArena(32, 64, "cuda", max_requests=2)      # 2 lease records
    src = wl.source(contents)
    a, b = sorted(wl.chains)
    arena.prepare(a, 2 * 1024 + 5, src)
    arena.check()
    refs = arena.refs.clone()
    with pytest.raises(RuntimeError, match="bucket records exhausted"):
        arena.prepare(b, 1024, src)
    assert torch.equal(arena.refs, refs) and arena.free_leases == []
    with pytest.raises(ValueError):
        arena.prepare(a, 64 * 64 + 1, src)
    arena.prepare(a, 1024, src)              # shorter: released, then one bucket rebuilt
    arena.check()
    assert len(arena.states[a].leases) == 1 and int(arena.free_count.item()) == 16
    arena.release(a)
    assert int(arena.free_count.item()) == 32 and bool((arena.refs == 0).all())
