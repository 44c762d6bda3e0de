"""The N > 1 host path on CPU: two gloo ranks shard a batch of requests by bytes,
each runs the CPU restatement of the step on its own requests only, and the
gathered results equal a single-process run over the whole batch; the timing
reduction (max over ranks) is checked on the same process group."""
import importlib
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2
CFG = dict(B=6, H=4, P=160, take=8, window=64, topk=256)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    synth = importlib.import_module("10_20_b200.synth")
    lens = synth.decode_lens(CFG["B"], 1500, CFG["P"] * 64, 11)
    case = synth.make_query_case(CFG["B"], CFG["H"], lens, P=CFG["P"], take=CFG["take"], window=CFG["window"],
                                 topk=CFG["topk"], seed=5, device="cpu")
    return lens, case


def _worker(rank, port, out_q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=timedelta(seconds=120))
    try:
        sharding = importlib.import_module("10_20_b200.sharding")
        port_mod = importlib.import_module("oracle.port")
        lens, case = _case()
        costs = [sharding.row_bytes(n, CFG["H"], CFG["take"], CFG["window"], CFG["topk"])["total"] for n in lens]
        shards = sharding.shard_requests(costs, WORLD, per_rank=CFG["B"] // WORLD)
        seen = [None] * WORLD
        dist.all_gather_object(seen, shards)
        c = port_mod.to_numpy_case(case)
        mine = {i: r["physical"].tolist() for i, r in zip(shards[rank], port_mod.run_rows(c, rows=shards[rank]))}
        parts = [None] * WORLD
        dist.all_gather_object(parts, mine)
        t = torch.tensor([1.5 + rank], dtype=torch.float64)      # a per-rank duration
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            out_q.put(dict(shards=shards, seen=seen, parts=parts, tmax=float(t.item()), costs=costs))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_step_matches_single_process():
    sys.path.insert(0, ROOT)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    shards = res["shards"]
    # every rank computed the same assignment; it partitions the batch evenly
    assert all(s == shards for s in res["seen"])
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(CFG["B"])) and all(len(s) == CFG["B"] // WORLD for s in shards)
    # gathered per-request results == one process over the whole batch
    merged = {}
    for part in res["parts"]:
        merged.update(part)
    port_mod = importlib.import_module("oracle.port")
    _, case = _case()
    full = port_mod.run_rows(port_mod.to_numpy_case(case))
    for i, r in enumerate(full):
        assert merged[i] == r["physical"].tolist()
    assert res["tmax"] == 1.5 + (WORLD - 1)


def test_shard_requests_balance_and_errors():
    sharding = importlib.import_module("10_20_b200.sharding")
    rng = np.random.default_rng(3)
    costs = rng.integers(1, 1000, size=64).tolist()
    shards = sharding.shard_requests(costs, 8, per_rank=8)
    loads = [sum(costs[i] for i in s) for s in shards]
    assert sorted(i for s in shards for i in s) == list(range(64))
    assert max(loads) - min(loads) <= max(costs)
    assert sharding.shard_requests(costs, 1) == [list(range(64))]
    try:
        sharding.shard_requests(costs, 8, per_rank=7)
        raise AssertionError("expected ValueError")
    except ValueError:
        pass
