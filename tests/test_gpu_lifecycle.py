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


def _rounds_batched(gpu, cpu, wl, contents, host, pool=False):
    """Each round's consecutive prepares as one prepare_many call and its
    consecutive releases as one release_many call; the CPU port takes the same
    operations one by one.  pool: the bucket contents are read in place from
    the content pool (source ids) instead of copied out per call."""
    bsrc = wl.pool_source(contents) if pool else wl.batch_source(contents)
    src_cpu = wl.source(host)
    for ops in wl.ops:
        prep, rel = [], []
        for op in ops + [("end",)]:
            if op[0] != "prepare" and prep:
                gpu.prepare_many(prep, bsrc)
                prep = []
            if op[0] != "release" and rel:
                gpu.release_many(rel)
                rel = []
            if op[0] == "prepare":
                prep.append((op[1], op[2]))
                cpu.prepare(op[1], op[2], src_cpu)
            elif op[0] == "release":
                rel.append(op[1])
                cpu.release(op[1])
        gpu.check()
        torch.cuda.synchronize()
        _compare(gpu, cpu)


@pytest.mark.parametrize("requests,grow,pool", [(10, 3, False), (40, 4, False), (40, 4, True)])
def test_prepare_many_matches_cpu_port(requests, grow, pool, cuda_dev):
    """Batched prepare (extension) == the reference's per-bucket sequence: every
    arena array and request table after every round.  (40, 4) puts more than 64
    buckets in a round (several calls); shared prefixes give matches both
    against pages live before a call and against pages published inside it."""
    cap, pages = 4096, 256
    wl = synth.LifecycleWorkload(requests=requests, max_buckets=8, rounds=4, seed=11 + requests,
                                 max_leases=cap // 16, share=0.6, grow=grow)
    contents = wl.contents("cuda")
    host = tuple(x.cpu().numpy() for x in contents)
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=64)
    cpu = port.ArenaPort(cap, pages, max_requests=64)
    _rounds_batched(gpu, cpu, wl, contents, host, pool)
    assert (cpu.refs > 1).sum() > 0


def test_prepare_many_inside_batch_sharing(cuda_dev):
    """Two requests with the same chain prepared in ONE call: the second one's
    pages match the pages the first one published earlier in the same call."""
    cap, pages = 1024, 128
    wl = synth.LifecycleWorkload(requests=1, max_buckets=4, rounds=1, seed=2, max_leases=cap // 16, share=0.0)
    (a,) = list(wl.chains)
    wl.chains[a + 1] = list(wl.chains[a])
    contents = wl.contents("cuda")
    host = tuple(x.cpu().numpy() for x in contents)
    n = len(wl.chains[a]) * 1024 + 3
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=4)
    cpu = port.ArenaPort(cap, pages, max_requests=4)
    gpu.prepare_many([(a, n), (a + 1, n)], wl.batch_source(contents))
    for o in (a, a + 1):
        cpu.prepare(o, n, wl.source(host))
    gpu.check()
    _compare(gpu, cpu)
    assert int((cpu.refs == 2).sum()) == 16 * len(wl.chains[a])


@pytest.mark.parametrize("batched", [False, True])
def test_exhausted_free_stack_changes_nothing(batched, cuda_dev):
    """A free stack shorter than a bucket needs (only reachable by changing the
    arena by hand: the driver's lease records bound the live pages): the status
    word reports it and that bucket and the later ones change nothing -- the
    arena equals the CPU port's at the failing bucket (the reference traps)."""
    cap, pages = 256, 64
    wl = synth.LifecycleWorkload(requests=3, max_buckets=3, rounds=1, seed=4, max_leases=cap // 16, share=0.0)
    a = min(wl.chains)
    wl.chains[a] = [0, 1, 2]                 # three distinct buckets
    contents = wl.contents("cuda")
    host = tuple(x.cpu().numpy() for x in contents)
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=2)
    cpu = port.ArenaPort(cap, pages, max_requests=2)
    gpu.free_count.fill_(20)
    cpu.count = 20
    n = 3 * 1024
    if batched:
        gpu.prepare_many([(a, n)], wl.batch_source(contents))
    else:
        gpu.prepare(a, n, wl.source(contents))
    with pytest.raises(port.O.ArenaExhausted):
        cpu.prepare(a, n, wl.source(host))
    with pytest.raises(Exception, match="exhausted"):
        gpu.check()
    torch.cuda.synchronize()
    assert int(gpu.free_count.item()) == cpu.count == 4
    for name in ("refs", "free", "members", "hashes"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(cpu, name)), name
    assert np.array_equal(gpu.fine.cpu().numpy(), cpu.fine)
    assert np.array_equal(gpu.centers.cpu().numpy(), cpu.centers)
    assert np.array_equal(gpu.tables.cpu().numpy(), cpu.tables)
    # the host state again describes the arena: the owner keeps its first
    # bucket, the aborted leases are free, their page-table entries read 0
    st = gpu.states[a]
    assert len(st.leases) == len(cpu.states[a]["leases"]) == 1 and st.length == 1024
    assert not st.table[16:48].any() and gpu.pending_check is False
    # releasing the owner afterwards touches only its allocated pages
    if batched:
        gpu.release_many([a])
    else:
        gpu.release(a)
    cpu.release(a)
    torch.cuda.synchronize()
    assert int(gpu.free_count.item()) == cpu.count == 20
    for name in ("refs", "free"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(cpu, name)), name
    assert len(gpu.free_leases) == gpu.max_leases


def _collide(mapping_page):
    """Members whose fingerprint equals the page's (same bytes): +1, -2, +1 at
    members 0..2 leave both fingerprint sums unchanged, the content differs."""
    m = mapping_page.clone()
    m[0] += 1
    m[1] -= 2
    m[2] += 1
    return m


def test_prepare_many_fingerprint_collisions(cuda_dev):
    """Pages with equal fingerprints but different members must never match:
    against a live arena page (the confirmation fails), and inside one call,
    where a page's lowest equal-fingerprint earlier page is the colliding one
    and its true equal page comes later in the call (the decision warp's exact
    search)."""
    cap, pages = 1024, 128
    gen = torch.Generator().manual_seed(8)
    n = 4
    tmp = torch.randint(0, 256, (n, 16, 8448), generator=gen, dtype=torch.uint8)
    centers = torch.randint(0, 256, (n, 2, 8448), generator=gen, dtype=torch.uint8)
    mapping = torch.stack([torch.randperm(1024, generator=gen).to(torch.int32).view(16, 64) for _ in range(n)])
    # one call: content 0 (X at page 3), content 1 (Y at page 3: X's bytes with
    # colliding members), content 2 (Y again at page 3): the lowest earlier
    # equal-fingerprint page of the second Y is X, its true copy the first Y.
    # Second call: content 3 page 5 collides with content 0 page 5, live by then.
    tmp[1, 3] = tmp[0, 3]
    mapping[1, 3] = _collide(mapping[0, 3])
    tmp[2, 3] = tmp[1, 3]
    mapping[2, 3] = mapping[1, 3]
    tmp[3, 5] = tmp[0, 5]
    mapping[3, 5] = _collide(mapping[0, 5])
    chains = {10: [0], 11: [1, 2], 12: [3]}
    host = (tmp.numpy(), mapping.numpy(), centers.numpy())
    dev_c = (tmp.cuda(), mapping.cuda(), centers.cuda())

    def src(c):
        return lambda o, b: tuple(x[chains[o][b]] for x in c)

    def bsrc(pairs):
        ids = torch.tensor([chains[o][b] for o, b in pairs], dtype=torch.long, device="cuda")
        return tuple(x.index_select(0, ids) for x in dev_c)

    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=4)
    cpu = port.ArenaPort(cap, pages, max_requests=4)
    for group in ([(10, 1024), (11, 2048)], [(12, 1024)]):
        gpu.prepare_many(group, bsrc)
        for o, length in group:
            cpu.prepare(o, length, src(host))
        gpu.check()
        torch.cuda.synchronize()
        _compare(gpu, cpu)
    t = {o: cpu.states[o]["table"] for o in chains}
    assert t[11][16 + 3] == t[11][3] != t[10][3]     # the copy shares its page, not the collision's
    assert t[12][5] != t[10][5]


def test_prepare_many_error_matches_prepare(cuda_dev):
    """Lease records running out inside a batched call: the same error as the
    per-bucket driver, raised at the same bucket, and the same arena (the
    buckets granted before it are indexed, none twice)."""
    cap, pages = 64, 64                      # 4 lease records
    wl = synth.LifecycleWorkload(requests=6, max_buckets=3, rounds=1, seed=9, max_leases=cap // 16, share=0.0)
    a, b = sorted(wl.chains)[:2]
    wl.chains[a], wl.chains[b] = [0, 1, 2], [3, 4, 5]
    contents = wl.contents("cuda")
    batched = lifecycle.PageArena(cap, pages, "cuda", max_requests=2)
    single = lifecycle.PageArena(cap, pages, "cuda", max_requests=2)
    with pytest.raises(RuntimeError, match="bucket records exhausted"):
        batched.prepare_many([(a, 3 * 1024), (b, 3 * 1024)], wl.batch_source(contents))
    single.prepare(a, 3 * 1024, wl.source(contents))
    with pytest.raises(RuntimeError, match="bucket records exhausted"):
        single.prepare(b, 3 * 1024, wl.source(contents))
    batched.check()
    single.check()
    torch.cuda.synchronize()
    for name in ("refs", "free", "free_count", "tables", "members", "hashes", "fine", "centers"):
        assert torch.equal(getattr(batched, name), getattr(single, name)), name
    for o in (a, b):
        assert batched.states[o].leases == single.states[o].leases
        assert torch.equal(batched.states[o].table, single.states[o].table)
    assert len(batched.states[b].leases) == 1 and int(batched.free_count.item()) == 0


@pytest.mark.parametrize("seed", range(4))
def test_prepare_buckets_entry_point_random_batches(seed, cuda_dev):
    """v1x_prepare_buckets called directly (the C ABI), on randomised calls with
    inactive buckets, pages live before the call, pages published earlier in the
    call, fingerprint collisions and (some seeds) a short free stack, against the
    numpy restatement of the batched algorithm -- which the CPU tests tie to the
    reference's per-bucket sequence.  Seeds 2-3 pass the bucket contents as ids
    into a shuffled pool (src)."""
    import copy

    import oracle.v1x_oracle as O
    _lib = importlib.import_module("10_20_b200._lib")
    rng = np.random.default_rng(200 + seed)
    cap, pages = 512, 256
    cpu = port.ArenaPort(cap, pages, max_requests=8)
    live = []
    for b in range(3):
        tmp = rng.integers(0, 256, (16, 8448), dtype=np.uint8)
        mp = (100000 * (b + 1) + np.arange(1024)).astype(np.int32).reshape(16, 64)
        cpu._bucket(tmp, mp, rng.integers(0, 256, (2, 8448), dtype=np.uint8), b * 1024, b)
        live += [(tmp[i], mp[i]) for i in range(16)]
    nb = 8
    tmp = np.zeros((nb, 16, 8448), np.uint8)
    mp = np.zeros((nb, 16, 64), np.int32)
    made = []
    for b in range(nb):
        seen = set()
        for i in range(16):
            while True:
                kind = rng.integers(0, 4)
                if kind == 0 or (kind == 2 and not made):
                    x = rng.integers(0, 256, 8448, dtype=np.uint8)
                    m = (900000 + 4096 * b + 64 * i + np.arange(64)).astype(np.int32)
                elif kind == 1:
                    x, m = live[int(rng.integers(len(live)))]
                elif kind == 2:
                    x, m = made[int(rng.integers(len(made)))]
                else:
                    x, m = (live + made)[int(rng.integers(len(live) + len(made)))]
                    m = m.copy()
                    m[:3] += np.array([1, -2, 1], np.int32)
                if (x.tobytes(), m.tobytes()) not in seen:
                    seen.add((x.tobytes(), m.tobytes()))
                    break
            tmp[b, i], mp[b, i] = x, m
        made += [(tmp[b, i].copy(), mp[b, i].copy()) for i in range(16)]
    centers = rng.integers(0, 256, (nb, 2, 8448), dtype=np.uint8)
    active = (rng.random(nb) > 0.25).astype(np.int32)
    meta3 = np.array([[b * 1024, 3 + b, active[b]] for b in range(nb)], np.int32)
    if seed % 2:
        cpu.count = int(rng.integers(10, 60))
    exp = copy.deepcopy(cpu)
    new_exp, exhausted_exp = port.prepare_buckets_batched(exp, tmp, centers, mp, meta3)
    # the same starting arena on the GPU
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=8)
    for name in ("refs", "free", "tables", "members", "hashes", "fine", "centers"):
        getattr(gpu, name).copy_(torch.from_numpy(np.ascontiguousarray(getattr(cpu, name))))
    gpu.free_count.fill_(cpu.count)
    meta = np.array([[b * 1024, 3 + b, active[b], 0] for b in range(nb)], dtype=np.int32)   # host records
    t, m, c = (torch.from_numpy(a).cuda() for a in (tmp, mp, centers))
    src, nsrc = None, 0
    if seed >= 2:
        # the bucket contents read through ids from a shuffled pool of nb + 3 entries
        nsrc = nb + 3
        perm = torch.as_tensor(rng.permutation(nsrc)[:nb], device="cuda")
        pools = [torch.zeros((nsrc,) + tuple(x.shape[1:]), dtype=x.dtype, device="cuda") for x in (t, m, c)]
        for pool, x in zip(pools, (t, m, c)):
            pool[perm] = x
        t, m, c = pools
        src = perm.cpu().numpy().astype(np.int32)   # host ids
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    work = torch.zeros(lifecycle.PREPARE_WORK_INTS, dtype=torch.int32, device="cuda")
    hsh = torch.zeros((nb * 16, 2), dtype=torch.int64, device="cuda")
    match = torch.zeros(nb * 16, dtype=torch.int32, device="cuda")
    new = torch.zeros(nb * 16, dtype=torch.uint8, device="cuda")
    p = _lib.ptr
    _lib.call("v1x_prepare_buckets", p(t), p(c), p(c.view(torch.float32)), p(m), meta.ctypes.data,
              None if src is None else src.ctypes.data, nsrc, nb, p(hsh),
              p(match),
              p(new), p(gpu.fine), p(gpu.centers), p(gpu.centers.view(torch.float32)), p(gpu.members),
              p(gpu.hashes), p(gpu.refs), p(gpu.free), p(gpu.free_count), p(gpu.tables), p(gpu.center_pages),
              None, 0, None, 0, cap, p(work), p(status), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(gpu.free_count.item()) == exp.count
    for name in ("refs", "free", "tables", "members", "hashes", "fine", "centers"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(exp, name)), name
    assert (int(status.item()) == _lib.V1X_STATUS_ARENA_EXHAUSTED) == exhausted_exp
    assert np.array_equal(new.cpu().numpy(), new_exp)


def test_prepare_buckets_pair_list_overflow(cuda_dev):
    """More fingerprint-equal (live page, batch page) pairs than the pair list
    holds: 80 live arena pages and 128 batch pages that all share one
    fingerprint (the same bytes, members differing by multiples of the
    +1/-2/+1 collision pattern) give 10,240 pairs, so the call takes its exact
    fallback (the sweep with inline confirmation).  Some batch pages equal a
    live page, some are new, some repeat a new page of an earlier bucket behind
    a colliding one.  The arena afterwards equals the restated algorithm's."""
    import copy

    _lib = importlib.import_module("10_20_b200._lib")
    cap, pages = 2048, 256
    rng = np.random.default_rng(77)
    x = rng.integers(0, 256, 8448, dtype=np.uint8)
    m0 = (5000 + np.arange(64)).astype(np.int32)
    delta = np.zeros(64, np.int32)
    delta[:3] = (1, -2, 1)
    variant = lambda k: (m0 + k * delta).astype(np.int32)
    cpu = port.ArenaPort(cap, pages, max_requests=8)
    for b in range(5):                       # 80 live variants k = 0..79
        tmp = np.stack([x] * 16)
        mp = np.stack([variant(16 * b + i) for i in range(16)])
        cpu._bucket(tmp, mp, rng.integers(0, 256, (2, 8448), dtype=np.uint8), b * 1024, b)
    nb = 8
    ks = []
    for b in range(nb):                      # live k < 80, new k in [80, 120): repeats across buckets
        ks.append(rng.choice(np.arange(120), size=16, replace=False))
    tmp = np.stack([np.stack([x] * 16) for _ in range(nb)])
    mp = np.stack([np.stack([variant(int(k)) for k in row]) for row in ks])
    centers = rng.integers(0, 256, (nb, 2, 8448), dtype=np.uint8)
    meta3 = np.array([[b * 1024, 5 + b, 1] for b in range(nb)], np.int32)
    exp = copy.deepcopy(cpu)
    new_exp, exhausted_exp = port.prepare_buckets_batched(exp, tmp, centers, mp, meta3)
    gpu = lifecycle.PageArena(cap, pages, "cuda", max_requests=8)
    for name in ("refs", "free", "tables", "members", "hashes", "fine", "centers"):
        getattr(gpu, name).copy_(torch.from_numpy(np.ascontiguousarray(getattr(cpu, name))))
    gpu.free_count.fill_(cpu.count)
    meta = np.array([[b * 1024, 5 + b, 1, 0] for b in range(nb)], dtype=np.int32)   # host records
    t, m, c = (torch.from_numpy(a).cuda() for a in (tmp, mp, centers))
    # the bucket contents read through ids from a pool of nb + 3 entries, in
    # reverse order (the inline-confirmation sweep reads them through the ids)
    nsrc = nb + 3
    perm = torch.arange(nb, 0, -1, device="cuda")
    pools = [torch.zeros((nsrc,) + tuple(x.shape[1:]), dtype=x.dtype, device="cuda") for x in (t, m, c)]
    for pool, x in zip(pools, (t, m, c)):
        pool[perm] = x
    t, m, c = pools
    src = perm.cpu().numpy().astype(np.int32)   # host ids
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    work = torch.zeros(lifecycle.PREPARE_WORK_INTS, dtype=torch.int32, device="cuda")
    hsh = torch.zeros((nb * 16, 2), dtype=torch.int64, device="cuda")
    match = torch.zeros(nb * 16, dtype=torch.int32, device="cuda")
    new = torch.zeros(nb * 16, dtype=torch.uint8, device="cuda")
    p = _lib.ptr
    _lib.call("v1x_prepare_buckets", p(t), p(c), p(c.view(torch.float32)), p(m), meta.ctypes.data,
              None if src is None else src.ctypes.data, nsrc, nb, p(hsh),
              p(match),
              p(new), p(gpu.fine), p(gpu.centers), p(gpu.centers.view(torch.float32)), p(gpu.members),
              p(gpu.hashes), p(gpu.refs), p(gpu.free), p(gpu.free_count), p(gpu.tables), p(gpu.center_pages),
              None, 0, None, 0, cap, p(work), p(status), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(work[2].item()) & 1, "the pair list did not overflow"
    assert not exhausted_exp and int(status.item()) == 0
    assert int(gpu.free_count.item()) == exp.count
    for name in ("refs", "free", "tables", "members", "hashes", "fine", "centers"):
        assert np.array_equal(getattr(gpu, name).cpu().numpy(), getattr(exp, name)), name
    assert np.array_equal(new.cpu().numpy(), new_exp)
    assert 0 < int(new_exp.sum()) < nb * 16          # both fresh pages and matches occurred
