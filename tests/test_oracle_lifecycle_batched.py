"""CPU: the batched page-lifecycle algorithm (v1x_prepare_buckets,
v1x_release_many), restated in numpy, leaves the arena exactly as the
reference's per-bucket and per-lease sequence does -- over randomised calls
mixing fresh pages, pages live before the call, pages first published earlier in
the same call, fingerprint collisions (equal fingerprints, different members),
inactive buckets and a free stack that runs short.  This checks the argument the
GPU kernels rest on; the GPU tests check the kernels against the same sequence."""
import copy

import numpy as np
import pytest

import oracle.port as port
import oracle.v1x_oracle as O

ARRAYS = ("refs", "free", "tables", "fine", "members", "hashes", "centers")


def _page(rng, base):
    return rng.integers(0, 256, O.PAGE_BYTES, dtype=np.uint8), (base + rng.permutation(64)).astype(np.int32)


def _collide(members):
    m = members.copy()
    m[0] += 1
    m[1] -= 2
    m[2] += 1
    return m


def _compare(a, b):
    assert a.count == b.count
    for n in ARRAYS:
        assert np.array_equal(getattr(a, n), getattr(b, n)), n


@pytest.mark.parametrize("seed", range(12))
def test_batched_prepare_equals_per_bucket_sequence(seed):
    rng = np.random.default_rng(seed)
    cap = 512
    seq = port.ArenaPort(cap, 256, max_requests=8)
    live_pages = []                       # (bytes, members) published before the call
    for b in range(3):
        pages = [_page(rng, 100000 * (b + 1) + 64 * i) for i in range(16)]
        tmp = np.stack([p[0] for p in pages])
        mp = np.stack([p[1] for p in pages])
        seq._bucket(tmp, mp, rng.integers(0, 256, (2, O.PAGE_BYTES), dtype=np.uint8), b * 1024, b)
        live_pages += pages
    if seed % 3 == 0:                     # a released bucket: its pages are dead but keep their bytes
        seq.count = O.release(seq.tables[2], seq.refs, seq.free, seq.count)
    bat = copy.deepcopy(seq)
    nb = int(rng.integers(2, 9))
    batch_pages = []
    tmp = np.zeros((nb, 16, O.PAGE_BYTES), np.uint8)
    mp = np.zeros((nb, 16, 64), np.int32)
    for b in range(nb):
        seen = set()
        for i in range(16):
            while True:
                kind = rng.integers(0, 5)
                if kind == 0 or (kind == 2 and not batch_pages):
                    x, m = _page(rng, 900000 + 4096 * b + 64 * i)
                elif kind == 1:
                    x, m = live_pages[int(rng.integers(len(live_pages)))]
                elif kind == 2:
                    x, m = batch_pages[int(rng.integers(len(batch_pages)))]
                else:                     # fingerprint collision with a live or earlier batch page
                    src = live_pages + batch_pages
                    x, m = src[int(rng.integers(len(src)))]
                    m = _collide(m)
                key = (x.tobytes(), m.tobytes())
                if key not in seen:       # a bucket's pages are distinct (disjoint token positions)
                    seen.add(key)
                    break
            tmp[b, i], mp[b, i] = x, m
        batch_pages += [(tmp[b, i], mp[b, i]) for i in range(16)]
    centers = rng.integers(0, 256, (nb, 2, O.PAGE_BYTES), dtype=np.uint8)
    active = rng.random(nb) > 0.15
    meta = np.array([[b * 1024, 3 + b, int(active[b])] for b in range(nb)], np.int32)
    if seed % 4 == 1:                     # a free stack shorter than the call needs
        seq.count = bat.count = int(rng.integers(0, 40))
    # the reference: one bucket after another; it traps at the first short stack
    # (here: that bucket and, the status being sticky, every later one abort,
    # each leaving its lease table row at -1)
    trapped = False
    for b in range(nb):
        if not active[b]:
            continue
        if trapped:
            seq.tables[int(meta[b, 1])] = -1
            continue
        try:
            seq._bucket(tmp[b], mp[b], centers[b], int(meta[b, 0]), int(meta[b, 1]))
        except O.ArenaExhausted:
            trapped = True
    new, exhausted = port.prepare_buckets_batched(bat, tmp, centers, mp, meta)
    _compare(seq, bat)
    assert set(np.unique(new)) <= {0, 1, 2}


def test_batched_prepare_covers_every_path():
    """The generator above reaches every branch: live matches, in-call matches,
    collisions and exhaustion (checked on a fixed case)."""
    rng = np.random.default_rng(0)
    arena = port.ArenaPort(64, 64, max_requests=2)
    x0, m0 = _page(rng, 0)
    tmp = np.stack([np.stack([_page(rng, 64 * i + 4096 * b)[0] for i in range(16)]) for b in range(3)])
    mp = np.stack([np.stack([(4096 * b + 64 * i + np.arange(64)).astype(np.int32) for i in range(16)])
                   for b in range(3)])
    tmp[0, 0], mp[0, 0] = x0, m0                 # X
    tmp[1, 0], mp[1, 0] = x0, _collide(m0)       # Y: X's fingerprint, different members
    tmp[2, 0], mp[2, 0] = x0, _collide(m0)       # Y again: earliest equal fingerprint is X
    centers = np.zeros((3, 2, O.PAGE_BYTES), np.uint8)
    meta = np.array([[0, 0, 1], [1024, 1, 1], [2048, 2, 1]], np.int32)
    new, exhausted = port.prepare_buckets_batched(arena, tmp, centers, mp, meta)
    assert not exhausted
    assert arena.tables[2, 0] == arena.tables[1, 0] != arena.tables[0, 0]
    assert new[32] == 0 and new[16] == 1
    arena2 = port.ArenaPort(64, 64, max_requests=2)
    arena2.count = 20
    new, exhausted = port.prepare_buckets_batched(arena2, tmp, centers, mp, meta)
    assert exhausted and list(new[16:]) == [2] * 32 and arena2.count == 4


@pytest.mark.parametrize("seed", range(6))
def test_batched_release_equals_per_lease_sequence(seed):
    """Requests built by the driver hold distinct pages; releasing several at
    once (all of a request's leases together) equals the per-lease sequence."""
    rng = np.random.default_rng(100 + seed)
    import torch
    import importlib
    synth = importlib.import_module("10_20_b200.synth")
    wl = synth.LifecycleWorkload(requests=8, max_buckets=5, rounds=3, seed=seed, max_leases=1024 // 16,
                                 share=0.6, grow=3)
    contents = tuple(x.numpy() for x in wl.contents("cpu"))
    seq = port.ArenaPort(1024, 128, max_requests=16)
    src = wl.source(contents)
    for ops in wl.ops:
        for op in ops:
            if op[0] == "prepare":
                seq.prepare(op[1], op[2], src)
            else:
                seq.release(op[1])
    owners = sorted(seq.states)
    for o in owners:                     # the precondition of the batched release
        pages = seq.tables[seq.states[o]["leases"]].reshape(-1)
        assert len(set(pages.tolist())) == pages.size
    bat = copy.deepcopy(seq)
    pick = [o for o in owners if rng.random() < 0.7]
    for o in pick:
        seq.release(o)
    port.release_many(bat, [bat.states.pop(o)["leases"] for o in pick])
    _compare(seq, bat)
