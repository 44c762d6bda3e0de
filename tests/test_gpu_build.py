"""GPU: the index build of 1024-token buckets (Build.compute's initialize /
grouping / assemble, DS/runtime.py:170-233) against the CPU oracle, bit-exact:
the fused many-bucket launch, the reference's own op sequence through the
drop-in ops, the 4K FusedGroups grouping, and the Indexer building its arena
from the native cache."""
import importlib

import numpy as np
import pytest
import torch

from oracle import v1x_oracle as O
from oracle.port import ArenaPort

pytestmark = pytest.mark.gpu

ib = importlib.import_module("10_20_b200.index_build")
K = importlib.import_module("10_20_b200.kernels")
FG = importlib.import_module("10_20_b200.fused_grouping")
indexer_mod = importlib.import_module("10_20_b200.indexer")
Config = importlib.import_module("10_20_b200.config").Config
_lib = importlib.import_module("10_20_b200._lib")


def _pool(seed, pages, adversarial=False):
    gen = torch.Generator().manual_seed(seed)
    k = torch.randn((pages, 64, 128), generator=gen).to(torch.float8_e4m3fn)
    buf = torch.zeros((pages, 8448), dtype=torch.uint8)
    buf[:, :8192] = k.view(torch.uint8).reshape(pages, 8192)
    buf.view(torch.float32)[:, 2048:] = torch.rand((pages, 64), generator=gen) + 0.25
    if adversarial:   # duplicated tokens, zero tokens, constant pages
        kb = buf[:, :8192].view(pages, 64, 128)
        sc = buf.view(torch.float32)[:, 2048:]
        for _ in range(pages * 8):
            a, b = torch.randint(0, pages * 64, (2,), generator=gen).tolist()
            kb[b // 64, b % 64] = kb[a // 64, a % 64]
            sc[b // 64, b % 64] = sc[a // 64, a % 64]
        for t in torch.randint(0, pages * 64, (pages * 3,), generator=gen).tolist():
            kb[t // 64, t % 64] = 0
        kb[::7] = kb[::7, :1]
        sc[::7] = sc[::7, :1]
    return buf.numpy()


def _oracle_bucket(pool, table, start):
    unit, _ = O.build_initialize(pool, table)
    perm = O.group_bucket(unit)
    return (perm,) + O.build_assemble(pool, table, start, perm)


def test_build_buckets_golden(golden, cuda_dev):
    """The reference's bucket (interpreter fixture): same member order, tmp
    pages and mapping; centres as the round-to-nearest cast gives them."""
    g = golden("build")
    native = torch.from_numpy(g["native"]).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    tmp, centers, mapping, perm = ib.build_buckets(native, torch.from_numpy(g["tables"]).cuda(),
                                                   [int(x) for x in g["starts"]], status)
    for b in range(2):
        assert np.array_equal(perm[b].cpu().numpy(), g[f"perm{b}"])
        assert np.array_equal(tmp[b].cpu().numpy(), g[f"tmp{b}"])
        assert np.array_equal(mapping[b].cpu().numpy(), g[f"mapping{b}"])
        exp = O.build_assemble(g["native"], g["tables"][b], int(g["starts"][b]), g[f"perm{b}"])[1]
        assert np.array_equal(centers[b].cpu().numpy(), exp)
    assert int(status.item()) == 0


@pytest.mark.parametrize("seed", [1, 2])
def test_build_buckets_vs_oracle(seed, cuda_dev):
    pages, nb = 96, 6
    pool = _pool(seed, pages, adversarial=seed == 2)
    rng = np.random.default_rng(seed)
    tables = np.stack([rng.permutation(pages)[:16] for _ in range(nb)]).astype(np.int32)
    starts = [int(x) * 1024 for x in rng.integers(0, 100, nb)]
    builder = ib.BucketBuilder("cuda", max_buckets=8)
    native = torch.from_numpy(pool).cuda()
    out = [x.clone() for x in builder.build(native, torch.from_numpy(tables).cuda(), starts)]
    again = builder.build(native, torch.from_numpy(tables).cuda(), starts)     # buffers reused
    for x, y in zip(out, again):
        assert torch.equal(x, y)
    tmp, centers, mapping, perm = (x.cpu().numpy() for x in out)
    for b in range(nb):
        e_perm, e_tmp, e_centers, e_map = _oracle_bucket(pool, tables[b], starts[b])
        assert np.array_equal(perm[b], e_perm), b
        assert np.array_equal(tmp[b], e_tmp), b
        assert np.array_equal(centers[b], e_centers), b
        assert np.array_equal(mapping[b], e_map), b


def test_reference_op_sequence(cuda_dev):
    """Build.compute's own launch sequence (DS/runtime.py:170-233) through the
    drop-in ops equals the oracle stage by stage and the fused launch."""
    pool = _pool(3, 40, adversarial=True)
    table = np.random.default_rng(3).permutation(40)[:16].astype(np.int32)
    start = 7 * 1024
    native = torch.from_numpy(pool).cuda()
    fp8, f32 = native.view(torch.float8_e4m3fn), native.view(torch.float32)
    source = torch.from_numpy(table).cuda()
    meta = torch.tensor([start, 0, 1], dtype=torch.int32, device="cuda")
    unit = torch.empty((1024, 128), device="cuda")
    perm = [torch.empty(1024, dtype=torch.int32, device="cuda") for _ in range(2)]
    anchor = torch.empty((64, 2), dtype=torch.int32, device="cuda")
    scores = torch.empty(1024, device="cuda")
    flag = torch.zeros((), dtype=torch.int32, device="cuda")
    K.initialize[(64,)](fp8, f32, source, meta, unit, perm[0], flag, num_warps=4)
    e_unit, _ = O.build_initialize(pool, table)
    assert np.array_equal(unit.cpu().numpy().view(np.uint32), e_unit.view(np.uint32))
    assert int(flag.item()) == -1 and torch.equal(perm[0].cpu(), torch.arange(1024, dtype=torch.int32))
    cur = 0
    for n in (1024, 512, 256, 128, 64, 32, 16):
        for mode in (0, 1, 2):
            FG._dots[(64, 1)](unit, perm[cur], anchor, scores, flag, n, 0, mode, num_warps=4, enable_fp_fusion=False)
            if mode < 2:
                FG._anchor[(1024 // n, 1)](perm[cur], anchor, scores, flag, n, mode, num_warps=4)
        FG._sort[(1024 // n, 1)](perm[cur], perm[1 - cur], scores, flag, n, num_warps=4)
        cur = 1 - cur
    e_perm, e_tmp, e_centers, e_map = _oracle_bucket(pool, table, start)
    assert np.array_equal(perm[cur].cpu().numpy(), e_perm)
    tmp = torch.zeros((16, 8448), dtype=torch.uint8, device="cuda")
    centers = torch.zeros((2, 8448), dtype=torch.uint8, device="cuda")
    mapping = torch.zeros((16, 64), dtype=torch.int32, device="cuda")
    K.assemble[(16, 8)](fp8, f32, source, meta, perm[cur], tmp.view(torch.float8_e4m3fn), tmp.view(torch.float32),
                        centers.view(torch.float8_e4m3fn), centers.view(torch.float32), mapping, num_warps=4)
    assert np.array_equal(tmp.cpu().numpy(), e_tmp)
    assert np.array_equal(centers.cpu().numpy(), e_centers)
    assert np.array_equal(mapping.cpu().numpy(), e_map)
    fused = ib.build_buckets(native, source.view(1, 16), [start])
    assert torch.equal(fused[0][0], tmp) and torch.equal(fused[1][0], centers) and torch.equal(fused[3][0], perm[cur])
    # inactive: initialize clears the flag and the grouping ops do nothing
    meta[2] = 0
    unit.fill_(7.0)
    K.initialize[(64,)](fp8, f32, source, meta, unit, perm[0], flag)
    assert int(flag.item()) == 0 and bool((unit == 7.0).all())
    scores.fill_(3.0)
    FG._dots[(64, 1)](unit, perm[0], anchor, scores, flag, 1024, 0, 0)
    assert bool((scores == 3.0).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_groups_4k(dtype, cuda_dev):
    """FusedGroups.run (NA/fused_grouping.py:78-111, fused mode), two heads,
    a strided K pool and a slot map, against the oracle's op chain."""
    gen = torch.Generator().manual_seed(4)
    heads, slots, start = 2, 4500, 150
    base = torch.randn((slots, heads, 160), generator=gen).to(dtype)
    k = base[:, :, :128]                        # padded head rows: stride(1) = 160
    k[100:140] = k[40]                          # duplicated keys
    k[200:230] = 0                              # zero keys
    req = torch.randperm(slots, generator=gen).to(torch.int32)
    flag = torch.full((), -1, dtype=torch.int32)
    fg = FG.FusedGroups(heads, "cuda")
    kd = base.cuda()[:, :, :128]
    assert kd.stride(1) == 160
    out = fg.run(kd, req.cuda(), start, flag.cuda()).cpu().numpy()
    unit, P = O.group_init(k.float().numpy(), req.numpy(), start, heads)
    exp = O.group_levels(unit, P, start, (4096, 2048, 1024, 512, 256, 128, 64, 32, 16), 4096, heads)
    assert np.array_equal(out.reshape(-1), exp)
    for h in range(heads):
        assert sorted(out[h].tolist()) == list(range(start, start + 4096))


def test_bad_source_page_reports_status(cuda_dev):
    pool = _pool(5, 20)
    table = np.arange(16, dtype=np.int32)
    table[3] = 20                               # outside the 20-page pool
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    tmp, centers, mapping, perm = ib.build_buckets(torch.from_numpy(pool).cuda(),
                                                   torch.from_numpy(table).cuda().view(1, 16), [0], status)
    assert int(status.item()) == _lib.V1X_STATUS_BAD_PAGE
    m = mapping[0].cpu().numpy().reshape(-1)
    rows = np.nonzero((m >= 3 * 64) & (m < 4 * 64))[0]
    t = tmp[0].cpu().numpy()
    assert len(rows) == 64 and all((t[r // 64, (r % 64) * 128:(r % 64) * 128 + 128] == 0).all() for r in rows)


def test_indexer_builds_from_native_cache(cuda_dev):
    """Indexer.prepare without a bucket source builds every bucket from the
    native cache (Build.compute): the arena equals the CPU port fed by the
    oracle's build, including pages shared through a common prefix."""
    P, pages = 128, 160
    pool = _pool(6, pages)
    rng = np.random.default_rng(6)
    t0 = rng.permutation(pages)[:P].astype(np.int32)
    t1 = np.concatenate([t0[:32], rng.permutation(pages)[:P - 32]]).astype(np.int32)   # 2 shared buckets
    tables = {0: t0, 1: t1}
    cfg = Config(max_context=P * 64, heads=32, max_requests=4, topk=512, page_fraction=0.25, window=64,
                 q_buckets=(1, 4))
    ix = indexer_mod.Indexer(torch.from_numpy(pool).cuda(), cfg)
    cpu = ArenaPort(ix.arena.capacity, ix.arena.pages, max_requests=cfg.max_requests)

    def src(owner, bucket):
        tab = tables[owner][bucket * 16:(bucket + 1) * 16]
        tmp, centers, mapping = O.build_assemble(pool, tab, bucket * 1024,
                                                 O.group_bucket(O.build_initialize(pool, tab)[0]))
        return tmp, mapping, centers

    for owner, length in ((0, 3 * 1024 + 100), (1, 4 * 1024), (0, 4 * 1024 + 5)):
        ix.prepare(owner, torch.from_numpy(tables[owner]).cuda(), length)
        cpu.prepare(owner, length, src)
    ix.arena.check()
    a = ix.arena
    cap = a.capacity
    assert np.array_equal(a.fine[:cap].cpu().numpy(), cpu.fine)
    assert np.array_equal(a.centers.cpu().numpy(), cpu.centers)
    for name in ("refs", "free", "tables", "members", "hashes"):
        assert np.array_equal(getattr(a, name).cpu().numpy(), getattr(cpu, name)), name
    assert int(a.free_count.item()) == cpu.count
    assert int((cpu.refs > 1).sum()) == 32      # the two shared buckets' pages
    for owner in (0, 1):
        assert np.array_equal(a.states[owner].table.cpu().numpy(), cpu.states[owner]["table"])
    ix.close()
