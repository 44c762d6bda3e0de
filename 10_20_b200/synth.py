"""Seeded synthetic workloads with the shapes of the benchmark configurations.

There is no dataset for this path: the reference tests and benchmarks use
synthetic tensors only.  Everything is generated on the target device with
torch and laid out exactly as the reference's pools:

  * native pool  uint8 [NP, 8448]: 64-token pages of FP8 e4m3 index keys (bf16
    N(0,1) keys quantised per token with an fp32 absmax/448 scale), pages of
    every request scattered over the pool by a shuffled native page table;
  * fine pool    uint8 [CAP + B*68, 8448]: the index build's reordered pages
    (each complete 1K-token bucket = 16 pages holding a random permutation of
    the bucket's tokens, `members` = their logical positions) plus 68 staging
    pages per query row;
  * centre pool  uint8 [ceil(CAP/8), 8448]: 8 centres per reordered page, each
    the mean of 8 consecutive members' dequantised keys, quantised with the
    reference's power-of-two scale (v1_deepseek/kernels.py:45-54);
  * latent pool  bf16 [NP*64, 1, D] for the K/V gather (slot = page*64+offset);
  * queries: q bf16 N(0,1) per (row, head) quantised to e4m3 with a power-of-two
    scale folded into the head weight (qwen_gqa_probe_kernels.py:15-20), head
    weights U(0,1).
"""
from __future__ import annotations

import dataclasses
import math

import torch

PAGE = 8448


def quantize_tokens(x: torch.Tensor, pow2: bool = False):
    """x float [T, 128] -> (e4m3 bytes uint8 [T, 128], fp32 scale [T])."""
    amax = x.abs().amax(dim=1).float()
    if pow2:
        scale = torch.exp2(torch.ceil(torch.log2(amax.clamp_min(1e-4) / 448.0)))
    else:
        scale = amax.clamp_min(1e-12) / 448.0
    q = (x.float() / scale[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(torch.uint8), scale


def pack_pages(kbytes: torch.Tensor, scales: torch.Tensor, out: torch.Tensor):
    """kbytes uint8 [pages, 64, 128], scales f32 [pages, 64] -> packed pages (in place)."""
    n = kbytes.shape[0]
    out[:n, :8192] = kbytes.reshape(n, 8192)
    out[:n].view(torch.float32)[:, 2048:] = scales


@dataclasses.dataclass
class QueryCase:
    """Device-resident inputs of one batch of index queries (one query per row)."""
    B: int
    H: int
    P: int                     # page-table capacity per row (max_context / 64)
    take: int                  # fixed page budget (BudgetMetadata)
    window: int
    topk: int
    lens: torch.Tensor         # int32 [B]
    q8: torch.Tensor           # float8_e4m3fn [B, H, 128]
    w: torch.Tensor            # float32 [B, H]
    native: torch.Tensor       # uint8 [NP, 8448]
    fine: torch.Tensor         # uint8 [CAP + B*68, 8448]
    centers: torch.Tensor      # uint8 [ceil(CAP/8), 8448]
    members: torch.Tensor      # int32 [CAP, 64]
    native_table: torch.Tensor     # int32 [B, P]
    reordered_table: torch.Tensor  # int32 [B, P]
    center_table: torch.Tensor     # int32 [B, P // 8]
    capacity: int
    latent: torch.Tensor | None = None  # bf16 [NP*64, 1, D]

    @property
    def width(self) -> int:
        return -(-(self.take * 64 + 64 + 4096) // 256) * 256


def make_query_case(B: int, H: int, lens, P: int, take: int, window: int = 64, topk: int = 2048,
                    seed: int = 0, device="cuda", latent_dim: int = 0, chunk_pages: int = 8192,
                    lens_tensor: torch.Tensor | None = None) -> QueryCase:
    """Build a QueryCase.  `lens` is a list of per-row visible lengths."""
    dev = torch.device(device)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    lens = [int(x) for x in lens]
    assert len(lens) == B and all(0 <= n <= P * 64 for n in lens)
    npages = [-(-n // 64) for n in lens]
    NP = max(sum(npages), 1)
    # native pages: every row owns its own pages, scattered over the pool
    perm = torch.randperm(NP, generator=gen).to(torch.int32)
    native_table = torch.zeros((B, P), dtype=torch.int32)
    off = 0
    for b, m in enumerate(npages):
        native_table[b, :m] = perm[off:off + m]
        off += m
    native = torch.empty((NP, PAGE), dtype=torch.uint8, device=dev)
    dgen = torch.Generator(device=dev).manual_seed(seed + 1)
    for s in range(0, NP, chunk_pages):
        e = min(NP, s + chunk_pages)
        x = torch.randn(((e - s) * 64, 128), generator=dgen, device=dev, dtype=torch.bfloat16)
        kb, sc = quantize_tokens(x)
        pack_pages(kb.view(e - s, 64, 128), sc.view(e - s, 64), native[s:e])
        del x, kb, sc
    # index build result: complete 1K buckets, shuffled within the bucket
    nbk = [max(n - 1, 0) // 1024 for n in lens]
    CAP = max(sum(nbk) * 16, 16)
    rperm = torch.randperm(CAP, generator=gen).to(torch.int32)
    reordered_table = torch.zeros((B, P), dtype=torch.int32)
    center_table = torch.zeros((B, P // 8), dtype=torch.int32)
    members = torch.full((CAP, 64), -1, dtype=torch.int32, device=dev)
    fine = torch.zeros((CAP + B * 68, PAGE), dtype=torch.uint8, device=dev)
    centers = torch.zeros((-(-CAP // 8), PAGE), dtype=torch.uint8, device=dev)
    off = 0
    lease = 0
    nt_dev = native_table.to(dev)
    for b in range(B):
        k = nbk[b]
        if k == 0:
            continue
        pages = rperm[off:off + k * 16]
        reordered_table[b, :k * 16] = pages
        center_table[b, :k * 2] = torch.arange(lease * 2, (lease + k) * 2, dtype=torch.int32)
        # random permutation of each bucket's 1024 positions
        keys = torch.rand((k, 1024), generator=gen)
        order = keys.argsort(dim=1).to(torch.int32) + (torch.arange(k, dtype=torch.int32) * 1024)[:, None]
        logical = order.reshape(k * 16, 64).to(dev)
        pg = pages.to(dev).long()
        members[pg] = logical
        lg = logical.reshape(-1).long()
        src_page = nt_dev[b, lg // 64].long()
        src_slot = lg % 64
        kbytes = native[:, :8192].reshape(-1, 64, 128)[src_page, src_slot]
        scales = native.view(torch.float32)[:, 2048:][src_page, src_slot]
        fine[pg, :8192] = kbytes.reshape(k * 16, 8192)
        fine.view(torch.float32)[pg, 2048:] = scales.reshape(k * 16, 64)
        # centres: mean of 8 consecutive members (DS/kernels.py:45-54)
        x = kbytes.view(torch.float8_e4m3fn).float() * scales[:, None]
        mean = x.reshape(k * 128, 8, 128).mean(1)
        cb, cs = quantize_tokens(mean, pow2=True)
        cpages = torch.arange(lease * 2, (lease + k) * 2, device=dev)
        centers[cpages, :8192] = cb.reshape(k * 2, 8192)
        centers.view(torch.float32)[cpages, 2048:] = cs.reshape(k * 2, 64)
        off += k * 16
        lease += k
    # queries
    q = torch.randn((B, H, 128), generator=dgen, device=dev, dtype=torch.bfloat16).float()
    qscale = torch.exp2(torch.ceil(torch.log2(q.abs().amax(-1).clamp_min(1e-4) / 448.0)))
    q8 = (q / qscale[..., None]).to(torch.float8_e4m3fn)
    w = (torch.rand((B, H), generator=dgen, device=dev) * qscale).float()
    latent = None
    if latent_dim:
        latent = torch.empty((NP * 64, 1, latent_dim), dtype=torch.bfloat16, device=dev)
        step = 1 << 22
        flat = latent.view(-1, latent_dim)
        for s in range(0, flat.shape[0], step):
            e = min(flat.shape[0], s + step)
            flat[s:e] = torch.randn((e - s, latent_dim), generator=dgen, device=dev, dtype=torch.bfloat16)
    return QueryCase(B=B, H=H, P=P, take=take, window=window, topk=topk,
                     lens=torch.tensor(lens, dtype=torch.int32, device=dev), q8=q8, w=w, native=native,
                     fine=fine, centers=centers, members=members, native_table=nt_dev,
                     reordered_table=reordered_table.to(dev), center_table=center_table.to(dev),
                     capacity=CAP, latent=latent)


def decode_lens(B: int, lo: int, hi: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (B,), generator=g).tolist()


# ---------------------------------------------------------------------------
# page-lifecycle schedules
# ---------------------------------------------------------------------------

class LifecycleWorkload:
    """A seeded request schedule for the page arena.

    Requests grow bucket by bucket over `rounds`; each new request shares, with
    probability `share`, a prefix of another request's bucket chain (identical
    pages and members at identical logical offsets, so match_pages finds them),
    and about a quarter of the live requests complete (release) after every
    round.  Bucket contents are indexed by a content id; `contents(device)`
    materialises them: tmp uint8 [U, 16, 8448] (random packed pages), mapping
    int32 [U, 16, 64] (the bucket's 1024 logical positions, shuffled) and
    centers uint8 [U, 2, 8448].  `ops` is a list of rounds, each a list of
    ("prepare", owner, length) and ("release", owner) in canonical order."""

    def __init__(self, requests: int, max_buckets: int, rounds: int, seed: int, max_leases: int,
                 share: float = 0.5, grow: int = 8):
        g = torch.Generator().manual_seed(seed)
        rnd = lambda n: int(torch.randint(0, n, (1,), generator=g).item())
        self.chains: dict[int, list[int]] = {}
        self.bucket_of: list[int] = []            # content id -> its bucket index
        prepared: dict[int, int] = {}
        live: list[int] = []
        next_owner = 0
        self.ops = []
        for _ in range(rounds):
            ops = []
            while len(live) < requests:
                owner = next_owner
                next_owner += 1
                n = 1 + rnd(max_buckets)
                chain = []
                if self.chains and rnd(1000) < share * 1000:
                    other = self.chains[list(self.chains)[rnd(len(self.chains))]]
                    k = 1 + rnd(min(len(other), n))
                    chain = other[:k]
                while len(chain) < n:
                    self.bucket_of.append(len(chain))
                    chain.append(len(self.bucket_of) - 1)
                self.chains[owner] = chain
                prepared[owner] = 0
                live.append(owner)
            used = sum(prepared[o] for o in live)
            for owner in live:
                add = min(1 + rnd(grow), len(self.chains[owner]) - prepared[owner])
                add = min(add, max_leases - used)
                if add <= 0:
                    continue
                prepared[owner] += add
                used += add
                ops.append(("prepare", owner, prepared[owner] * 1024 + rnd(1024)))
            done = [o for o in live if rnd(4) == 0]
            for owner in done:
                ops.append(("release", owner))
                live.remove(owner)
                prepared.pop(owner)
            self.ops.append(ops)
        self.n_contents = len(self.bucket_of)

    def contents(self, device):
        U = self.n_contents
        gen = torch.Generator(device=device).manual_seed(7)
        tmp = torch.randint(0, 256, (U, 16, PAGE), generator=gen, device=device, dtype=torch.uint8)
        centers = torch.randint(0, 256, (U, 2, PAGE), generator=gen, device=device, dtype=torch.uint8)
        perm = torch.argsort(torch.rand((U, 1024), generator=gen, device=device), dim=1).to(torch.int32)
        base = torch.as_tensor(self.bucket_of, dtype=torch.int32, device=device)[:, None] * 1024
        mapping = (base + perm).reshape(U, 16, 64).contiguous()
        return tmp, mapping, centers

    def source(self, contents):
        """bucket_source(owner, bucket) for PageArena / ArenaPort over materialised contents."""
        tmp, mapping, centers = contents
        return lambda owner, bucket: (tmp[self.chains[owner][bucket]], mapping[self.chains[owner][bucket]],
                                      centers[self.chains[owner][bucket]])

    def batch_source(self, contents):
        """batch_source(pairs) for PageArena.prepare_many: the (owner, bucket)
        pairs' contents stacked in order."""
        from .lifecycle import BATCH_BUCKETS, HostStaging

        tmp, mapping, centers = contents
        ids_dev = torch.zeros(BATCH_BUCKETS, dtype=torch.long, device=tmp.device)
        staging = HostStaging(BATCH_BUCKETS, tmp.device, dtype=torch.long)

        def fetch(pairs):
            ids = staging.copy([self.chains[o][b] for o, b in pairs], ids_dev)[:len(pairs)]
            return tmp.index_select(0, ids), mapping.index_select(0, ids), centers.index_select(0, ids)
        return fetch

    def pool_source(self, contents):
        """batch_source(pairs) for PageArena.prepare_many that hands over the
        materialised contents as pools with each pair's entry (read in place)."""
        tmp, mapping, centers = contents
        return lambda pairs: (tmp, mapping, centers, [self.chains[o][b] for o, b in pairs])
