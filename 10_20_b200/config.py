"""Index geometry and budget of the query path: the reference's ``Config``
(sglang/srt/layers/attention/v1_deepseek/runtime.py:19-96), same fields,
validation and derived sizes, so callers that build one for the reference build
it unchanged here.

Derived sizes (kept identical to the reference, since buffers are sized by them):
  pages        max_context / 64                         (:58-60)
  take         min(pages, max(ceil(pages * page_fraction), ceil(topk / 64)))  (:66-71)
  width        ceil((take * 64 + 64 + 4096) / 256) * 256   fine candidate columns (:73-75)
  reservation  arena + scratch + per-bucket query buffers  bytes (:77-96)
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from fractions import Fraction


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


@dataclass(frozen=True)
class Config:
    max_context: int = 65536
    heads: int = 32
    max_requests: int = 1
    topk: int = 512
    page_fraction: float = 0.5
    q_buckets: tuple = (1, 4, 16, 64)
    sink: int = 64
    window: int = 2048
    score_mode: str = "relu"
    graphs: bool = True
    budget_bytes: int = 2 << 30
    query_optimizations: bool = True
    query_mask_fusion: bool = True
    query_bucket_rank_mask: bool = True
    query_direct_fine_map: bool = False
    query_int32_selected: bool = True
    query_tail_compaction: bool = True
    query_inplace_metadata: bool = False
    query_output_mapping_optimization: bool = True
    expand_output: bool = False
    query_route_table_fusion: bool = False

    def __post_init__(self):
        if (
            self.max_context < 4096
            or self.max_context % 4096
            or (self.expand_output and self.max_context > (1 << 29))
            or self.max_requests < 1
            or not 0 < self.topk <= 2048
            or not 0 < self.page_fraction <= 1
            or self.heads not in (32, 64)
            or self.score_mode not in ("relu", "signed")
            or self.sink != 64
            or not 0 <= self.window <= 4096
            or not self.q_buckets
            or tuple(sorted(set(self.q_buckets))) != tuple(self.q_buckets)
            or self.q_buckets[0] != 1
            or self.budget_bytes <= 0
        ):
            raise ValueError("Invalid DeepSeek V1 geometry/budget")

    @property
    def pages(self) -> int:
        return self.max_context // 64

    @property
    def ratio(self) -> Fraction:
        return Fraction(str(self.page_fraction)).limit_denominator(1000000)

    @property
    def take(self) -> int:
        return min(self.pages, max(math.ceil(self.pages * self.page_fraction), _cdiv(self.topk, 64)))

    @property
    def width(self) -> int:
        return _cdiv(self.take * 64 + 64 + 4096, 256) * 256

    @property
    def reservation(self) -> int:
        cap = self.pages * self.max_requests
        arena = cap * (8448 + 1056 + 256 + 32) + self.q_buckets[-1] * 68 * 8448 + self.max_requests * self.pages * 4
        scratch = 32 << 20
        query = sum((8 << 20) + r * (self.width * 24 + self.pages * 64 + 32768) for r in self.q_buckets)
        expand = sum(self.q_buckets) * (self.topk * 4 + 64) * 4 if self.expand_output else 0
        return arena + scratch + query + expand
