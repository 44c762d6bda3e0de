"""Drop-in for the in-scope Triton ops of ``v1_deepseek/kernels.py``.

Each op is an object used exactly like the reference's Triton kernels,
``op[grid](*args, **constexprs)``, with the reference's positional argument
order; ``num_warps``/``debug`` and other Triton launch options are accepted and
ignored.  Every launch goes to a hand-written sm_100a kernel in libv1x.so on
the current CUDA stream.

Ops (reference sglang/srt/layers/attention/v1_deepseek/kernels.py):
  initialize :9-29, assemble :32-54, fingerprint :57-69, match_pages :72-113, allocate :116-131, publish :134-167,
  release :170-179, query_lengths :224-245, output_ids :323-376,
  mask_fine :444-472, reduce_centers :475-486, fine_table_shared :488-514,
  stage_tail_shared :518-564, query_metadata :568-591, expand_logical :594-600;
  and BudgetMetadata (bench_v1_dynamic_budget_metadata.py:30-34).

Failure reporting: where the reference's ``allocate`` traps on an exhausted
arena (device_assert at :125), this ``allocate`` records the condition in a
per-device status word and leaves the arena untouched.  Outside CUDA-graph
capture the launch checks that word immediately and raises ArenaExhausted;
inside capture, call :func:`check_status` after the graph runs.
"""
from __future__ import annotations

import threading

import torch

from . import _lib
from ._lib import ptr, require


class ArenaExhausted(RuntimeError):
    """The page arena's free stack held fewer pages than a bucket needed."""


_status_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32 status word the page-lifecycle kernels report into."""
    idx = torch.device(device).index or 0
    with _status_lock:
        t = _status.get(idx)
        if t is None:
            # a normal tensor even when first asked for under inference mode, so
            # that check_status can reset it anywhere
            with torch.inference_mode(False):
                t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _status[idx] = t
    return t


def check_status(device=None, reset: bool = True):
    """Raise ArenaExhausted if a kernel on `device` reported an exhausted arena."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = status_word(dev)
    code = int(st.item())
    if code != 0:
        if reset:
            st.zero_()
        if code == _lib.V1X_STATUS_ARENA_EXHAUSTED:
            raise ArenaExhausted("V1 DeepSeek page arena exhausted")
        raise RuntimeError(f"v1x device status {code}")


class _Op:
    """Triton-style launcher: ``op[grid](*args, **kwargs)``."""

    def __init__(self, fn):
        self.fn = fn
        self.__name__ = fn.__name__
        self.__doc__ = fn.__doc__

    def __getitem__(self, grid):
        grid = tuple(grid) if isinstance(grid, (tuple, list)) else (grid,)

        def launch(*args, **kwargs):
            for k in ("num_warps", "num_stages", "debug", "enable_fp_fusion", "num_ctas"):
                kwargs.pop(k, None)
            return self.fn(grid, *args, **kwargs)

        return launch

    def __call__(self, *args, **kwargs):
        raise TypeError(f"{self.__name__} is launched as {self.__name__}[grid](...)")


def _op(fn):
    return _Op(fn)


def _s(t):
    return _lib.stream_of(t)


def _sel64(sel):
    require(sel.dtype in (torch.int32, torch.int64), "SELECTED: int32 or int64 required")
    return 1 if sel.dtype == torch.int64 else 0


# ---------------------------------------------------------------------------
# index build of one bucket (the fused many-bucket form is index_build.py)
# ---------------------------------------------------------------------------

def _native_pages(K):
    require(K.dtype in (torch.uint8, torch.float8_e4m3fn) and K.is_contiguous() and K.numel() % 8448 == 0,
            "K: contiguous packed native pool (uint8 / float8 view, 8448 bytes per page)")
    return K.numel() // 8448


@_op
def initialize(grid, K, KS, TABLE, META, UNIT, PERM, FLAG):
    """Dequantise + normalise the bucket's 1024 keys (DS/kernels.py:9-29).
    K / KS: the native pool's FP8 and float32 views; UNIT f32 [1024, 128];
    PERM i32 [1024]; FLAG i32 (-1 when META[2] is set).  grid = (64,)."""
    require(UNIT.dtype == torch.float32 and UNIT.numel() >= 1024 * 128, "UNIT: float32 [1024, 128]")
    require(PERM.dtype == torch.int32 and FLAG.dtype == torch.int32 and TABLE.dtype == torch.int32,
            "initialize: PERM/FLAG/TABLE int32")
    _lib.call("v1x_initialize", ptr(K), _native_pages(K), ptr(TABLE), ptr(META), ptr(UNIT), ptr(PERM),
              ptr(FLAG), ptr(status_word(K.device)), _s(K), device=K.device)


@_op
def assemble(grid, K, KS, TABLE, META, IDS, TMP, TMPS, CENTERS, CS, MAP):
    """Reordered tmp pages, centres and logical members (DS/kernels.py:32-54).
    TMP/TMPS and CENTERS/CS are FP8 and float32 views of [16, 8448] and
    [2, 8448] byte buffers.  grid = (16, 8)."""
    require(IDS.dtype == torch.int32 and MAP.dtype == torch.int32, "assemble: IDS/MAP int32")
    require(TMP.numel() >= 16 * 8448 and CENTERS.numel() >= 2 * 8448, "assemble: TMP [16, 8448], CENTERS [2, 8448]")
    _lib.call("v1x_assemble", ptr(K), _native_pages(K), ptr(TABLE), ptr(META), ptr(IDS), ptr(TMP), ptr(CENTERS),
              ptr(MAP), _s(K), device=K.device)


# ---------------------------------------------------------------------------
# page lifecycle
# ---------------------------------------------------------------------------

@_op
def fingerprint(grid, TMP, MAP, META, HASH):
    """Two int64 hashes per tmp page (DS/kernels.py:57-69). grid = (pages,)."""
    n = int(grid[0])
    require(TMP.dtype == torch.uint8 and TMP.numel() >= n * 8448, "TMP: uint8 [pages, 8448]")
    require(HASH.dtype == torch.int64, "HASH: int64 [pages, 2]")
    _lib.call("v1x_fingerprint", ptr(TMP), ptr(MAP), ptr(META), ptr(HASH), n, _s(TMP), device=TMP.device)


@_op
def match_pages(grid, TMP, MAP, HASH, META, FINE, MEMBERS, HASHES, REFS, MATCH, CAP, SCAN=None):
    """Lowest live page with equal hashes, bytes and members (DS/kernels.py:72-113)."""
    n = int(grid[0])
    require(FINE.dtype == torch.uint8 and MEMBERS.dtype == torch.int32 and HASHES.dtype == torch.int64,
            "match_pages: FINE uint8, MEMBERS int32, HASHES int64")
    require(REFS.dtype == torch.int32 and MATCH.dtype == torch.int32, "match_pages: REFS/MATCH int32")
    _lib.call("v1x_match_pages", ptr(TMP), ptr(MAP), ptr(HASH), ptr(META), ptr(FINE), ptr(MEMBERS),
              ptr(HASHES), ptr(REFS), ptr(MATCH), int(CAP), n, _s(TMP), device=TMP.device)


@_op
def allocate(grid, META, MATCH, FREE, COUNT, REFS, TABLES, NEW, status=None, check=None):
    """Pop fresh pages, share matched ones, bump refcounts (DS/kernels.py:116-131).

    status: optional int32 device word (default: the per-device status word).
    check: raise right after the launch (default: when not capturing a graph).
    """
    require(NEW.dtype in (torch.bool, torch.uint8), "NEW: bool [16]")
    require(FREE.dtype == torch.int32 and COUNT.dtype == torch.int32 and TABLES.dtype == torch.int32,
            "allocate: FREE/COUNT/TABLES int32")
    st = status if status is not None else status_word(META.device)
    _lib.call("v1x_allocate", ptr(META), ptr(MATCH), ptr(FREE), ptr(COUNT), ptr(REFS), ptr(TABLES),
              ptr(NEW), ptr(st), _s(META), device=META.device)
    if check is None:
        check = not torch.cuda.is_current_stream_capturing()
    if check and status is None:
        check_status(META.device)


@_op
def publish(grid, TMP, TC, TCS, MAP, HASH, META, TABLES, NEW, FINE, CENTERS, CS, MEMBERS, HASHES):
    """Copy fresh pages + the bucket's centres into the arena (DS/kernels.py:134-167)."""
    require(TCS.dtype == torch.float32 and CS.dtype == torch.float32, "publish: TCS/CS float32 views")
    _lib.call("v1x_publish", ptr(TMP), ptr(TC), ptr(TCS), ptr(MAP), ptr(HASH), ptr(META), ptr(TABLES),
              ptr(NEW), ptr(FINE), ptr(CENTERS), ptr(CS), ptr(MEMBERS), ptr(HASHES), _s(TMP),
              device=TMP.device)


@_op
def release(grid, TABLE, REFS, FREE, COUNT):
    """Drop one lease's references; dead pages return to the free stack (:170-179)."""
    _lib.call("v1x_release", ptr(TABLE), ptr(REFS), ptr(FREE), ptr(COUNT), _s(REFS), device=REFS.device)


# ---------------------------------------------------------------------------
# per-row query metadata and staging
# ---------------------------------------------------------------------------

@_op
def query_lengths(grid, LENS, FLENS, TAKES, MAXTAKE, TOPK, NUM, DEN, SINK, WINDOW):
    """fine_lens / takes per row (DS/kernels.py:224-245). grid = (rows,)."""
    _lib.call("v1x_query_lengths", ptr(LENS), ptr(FLENS), ptr(TAKES), int(TOPK), int(NUM), int(DEN),
              int(SINK), int(WINDOW), int(grid[0]), _s(LENS), device=LENS.device)


def _query_metadata(grid, LENS, NT, FLENS, TAKES, DG_LENS, CENTER_LENS, TAIL_ROWS, NP, TOPK, NUM,
                    DEN, SINK, WINDOW, budget=None):
    _lib.call("v1x_query_metadata", ptr(LENS), ptr(NT), ptr(FLENS), ptr(TAKES), ptr(DG_LENS),
              ptr(CENTER_LENS), ptr(TAIL_ROWS), int(NP), int(TOPK), int(NUM), int(DEN), int(SINK),
              int(WINDOW), ptr(budget) if budget is not None else None, int(grid[0]), _s(LENS),
              device=LENS.device)


query_metadata = _Op(_query_metadata)
query_metadata.__doc__ = "Per-row fine/center lengths, take and shared-tail owner (DS/kernels.py:568-591)."


class BudgetMetadata:
    """Fixed page budget metadata: ``take = min(pages, budget)``
    (reference bench_v1_dynamic_budget_metadata.py:5-34; `budget` is an int32
    device tensor read by the kernel, as in the reference)."""

    def __init__(self, budget):
        self.budget = budget

    def __getitem__(self, grid):
        def launch(*args, **kwargs):
            for k in ("num_warps", "num_stages"):
                kwargs.pop(k, None)
            return _query_metadata(tuple(grid), *args, budget=self.budget, **kwargs)

        return launch


@_op
def fine_table_shared(grid, RT, SELECTED, TAKES, LENS, FT, TAIL_ROWS, CAP, MAXP, TAKE, FP, SCRATCH,
                      B=None):
    """Fine page table: selected pages then the owner's staging pages (:488-514)."""
    _lib.call("v1x_fine_table_shared", ptr(RT), ptr(SELECTED), _sel64(SELECTED), ptr(TAKES), ptr(FT),
              ptr(TAIL_ROWS), int(CAP), int(MAXP), int(TAKE), int(FP), int(SCRATCH), int(grid[0]),
              _s(RT), device=RT.device)


@_op
def stage_tail_shared(grid, NATIVE, NS, NT, LENS, K, KS, TAIL_ROWS, CAP, NP, SCRATCH, SINK, WINDOW,
                      ROWS=0, GROUP=1):
    """Copy each owner row's sink + tail tokens into its staging pages (:518-564).
    grid = (row groups, staging pages per row)."""
    require(NS.dtype == torch.float32 and KS.dtype == torch.float32, "NS/KS must be float32 views")
    g = grid + (1,) * (2 - len(grid))
    _lib.call("v1x_stage_tail_shared", ptr(NATIVE), ptr(NS), ptr(NT), ptr(LENS), ptr(K), ptr(KS),
              ptr(TAIL_ROWS), int(CAP), int(NP), int(SCRATCH), int(SINK), int(WINDOW), int(ROWS),
              int(GROUP), int(g[0]), int(g[1]), _s(NT), device=NT.device)


def query_prepare(LENS, NT, FLENS, TAKES, DG_LENS, CENTER_LENS, TAIL_ROWS, NP, TOPK, NUM, DEN, SINK, WINDOW,
                  NATIVE, NS, K, KS, CAP, SCRATCH, budget=None):
    """Extension: query_metadata + stage_tail_shared in one launch (one program per
    row and group of 4 staging pages).  Same arguments and outputs as the two
    reference ops; `budget` as in BudgetMetadata."""
    require(NS.dtype == torch.float32 and KS.dtype == torch.float32, "NS/KS must be float32 views")
    _lib.call("v1x_query_prepare", ptr(LENS), ptr(NT), ptr(FLENS), ptr(TAKES), ptr(DG_LENS), ptr(CENTER_LENS),
              ptr(TAIL_ROWS), int(NP), int(TOPK), int(NUM), int(DEN), int(SINK), int(WINDOW),
              ptr(budget) if budget is not None else None, ptr(NATIVE), ptr(NS), ptr(K), ptr(KS), int(CAP),
              int(SCRATCH), LENS.shape[0], _s(LENS), device=LENS.device)


@_op
def mask_fine(grid, SCORES, SELECTED, RT, MEMBERS, LENS, TAKES, MAXP, TAKE, STRIDE, WIDTH, SINK,
              WINDOW):
    """Non-fused -inf mask of fine scores (DS/kernels.py:444-472). grid = (rows, .)."""
    _lib.call("v1x_mask_fine", ptr(SCORES), ptr(SELECTED), _sel64(SELECTED), ptr(RT), ptr(MEMBERS),
              ptr(LENS), ptr(TAKES), int(MAXP), int(TAKE), int(STRIDE), int(WIDTH), int(SINK),
              int(WINDOW), int(grid[0]), _s(SCORES), device=SCORES.device)


@_op
def reduce_centers(grid, LOGITS, LENS, SCORES, MAXP, STRIDE):
    """Page max of 8 centre logits (DS/kernels.py:475-486). grid = (rows, pages/32)."""
    pcount = int(grid[1]) * 32 if len(grid) > 1 else int(MAXP)
    _lib.call("v1x_reduce_centers", ptr(LOGITS), ptr(LENS), ptr(SCORES), int(MAXP), pcount, int(STRIDE),
              int(grid[0]), _s(LOGITS), device=LOGITS.device)


@_op
def output_ids(grid, RAW, SCORES, MEMBERS, RT, NT, SELECTED, LENS, TAKES, OUT, LOGICAL, FT, MAXP, NP,
               TAKE, WIDTH, TOPK, SINK, WINDOW, MAP_PHYSICAL=True, DIRECT_FINE=False, FP=0):
    """Non-fused raw -> logical -> physical mapping (DS/kernels.py:323-376)."""
    _lib.call("v1x_output_ids", ptr(RAW), ptr(SCORES), ptr(MEMBERS), ptr(RT), ptr(NT), ptr(SELECTED),
              _sel64(SELECTED), ptr(LENS), ptr(TAKES), ptr(OUT) if MAP_PHYSICAL else None,
              ptr(LOGICAL), ptr(FT), int(MAXP), int(NP), int(TAKE), int(WIDTH), int(TOPK), int(SINK),
              int(WINDOW), int(bool(MAP_PHYSICAL)), int(bool(DIRECT_FINE)), int(FP), int(grid[0]),
              _s(RAW), device=RAW.device)


@_op
def expand_logical(grid, LOGICAL, OUT, TOPK, STRIDE, BLOCK=None):
    """logical p -> 4p..4p+3, -1 padding (DS/kernels.py:594-600)."""
    _lib.call("v1x_expand_logical", ptr(LOGICAL), ptr(OUT), int(TOPK), int(STRIDE), int(grid[0]),
              _s(LOGICAL), device=LOGICAL.device)
