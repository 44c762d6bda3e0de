"""FP8 paged index scoring with the DeepGEMM ``fp8_paged_mqa_logits`` contract.

The reference calls DeepGEMM (an external, unvendored dependency) at
sglang/srt/layers/attention/v1_deepseek/runtime.py:434-444 (centre logits) and
:538-548 (fine logits); its formula is restated by the reference at
kernels.py:310-313 and pinned against DeepGEMM at
experiments/fine_pool_shared_20261021/test_and_bench.py:37-41:

    logits[b, j] = sum_h w[b, h] * relu(q[b, h, :] . k_j) * scale_j,  j < len[b]

This module mirrors the DeepGEMM call surface used there (next_n = 1) and runs
libv1x.so's sm_100a kernel.  The schedule argument is accepted for signature
compatibility and ignored: the kernel needs no host-built schedule.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import ptr, require


def get_paged_mqa_logits_metadata(context_lens: torch.Tensor, block_size: int, num_sms: int):
    """Signature-compatible schedule stub: an int32 [num_sms + 1, 2] zero tensor."""
    require(block_size == 64, "only 64-token pages are supported")
    return torch.zeros((num_sms + 1, 2), dtype=torch.int32, device=context_lens.device)


IMPLS = {"auto": 0, "simt": 1, "tensor_core": 2}
LENS_KINDS = {"tokens": 0, "centres": 1}


def fp8_paged_mqa_logits(q, kv_cache, weights, context_lens, block_table, schedule_meta,
                         max_context_len: int, clean_logits: bool = True, relu: bool = True,
                         out: torch.Tensor | None = None, impl: str = "auto",
                         page_max: torch.Tensor | None = None, logits: bool = True,
                         lens_kind: str = "tokens", max_ctas: int = 0):
    """Logits [B, max_context_len] (float32); columns >= context_lens[b] are -inf.

    q: e4m3 [B, H, 128] or [B, 1, H, 128]; kv_cache: packed uint8 [pages, 8448] or
    [pages, 64, 1, 132]; weights: float32 [B, H]; context_lens: int32 [B] or [B, 1];
    block_table: int32 [B, max_blocks].  impl: "auto" (tensor cores when H is a
    multiple of 32, or 1), "simt" (fixed fp32 evaluation order, H <= 64) or "tensor_core".
    clean_logits=False leaves columns >= context_lens[b] untouched.
    page_max (extension): float32 [B, >= ceil(max_context_len / 8)] receiving the max of
    every 8 consecutive logits (fused.route's page score); logits=False skips the
    logits output (then `page_max` is required and the call returns it).
    lens_kind (extension): "tokens" scores context_lens[b] keys; "centres" scores
    the centre count of a token length n, max(8 * ((n-1)//1024*16), 1) -- the
    center_lens the query metadata derives (DS/kernels.py:589) -- so centre scoring
    can take the raw token lengths and need not wait for the metadata kernel.
    max_ctas (extension): > 0 caps the tensor-core scorer's persistent grid.
    """
    if q.dim() == 4:
        require(q.shape[1] == 1, "only next_n == 1 is supported")
        q = q[:, 0]
    require(q.dim() == 3 and q.shape[2] == 128, "q: [B, H, 128]")
    require(q.dtype in (torch.float8_e4m3fn, torch.uint8), "q: float8_e4m3fn")
    require(q.is_contiguous(), "q must be contiguous")
    B, H = q.shape[0], q.shape[1]
    require(kv_cache.dtype == torch.uint8 and kv_cache.is_contiguous() and kv_cache.numel() % 8448 == 0,
            "kv_cache: contiguous packed uint8 pages of 8448 bytes")
    require(weights.shape == (B, H) and weights.dtype == torch.float32 and weights.is_contiguous(),
            "weights: float32 [B, H]")
    lens = context_lens.reshape(-1)
    require(lens.numel() == B and lens.dtype == torch.int32, "context_lens: int32 [B]")
    require(block_table.dim() == 2 and block_table.shape[0] == B and block_table.dtype == torch.int32
            and block_table.stride(1) == 1, "block_table: int32 [B, max_blocks]")
    if logits:
        if out is None:
            out = torch.empty((B, max_context_len), dtype=torch.float32, device=q.device)
        require(out.dtype == torch.float32 and out.stride(1) == 1 and out.shape[1] >= max_context_len,
                "out: float32 [B, >= max_context_len]")
    else:
        require(page_max is not None, "logits=False needs page_max")
        out = None
    if page_max is not None:
        require(page_max.dtype == torch.float32 and page_max.stride(1) == 1 and page_max.shape[0] == B
                and page_max.shape[1] * 8 >= max_context_len, "page_max: float32 [B, >= max_len/8]")
    require(lens_kind in LENS_KINDS, "lens_kind: 'tokens' or 'centres'")
    from .kernels import status_word
    _lib.call("v1x_score_fp8_ex", ptr(q), ptr(weights), ptr(kv_cache), kv_cache.numel() // 8448, ptr(lens),
              ptr(block_table), block_table.stride(0), ptr(out), out.stride(0) if out is not None else 0,
              int(max_context_len), ptr(page_max), page_max.stride(0) if page_max is not None else 0, H,
              int(bool(relu)), int(bool(clean_logits)), IMPLS[impl], LENS_KINDS[lens_kind], int(max_ctas),
              ptr(status_word(q.device)), B,
              _lib.stream_of(q), device=q.device)
    return out if logits else page_max


def fp8_mqa_logits(q, kv, weights, cu_seqlen_ks, cu_seqlen_ke, clean_logits: bool = True, relu: bool = True,
                   out: torch.Tensor | None = None):
    """DeepGEMM ``fp8_mqa_logits`` over a flat key array, as the signed-score
    Scorer's ``dsa`` mode (NA/scoring.py:74-78) and the probe backend
    (qwen_gqa_probe_backend.py:184) call it: logits [M, N] float32 with
    logits[i, j] = sum_h w[i, h] * relu(q[i, h, :] . k[j]) * k_scale[j] for
    ks[i] <= j < ke[i] (-inf elsewhere when clean_logits, else untouched).

    q: e4m3 [M, H, 128] (H <= 64); kv = (k e4m3 [N, 128], k_scale float32 [N]);
    weights float32 [M, H]; cu_seqlen_ks / cu_seqlen_ke int32 [M].  relu=False
    (extension) is the signed variant the Scorer uses.
    """
    k, k_scale = kv
    require(q.dim() == 3 and q.shape[2] == 128 and q.dtype in (torch.float8_e4m3fn, torch.uint8)
            and q.is_contiguous(), "q: contiguous float8_e4m3fn [M, H, 128]")
    M, H = q.shape[0], q.shape[1]
    require(k.dim() == 2 and k.shape[1] == 128 and k.dtype in (torch.float8_e4m3fn, torch.uint8)
            and k.is_contiguous(), "kv[0]: contiguous float8_e4m3fn [N, 128]")
    N = k.shape[0]
    k_scale = k_scale.reshape(-1)
    require(k_scale.numel() == N and k_scale.dtype == torch.float32 and k_scale.is_contiguous(),
            "kv[1]: float32 [N]")
    require(weights.shape == (M, H) and weights.dtype == torch.float32 and weights.is_contiguous(),
            "weights: float32 [M, H]")
    for name, t in (("cu_seqlen_ks", cu_seqlen_ks), ("cu_seqlen_ke", cu_seqlen_ke)):
        require(t.shape == (M,) and t.dtype == torch.int32 and t.is_contiguous(), f"{name}: int32 [M]")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=q.device)
    require(out.dtype == torch.float32 and out.dim() == 2 and out.shape[0] == M and out.shape[1] >= N
            and out.stride(1) == 1, "out: float32 [M, >= N]")
    _lib.same_device(q, k, k_scale, weights, cu_seqlen_ks, cu_seqlen_ke, out)
    _lib.call("v1x_mqa_logits_fp8", ptr(q), ptr(weights), ptr(k), ptr(k_scale), N, ptr(cu_seqlen_ks),
              ptr(cu_seqlen_ke), ptr(out), out.stride(0), H, int(bool(relu)), int(bool(clean_logits)), M,
              _lib.stream_of(q), device=q.device)
    return out


def paged_logits_grouped(q8, weights, kv_cache, table, keys: int, out, row_tables=None, group_rows: int = 32,
                         relu: bool = False, rows: int | None = None, key_valid=None, mask=None):
    """Extension: the signed-score Scorer's paged logits for query rows of four
    heads that share one key table (``v1x_score_fp8_grouped``).  q8 e4m3 [R, 4,
    128] and weights float32 [R, 4] with R a multiple of group_rows (rows past
    ``rows`` zero); table int32 [>= ceil(keys / 64)] of pool pages.  Without
    ``row_tables``: out[r, j] = the logit of key j (j < keys).  With
    ``row_tables`` int32 [rows, P]: out[r, c] = the logit of key (row_tables[r,
    c // 64], c % 64) for c < 64 * P, every page a row names being in ``table``.
    ``key_valid`` (bool / uint8 [>= keys], without row tables): logits of the
    keys where it is 0 are -inf.  ``mask`` = (mapping int32 [pool pages * 64],
    positions int32 [rows]) with row tables: ``gather.mask_scores(out, row_tables,
    mapping, positions)`` applied in the same pass."""
    R = q8.shape[0]
    rows = R if rows is None else int(rows)
    require(q8.dim() == 3 and q8.shape[1:] == (4, 128) and q8.is_contiguous()
            and q8.dtype in (torch.float8_e4m3fn, torch.uint8), "q8: contiguous e4m3 [R, 4, 128]")
    require(weights.shape == (R, 4) and weights.dtype == torch.float32 and weights.is_contiguous(),
            "weights: contiguous float32 [R, 4]")
    require(R % group_rows == 0 and rows <= R, "q8 rows: a multiple of group_rows, at least rows")
    require(kv_cache.dtype == torch.uint8 and kv_cache.is_contiguous() and kv_cache.numel() % 8448 == 0,
            "kv_cache: contiguous packed uint8 pages of 8448 bytes")
    require(table.dtype == torch.int32 and table.dim() == 1 and table.is_contiguous()
            and table.numel() * 64 >= keys, "table: int32 [>= ceil(keys / 64)]")
    require(out.dtype == torch.float32 and out.dim() == 2 and out.shape[0] >= rows and out.stride(1) == 1,
            "out: float32 [rows, -1]")
    pool_pages = kv_cache.numel() // 8448
    ws = None
    if row_tables is not None:
        require(row_tables.dtype == torch.int32 and row_tables.dim() == 2 and row_tables.shape[0] == rows
                and row_tables.stride(1) == 1, "row_tables: int32 [rows, P]")
        P = row_tables.shape[1]
        require(out.shape[1] >= P * 64, "out: at least 64 columns per row-table page")
        padded = -(-rows // group_rows) * group_rows
        ws = torch.empty(padded * pool_pages + 1 + 3 * rows * P, dtype=torch.int32, device=q8.device)
    else:
        require(out.shape[1] >= keys, "out: at least `keys` columns")
    if key_valid is not None:
        require(row_tables is None, "key_valid applies without row tables")
        require(key_valid.dtype in (torch.bool, torch.uint8) and key_valid.is_contiguous()
                and key_valid.numel() >= keys, "key_valid: contiguous bool / uint8 [>= keys]")
        key_valid = key_valid.view(torch.uint8)
    mmap = mpos = None
    if mask is not None:
        mmap, mpos = mask
        require(row_tables is not None, "mask applies with row tables")
        require(mmap.dtype == torch.int32 and mmap.is_contiguous() and mmap.numel() >= pool_pages * 64,
                "mask mapping: contiguous int32 [pool pages * 64]")
        require(mpos.dtype == torch.int32 and mpos.is_contiguous() and mpos.numel() >= rows, "positions: int32 [rows]")
    from .kernels import status_word
    _lib.same_device(q8, weights, kv_cache, table, out, row_tables, key_valid, mmap, mpos)
    _lib.call("v1x_score_fp8_grouped", ptr(q8), ptr(weights), ptr(kv_cache), pool_pages, int(keys), ptr(table),
              ptr(row_tables), row_tables.stride(0) if row_tables is not None else 0,
              row_tables.shape[1] if row_tables is not None else 0, ptr(key_valid), ptr(mmap), ptr(mpos), ptr(ws),
              ptr(out), out.stride(0), 4,
              int(group_rows), rows, int(bool(relu)), ptr(status_word(q8.device)), _lib.stream_of(q8),
              device=q8.device)
    return out


def mqa_logits_grouped(q8, weights, kv, cu_seqlen_ks, cu_seqlen_ke, rows: int | None = None, group_rows: int = 32,
                       relu: bool = False, out=None):
    """Extension: ``fp8_mqa_logits(..., clean_logits=True)`` for query rows of
    four heads on the tensor cores (``v1x_mqa_logits_fp8_grouped``).  q8 e4m3
    [R, 4, 128] and weights float32 [R, 4], R a multiple of group_rows, rows
    past ``rows`` zero; kv = (k e4m3 [N, 128], k_scale float32 [N]); returns
    logits [rows, N], -inf outside [ks[r], ke[r])."""
    k, k_scale = kv
    R = q8.shape[0]
    rows = R if rows is None else int(rows)
    require(q8.dim() == 3 and q8.shape[1:] == (4, 128) and q8.is_contiguous()
            and q8.dtype in (torch.float8_e4m3fn, torch.uint8), "q8: contiguous e4m3 [R, 4, 128]")
    require(weights.shape == (R, 4) and weights.dtype == torch.float32 and weights.is_contiguous(),
            "weights: contiguous float32 [R, 4]")
    require(R % group_rows == 0 and rows <= R, "q8 rows: a multiple of group_rows, at least rows")
    require(k.dim() == 2 and k.shape[1] == 128 and k.dtype in (torch.float8_e4m3fn, torch.uint8)
            and k.is_contiguous(), "kv[0]: contiguous float8_e4m3fn [N, 128]")
    N = k.shape[0]
    k_scale = k_scale.reshape(-1)
    require(k_scale.numel() == N and k_scale.dtype == torch.float32 and k_scale.is_contiguous(),
            "kv[1]: float32 [N]")
    for name, t in (("cu_seqlen_ks", cu_seqlen_ks), ("cu_seqlen_ke", cu_seqlen_ke)):
        require(t.dtype == torch.int32 and t.is_contiguous() and t.numel() >= rows, f"{name}: int32 [rows]")
    if out is None:
        out = torch.empty((rows, N), dtype=torch.float32, device=q8.device)
    require(out.dtype == torch.float32 and out.dim() == 2 and out.shape[0] >= rows and out.shape[1] >= N
            and out.stride(1) == 1, "out: float32 [rows, >= N]")
    from .kernels import status_word
    _lib.same_device(q8, weights, k, k_scale, cu_seqlen_ks, cu_seqlen_ke, out)
    _lib.call("v1x_mqa_logits_fp8_grouped", ptr(q8), ptr(weights), ptr(k), ptr(k_scale), N, ptr(cu_seqlen_ks),
              ptr(cu_seqlen_ke), ptr(out), out.stride(0), 4, int(group_rows), rows, int(bool(relu)),
              ptr(status_word(q8.device)), _lib.stream_of(q8), device=q8.device)
    return out
