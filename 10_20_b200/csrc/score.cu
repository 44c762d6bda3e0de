// FP8 paged scoring for sm_100a: out[b, j] = sum_h w[b,h] * relu(q[b,h,:] . k_j) * s_j.
//
// Reference contract: DeepGEMM fp8_paged_mqa_logits as called at
// sglang/srt/layers/attention/v1_deepseek/runtime.py:434-444 (centres) and
// :538-548 (fine candidates); the formula is the reference's own restatement in
// kernels.py:310-313 (fine) / :210-213 (coarse), pinned against DeepGEMM at
// experiments/fine_pool_shared_20261021/test_and_bench.py:37-41.
//
// This file holds the SIMT path for few heads (the single-head config is 2
// FLOP/byte).  Eight lanes share a key, each holding 16 of its 128 FP8 bytes, so
// one warp load covers four consecutive keys (512 contiguous bytes) and the row's
// query sits in registers (one head) or shared memory.  Exact e4m3 -> fp32
// conversion and a FIXED fp32 evaluation order make the result bit-identical to
// the CPU oracle: per head, each lane accumulates its 16 products with fma from
// 0 (every e4m3 x e4m3 product is exact in fp32), the eight partial sums combine
// as ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)), then acc += w_h * relu with separately
// rounded multiply and add, then one multiply by the key's scale.
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace v1x {
namespace {

constexpr int kScoreThreads = 128;
constexpr int kSimtMaxHeads = 64;
constexpr int64_t kTcMaxRows = 8192;  // rows the tensor-core scorer takes per call (score_tc.cu)

struct ScoreArgs {
  const uint8_t* q;
  const float* w;
  const uint8_t* pool;
  const int32_t* lens;
  const int32_t* table;
  int64_t table_stride;
  float* out;
  int64_t out_stride, max_len;
  float* page_max;
  int64_t page_stride;
  int heads, relu, clean;
  int lens_kind;
  // flat layout (fp8_mqa_logits): `pool` holds key j at j * 128, `flat_scale`
  // its scale, `lens` the row's end ke and `starts` its start ks
  const float* flat_scale;
  const int32_t* starts;
};

__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Keys per warp iteration: kKeyLoads loads of four keys each.
constexpr int kKeyLoads = 8;
constexpr int kWarpKeys = 4 * kKeyLoads;

// kHeads: 1 compiles the single-head case (the lane's 16 query values in
// registers, 128 registers per thread for four resident CTAs per SM); 0 takes the
// head count from the arguments (up to kSimtMaxHeads) with the query in shared
// memory.  The arithmetic per key is the same.  kFlat: keys and scales in two
// flat arrays instead of pages, and a row scores keys [starts[b], lens[b]).
template <int kHeads, bool kFlat = false>
__global__ void __launch_bounds__(kScoreThreads, kHeads == 1 ? 4 : 1)
    score_simt_kernel(const __grid_constant__ ScoreArgs a) {
  __shared__ __align__(16) float qs[kHeads == 1 ? 4 : kSimtMaxHeads * 128];
  __shared__ float ws[kHeads == 1 ? 1 : kSimtMaxHeads];
  const int64_t b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, part = lane & 7;  // key of the load, 16-byte part of it
  const int H = kHeads ? kHeads : a.heads;
  float qr[kHeads == 1 ? 16 : 1];
  float w0 = 0.0f;
  if constexpr (kHeads == 1) {
    const uint4 qw = reinterpret_cast<const uint4*>(a.q + b * 128)[part];
    const uint32_t q4[4] = {qw.x, qw.y, qw.z, qw.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 lo = e4m3x2_to_float2(static_cast<uint16_t>(q4[u] & 0xFFFFu));
      const float2 hi = e4m3x2_to_float2(static_cast<uint16_t>(q4[u] >> 16));
      qr[4 * u] = lo.x;
      qr[4 * u + 1] = lo.y;
      qr[4 * u + 2] = hi.x;
      qr[4 * u + 3] = hi.y;
    }
    w0 = a.w[b];
  } else {
    for (int i = threadIdx.x; i < H * 64; i += blockDim.x) {
      const uint16_t two = reinterpret_cast<const uint16_t*>(a.q + b * H * 128)[i];
      const float2 f = e4m3x2_to_float2(two);
      qs[2 * i] = f.x;
      qs[2 * i + 1] = f.y;
    }
    for (int h = threadIdx.x; h < H; h += blockDim.x) ws[h] = a.w[b * H + h];
    __syncthreads();
  }
  // A warp takes blocks of kWarpKeys keys (inside one page), striding over the
  // row; the next block's bytes are loaded while the current one is evaluated.
  const int64_t n = score_len(a.lens[b], a.lens_kind);
  const int64_t lim = min(n, a.max_len);  // keys j < lim are scored
  const int64_t lo = kFlat ? max(a.starts[b], 0) : 0;  // and j >= lo
  const int64_t live = (lim + kWarpKeys - 1) / kWarpKeys;  // blocks holding a scored key
  const int64_t wstep = static_cast<int64_t>(gridDim.y) * (kScoreThreads / 32);
  auto load = [&](int64_t blk, uint4 (&kw)[kKeyLoads], float& scale) {
    const int64_t k0 = blk * kWarpKeys;
    if (blk < live) {
      if constexpr (kFlat) {
#pragma unroll
        for (int u = 0; u < kKeyLoads; ++u) {
          const int64_t key = k0 + u * 4 + grp;
          kw[u] = key < lim && key >= lo ? reinterpret_cast<const uint4*>(a.pool + key * 128)[part]
                                         : make_uint4(0, 0, 0, 0);
        }
        const int64_t ks = k0 + lane;
        scale = ks < lim && ks >= lo ? a.flat_scale[ks] : 0.0f;
      } else {
        const int64_t page = a.table[b * a.table_stride + k0 / 64];
        const uint8_t* base = a.pool + page * kPageBytes;
#pragma unroll
        for (int u = 0; u < kKeyLoads; ++u) {
          const int64_t key = k0 + u * 4 + grp;
          kw[u] = key < lim ? reinterpret_cast<const uint4*>(base + (key % 64) * 128)[part] : make_uint4(0, 0, 0, 0);
        }
        const int64_t ks = k0 + lane;  // lane i holds the scale of the block's key i
        scale = ks < lim ? reinterpret_cast<const float*>(base)[kScaleWord + ks % 64] : 0.0f;
      }
    }
  };
  uint4 cur[kKeyLoads], nxt[kKeyLoads];
  float cur_scale = 0.0f, nxt_scale = 0.0f;
  int64_t blk = static_cast<int64_t>(blockIdx.y) * (kScoreThreads / 32) + warp;
  load(blk, cur, cur_scale);
  for (; blk < live; blk += wstep) {
    load(blk + wstep, nxt, nxt_scale);
    const int64_t k0 = blk * kWarpKeys;
    float res[kKeyLoads];
#pragma unroll
    for (int u = 0; u < kKeyLoads; ++u) {
      const uint32_t k4[4] = {cur[u].x, cur[u].y, cur[u].z, cur[u].w};
      float kf[16];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const float2 lo = e4m3x2_to_float2(static_cast<uint16_t>(k4[v] & 0xFFFFu));
        const float2 hi = e4m3x2_to_float2(static_cast<uint16_t>(k4[v] >> 16));
        kf[4 * v] = lo.x;
        kf[4 * v + 1] = lo.y;
        kf[4 * v + 2] = hi.x;
        kf[4 * v + 3] = hi.y;
      }
      float acc = 0.0f;
      for (int h = 0; h < H; ++h) {
        // a zero weight adds +-0, which leaves the sum unchanged (finite
        // inputs): skipped, so zero-padded heads cost nothing
        if constexpr (kHeads != 1) {
          if (ws[h] == 0.0f) continue;
        }
        float p = 0.0f;
        if constexpr (kHeads == 1) {
#pragma unroll
          for (int d = 0; d < 16; ++d) p = __fmaf_rn(qr[d], kf[d], p);
        } else {
          const float4* qh = reinterpret_cast<const float4*>(qs + h * 128 + part * 16);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float4 qq = qh[v];
            p = __fmaf_rn(qq.x, kf[4 * v], p);
            p = __fmaf_rn(qq.y, kf[4 * v + 1], p);
            p = __fmaf_rn(qq.z, kf[4 * v + 2], p);
            p = __fmaf_rn(qq.w, kf[4 * v + 3], p);
          }
        }
        p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 1));
        p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 2));
        p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 4));
        const float r = a.relu ? (p > 0.0f ? p : 0.0f) : p;
        acc = __fadd_rn(acc, __fmul_rn(kHeads == 1 ? w0 : ws[h], r));
      }
      const float scale = __shfl_sync(0xffffffffu, cur_scale, u * 4 + grp);
      const int64_t key = k0 + u * 4 + grp;
      const bool in = key < lim && key >= lo;
      res[u] = in ? __fmul_rn(acc, scale) : -CUDART_INF_F;
      if (part == u && a.out && key < a.max_len && ((key < n && key >= lo) || a.clean))
        a.out[b * a.out_stride + key] = res[u];
    }
    if (a.page_max) {  // max over each group of 8 consecutive keys: loads u, u+1 of the four key lanes
#pragma unroll
      for (int u = 0; u < kKeyLoads; u += 2) {
        float m = fmaxf(res[u], res[u + 1]);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        const int64_t first = k0 + u * 4;
        if (lane == 0 && first < a.max_len) a.page_max[b * a.page_stride + first / 8] = m;
      }
    }
#pragma unroll
    for (int u = 0; u < kKeyLoads; ++u) cur[u] = nxt[u];
    cur_scale = nxt_scale;
  }
  // blocks past the row's length: -inf logits (clean) and page maxima only
  if ((a.out && a.clean) || a.page_max) {
    const int64_t nblk = (a.max_len + kWarpKeys - 1) / kWarpKeys;
    for (; blk < nblk; blk += wstep) {
      const int64_t key = blk * kWarpKeys + lane;
      if (a.out && a.clean && key < a.max_len) a.out[b * a.out_stride + key] = -CUDART_INF_F;
      const int64_t first = blk * kWarpKeys + lane * 8;
      if (a.page_max && lane < kWarpKeys / 8 && first < a.max_len)
        a.page_max[b * a.page_stride + first / 8] = -CUDART_INF_F;
    }
  }
}

}  // namespace

int score_fp8_tc(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                 const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                 float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int lens_kind,
                 int64_t batch, int32_t* status, cudaStream_t stream, int64_t max_ctas);
int mqa_tc_grouped(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale, int64_t keys,
                   const int32_t* win_lo, const int32_t* win_hi, float* out, int64_t out_stride, int64_t group_rows,
                   int64_t real_rows, int relu, int64_t vrows, int32_t* status, cudaStream_t stream);
int score_fp8_tc_grouped(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                         const int32_t* lens, const int32_t* table, int64_t table_stride, int64_t max_len,
                         const int32_t* colmap, int64_t colmap_stride, int64_t colmap_pages,
                         const uint8_t* key_valid, const int32_t* mask_map, const int32_t* mask_pos, float* out,
                         int64_t out_stride, int64_t group_rows, int64_t real_rows, int relu, int64_t vrows,
                         int32_t* status, cudaStream_t stream);

namespace {
int score_dispatch(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                   const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                   float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int impl,
                   int lens_kind, int32_t* status, int64_t batch, void* stream, int64_t max_ctas = 0) {
  clear_error();
  V1X_CHECK_ARG(heads >= 1 && heads <= 256, "score_fp8: heads must be in [1, 256]");
  V1X_CHECK_ARG(batch >= 0 && max_len >= 0 && pool_pages > 0, "score_fp8: bad geometry");
  V1X_CHECK_ARG(!out || out_stride >= max_len, "score_fp8: out row stride < max_len");
  V1X_CHECK_ARG(!page_max || page_stride * 8 >= max_len, "score_fp8: page_max row stride < max_len / 8");
  V1X_CHECK_ARG(out || page_max, "score_fp8: no output requested");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(pool) & 15) == 0, "score_fp8: pool must be 16-byte aligned");
  V1X_CHECK_ARG(table_stride >= 0 && impl >= 0 && impl <= 2, "score_fp8: bad table stride / impl");
  V1X_CHECK_ARG(lens_kind == 0 || lens_kind == 1, "score_fp8: lens_kind must be 0 or 1");
  if (batch == 0 || max_len == 0) return V1X_OK;
  // automatic: the tensor cores where they take the shape (one head, or a
  // multiple of 32 up to 128; batch <= kTcMaxRows; pool < 2^31 pages), else SIMT
  const bool tc_shape = (heads == 1 || (heads % 32 == 0 && heads <= 128)) && batch <= kTcMaxRows &&
                        pool_pages < (int64_t(1) << 31);
  const bool tc = impl == 2 || (impl == 0 && tc_shape);
  if (tc)
    return score_fp8_tc(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                        page_stride, heads, relu, clean, lens_kind, batch, status, as_stream(stream), max_ctas);
  if (heads > kSimtMaxHeads) {
    set_error("score_fp8: the SIMT path takes heads <= %d", kSimtMaxHeads);
    return V1X_ERR_UNSUPPORTED;
  }
  ScoreArgs a{q, w, pool, lens, table, table_stride, out, out_stride, max_len, page_max, page_stride,
              static_cast<int>(heads), relu, clean, lens_kind};
  // CTAs per row: about one wave of resident CTAs over the batch (four per SM),
  // at most one per 128 keys and 8 per row.  Fewer CTAs per row give each warp
  // several blocks, so its next block's loads overlap the current evaluation.
  const int64_t blocks = (max_len + kScoreThreads - 1) / kScoreThreads;  // 128 keys per CTA iteration
  const int64_t wave = static_cast<int64_t>(num_sms()) * 4;
  const int64_t per_row = std::max<int64_t>(1, std::min<int64_t>({(wave + batch - 1) / batch, blocks, 8}));
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(per_row));
  if (heads == 1) launch_kernel(score_simt_kernel<1>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  else launch_kernel(score_simt_kernel<0>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  return launch_status("v1x_score_fp8");
}

int mqa_flat(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale, int64_t kv_len,
             const int32_t* starts, const int32_t* ends, float* out, int64_t out_stride, int64_t heads, int relu,
             int clean, int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(heads >= 1 && heads <= kSimtMaxHeads, "mqa_logits: heads must be in [1, 64]");
  V1X_CHECK_ARG(batch >= 0 && kv_len >= 0 && out_stride >= kv_len, "mqa_logits: bad geometry");
  V1X_CHECK_ARG(batch < (int64_t(1) << 31), "mqa_logits: too many rows");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(k) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0,
                "mqa_logits: q and k must be 16-byte aligned");
  if (batch == 0 || kv_len == 0) return V1X_OK;
  ScoreArgs a{q, w, k, ends, nullptr, 0, out, out_stride, kv_len, nullptr, 0,
              static_cast<int>(heads), relu, clean, 0, k_scale, starts};
  const int64_t blocks = (kv_len + kScoreThreads - 1) / kScoreThreads;
  const int64_t wave = static_cast<int64_t>(num_sms()) * 4;
  const int64_t per_row = std::max<int64_t>(1, std::min<int64_t>({(wave + batch - 1) / batch, blocks, 8}));
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(per_row));
  if (heads == 1) launch_kernel(score_simt_kernel<1, true>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  else launch_kernel(score_simt_kernel<0, true>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  return launch_status("v1x_mqa_logits_fp8");
}
// Column map of the grouped scorer, page-major: colmap[p, r] (row stride
// `cstride`) = a column c of row r whose page table entry is p (-1: none).
// Every other column of the row -- a second column of the same page, or a page
// outside the pool -- is listed in `fix` as (row, column, source column or -1)
// behind a count in fix[0].
__global__ void column_map_kernel(const int32_t* __restrict__ tables, int64_t tstride, int64_t cols, int64_t rows,
                                  int64_t pool_pages, int64_t cstride, int32_t* __restrict__ colmap,
                                  int32_t* __restrict__ fix) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * cols) return;
  const int64_t r = t / cols, c = t % cols;
  const int64_t p = tables[r * tstride + c];
  int old = -1;
  if (p >= 0 && p < pool_pages) {
    old = atomicCAS(&colmap[p * cstride + r], -1, static_cast<int>(c));
    if (old == -1) return;
  }
  const int k = atomicAdd(fix, 1);
  fix[1 + 3 * k] = static_cast<int>(r);
  fix[2 + 3 * k] = static_cast<int>(c);
  fix[3 + 3 * k] = old;
}

// The listed columns: a copy of the source column's 64 logits (the same page's
// keys), or for a page outside the pool zeros (what the per-row scorer's
// zero-filled loads give) -- -inf when the mask is applied (no token there).
// One warp per entry.
__global__ void fix_columns_kernel(const int32_t* __restrict__ fix, float* __restrict__ out, int64_t out_stride,
                                   float outside) {
  const int n = fix[0];
  const int lane = threadIdx.x & 31;
  for (int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; e < n; e += (gridDim.x * blockDim.x) >> 5) {
    const int64_t r = fix[1 + 3 * e], c = fix[2 + 3 * e], src = fix[3 + 3 * e];
    float* row = out + r * out_stride;
    for (int j = lane; j < 64; j += 32) row[c * 64 + j] = src >= 0 ? row[src * 64 + j] : outside;
  }
}
}  // namespace
}  // namespace v1x

extern "C" int v1x_score_fp8_grouped(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                                     int64_t keys, const int32_t* table, const int32_t* row_tables,
                                     int64_t row_table_stride, int64_t row_table_cols, const uint8_t* key_valid,
                                     const int32_t* mask_map, const int32_t* mask_pos, int32_t* workspace,
                                     float* out, int64_t out_stride,
                                     int64_t heads, int64_t group_rows, int64_t rows, int relu, int32_t* status,
                                     void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(heads == 4, "score_fp8_grouped: four heads per query row");
  V1X_CHECK_ARG(group_rows == 8 || group_rows == 16 || group_rows == 32,
                "score_fp8_grouped: group_rows must be 8, 16 or 32");
  V1X_CHECK_ARG(rows >= 0 && keys >= 0 && pool_pages > 0 && pool_pages < (int64_t(1) << 31),
                "score_fp8_grouped: bad geometry");
  V1X_CHECK_ARG(table, "score_fp8_grouped: the shared key table is required");
  V1X_CHECK_ARG(!(key_valid && row_tables), "score_fp8_grouped: key_valid applies without row tables only");
  V1X_CHECK_ARG(!mask_map || (row_tables && mask_pos), "score_fp8_grouped: the mask needs row tables and positions");
  const int64_t vrows = (rows + group_rows - 1) / group_rows;
  V1X_CHECK_ARG(vrows <= kTcMaxRows, "score_fp8_grouped: too many rows");
  if (row_tables) {
    V1X_CHECK_ARG(workspace && row_table_cols >= 0 && row_table_stride >= row_table_cols &&
                      out_stride >= row_table_cols * 64,
                  "score_fp8_grouped: bad row tables / workspace / out stride");
    V1X_CHECK_ARG(rows * row_table_cols < (int64_t(1) << 31) / 3, "score_fp8_grouped: row tables too large");
  } else {
    V1X_CHECK_ARG(out_stride >= keys, "score_fp8_grouped: out row stride < keys");
  }
  if (rows == 0 || keys == 0 || (row_tables && row_table_cols == 0)) return V1X_OK;
  cudaStream_t s = as_stream(stream);
  int32_t* colmap = nullptr;
  int32_t* fix = nullptr;
  const int64_t padded = vrows * group_rows;
  if (row_tables) {
    colmap = workspace;
    fix = workspace + pool_pages * padded;
    cudaMemsetAsync(colmap, 0xFF, static_cast<size_t>(pool_pages * padded) * 4, s);
    cudaMemsetAsync(fix, 0, 4, s);
    const int64_t n = rows * row_table_cols;
    column_map_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
        row_tables, row_table_stride, row_table_cols, rows, pool_pages, padded, colmap, fix);
    if (int rc = launch_status("v1x_score_fp8_grouped (column map)")) return rc;
  }
  if (int rc = score_fp8_tc_grouped(q, w, pool, pool_pages, nullptr, table, 0, keys, colmap, padded, pool_pages,
                                    key_valid, mask_map, mask_pos, out, out_stride, group_rows, rows, relu, vrows,
                                    status, s))
    return rc;
  if (row_tables) {
    fix_columns_kernel<<<static_cast<unsigned>(num_sms()), 256, 0, s>>>(fix, out, out_stride,
                                                                         mask_map ? -INFINITY : 0.0f);
    return launch_status("v1x_score_fp8_grouped (fix columns)");
  }
  return V1X_OK;
}

extern "C" int v1x_score_fp8(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                             const int32_t* lens, const int32_t* table, int64_t table_stride,
                             float* out, int64_t out_stride, int64_t max_len, float* page_max,
                             int64_t page_stride, int64_t heads, int relu, int clean, int impl,
                             int32_t* status, int64_t batch, void* stream) {
  return v1x::score_dispatch(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                             page_stride, heads, relu, clean, impl, 0, status, batch, stream);
}

extern "C" int v1x_score_fp8_ex(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                                const int32_t* lens, const int32_t* table, int64_t table_stride,
                                float* out, int64_t out_stride, int64_t max_len, float* page_max,
                                int64_t page_stride, int64_t heads, int relu, int clean, int impl,
                                int lens_kind, int64_t max_ctas, int32_t* status, int64_t batch, void* stream) {
  using namespace v1x;
  V1X_CHECK_ARG(max_ctas >= 0, "score_fp8: max_ctas must be >= 0");
  return v1x::score_dispatch(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                             page_stride, heads, relu, clean, impl, lens_kind, status, batch, stream, max_ctas);
}

extern "C" int v1x_mqa_logits_fp8(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale,
                                  int64_t kv_len, const int32_t* starts, const int32_t* ends, float* out,
                                  int64_t out_stride, int64_t heads, int relu, int clean, int64_t batch,
                                  void* stream) {
  return v1x::mqa_flat(q, w, k, k_scale, kv_len, starts, ends, out, out_stride, heads, relu, clean, batch, stream);
}

extern "C" int v1x_mqa_logits_fp8_grouped(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale,
                                          int64_t kv_len, const int32_t* starts, const int32_t* ends, float* out,
                                          int64_t out_stride, int64_t heads, int64_t group_rows, int64_t rows,
                                          int relu, int32_t* status, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(heads == 4, "mqa_logits_grouped: four heads per query row");
  V1X_CHECK_ARG(group_rows == 8 || group_rows == 16 || group_rows == 32,
                "mqa_logits_grouped: group_rows must be 8, 16 or 32");
  V1X_CHECK_ARG(rows >= 0 && kv_len >= 0 && out_stride >= kv_len && kv_len < (int64_t(1) << 31) - 128,
                "mqa_logits_grouped: bad geometry");
  V1X_CHECK_ARG(((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(k_scale)) & 15) == 0,
                "mqa_logits_grouped: k and k_scale must be 16-byte aligned");
  V1X_CHECK_ARG(starts && ends, "mqa_logits_grouped: starts and ends are required");
  const int64_t vrows = (rows + group_rows - 1) / group_rows;
  V1X_CHECK_ARG(vrows <= kTcMaxRows, "mqa_logits_grouped: too many rows");
  if (rows == 0 || kv_len == 0) return V1X_OK;
  return mqa_tc_grouped(q, w, k, k_scale, kv_len, starts, ends, out, out_stride, group_rows, rows, relu, vrows,
                        status, as_stream(stream));
}
