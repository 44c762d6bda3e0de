// Per-row query metadata, fine page tables, shared sink/tail staging and the
// non-fused mask / mapping kernels for sm_100a.
//
// Reference behaviour (sglang/srt/layers/attention/v1_deepseek/kernels.py):
//   query_lengths :224-245, output_ids :323-376, mask_fine :444-472,
//   reduce_centers :475-486, fine_table_shared :488-514,
//   stage_tail_shared :518-564, query_metadata :568-591, expand_logical :594-600;
//   the fixed-budget take rule of bench_v1_dynamic_budget_metadata.py:5-27.
// All index arithmetic is 64-bit (the pools exceed 2 GiB).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>

#include "common.cuh"

namespace v1x {
namespace {

__device__ __forceinline__ int64_t take_rule(int64_t pages, int64_t topk, int64_t num, int64_t den,
                                             const int32_t* budget) {
  if (budget) return min(pages, static_cast<int64_t>(*budget));
  return min(pages, max((pages * num + den - 1) / den, (topk + 63) / 64));
}

struct MetaArgs {
  const int32_t* lens;
  const int32_t* nt;
  int32_t* fine_lens;
  int32_t* takes;
  int32_t* dg_lens;
  int32_t* center_lens;
  int32_t* tail_rows;
  int64_t np, topk, num, den, sink_cfg, window;
  const int32_t* budget;
};

struct RowMeta {
  int n;
  RowBounds rb;
  int64_t pages, take, fine;
  bool owner;  // tail_rows[row] == row: the row stages its own sink/tail pages
};

// Per-row metadata (:568-591) computed by one CTA (threads 0..127 take part in
// the page-id comparison).
__device__ __forceinline__ RowMeta row_meta(const MetaArgs& a, int64_t row) {
  RowMeta m;
  m.n = a.lens[row];
  m.pages = static_cast<int64_t>(max(m.n - 1, 0) / 1024) * 16;
  m.take = take_rule(m.pages, a.topk, a.num, a.den, a.budget);
  m.rb = row_bounds(m.n, static_cast<int>(a.sink_cfg), static_cast<int>(a.window));
  m.fine = m.take * 64 + m.rb.sink + m.n - m.rb.tail;
  // share the staging copy with row 0 only if the length and every page id the
  // sink/tail copy touches are identical (:583-591)
  const int i = threadIdx.x;
  const int64_t page = i == 0 ? 0 : m.rb.tail / 64 + i - 1;
  const bool valid = i < 128 && (m.n > 0) && ((i == 0) || (page < (static_cast<int64_t>(m.n) + 63) / 64)) &&
                     (page < a.np);
  const int mine = valid ? a.nt[row * a.np + page] : -1;
  const int first = valid ? a.nt[page] : -1;
  const int differs = __syncthreads_or(mine != first);
  const bool share = (m.n == a.lens[0]) && !differs;
  m.owner = !share || row == 0;
  return m;
}

__device__ __forceinline__ void write_meta(const MetaArgs& a, int64_t row, const RowMeta& m) {
  a.fine_lens[row] = static_cast<int32_t>(m.fine);
  a.takes[row] = static_cast<int32_t>(m.take);
  a.dg_lens[row] = static_cast<int32_t>(max(m.fine, int64_t(1)));
  a.center_lens[row] = static_cast<int32_t>(max(m.pages * 8, int64_t(1)));
  a.tail_rows[row] = m.owner ? static_cast<int32_t>(row) : 0;
}

__global__ void __launch_bounds__(128) query_metadata_kernel(const __grid_constant__ MetaArgs a) {
  const int64_t row = blockIdx.x;
  const RowMeta m = row_meta(a, row);
  if (threadIdx.x == 0) write_meta(a, row, m);
}

__global__ void query_lengths_kernel(const int32_t* __restrict__ lens, int32_t* __restrict__ fine_lens,
                                     int32_t* __restrict__ takes, int64_t topk, int64_t num,
                                     int64_t den, int64_t sink_cfg, int64_t window, int64_t batch) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= batch) return;
  const int n = lens[row];
  const int64_t pages = static_cast<int64_t>(max(n - 1, 0) / 1024) * 16;
  const int64_t take = take_rule(pages, topk, num, den, nullptr);
  const RowBounds rb = row_bounds(n, static_cast<int>(sink_cfg), static_cast<int>(window));
  fine_lens[row] = static_cast<int32_t>(take * 64 + rb.sink + n - rb.tail);
  takes[row] = static_cast<int32_t>(take);
}

__global__ void fine_table_shared_kernel(const int32_t* __restrict__ rt, const void* selected,
                                         int sel64, const int32_t* __restrict__ takes,
                                         int32_t* __restrict__ ft, const int32_t* __restrict__ tail_rows,
                                         int64_t cap, int64_t maxp, int64_t take_stride, int64_t fp,
                                         int64_t scratch) {
  const int64_t row = blockIdx.x;
  const int take = takes[row];
  const int64_t pad_base = cap + static_cast<int64_t>(tail_rows[row]) * scratch;
  for (int64_t j = threadIdx.x; j < fp; j += blockDim.x) {
    int64_t page;
    if (j < take) {
      const int64_t rank = load_index(selected, sel64, row * take_stride + j);
      page = rt[row * maxp + rank];
    } else {
      page = pad_base + min(max(j - take, int64_t(0)), scratch - 1);
    }
    ft[row * fp + j] = static_cast<int32_t>(page);
  }
}

struct StageArgs {
  const uint8_t* native;
  const float* nscale;
  const int32_t* nt;
  const int32_t* lens;
  uint8_t* fine;
  float* fscale;
  const int32_t* tail_rows;
  int64_t cap, np, scratch, sink, window, rows_bound, group;
};

// Staging of each owner row's sink + tail candidates (:535-564).  The
// reference runs programs (group, page) that loop over the group's owner rows;
// rows write disjoint staging pages, so the order is free: here one CTA takes
// one row and kStagePages consecutive staging pages, copies every needed 16-byte
// chunk with several loads in flight, and zero-fills masked slots exactly as the
// reference does (pages p with p*64 < count, plus page 0).
constexpr int kStagePages = 4;

// Copies staging pages [p0, p1) of an owner row (any block size).
__device__ __forceinline__ void stage_pages(const StageArgs& a, int64_t row, const RowBounds& rb, int count, int p0,
                                            int p1) {
  const int chunks = (p1 - p0) * 512;
  constexpr int U = 4;
  for (int c0 = threadIdx.x; c0 < chunks; c0 += blockDim.x * U) {
    uint4 v[U];
    int64_t dst[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * blockDim.x;
      v[u] = make_uint4(0, 0, 0, 0);
      dst[u] = -1;
      if (c < chunks) {
        const int p = p0 + c / 512, tok = (c % 512) >> 3, part = c & 7;
        const int i = p * 64 + tok;
        if (i < count) {
          const int logical = i < rb.sink ? i : rb.tail + i - rb.sink;
          const int64_t page = a.nt[row * a.np + logical / 64];
          v[u] = reinterpret_cast<const uint4*>(a.native + page * kPageBytes + (logical % 64) * 128)[part];
        }
        dst[u] = (a.cap + row * a.scratch + p) * kPageBytes + tok * 128 + part * 16;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (dst[u] >= 0) *reinterpret_cast<uint4*>(a.fine + dst[u]) = v[u];
  }
  for (int e = threadIdx.x; e < (p1 - p0) * 64; e += blockDim.x) {
    const int p = p0 + e / 64, tok = e % 64;
    const int i = p * 64 + tok;
    float s = 0.0f;
    if (i < count) {
      const int logical = i < rb.sink ? i : rb.tail + i - rb.sink;
      const int64_t page = a.nt[row * a.np + logical / 64];
      s = a.nscale[page * kPageWords + kScaleWord + logical % 64];
    }
    a.fscale[(a.cap + row * a.scratch + p) * kPageWords + kScaleWord + tok] = s;
  }
}

__global__ void __launch_bounds__(256) stage_tail_shared_kernel(const __grid_constant__ StageArgs a,
                                                                int64_t grid_pages) {
  const int64_t row = blockIdx.x;
  if (a.rows_bound > 0 && row >= a.rows_bound) return;
  if (a.tail_rows[row] != row) return;
  const int n = a.lens[row];
  const RowBounds rb = row_bounds(n, static_cast<int>(a.sink), static_cast<int>(a.window));
  const int count = rb.sink + n - rb.tail;
  const int64_t need = min(grid_pages, static_cast<int64_t>(max((count + 63) / 64, 1)));
  const int p0 = blockIdx.y * kStagePages;
  const int p1 = static_cast<int>(min(need, static_cast<int64_t>(p0 + kStagePages)));
  if (p0 >= p1) return;
  stage_pages(a, row, rb, count, p0, p1);
}

// Metadata + sink/tail staging in one launch: CTA (row, g) derives the row's
// metadata itself (row 0's page ids decide the shared-tail owner), CTAs with
// g == 0 write it, and an owner row's CTAs stage pages [4g, 4g + 4).  Equal to
// query_metadata followed by stage_tail_shared (every owner row stages its own
// pages; the reference's row grouping only changes which program copies them).
// Light CTAs (128 threads, no shared memory), so the centre scorer launched
// next can be resident beside them.
__global__ void __launch_bounds__(128) query_prepare_kernel(const __grid_constant__ MetaArgs m,
                                                            const __grid_constant__ StageArgs s) {
  const int64_t row = blockIdx.x;
  const RowMeta r = row_meta(m, row);
  if (blockIdx.y == 0 && threadIdx.x == 0) write_meta(m, row, r);
  if (!r.owner) return;
  const int count = r.rb.sink + r.n - r.rb.tail;
  const int64_t need = min(s.scratch, static_cast<int64_t>(max((count + 63) / 64, 1)));
  for (int p0 = blockIdx.y * kStagePages; p0 < need; p0 += gridDim.y * kStagePages) {
    const int p1 = static_cast<int>(min(need, static_cast<int64_t>(p0 + kStagePages)));
    stage_pages(s, row, r.rb, count, p0, p1);
  }
}

__global__ void mask_fine_kernel(float* __restrict__ scores, const void* selected, int sel64,
                                 const int32_t* __restrict__ rt, const int32_t* __restrict__ members,
                                 const int32_t* __restrict__ lens, const int32_t* __restrict__ takes,
                                 int64_t maxp, int64_t take_stride, int64_t stride, int64_t width,
                                 int64_t sink_cfg, int64_t window) {
  const int64_t row = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  if (j >= width) return;
  const int n = lens[row];
  const int take = takes[row];
  const RowBounds rb = row_bounds(n, static_cast<int>(sink_cfg), static_cast<int>(window));
  const int64_t count = static_cast<int64_t>(take) * 64 + rb.sink + n - rb.tail;
  const bool fine = j < static_cast<int64_t>(take) * 64;
  bool good = j < count;
  if (fine && good) {
    const int64_t rank = load_index(selected, sel64, row * take_stride + j / 64);
    const int64_t page = rt[row * maxp + rank];
    const int logical = members[page * 64 + j % 64];
    good = logical >= rb.sink && logical < rb.tail;
  }
  if (!good) scores[row * stride + j] = -CUDART_INF_F;
}

__global__ void reduce_centers_kernel(const float* __restrict__ logits, const int32_t* __restrict__ lens,
                                      float* __restrict__ out, int64_t maxp, int64_t cols, int64_t stride) {
  const int64_t row = blockIdx.x;
  const int64_t p = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  if (p >= cols) return;
  const int64_t pages = static_cast<int64_t>(max(lens[row] - 1, 0) / 1024) * 16;
  float best = -CUDART_INF_F;
  if (p < pages) {
    const float* s = logits + row * stride + p * 8;
#pragma unroll
    for (int g = 0; g < 8; ++g) best = fmaxf(best, s[g]);
  }
  out[row * maxp + p] = best;
}

struct OutputIdsArgs {
  const int32_t* raw;
  const float* scores;
  const int32_t* members;
  const int32_t* rt;
  const int32_t* nt;
  const void* selected;
  int sel64;
  const int32_t* lens;
  const int32_t* takes;
  int32_t* out;
  int32_t* logical;
  const int32_t* ft;
  int64_t maxp, np, take_stride, width, topk, sink, window;
  int map_physical, direct_fine;
  int64_t fp;
};

__global__ void output_ids_kernel(const __grid_constant__ OutputIdsArgs a) {
  const int64_t row = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  if (j >= a.topk) return;
  const int raw = a.raw[row * a.topk + j];
  const int take = a.takes[row];
  const int n = a.lens[row];
  const RowBounds rb = row_bounds(n, static_cast<int>(a.sink), static_cast<int>(a.window));
  bool valid = raw >= 0 && raw < a.width;
  int logical = -1;
  if (valid) {
    if (raw < take * 64) {
      int64_t page;
      if (a.direct_fine) {
        page = a.ft[row * a.fp + raw / 64];
      } else {
        const int64_t rank = load_index(a.selected, a.sel64, row * a.take_stride + raw / 64);
        page = a.rt[row * a.maxp + rank];
      }
      logical = a.members[page * 64 + raw % 64];
    } else {
      const int off = raw - take * 64;
      logical = off < rb.sink ? off : rb.tail + off - rb.sink;
    }
    valid = a.scores[row * a.width + raw] != -CUDART_INF_F && logical >= 0 && logical < n;
  }
  if (a.map_physical)
    a.out[row * a.topk + j] = valid ? a.nt[row * a.np + logical / 64] * 64 + logical % 64 : -1;
  a.logical[row * a.topk + j] = valid ? logical : -1;
}

__global__ void expand_logical_kernel(const int32_t* __restrict__ logical, int32_t* __restrict__ out,
                                      int64_t topk, int64_t stride) {
  const int64_t row = blockIdx.x;
  for (int64_t j = threadIdx.x; j < stride; j += blockDim.x) {
    int32_t v = -1;
    if (j < topk * 4) {
      const int32_t lg = logical[row * topk + j / 4];
      if (lg >= 0) v = lg * 4 + static_cast<int32_t>(j % 4);
    }
    out[row * stride + j] = v;
  }
}

// ---- row staging of a query bucket (runtime.py:643-666) ----------------------
// One CTA per bucket row: the caller's q, weights, length and native page table
// row, the request's reordered and centre table rows (arena rows named by id),
// or zeros for a row past the caller's n.  The ids travel in the launch's
// parameters, so no host -> device copy precedes the kernel.
constexpr int kStageRowsMax = 256;

struct QueryStageArgs {
  const uint8_t* q;
  const float* w;
  const int32_t* lens;
  const int32_t* nt;
  const int32_t* state_tables;
  const int32_t* state_centers;
  uint8_t* q_out;
  float* w_out;
  int32_t* lens_out;
  int32_t* nt_out;
  int32_t* rt_out;
  int32_t* ct_out;
  int64_t heads, width, pages, n;
  int32_t rows[kStageRowsMax];
};

// dst[0, bytes) = src[0, bytes) (src null: zeros) by the CTA's threads, with
// 16-byte accesses where both addresses allow them.
__device__ __forceinline__ void stage_bytes(uint8_t* dst, const uint8_t* src, int64_t bytes) {
  const int t = threadIdx.x, nt = blockDim.x;
  const uintptr_t al = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
  int64_t done = 0;
  if ((al & 15) == 0) {
    const int64_t n16 = bytes >> 4;
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    for (int64_t i = t; i < n16; i += nt) d[i] = src ? s[i] : make_uint4(0, 0, 0, 0);
    done = n16 << 4;
  } else if ((al & 3) == 0) {
    const int64_t n4 = bytes >> 2;
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    for (int64_t i = t; i < n4; i += nt) d[i] = src ? s[i] : 0u;
    done = n4 << 2;
  }
  for (int64_t i = done + t; i < bytes; i += nt) dst[i] = src ? src[i] : 0;
}

__global__ void __launch_bounds__(256) query_stage_kernel(const __grid_constant__ QueryStageArgs a) {
  const int64_t i = blockIdx.x;
  const bool live = i < a.n;
  const int64_t qb = a.heads * 128, cp = a.pages / 8;
  const int64_t wb = live ? a.width * 4 : 0;
  stage_bytes(a.q_out + i * qb, live ? a.q + i * qb : nullptr, qb);
  stage_bytes(reinterpret_cast<uint8_t*>(a.w_out + i * a.heads),
              live ? reinterpret_cast<const uint8_t*>(a.w + i * a.heads) : nullptr, a.heads * 4);
  uint8_t* nt = reinterpret_cast<uint8_t*>(a.nt_out + i * a.pages);
  stage_bytes(nt, live ? reinterpret_cast<const uint8_t*>(a.nt + i * a.width) : nullptr, wb);
  stage_bytes(nt + wb, nullptr, a.pages * 4 - wb);
  const int64_t r = live ? a.rows[i] : 0;
  stage_bytes(reinterpret_cast<uint8_t*>(a.rt_out + i * a.pages),
              live ? reinterpret_cast<const uint8_t*>(a.state_tables + r * a.pages) : nullptr, a.pages * 4);
  stage_bytes(reinterpret_cast<uint8_t*>(a.ct_out + i * cp),
              live ? reinterpret_cast<const uint8_t*>(a.state_centers + r * cp) : nullptr, cp * 4);
  if (threadIdx.x == 0) a.lens_out[i] = live ? a.lens[i] : 0;
}

}  // namespace
}  // namespace v1x

using namespace v1x;

extern "C" int v1x_query_metadata(const int32_t* lens, const int32_t* nt, int32_t* fine_lens,
                                  int32_t* takes, int32_t* dg_lens, int32_t* center_lens,
                                  int32_t* tail_rows, int64_t np, int64_t topk, int64_t num,
                                  int64_t den, int64_t sink, int64_t window, const int32_t* budget,
                                  int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && np > 0 && den > 0 && num >= 0, "query_metadata: bad geometry");
  if (batch == 0) return V1X_OK;
  const MetaArgs a{lens, nt, fine_lens, takes, dg_lens, center_lens, tail_rows, np, topk, num, den, sink, window,
                   budget};
  launch_kernel(query_metadata_kernel, dim3(static_cast<unsigned>(batch)), dim3(128), 0, as_stream(stream), a);
  return launch_status("v1x_query_metadata");
}

extern "C" int v1x_query_prepare(const int32_t* lens, const int32_t* nt, int32_t* fine_lens, int32_t* takes,
                                 int32_t* dg_lens, int32_t* center_lens, int32_t* tail_rows, int64_t np,
                                 int64_t topk, int64_t num, int64_t den, int64_t sink, int64_t window,
                                 const int32_t* budget, const uint8_t* native_bytes, const float* native_scales,
                                 uint8_t* fine_bytes, float* fine_scales, int64_t cap, int64_t scratch,
                                 int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && np > 0 && den > 0 && num >= 0, "query_prepare: bad geometry");
  V1X_CHECK_ARG(scratch >= 1 && scratch < 65536 * kStagePages && cap >= 0, "query_prepare: bad staging geometry");
  V1X_CHECK_ARG(((reinterpret_cast<uintptr_t>(native_bytes) | reinterpret_cast<uintptr_t>(fine_bytes)) & 15) == 0,
                "query_prepare: page pools must be 16-byte aligned");
  if (batch == 0) return V1X_OK;
  const MetaArgs m{lens, nt, fine_lens, takes, dg_lens, center_lens, tail_rows, np, topk, num, den, sink, window,
                   budget};
  const StageArgs s{native_bytes, native_scales, nt, lens, fine_bytes, fine_scales, tail_rows, cap, np,
                    scratch, sink, window, batch, 1};
  // CTA (row, g) stages page groups g, g + gridDim.y, ...: enough CTAs in total to
  // fill the GPU (about 2560), but not one per group when rows are many
  const int64_t groups = (scratch + kStagePages - 1) / kStagePages;
  const int64_t gy = std::min<int64_t>(groups, std::max<int64_t>(1, (2560 + batch - 1) / batch));
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(gy));
  launch_kernel(query_prepare_kernel, grid, dim3(128), 0, as_stream(stream), m, s);
  return launch_status("v1x_query_prepare");
}

extern "C" int v1x_query_lengths(const int32_t* lens, int32_t* fine_lens, int32_t* takes,
                                 int64_t topk, int64_t num, int64_t den, int64_t sink,
                                 int64_t window, int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && den > 0 && num >= 0, "query_lengths: bad geometry");
  if (batch == 0) return V1X_OK;
  query_lengths_kernel<<<static_cast<unsigned>((batch + 127) / 128), 128, 0, as_stream(stream)>>>(
      lens, fine_lens, takes, topk, num, den, sink, window, batch);
  return launch_status("v1x_query_lengths");
}

extern "C" int v1x_fine_table_shared(const int32_t* rt, const void* selected, int selected_is_i64,
                                     const int32_t* takes, int32_t* ft, const int32_t* tail_rows,
                                     int64_t cap, int64_t maxp, int64_t take, int64_t fp,
                                     int64_t scratch, int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && fp >= 0 && scratch >= 1, "fine_table_shared: bad geometry");
  if (batch == 0 || fp == 0) return V1X_OK;
  fine_table_shared_kernel<<<static_cast<unsigned>(batch), 128, 0, as_stream(stream)>>>(
      rt, selected, selected_is_i64, takes, ft, tail_rows, cap, maxp, take, fp, scratch);
  return launch_status("v1x_fine_table_shared");
}

extern "C" int v1x_stage_tail_shared(const uint8_t* native_bytes, const float* native_scales,
                                     const int32_t* nt, const int32_t* lens, uint8_t* fine_bytes,
                                     float* fine_scales, const int32_t* tail_rows, int64_t cap,
                                     int64_t np, int64_t scratch, int64_t sink, int64_t window,
                                     int64_t rows_bound, int64_t group, int64_t grid_groups,
                                     int64_t grid_pages, void* stream) {
  clear_error();
  V1X_CHECK_ARG(group >= 1 && grid_groups >= 0 && grid_pages >= 0 && grid_pages < 65536,
                "stage_tail_shared: bad grid");
  V1X_CHECK_ARG(((reinterpret_cast<uintptr_t>(native_bytes) | reinterpret_cast<uintptr_t>(fine_bytes)) & 15) == 0,
                "stage_tail_shared: page pools must be 16-byte aligned");
  if (grid_groups == 0 || grid_pages == 0) return V1X_OK;
  StageArgs a{native_bytes, native_scales, nt, lens, fine_bytes, fine_scales, tail_rows, cap, np,
              scratch, sink, window, rows_bound, group};
  int64_t rows = grid_groups * group;
  if (rows_bound > 0 && rows > rows_bound) rows = rows_bound;
  if (rows <= 0) return V1X_OK;
  const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>((grid_pages + kStagePages - 1) / kStagePages));
  launch_kernel(stage_tail_shared_kernel, grid, dim3(256), 0, as_stream(stream), a, grid_pages);
  return launch_status("v1x_stage_tail_shared");
}

extern "C" int v1x_mask_fine(float* scores, const void* selected, int selected_is_i64,
                             const int32_t* rt, const int32_t* members, const int32_t* lens,
                             const int32_t* takes, int64_t maxp, int64_t take, int64_t stride,
                             int64_t width, int64_t sink, int64_t window, int64_t batch,
                             void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && width >= 0, "mask_fine: bad geometry");
  if (batch == 0 || width == 0) return V1X_OK;
  mask_fine_kernel<<<dim3(static_cast<unsigned>(batch), static_cast<unsigned>((width + 255) / 256)), 256, 0,
                     as_stream(stream)>>>(scores, selected, selected_is_i64, rt, members, lens, takes,
                                          maxp, take, stride, width, sink, window);
  return launch_status("v1x_mask_fine");
}

extern "C" int v1x_reduce_centers(const float* logits, const int32_t* lens, float* out,
                                  int64_t maxp, int64_t pcount, int64_t stride, int64_t batch,
                                  void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && maxp >= 0 && pcount >= 0, "reduce_centers: bad geometry");
  const int64_t cols = pcount < maxp ? pcount : maxp;
  if (batch == 0 || cols == 0) return V1X_OK;
  reduce_centers_kernel<<<dim3(static_cast<unsigned>(batch), static_cast<unsigned>((cols + 127) / 128)), 128,
                          0, as_stream(stream)>>>(logits, lens, out, maxp, cols, stride);
  return launch_status("v1x_reduce_centers");
}

extern "C" int v1x_output_ids(const int32_t* raw, const float* scores, const int32_t* members,
                              const int32_t* rt, const int32_t* nt, const void* selected,
                              int selected_is_i64, const int32_t* lens, const int32_t* takes,
                              int32_t* out, int32_t* logical, const int32_t* ft, int64_t maxp,
                              int64_t np, int64_t take, int64_t width, int64_t topk, int64_t sink,
                              int64_t window, int map_physical, int direct_fine, int64_t fp,
                              int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && topk >= 0, "output_ids: bad geometry");
  if (batch == 0 || topk == 0) return V1X_OK;
  OutputIdsArgs a{raw, scores, members, rt, nt, selected, selected_is_i64, lens, takes, out, logical,
                  ft, maxp, np, take, width, topk, sink, window, map_physical, direct_fine, fp};
  output_ids_kernel<<<dim3(static_cast<unsigned>(batch), static_cast<unsigned>((topk + 255) / 256)), 256, 0,
                      as_stream(stream)>>>(a);
  return launch_status("v1x_output_ids");
}

extern "C" int v1x_expand_logical(const int32_t* logical, int32_t* out, int64_t topk, int64_t stride,
                                  int64_t batch, void* stream) {
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && topk >= 0 && stride >= 0, "expand_logical: bad geometry");
  if (batch == 0 || stride == 0) return V1X_OK;
  expand_logical_kernel<<<static_cast<unsigned>(batch), 256, 0, as_stream(stream)>>>(logical, out, topk, stride);
  return launch_status("v1x_expand_logical");
}

extern "C" int v1x_query_stage(const uint8_t* q, const float* w, const int32_t* lens, const int32_t* native_tables,
                               int64_t width, const int32_t* rows, const int32_t* state_tables,
                               const int32_t* state_centers, int64_t state_rows, uint8_t* q_out, float* w_out,
                               int32_t* lens_out, int32_t* nt_out, int32_t* rt_out, int32_t* ct_out,
                               int64_t heads, int64_t pages, int64_t n, int64_t filled, void* stream) {
  clear_error();
  V1X_CHECK_ARG(heads > 0 && pages > 0 && pages % 8 == 0 && width >= 0 && width <= pages && n >= 0 &&
                    filled >= 0 && state_rows >= 0,
                "query_stage: bad geometry");
  V1X_CHECK_ARG(q_out && w_out && lens_out && nt_out && rt_out && ct_out, "query_stage: null output");
  V1X_CHECK_ARG(n == 0 || (q && w && lens && rows && state_tables && state_centers && (native_tables || !width)),
                "query_stage: null input");
  for (int64_t i = 0; i < n; ++i)
    V1X_CHECK_ARG(rows[i] >= 0 && rows[i] < state_rows, "query_stage: row id %d of row %lld out of range",
                  rows[i], static_cast<long long>(i));
  const int64_t total = std::max(n, filled);
  for (int64_t s = 0; s < total; s += kStageRowsMax) {
    const int64_t m = std::min<int64_t>(kStageRowsMax, total - s);
    const int64_t live = std::min<int64_t>(std::max<int64_t>(n - s, 0), m);
    QueryStageArgs a{};
    a.q = live ? q + s * heads * 128 : nullptr;
    a.w = live ? w + s * heads : nullptr;
    a.lens = live ? lens + s : nullptr;
    a.nt = live ? native_tables + s * width : nullptr;
    a.state_tables = state_tables;
    a.state_centers = state_centers;
    a.q_out = q_out + s * heads * 128;
    a.w_out = w_out + s * heads;
    a.lens_out = lens_out + s;
    a.nt_out = nt_out + s * pages;
    a.rt_out = rt_out + s * pages;
    a.ct_out = ct_out + s * (pages / 8);
    a.heads = heads;
    a.width = width;
    a.pages = pages;
    a.n = live;
    for (int64_t i = 0; i < live; ++i) a.rows[i] = rows[s + i];
    launch_kernel(query_stage_kernel, dim3(static_cast<unsigned>(m)), dim3(256), 0, as_stream(stream), a);
  }
  return launch_status("v1x_query_stage");
}

namespace v1x {
namespace {

// mask_scores of the v1_native backend (NA/kernels.py:47-59): a candidate column
// whose logical token (members of its fine page) is missing, in the query's
// future, or -- among the first dedup_cols columns -- a sink token or one at or
// past fixed_start, scores -inf.
constexpr int kMaskCols = 4096;

__global__ void mask_scores_kernel(float* __restrict__ scores, int64_t score_stride, int64_t width,
                                   const int32_t* __restrict__ table, int64_t table_stride,
                                   const int32_t* __restrict__ mapping, int64_t mapping_pages,
                                   const int32_t* __restrict__ positions, int64_t dedup_cols, int64_t fixed_start) {
  // a CTA takes kMaskCols columns of one row, a thread every 256th of them
  const int64_t row = blockIdx.y;
  const int pos = positions[row];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kMaskCols + threadIdx.x;
  const int64_t last = min(width, static_cast<int64_t>(blockIdx.x + 1) * kMaskCols);
#pragma unroll 4
  for (int64_t col = first; col < last; col += 256) {
    const int64_t page = table[row * table_stride + col / 64];
    // a page outside the mapping reads as no token (masked)
    const int logical = page >= 0 && page < mapping_pages ? mapping[page * 64 + col % 64] : -1;
    if (logical < 0 || logical > pos || (col < dedup_cols && (logical < 64 || logical >= fixed_start)))
      scores[row * score_stride + col] = -CUDART_INF_F;
  }
}

// pack_q of the signed-score path (qwen_gqa_probe_kernels.py:15-20; the same
// math as the Scorer's quantize + head padding, NA/scoring.py:66-71 with
// NA/grouping.py:41-44): one warp per (row, head) of the padded output; heads
// below qheads of rows below `rows` are quantised with the power of two
// >= max(absmax, 1e-4) / 448 (exactly) and get weight scale * w_mul, the rest
// are zero.  A lane holds 4 of the 128 values.
__device__ __forceinline__ float pq_pow2_ceil(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x007FFFFFu) == 0 ? v : __uint_as_float(((b >> 23) + 1u) << 23);
}

__global__ void pack_q_kernel(const void* __restrict__ q, int dtype, int64_t qs0, int64_t qs1, int64_t rows,
                              int64_t out_rows, int64_t qheads, int64_t out_heads, float w_mul,
                              uint8_t* __restrict__ q8, float* __restrict__ w) {
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (unit >= out_rows * out_heads) return;
  const int64_t row = unit / out_heads, h = unit % out_heads;
  float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const bool live = row < rows && h < qheads;
  if (live) {
    const int64_t off = row * qs0 + h * qs1 + lane * 4;
    if (dtype == 0) {
      const float* src = static_cast<const float*>(q) + off;
      for (int i = 0; i < 4; ++i) x[i] = src[i];
    } else if (dtype == 1) {
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(q) + off;
      for (int i = 0; i < 4; ++i) x[i] = __bfloat162float(src[i]);
    } else {
      const __half* src = static_cast<const __half*>(q) + off;
      for (int i = 0; i < 4; ++i) x[i] = __half2float(src[i]);
    }
  }
  float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = pq_pow2_ceil(__fdiv_rn(fmaxf(m, 1e-4f), 448.0f));
  uint32_t packed = 0;
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(__fdiv_rn(x[i], scale), __NV_SATFINITE, __NV_E4M3);
    packed |= static_cast<uint32_t>(b) << (8 * i);
  }
  reinterpret_cast<uint32_t*>(q8 + unit * 128)[lane] = packed;
  if (lane == 0) w[unit] = live ? __fmul_rn(scale, w_mul) : 0.0f;
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_pack_q(const void* q, int dtype, int64_t qs0, int64_t qs1, int64_t rows, int64_t out_rows,
                          int64_t qheads, int64_t out_heads, float w_mul, uint8_t* q8, float* w, void* stream) {
  clear_error();
  V1X_CHECK_ARG(dtype >= 0 && dtype <= 2, "pack_q: dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
  V1X_CHECK_ARG(rows >= 0 && out_rows >= rows && qheads >= 0 && out_heads >= qheads && qs0 >= 0 && qs1 >= 0,
                "pack_q: bad geometry");
  const int64_t units = out_rows * out_heads;
  if (units == 0) return V1X_OK;
  V1X_CHECK_ARG(q8 && w && (q || rows == 0 || qheads == 0), "pack_q: a required buffer is NULL");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(q8) & 3) == 0, "pack_q: q8 must be 4-byte aligned");
  V1X_CHECK_ARG((units + 7) / 8 < (int64_t(1) << 31), "pack_q: too many rows");
  pack_q_kernel<<<static_cast<unsigned>((units + 7) / 8), 256, 0, as_stream(stream)>>>(
      q, dtype, qs0, qs1, rows, out_rows, qheads, out_heads, w_mul, q8, w);
  return launch_status("v1x_pack_q");
}

extern "C" int v1x_mask_scores(float* scores, int64_t score_stride, int64_t width, const int32_t* table,
                               int64_t table_stride, const int32_t* mapping, int64_t mapping_pages,
                               const int32_t* positions,
                               int64_t dedup_cols, int64_t fixed_start, int64_t rows, void* stream) {
  clear_error();
  V1X_CHECK_ARG(rows >= 0 && width >= 0 && score_stride >= width && table_stride >= 0,
                "mask_scores: bad geometry");
  if (rows == 0 || width == 0) return V1X_OK;
  V1X_CHECK_ARG(scores && table && mapping && positions, "mask_scores: a required buffer is NULL");
  V1X_CHECK_ARG(rows < 65536, "mask_scores: at most 65535 rows per call");
  const dim3 grid(static_cast<unsigned>((width + kMaskCols - 1) / kMaskCols), static_cast<unsigned>(rows));
  mask_scores_kernel<<<grid, 256, 0, as_stream(stream)>>>(scores, score_stride, width, table, table_stride, mapping,
                                                         mapping_pages, positions, dedup_cols, fixed_start);
  return launch_status("v1x_mask_scores");
}
