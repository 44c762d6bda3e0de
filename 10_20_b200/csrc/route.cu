// fused.route for sm_100a: per-page max of 8 centre logits, then the exact top
// pages in the reference's stable order, plus the fine-page-table write.
//
// Reference behaviour: sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:7-49
// (kernel) and :155-180 (host checks and the (THREADS, ITEMS) table).  The
// reference sorts all THREADS*ITEMS padded page slots with CUB BlockRadixSort
// (descending, stable); a slot's stable position is its blocked rank
//   rank(p) = (p % 128) * BASE + p / 128,  BASE = THREADS*ITEMS / 128,
// and CUB folds -0.0 onto +0.0.  Here the same total order -- key desc, blocked
// rank asc -- is produced by an exact radix select of the K-th key followed by a
// bitonic sort of only the K selected (key, rank) pairs.
#include "common.cuh"

namespace v1x {
namespace {

constexpr int kRouteThreads = 256;
constexpr int kRouteMaxItems = 4096;

struct RouteArgs {
  const float* scores;
  int64_t score_stride, score_cols;
  const int32_t* lens;
  const int32_t* takes;
  void* selected;
  int sel64;
  int64_t take_stride;
  int pages;
  const int32_t* rt;
  int32_t* ft;
  int64_t fine_pages;
  const int32_t* tail_rows;
  int64_t capacity;
  int fill_table;
  int n_items, base;  // padded slot count (THREADS*ITEMS) and BASE
};

struct RouteSmem {
  uint32_t keys[kRouteMaxItems];
  unsigned long long list[kRouteMaxItems];
  int hist[256];
  int warp_tot[kRouteThreads / 32 + 1];
  int digit, need;
};

__device__ __forceinline__ void store_sel(const RouteArgs& a, int64_t i, int64_t v) {
  if (a.sel64) static_cast<int64_t*>(a.selected)[i] = v;
  else static_cast<int32_t*>(a.selected)[i] = static_cast<int32_t>(v);
}

// kPages: `scores` already holds one value per page (the max of its 8 centres).
template <bool kPages>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const __grid_constant__ RouteArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RouteSmem& sm = *reinterpret_cast<RouteSmem*>(smem_raw);
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const int n = a.lens[row];
  const int take = a.takes[row];
  const int active = max(n - 1, 0) / 1024 * 16;
  if (a.fill_table) {
    const int64_t base = a.capacity + static_cast<int64_t>(a.tail_rows[row]) * 68;
    for (int64_t j = max(take, 0) + tid; j < a.fine_pages; j += nt)
      a.ft[row * a.fine_pages + j] = static_cast<int32_t>(base + min(j - take, int64_t(67)));
  }
  if (take >= active) {
    for (int64_t i = tid; i < a.take_stride; i += nt) {
      store_sel(a, row * a.take_stride + i, i);
      if (a.fill_table && i < take) a.ft[row * a.fine_pages + i] = a.rt[row * a.pages + i];
    }
    return;
  }
  // ---- page keys in blocked-rank order (VQ:26-41) ----------------------------
  // All loads of a thread are issued before any is consumed (a loop that stores
  // each load's result before the next load would serialise the latencies).
  const int act = static_cast<int>(min(static_cast<int64_t>(active), kPages ? a.score_cols : a.score_cols / 8));
  const float* srow = a.scores + row * a.score_stride;
  if (kPages) {
    // stage the row's page scores in smem (reusing the sort list), coalesced
    float* ps = reinterpret_cast<float*>(sm.list);
    const bool vec = (reinterpret_cast<uintptr_t>(srow) & 15) == 0;
    const int nv = vec ? act >> 2 : 0;
    for (int v = tid; v < nv; v += nt) reinterpret_cast<float4*>(ps)[v] = reinterpret_cast<const float4*>(srow)[v];
    for (int p = nv * 4 + tid; p < act; p += nt) ps[p] = srow[p];
    __syncthreads();
    for (int r = tid; r < a.n_items; r += nt) {
      const int p = r / a.base + (r % a.base) * 128;
      sm.keys[r] = order_key(p < act ? ps[p] : -CUDART_INF_F);
    }
  } else {
    const bool vec = (reinterpret_cast<uintptr_t>(srow) & 15) == 0;
    constexpr int kBatch = 4;
    for (int r0 = tid; r0 < a.n_items; r0 += nt * kBatch) {
      float4 x[kBatch], y[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = r0 + u * nt;
        const int p = r / a.base + (r % a.base) * 128;
        x[u] = y[u] = make_float4(-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F);
        if (r < a.n_items && p < act) {
          const float* sp = srow + static_cast<int64_t>(p) * 8;
          if (vec) {
            x[u] = reinterpret_cast<const float4*>(sp)[0];
            y[u] = reinterpret_cast<const float4*>(sp)[1];
          } else {
            x[u] = make_float4(sp[0], sp[1], sp[2], sp[3]);
            y[u] = make_float4(sp[4], sp[5], sp[6], sp[7]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = r0 + u * nt;
        if (r < a.n_items) {
          const float best = fmaxf(fmaxf(fmaxf(x[u].x, x[u].y), fmaxf(x[u].z, x[u].w)),
                                   fmaxf(fmaxf(y[u].x, y[u].y), fmaxf(y[u].z, y[u].w)));
          sm.keys[r] = order_key(best);
        }
      }
    }
  }
  // number of ranks the output needs: selected (take_stride) and ft (take)
  const int want = static_cast<int>(min(static_cast<int64_t>(a.n_items),
      max(a.take_stride, a.fill_table ? min(static_cast<int64_t>(take), a.fine_pages) : int64_t(0))));
  // ---- radix select of the want-th largest key ---------------------------------
  uint32_t prefix = 0, known = 0;
  int need = want;
  for (int pass = 0; pass < 4 && want > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += nt) sm.hist[b] = 0;
    __syncthreads();
    const int iters = (a.n_items + nt - 1) / nt;
    for (int j = 0; j < iters; ++j) {
      const int r = j * nt + tid;
      int bin = -1;
      if (r < a.n_items) {
        const uint32_t k = sm.keys[r];
        if ((k & known) == prefix) bin = (k >> shift) & 255;
      }
      const unsigned same = __match_any_sync(0xffffffffu, bin);
      if (bin >= 0 && lane == __ffs(same) - 1) atomicAdd(&sm.hist[bin], __popc(same));
    }
    __syncthreads();
    if (warp == 0) {
      int cnt[8], s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cnt[j] = sm.hist[255 - (lane * 8 + j)];
        s += cnt[j];
      }
      int cum = warp_inclusive_scan(s) - s;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cum < need && cum + cnt[j] >= need) {
          sm.digit = 255 - (lane * 8 + j);
          sm.need = need - cum;
        }
        cum += cnt[j];
      }
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(sm.digit) << shift;
    known |= 255u << shift;
    need = sm.need;
    __syncthreads();
  }
  const uint32_t thr = prefix;
  // ---- gather the `want` winners (ties: lowest blocked rank) --------------------
  const int chunk = (a.n_items + nt - 1) / nt;
  const int beg = min(tid * chunk, a.n_items), end = min(beg + chunk, a.n_items);
  int eq = 0, gt = 0;
  for (int r = beg; r < end; ++r) {
    eq += sm.keys[r] == thr;
    gt += sm.keys[r] > thr;
  }
  int tot;
  const int eq_before = block_exclusive_scan(eq, sm.warp_tot, &tot);
  const int take_eq = min(max(need - eq_before, 0), eq);
  int pos = block_exclusive_scan(gt + take_eq, sm.warp_tot, &tot);
  int eq_seen = eq_before;
  for (int r = beg; r < end; ++r) {
    const uint32_t k = sm.keys[r];
    bool sel = k > thr;
    if (k == thr) {
      sel = eq_seen < need;
      ++eq_seen;
    }
    if (sel && pos < want)
      sm.list[pos++] = (static_cast<unsigned long long>(k) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(r));
  }
  // pad to a power of two with the smallest composite, then sort descending
  int m = 1;
  while (m < want) m <<= 1;
  for (int i = want + tid; i < m; i += nt) sm.list[i] = 0ull;
  __syncthreads();
  bitonic_sort_desc(sm.list, m);
  for (int i = tid; i < want; i += nt) {
    const int r = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(sm.list[i] & 0xFFFFFFFFull));
    const int p = r / a.base + (r % a.base) * 128;
    if (i < a.take_stride) store_sel(a, row * a.take_stride + i, p);
    if (a.fill_table && i < take && i < a.fine_pages)
      a.ft[row * a.fine_pages + i] = p < a.pages ? a.rt[row * a.pages + p] : -1;
  }
}

}  // namespace
}  // namespace v1x

namespace v1x {
namespace {
int route_launch(bool pages_in, const float* scores, int64_t score_stride, int64_t score_cols,
                 const int32_t* lens, const int32_t* takes, void* selected, int selected_is_i64,
                 int64_t take_stride, int64_t pages, const int32_t* rt, int32_t* ft, int64_t fine_pages,
                 const int32_t* tail_rows, int64_t capacity, int fill_table, int64_t batch, void* stream) {
  int threads, items;
  if (pages <= 128) { threads = 64; items = 2; }
  else if (pages <= 256) { threads = 64; items = 4; }
  else if (pages <= 512) { threads = 64; items = 8; }
  else if (pages <= 1024) { threads = 128; items = 8; }
  else if (pages <= 2048) { threads = 128; items = 16; }
  else { threads = 128; items = 32; }
  const int n_items = threads * items;
  RouteArgs a{scores, score_stride, score_cols, lens, takes, selected, selected_is_i64,
              take_stride, static_cast<int>(pages), rt, ft, fine_pages, tail_rows, capacity,
              fill_table, n_items, n_items / 128};
  const size_t smem = sizeof(RouteSmem);
  static DeviceOnce once;
  if (once.first()) {
    cudaFuncSetAttribute(route_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(route_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  if (pages_in) route_kernel<true><<<static_cast<unsigned>(batch), kRouteThreads, smem, as_stream(stream)>>>(a);
  else route_kernel<false><<<static_cast<unsigned>(batch), kRouteThreads, smem, as_stream(stream)>>>(a);
  return launch_status(pages_in ? "v1x_route_pages" : "v1x_route");
}
}  // namespace
}  // namespace v1x

extern "C" int v1x_route(const float* scores, int64_t score_stride, int64_t score_cols,
                         const int32_t* lens, const int32_t* takes, void* selected,
                         int selected_is_i64, int64_t take_stride, int64_t pages,
                         const int32_t* rt, int32_t* ft, int64_t fine_pages,
                         const int32_t* tail_rows, int64_t capacity, int fill_table,
                         int64_t batch, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(capacity > 0 && fine_pages >= take_stride, "Invalid fine page table");
  V1X_CHECK_ARG(pages >= 64 && pages <= 4096 && score_cols >= pages * 8 && take_stride <= pages &&
                    score_stride % 4 == 0,
                "Invalid V1 route capacity");
  V1X_CHECK_ARG(batch >= 0 && take_stride >= 0 && score_stride >= score_cols,
                "route: bad batch / strides");
  if (batch == 0) return V1X_OK;
  return route_launch(false, scores, score_stride, score_cols, lens, takes, selected, selected_is_i64,
                      take_stride, pages, rt, ft, fine_pages, tail_rows, capacity, fill_table, batch, stream);
}

extern "C" int v1x_route_pages(const float* page_scores, int64_t page_stride, const int32_t* lens,
                               const int32_t* takes, void* selected, int selected_is_i64,
                               int64_t take_stride, int64_t pages, const int32_t* rt, int32_t* ft,
                               int64_t fine_pages, const int32_t* tail_rows, int64_t capacity,
                               int fill_table, int64_t batch, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(capacity > 0 && fine_pages >= take_stride, "Invalid fine page table");
  V1X_CHECK_ARG(pages >= 64 && pages <= 4096 && page_stride >= pages && take_stride <= pages,
                "Invalid V1 route capacity");
  V1X_CHECK_ARG(batch >= 0 && take_stride >= 0, "route: bad batch / strides");
  if (batch == 0) return V1X_OK;
  return route_launch(true, page_scores, page_stride, page_stride, lens, takes, selected, selected_is_i64,
                      take_stride, pages, rt, ft, fine_pages, tail_rows, capacity, fill_table, batch, stream);
}
