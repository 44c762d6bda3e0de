// fused.route for sm_100a: per-page max of 8 centre logits, then the exact top
// pages in the reference's stable order, plus the fine-page-table write.
//
// Reference behaviour: sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:7-49
// (kernel) and :155-180 (host checks and the (THREADS, ITEMS) table).  The
// reference sorts all THREADS*ITEMS padded page slots with CUB BlockRadixSort
// (descending, stable); a slot's stable position is its blocked rank
//   rank(p) = (p % 128) * BASE + p / 128,  BASE = THREADS*ITEMS / 128,
// and CUB folds -0.0 onto +0.0.  Here the same total order -- key desc, blocked
// rank asc -- is produced by an exact search for the K-th key (select.cuh)
// followed by ordering only the winners.
#include "common.cuh"
#include "select.cuh"

namespace v1x {
namespace {

constexpr int kRouteThreads = 256;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kRouteMaxItems = 4096;
constexpr int kRouteSmallItems = 512;  // tables up to this many padded slots take 2 keys per thread
constexpr int kRankDirect = 256;  // winner lists up to this size are ordered by counting
constexpr int kBucketRank = 256;  // longer lists: by bins, when no bin holds more keys

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
  int stage_rt;       // the row's rt entries are copied to shared memory up front
};

// Shared memory: this fixed head, then (dynamic, sized by the launch) the winner
// list of n_items composites (key << 32) | ~rank and, with stage_rt, the row's
// reordered-page table.
struct RouteSmem {
  int hist[kBins];
  int4 red[2 * kRouteWarps];
  int warp_tot[kRouteWarps + 1];
  int4 res;
  int count;
  int maxbin;
};
constexpr size_t kRouteListOff = (sizeof(RouteSmem) + 15) & ~size_t(15);

__device__ __forceinline__ void store_sel(const RouteArgs& a, int64_t i, int64_t v) {
  if (a.sel64) static_cast<int64_t*>(a.selected)[i] = v;
  else static_cast<int32_t*>(a.selected)[i] = static_cast<int32_t>(v);
}

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

// kPages: `scores` already holds one value per page (the max of its 8 centres).
// kPer: page keys per thread (n_items <= kPer * kRouteThreads); small tables
// take kPer = 2, which fits four CTAs per SM.
//
// Thread t owns pages p = t + j*256 (coalesced loads); the tie order of a page
// is its blocked rank, computed from p.  The want-th largest key comes from the
// bitwise search; the winners (keys above it and all keys equal to it) are then
// ordered by (key desc, rank asc) by counting, or by a bitonic sort when ties
// make the list long.
template <bool kPages, int kPer>
__global__ void __launch_bounds__(kRouteThreads, kPer <= 2 ? 4 : 2) route_kernel(const __grid_constant__ RouteArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RouteSmem& sm = *reinterpret_cast<RouteSmem*>(smem_raw);
  unsigned long long* list = reinterpret_cast<unsigned long long*>(smem_raw + kRouteListOff);
  int* srt = reinterpret_cast<int*>(list + a.n_items);
  const int tid = threadIdx.x, nt = kRouteThreads;
  const int64_t row = blockIdx.x;
  const int n = a.lens[row];
  const int active = max(n - 1, 0) / 1024 * 16;
  const int32_t* rtrow = a.rt + row * a.pages;
  if (a.stage_rt) {  // the row's reordered-page table, copied while the keys are selected
    if ((reinterpret_cast<uintptr_t>(rtrow) & 15) == 0 && (a.pages & 3) == 0) {
      for (int v = tid; v < (a.pages >> 2); v += nt) cp_async16(srt + 4 * v, rtrow + 4 * v);
    } else {
      for (int v = tid; v < a.pages; v += nt) cp_async4(srt + v, rtrow + v);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int take = a.takes[row];
  if (a.fill_table) {
    const int64_t base = a.capacity + static_cast<int64_t>(a.tail_rows[row]) * 68;
    for (int64_t j = max(take, 0) + tid; j < a.fine_pages; j += nt)
      a.ft[row * a.fine_pages + j] = static_cast<int32_t>(base + min(j - take, int64_t(67)));
  }
  // number of ranks the output needs: selected (take_stride) and ft (take)
  const int want = static_cast<int>(min(static_cast<int64_t>(a.n_items),
      max(a.take_stride, a.fill_table ? min(static_cast<int64_t>(take), a.fine_pages) : int64_t(0))));
  if (take >= active || want <= 0) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (take >= active) {
      for (int64_t i = tid; i < a.take_stride; i += nt) {
        store_sel(a, row * a.take_stride + i, i);
        if (a.fill_table && i < take) a.ft[row * a.fine_pages + i] = a.rt[row * a.pages + i];
      }
    }
    return;
  }
  if (tid == 0) {
    sm.count = 0;
    sm.maxbin = 0;
  }
  // ---- page keys (VQ:26-41): p < act -> key of the page's max centre, else -inf
  const int act = static_cast<int>(min(static_cast<int64_t>(active), kPages ? a.score_cols : a.score_cols / 8));
  const float* srow = a.scores + row * a.score_stride;
  uint32_t kr[kPer];
  float x[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = tid + j * nt;
    x[j] = -CUDART_INF_F;
    if (p < act) {
      if (kPages) {
        x[j] = srow[p];
      } else {
        const float* sp = srow + static_cast<int64_t>(p) * 8;
        float4 u, w;
        if ((reinterpret_cast<uintptr_t>(srow) & 15) == 0) {
          u = reinterpret_cast<const float4*>(sp)[0];
          w = reinterpret_cast<const float4*>(sp)[1];
        } else {
          u = make_float4(sp[0], sp[1], sp[2], sp[3]);
          w = make_float4(sp[4], sp[5], sp[6], sp[7]);
        }
        x[j] = fmaxf(fmaxf(fmaxf(u.x, u.y), fmaxf(u.z, u.w)), fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)));
      }
    }
  }
  const int nv = a.n_items > tid ? (a.n_items - tid + nt - 1) / nt : 0;  // pages of this thread
#pragma unroll
  for (int j = 0; j < kPer; ++j) kr[j] = order_key(x[j]);
  // ---- winners: a 12-bit histogram finds the bin of the want-th key; every key
  // in that bin or above is a winner candidate.  When ties make that list long,
  // the exact want-th key from the bitwise search bounds it instead.
  zero_hist<kRouteThreads>(sm.hist);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (j < nv) atomicAdd(&sm.hist[bin_of(kr[j])], 1);
  __syncthreads();
  const TopBin tb = find_top_bin<kRouteThreads>(want, sm.hist, sm.warp_tot, &sm.res);
  auto emit = [&](int pos, unsigned long long comp) {
    const int r = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(comp & 0xFFFFFFFFull));
    const int p = r / a.base + (r % a.base) * 128;
    if (pos < a.take_stride) store_sel(a, row * a.take_stride + pos, p);
    if (a.fill_table && pos < take && pos < a.fine_pages)
      a.ft[row * a.fine_pages + pos] = p < a.pages ? (a.stage_rt ? srt[p] : rtrow[p]) : -1;
  };
  if (tb.above + tb.in > kRankDirect) {
    // many winners: ordered through the bins.  The bins from the threshold bin
    // up are laid out in descending order (a block scan of their counts); each
    // winner-region key is placed into its bin's range, and its position is the
    // keys in higher bins plus its rank inside the bin -- counted, when no bin
    // holds more than kBucketRank keys (else the bitwise search and the sort
    // below).  hist[b] becomes the end of bin b's range; bin b starts where bin
    // b + 1 ends.
    constexpr int kPerBin = kBins / kRouteThreads;
    const int hib = kBins - tid * kPerBin;  // this thread's bins [hib - kPerBin, hib)
    int c[kPerBin];
    int s = 0, mx = 0;
#pragma unroll
    for (int j = 0; j < kPerBin; ++j) {
      const int b = hib - kPerBin + j;
      c[j] = b >= tb.bin ? sm.hist[b] : 0;
      s += c[j];
      mx = max(mx, c[j]);
    }
    int tot;
    int cum = block_exclusive_scan(s, sm.warp_tot, &tot);
    mx = __reduce_max_sync(0xffffffffu, mx);
    if ((tid & 31) == 0) atomicMax(&sm.maxbin, mx);
#pragma unroll
    for (int j = kPerBin - 1; j >= 0; --j) {
      const int b = hib - kPerBin + j;
      if (b >= tb.bin) {
        sm.hist[b] = cum;
        cum += c[j];
      }
    }
    __syncthreads();
    if (sm.maxbin <= kBucketRank) {
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (j < nv && bin_of(kr[j]) >= tb.bin) {
          const int p = tid + j * nt;
          const uint32_t rank = static_cast<uint32_t>((p & 127) * a.base + (p >> 7));
          const int e = atomicAdd(&sm.hist[bin_of(kr[j])], 1);
          list[e] = (static_cast<unsigned long long>(kr[j]) << 32) | (0xFFFFFFFFu - rank);
        }
      }
      if (a.stage_rt) asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
      for (int e = tid; e < tb.above + tb.in; e += nt) {
        const unsigned long long cc = list[e];
        const int b = bin_of(static_cast<uint32_t>(cc >> 32));
        const int beg = b == kBins - 1 ? 0 : sm.hist[b + 1], end = sm.hist[b];
        int r = 0;
        for (int f = beg; f < end; ++f) r += list[f] > cc;
        if (beg + r < want) emit(beg + r, cc);
      }
      return;
    }
  }
  uint32_t lo = static_cast<uint32_t>(tb.bin) << (32 - kBinBits);
  if (tb.above + tb.in > kRankDirect) {
    int gt = 0;
    lo = block_kth_largest<kRouteWarps>(
        want,
        [&](uint32_t c1, uint32_t c2, uint32_t c3, int& n1, int& n2, int& n3) {
          n1 = n2 = n3 = 0;
#pragma unroll
          for (int j = 0; j < kPer; ++j) {
            if (j < nv) {
              n1 += kr[j] >= c1;
              n2 += kr[j] >= c2;
              n3 += kr[j] >= c3;
            }
          }
        },
        sm.red, &gt);
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (j < nv && kr[j] >= lo) {
      const int p = tid + j * nt;
      const uint32_t rank = static_cast<uint32_t>((p & 127) * a.base + (p >> 7));
      const int e = atomicAdd(&sm.count, 1);
      list[e] = (static_cast<unsigned long long>(kr[j]) << 32) | (0xFFFFFFFFu - rank);
    }
  }
  if (a.stage_rt) asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int m = sm.count;
  if (m <= kRankDirect) {
    // composites are unique: a winner's position is the number of larger ones
    for (int e = tid; e < m; e += nt) {
      const unsigned long long c = list[e];
      int pos = 0;
      for (int f = 0; f < m; ++f) pos += list[f] > c;
      if (pos < want) emit(pos, c);
    }
  } else {
    int mp = 1;
    while (mp < m) mp <<= 1;
    for (int i = m + tid; i < mp; i += nt) list[i] = 0ull;
    bitonic_sort_desc(list, mp);
    for (int i = tid; i < want; i += nt) emit(i, list[i]);
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
              fill_table, n_items, n_items / 128,
              fill_table && pages <= kRouteMaxItems ? 1 : 0};
  const size_t smem = kRouteListOff + static_cast<size_t>(n_items) * 8 + (a.stage_rt ? static_cast<size_t>(pages) * 4 : 0);
  static DeviceOnce once;
  once.run([] {
    const int most = static_cast<int>(kRouteListOff + kRouteMaxItems * 12);
    cudaFuncSetAttribute(route_kernel<false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(route_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(route_kernel<false, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(route_kernel<true, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
  });
  const dim3 grid(static_cast<unsigned>(batch)), block(kRouteThreads);
  static_assert(kRouteSmallItems <= 2 * kRouteThreads && kRouteMaxItems <= 16 * kRouteThreads, "route slots per thread");
  if (n_items <= kRouteSmallItems) {
    if (pages_in) launch_kernel(route_kernel<true, 2>, grid, block, smem, as_stream(stream), a);
    else launch_kernel(route_kernel<false, 2>, grid, block, smem, as_stream(stream), a);
  } else {
    if (pages_in) launch_kernel(route_kernel<true, 16>, grid, block, smem, as_stream(stream), a);
    else launch_kernel(route_kernel<false, 16>, grid, block, smem, as_stream(stream), a);
  }
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
