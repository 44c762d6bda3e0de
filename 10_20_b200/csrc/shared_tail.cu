// Published-end shared-tail variant for sm_100a: one request's chunk of query
// rows (non-decreasing lengths) shares ONE staged copy of its sink and tail
// pages instead of a private copy per row.
//
// Reference (an experiment beside the production path):
//   experiments/tail_union_lab_20261021/union.py:10-40        bounds, stage_union
//   experiments/fine_pool_shared_20261021/kernels.py:8-76     tables, normalize, map_topk
//   experiments/fine_pool_shared_20261021/route_shared.cu:12-54  route_physical
// The tail of a row starts at the published index end (a device word), not at
// the last complete 1K bucket:
//   s = min(n, S);  t = max(s, min(min(max(end, 0), n), max(s, n - W)));  c = s + n - t.
//
// Kernels:
//   stage_union_kernel   grid-stride over the union pages, one CTA per page, 16-byte
//                        copies; per-row (s, t, c) and the chunk descriptor
//                        (sp, tp, ep, total) from the same launch.
//   shared_tables_kernel one CTA per row: fine page table, scored lengths, counts.
//   normalize_kernel     one thread per (row, candidate): canonical candidate order
//                        with the boundary/causality masks applied before Top-K.
//   map_topk_kernel      one thread per (row, pick): rank -> logical -> physical.
//   route_physical_kernel one CTA per row: the top `take` published pages by the
//                        max of their 8 centre scores, in the reference's stable
//                        order, written as physical page ids.
// Reads the reference leaves unguarded (a page id or a source column outside its
// buffer) are guarded here: such a candidate reads as masked (-inf / -1), a
// staged page from outside the source pool as zeros with V1X_STATUS_BAD_PAGE.
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "select.cuh"

namespace v1x {
namespace {

struct Bounds {
  int s, t, c;
};

__device__ __forceinline__ Bounds shared_bounds(int n, int end, int sink, int window) {
  const int s = min(n, sink);
  const int t = max(s, min(min(max(end, 0), n), max(s, n - window)));
  return {s, t, s + n - t};
}

// ---- stage_union (union.py:16-40) ---------------------------------------------
__global__ void __launch_bounds__(256) stage_union_kernel(const uint8_t* __restrict__ src, int64_t src_pages,
                                                          const int32_t* __restrict__ nt, int64_t nt_len,
                                                          const int32_t* __restrict__ lens, int rows,
                                                          const int32_t* __restrict__ indexed_end,
                                                          uint8_t* __restrict__ dst, int64_t dst_pages,
                                                          int32_t* __restrict__ meta, int32_t* __restrict__ desc,
                                                          int sink, int window, int32_t* status) {
  const int first = lens[0], last = lens[rows - 1];
  const int end = indexed_end[0];
  const int tail_first = shared_bounds(first, end, sink, window).t;
  const int sp = (min(last, sink) + 63) / 64;
  const int tp = max(sp, tail_first / 64);
  const int ep = (last + 63) / 64;
  const int total = sp + max(ep - tp, 0);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    desc[0] = sp;
    desc[1] = tp;
    desc[2] = ep;
    desc[3] = total;
    if (total > dst_pages && status) atomicExch(status, V1X_STATUS_CAPACITY);
  }
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const Bounds b = shared_bounds(lens[r], end, sink, window);
    meta[3 * r] = b.s;
    meta[3 * r + 1] = b.t;
    meta[3 * r + 2] = b.c;
  }
  const int64_t lim = min(static_cast<int64_t>(total), dst_pages);
  constexpr int kVec = kPageBytes / 16;  // 528 16-byte pieces per page
  for (int64_t u = blockIdx.x; u < lim; u += gridDim.x) {
    const int64_t lp = u < sp ? u : tp + u - sp;
    const int64_t phys = lp < nt_len ? nt[lp] : -1;
    const bool ok = phys >= 0 && phys < src_pages;
    if (!ok && threadIdx.x == 0 && status) atomicExch(status, V1X_STATUS_BAD_PAGE);
    const uint4* from = reinterpret_cast<const uint4*>(src + (ok ? phys : 0) * kPageBytes);
    uint4* to = reinterpret_cast<uint4*>(dst + u * kPageBytes);
    for (int v = threadIdx.x; v < kVec; v += blockDim.x) to[v] = ok ? __ldcs(from + v) : make_uint4(0, 0, 0, 0);
  }
}

// ---- tables (kernels.py:13-41) -------------------------------------------------
__global__ void __launch_bounds__(128) shared_tables_kernel(
    const int32_t* __restrict__ lens, const int32_t* __restrict__ indexed_end, const int32_t* __restrict__ takes,
    const int32_t* __restrict__ selected, const int32_t* __restrict__ desc, int32_t* __restrict__ ft,
    int32_t* __restrict__ dglens, int32_t* __restrict__ clens, int cap, int max_take, int scratch, int fp, int sink,
    int window, int shared) {
  const int r = blockIdx.x;
  const int n = lens[r], take = takes[r];
  const Bounds b = shared_bounds(n, indexed_end[0], sink, window);
  int pages, span, sp = 0, tp = 0, gsp = 0, gtp = 0;
  if (shared) {
    sp = (b.s + 63) / 64;
    tp = max(sp, b.t / 64);
    const int ep = (n + 63) / 64;
    gsp = desc[0];
    gtp = desc[1];
    pages = sp + max(ep - tp, 0);
    span = ep > tp ? sp * 64 + n - tp * 64 : n;
  } else {
    pages = (b.c + 63) / 64;
    span = b.c;
  }
  for (int j = threadIdx.x; j < fp; j += blockDim.x) {
    const int k = j - take;
    int page = 0;
    if (j < take) {
      page = j < max_take ? selected[static_cast<int64_t>(r) * max_take + j] : 0;
    } else if (k >= 0 && k < pages) {
      page = shared ? (k < sp ? cap + k : cap + gsp + tp - gtp + k - sp) : cap + r * scratch + k;
    }
    ft[static_cast<int64_t>(r) * fp + j] = page;
  }
  if (threadIdx.x == 0) {
    dglens[r] = max(take * 64 + span, 1);
    clens[r] = take * 64 + b.c;
  }
}

// ---- normalize (kernels.py:43-63) ----------------------------------------------
__global__ void __launch_bounds__(256) normalize_kernel(
    const float* __restrict__ raw, int64_t stride, const int32_t* __restrict__ lens,
    const int32_t* __restrict__ indexed_end, const int32_t* __restrict__ takes, const int32_t* __restrict__ selected,
    const int32_t* __restrict__ members, int64_t member_rows, float* __restrict__ out, int max_take, int width,
    int sink, int window, int shared) {
  const int r = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= width) return;
  const int n = lens[r], take = takes[r], end = indexed_end[0];
  const Bounds b = shared_bounds(n, end, sink, window);
  const int hist = take * 64;
  const bool fine = j < hist;
  const int x = j - hist;
  bool valid;
  int64_t source = j;
  if (fine) {
    const int col = j / 64;
    const int64_t page = col < max_take ? selected[static_cast<int64_t>(r) * max_take + col] : 0;
    const int member = page >= 0 && page < member_rows ? members[page * 64 + (j & 63)] : -1;
    valid = member >= b.s && member < b.t && member < n && member < end;
  } else {
    valid = x >= 0 && x < b.c;
    if (shared) {
      const int logical = x < b.s ? x : b.t + x - b.s;
      const int sp = (b.s + 63) / 64, tp = max(sp, b.t / 64);
      source = hist + (logical < sp * 64 ? logical : sp * 64 + logical - tp * 64);
    }
  }
  out[static_cast<int64_t>(r) * width + j] =
      valid && source < stride ? raw[static_cast<int64_t>(r) * stride + source] : -CUDART_INF_F;
}

// ---- map_topk (kernels.py:65-76) -----------------------------------------------
__global__ void __launch_bounds__(256) map_topk_kernel(
    const int64_t* __restrict__ ids, const float* __restrict__ values, const int32_t* __restrict__ lens,
    const int32_t* __restrict__ indexed_end, const int32_t* __restrict__ takes, const int32_t* __restrict__ selected,
    const int32_t* __restrict__ members, int64_t member_rows, const int32_t* __restrict__ nt, int64_t nt_len,
    int32_t* __restrict__ logical_out, int32_t* __restrict__ slots, int max_take, int top, int sink, int window) {
  const int r = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= top) return;
  const int64_t o = static_cast<int64_t>(r) * top + i;
  const int rank = static_cast<int>(ids[o]);
  const float value = values[o];
  const int n = lens[r], take = takes[r];
  const Bounds b = shared_bounds(n, indexed_end[0], sink, window);
  const bool fine = rank >= 0 && rank < take * 64;
  int logical;
  if (fine) {
    const int col = rank / 64;
    const int64_t page = col < max_take ? selected[static_cast<int64_t>(r) * max_take + col] : 0;
    logical = page >= 0 && page < member_rows ? members[page * 64 + (rank & 63)] : -1;
  } else {
    const int x = rank - take * 64;
    logical = x < b.s ? x : b.t + x - b.s;
  }
  const bool valid = value != -CUDART_INF_F && logical >= 0 && logical < n && logical / 64 < nt_len;
  logical_out[o] = valid ? logical : -1;
  slots[o] = valid ? nt[logical / 64] * 64 + (logical & 63) : -1;
}

// ---- route_physical (route_shared.cu:12-54) ------------------------------------
constexpr int kPhysThreads = 256;
constexpr int kPhysWarps = kPhysThreads / 32;
constexpr int kPhysMaxItems = 4096;
constexpr int kPhysDirect = 256;  // winner lists up to this size are ordered by counting

struct PhysSmem {
  int hist[kBins];
  int4 red[2 * kPhysWarps];
  int warp_tot[kPhysWarps + 1];
  int4 res;
  int count;
};
constexpr size_t kPhysListOff = (sizeof(PhysSmem) + 15) & ~size_t(15);

// Slot p of the padded layout (128 threads x `items`) has blocked rank
// (p % 128) * items + p / 128 (CUB's stable order over the blocked input);
// kPer page slots per thread (n_items <= kPer * 256).
template <int kPer>
__global__ void __launch_bounds__(kPhysThreads, kPer <= 2 ? 4 : 1) route_physical_kernel(
    const float* __restrict__ scores, int64_t score_stride, const int32_t* __restrict__ published,
    const int32_t* __restrict__ budgets, const int32_t* __restrict__ rt, int32_t* __restrict__ selected,
    int32_t* __restrict__ takes, int pages, int take_stride, int n_items, int items) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PhysSmem& sm = *reinterpret_cast<PhysSmem*>(smem_raw);
  unsigned long long* list = reinterpret_cast<unsigned long long*>(smem_raw + kPhysListOff);
  const int tid = threadIdx.x, nt = kPhysThreads;
  const int64_t row = blockIdx.x;
  const int active = min(max(published[row], 0), pages);
  const int take = min(min(max(budgets[row], 0), active), take_stride);
  const int32_t* rtrow = rt + row * pages;
  int32_t* out = selected + row * take_stride;
  if (tid == 0) takes[row] = take;
  for (int i = take + tid; i < take_stride; i += nt) out[i] = 0;  // padding stays a safe page id
  if (take == 0 || take == active) {
    for (int i = tid; i < take; i += nt) out[i] = rtrow[i];
    return;
  }
  if (tid == 0) sm.count = 0;
  uint32_t kr[kPer];
  const int nv = n_items > tid ? (n_items - tid + nt - 1) / nt : 0;  // slots of this thread
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = tid + j * nt;
    float x = -CUDART_INF_F;
    if (j < nv && p < active) {
      const float4* sp = reinterpret_cast<const float4*>(scores + row * score_stride + static_cast<int64_t>(p) * 8);
      const float4 u = sp[0], w = sp[1];
      x = fmaxf(fmaxf(fmaxf(u.x, u.y), fmaxf(u.z, u.w)), fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)));
      if (x == -CUDART_INF_F) x = -FLT_MAX;  // an all-masked published page still precedes padding
    }
    kr[j] = order_key(x);
  }
  zero_hist<kPhysThreads>(sm.hist);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (j < nv) atomicAdd(&sm.hist[bin_of(kr[j])], 1);
  __syncthreads();
  const TopBin tb = find_top_bin<kPhysThreads>(take, sm.hist, sm.warp_tot, &sm.res);
  uint32_t lo = static_cast<uint32_t>(tb.bin) << (32 - kBinBits);
  if (tb.above + tb.in > kPhysDirect) {
    int gt = 0;
    lo = block_kth_largest<kPhysWarps>(
        take,
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
      const uint32_t rank = static_cast<uint32_t>((p & 127) * items + (p >> 7));
      list[atomicAdd(&sm.count, 1)] = (static_cast<unsigned long long>(kr[j]) << 32) | (0xFFFFFFFFu - rank);
    }
  }
  __syncthreads();
  const int m = sm.count;
  auto emit = [&](int pos, unsigned long long comp) {
    const int rank = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(comp & 0xFFFFFFFFull));
    const int p = rank / items + (rank % items) * 128;
    if (pos < take) out[pos] = p < pages ? rtrow[p] : 0;
  };
  if (m <= kPhysDirect) {
    for (int e = tid; e < m; e += nt) {
      const unsigned long long c = list[e];
      int pos = 0;
      for (int f = 0; f < m; ++f) pos += list[f] > c;
      emit(pos, c);
    }
  } else {
    int mp = 1;
    while (mp < m) mp <<= 1;
    for (int i = m + tid; i < mp; i += nt) list[i] = 0ull;
    bitonic_sort_desc(list, mp);
    for (int i = tid; i < take; i += nt) emit(i, list[i]);
  }
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_stage_union(const uint8_t* src, int64_t src_pages, const int32_t* nt, int64_t nt_len,
                               const int32_t* lens, int64_t rows, const int32_t* indexed_end, uint8_t* dst,
                               int64_t dst_pages, int32_t* meta, int32_t* desc, int64_t sink, int64_t window,
                               int32_t* status, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(rows >= 1 && rows <= (int64_t(1) << 30), "stage_union: at least one row required");
  V1X_CHECK_ARG(src_pages > 0 && nt_len >= 0 && dst_pages >= 0 && sink >= 0 && window >= 0,
                "stage_union: bad geometry");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
                "stage_union: src and dst must be 16-byte aligned");
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>(dst_pages, (rows + 255) / 256),
                                                              static_cast<int64_t>(num_sms()) * 4));
  launch_kernel(stage_union_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, as_stream(stream), src,
                src_pages, nt, nt_len, lens, static_cast<int>(rows), indexed_end, dst, dst_pages, meta, desc,
                static_cast<int>(sink), static_cast<int>(window), status);
  return launch_status("v1x_stage_union");
}

extern "C" int v1x_shared_tables(const int32_t* lens, const int32_t* indexed_end, const int32_t* takes,
                                 const int32_t* selected, const int32_t* desc, int32_t* ft, int32_t* dglens,
                                 int32_t* clens, int64_t cap, int64_t max_take, int64_t scratch, int64_t fp,
                                 int64_t sink, int64_t window, int shared, int64_t rows, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(rows >= 0 && rows <= 2147483647 && fp >= 0 && max_take >= 0 && cap >= 0 && scratch >= 0,
                "tables: bad geometry");
  if (rows == 0) return V1X_OK;
  launch_kernel(shared_tables_kernel, dim3(static_cast<unsigned>(rows)), dim3(128), 0, as_stream(stream), lens,
                indexed_end, takes, selected, desc, ft, dglens, clens, static_cast<int>(cap),
                static_cast<int>(max_take), static_cast<int>(scratch), static_cast<int>(fp), static_cast<int>(sink),
                static_cast<int>(window), shared ? 1 : 0);
  return launch_status("v1x_shared_tables");
}

extern "C" int v1x_shared_normalize(const float* raw, int64_t stride, const int32_t* lens,
                                    const int32_t* indexed_end, const int32_t* takes, const int32_t* selected,
                                    const int32_t* members, int64_t member_rows, float* out, int64_t max_take,
                                    int64_t width, int64_t sink, int64_t window, int shared, int64_t rows,
                                    void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(rows >= 0 && rows <= 65535 && width >= 0 && stride >= 0 && max_take >= 0 && member_rows >= 0,
                "normalize: bad geometry");
  if (rows == 0 || width == 0) return V1X_OK;
  const dim3 grid(static_cast<unsigned>((width + 255) / 256), static_cast<unsigned>(rows));
  launch_kernel(normalize_kernel, grid, dim3(256), 0, as_stream(stream), raw, stride, lens, indexed_end, takes,
                selected, members, member_rows, out, static_cast<int>(max_take), static_cast<int>(width),
                static_cast<int>(sink), static_cast<int>(window), shared ? 1 : 0);
  return launch_status("v1x_shared_normalize");
}

extern "C" int v1x_shared_map_topk(const int64_t* ids, const float* values, const int32_t* lens,
                                   const int32_t* indexed_end, const int32_t* takes, const int32_t* selected,
                                   const int32_t* members, int64_t member_rows, const int32_t* nt, int64_t nt_len,
                                   int32_t* logical, int32_t* slots, int64_t max_take, int64_t top, int64_t sink,
                                   int64_t window, int64_t rows, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(rows >= 0 && rows <= 65535 && top >= 0 && max_take >= 0 && nt_len >= 0 && member_rows >= 0,
                "map_topk: bad geometry");
  if (rows == 0 || top == 0) return V1X_OK;
  const dim3 grid(static_cast<unsigned>((top + 255) / 256), static_cast<unsigned>(rows));
  launch_kernel(map_topk_kernel, grid, dim3(256), 0, as_stream(stream), ids, values, lens, indexed_end, takes,
                selected, members, member_rows, nt, nt_len, logical, slots, static_cast<int>(max_take),
                static_cast<int>(top), static_cast<int>(sink), static_cast<int>(window));
  return launch_status("v1x_shared_map_topk");
}

extern "C" int v1x_route_physical(const float* scores, int64_t score_stride, const int32_t* published,
                                  const int32_t* budgets, const int32_t* rt, int32_t* selected, int32_t* takes,
                                  int64_t pages, int64_t take_stride, int64_t rows, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(rows > 0 && pages > 0 && pages <= 4096 && take_stride > 0 && take_stride <= pages,
                "invalid capacity (1..4096 pages, 1..pages output width)");
  V1X_CHECK_ARG(score_stride >= pages * 8 && score_stride % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(scores) & 15) == 0,
                "route_physical: scores must be 16-byte aligned rows of >= pages*8 floats");
  int items = 1;
  while (items * 128 < pages) items *= 2;
  const int n_items = items * 128;
  const size_t smem = kPhysListOff + static_cast<size_t>(n_items) * 8;
  static DeviceOnce once;
  once.run([] {
    const int most = static_cast<int>(kPhysListOff + kPhysMaxItems * 8);
    cudaFuncSetAttribute(route_physical_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(route_physical_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
  });
  const dim3 grid(static_cast<unsigned>(rows)), block(kPhysThreads);
  if (n_items <= 2 * kPhysThreads)
    launch_kernel(route_physical_kernel<2>, grid, block, smem, as_stream(stream), scores, score_stride, published,
                  budgets, rt, selected, takes, static_cast<int>(pages), static_cast<int>(take_stride), n_items,
                  items);
  else
    launch_kernel(route_physical_kernel<16>, grid, block, smem, as_stream(stream), scores, score_stride, published,
                  budgets, rt, selected, takes, static_cast<int>(pages), static_cast<int>(take_stride), n_items,
                  items);
  return launch_status("v1x_route_physical");
}
