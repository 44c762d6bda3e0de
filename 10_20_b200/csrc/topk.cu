// fused.topk for sm_100a: in-place boundary mask + exact Top-T radix select +
// raw -> logical -> physical mapping (+ optional x4 expansion), one CTA per row.
//
// Reference behaviour: sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:62-153
// (kernel) and :181-220 (host checks).  Selection semantics: the T largest of
// scores[row, :fine_lens[row]] ordered by (value desc, index asc) -- exact ties at
// the boundary go to the lower index, where the reference falls back to
// shared-memory atomic order (topk_impl.cuh:400-401).  Outputs are written in
// ascending raw-index order (the reference leaves the order unspecified).
//
// Design: the row's candidate scores are staged once in shared memory as
// order-preserving uint32 keys; four 8-bit radix passes (warp-aggregated
// histogram atomics) find the exact T-th key and how many of its ties to keep;
// two block scans then place every selected candidate at its output slot in
// index order, and the selecting thread performs the mapping epilogue itself.
#include <algorithm>

#include "common.cuh"

namespace v1x {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkMaxSmemKeys = 48 * 1024;  // 192 KB of staged keys per CTA
constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // order_key(-inf)

struct TopkArgs {
  float* scores;
  int64_t score_stride, cols;
  const int32_t* fine_lens;
  const int32_t* members;
  int64_t member_rows;
  const int32_t* rt;
  const int32_t* nt;
  int64_t pages;
  const void* selected;
  int sel64;
  int64_t take_stride;
  const int32_t* lens;
  const int32_t* takes;
  int32_t* physical;
  int32_t* logical;
  int32_t* raw;
  int topk, window, mask;
  int32_t* expanded;
  int64_t expansion_stride;
  int physical_output, bucket_from_rank;
  const int32_t* fine_table;
  int64_t fine_table_cols;
  int direct_fine;
};

struct RowCtx {
  int64_t row;
  int n, take, sink, tail, L;
};

constexpr int kPageCache = 256;   // page ids of the first 256 selected ranks, cached in smem
constexpr int kMaxTopk = 2048;

struct TopkSmem {
  int hist[256];
  int warp_tot[kTopkThreads / 32 + 1];
  int digit, need;
  int nbnd;
  int pgc[kPageCache];
  int2 bnd[kPageCache];            // (rank index, reordered page) of boundary buckets
  int rawbuf[kMaxTopk];            // selected raw candidate ids in output order
};

// Page holding raw candidate r*64+x (r < take): the fine table's entry (direct)
// or the reordered page of the r-th selected rank (VQ:124-132).
__device__ __forceinline__ int64_t page_of_rank(const TopkArgs& a, const RowCtx& c, int r) {
  int64_t page = -1;
  if (a.direct_fine) {
    if (r < a.fine_table_cols) page = a.fine_table[c.row * a.fine_table_cols + r];
  } else if (r < a.take_stride) {
    const int64_t rank = load_index(a.selected, a.sel64, c.row * a.take_stride + r);
    if (rank >= 0 && rank < a.pages) page = a.rt[c.row * a.pages + rank];
  }
  return page;
}

// Members of the boundary bucket page `page` outside [sink, tail) -> -inf, in
// global memory and in the staged-key bitmap (VQ:94-103).
__device__ __forceinline__ void mask_page(const TopkArgs& a, const RowCtx& c, float* srow, uint32_t* bitmap,
                                          int r, int64_t page, int lane_lo, int lane_step) {
  for (int off = lane_lo; off < 64; off += lane_step) {
    const int lg = a.members[page * 64 + off];
    const int64_t col = static_cast<int64_t>(r) * 64 + off;
    if ((lg < c.sink || lg >= c.tail) && col < a.cols) {
      srow[col] = -CUDART_INF_F;
      if (bitmap) atomicOr(&bitmap[col >> 5], 1u << (col & 31));
    }
  }
}

// Selected ranks: every thread resolves its own ranks (selected -> reordered
// page, and the bucket identity) so the loads of all ranks are in flight at
// once; pages are cached for the epilogue and boundary buckets are queued.
// Then one warp per boundary page masks its members (VQ:71-107).
__device__ void ranks_and_mask(const TopkArgs& a, const RowCtx& c, float* srow, TopkSmem& sm, uint32_t* bitmap) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  for (int r = tid; r < c.take; r += nt) {
    int64_t rank = -1, rpage = -1;
    if (r < a.take_stride) rank = load_index(a.selected, a.sel64, c.row * a.take_stride + r);
    const bool rank_ok = rank >= 0 && rank < a.pages;
    if (rank_ok) rpage = a.rt[c.row * a.pages + rank];
    const int64_t epage =
        a.direct_fine ? (r < a.fine_table_cols ? a.fine_table[c.row * a.fine_table_cols + r] : -1) : rpage;
    if (r < kPageCache) sm.pgc[r] = static_cast<int>(epage);
    if (!a.mask || !rank_ok || rpage < 0 || rpage >= a.member_rows) continue;
    const int bucket = a.bucket_from_rank ? static_cast<int>(rank / 16) * 1024 : (a.members[rpage * 64] / 1024) * 1024;
    if (bucket < c.sink || bucket + 1024 > c.tail) {
      const int k = atomicAdd(&sm.nbnd, 1);
      if (k < kPageCache) sm.bnd[k] = make_int2(r, static_cast<int>(rpage));
      else mask_page(a, c, srow, bitmap, r, rpage, 0, 1);   // queue full: this thread masks it
    }
  }
  __syncthreads();
  const int nb = min(sm.nbnd, kPageCache);
  for (int k = warp; k < nb; k += nw) mask_page(a, c, srow, bitmap, sm.bnd[k].x, sm.bnd[k].y, lane, 32);
}

// Mapping epilogue for output slots tid, tid+nt, ... (VQ:121-148).  Each
// thread issues the loads of all its slots before consuming any of them.
template <bool kStaged>
__device__ void emit_all(const TopkArgs& a, const RowCtx& c, const TopkSmem& sm, const uint32_t* keys,
                         const float* srow) {
  constexpr int kPer = (kMaxTopk + kTopkThreads - 1) / kTopkThreads;
  const int tid = threadIdx.x, nt = blockDim.x;
  int raw[kPer], lg[kPer];
  bool live[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int t = tid + k * nt;
    raw[k] = t < a.topk ? sm.rawbuf[t] : -1;
    live[k] = false;
    if (raw[k] >= 0 && raw[k] < c.L) {
      if constexpr (kStaged) live[k] = keys[raw[k]] != kNegInfKey;
      else live[k] = srow[raw[k]] != -CUDART_INF_F;
    }
  }
  // raw -> logical (members load for reordered candidates)
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    lg[k] = -1;
    if (!live[k]) continue;
    const int x = raw[k];
    if (x < c.take * 64) {
      const int r = x >> 6;
      const int64_t page = r < kPageCache ? sm.pgc[r] : page_of_rank(a, c, r);
      if (page >= 0 && page < a.member_rows) lg[k] = a.members[page * 64 + (x & 63)];
    } else {
      const int off = x - c.take * 64;
      lg[k] = off < c.sink ? off : c.tail + off - c.sink;
    }
  }
  // logical -> physical (current native table) and stores
  int ph[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    ph[k] = -1;
    if (!(lg[k] >= 0 && lg[k] < c.n)) {
      lg[k] = -1;
      continue;
    }
    if (a.physical_output) {
      const int64_t p = lg[k] >> 6;
      ph[k] = p < a.pages ? a.nt[c.row * a.pages + p] * 64 + (lg[k] & 63) : -1;
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int t = tid + k * nt;
    if (t >= a.topk) continue;
    const int64_t dst = c.row * a.topk + t;
    a.logical[dst] = lg[k];
    if (a.physical_output) {
      a.physical[dst] = ph[k];
      a.raw[dst] = raw[k];
    }
    if (a.expansion_stride) {
      const int b = lg[k] * 4;
      reinterpret_cast<int4*>(a.expanded + c.row * a.expansion_stride)[t] =
          lg[k] < 0 ? make_int4(-1, -1, -1, -1) : make_int4(b, b + 1, b + 2, b + 3);
    }
  }
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

template <bool kStaged>
__device__ __forceinline__ uint32_t key_at(const uint32_t* keys, const float* srow, int i) {
  if constexpr (kStaged) return keys[i];
  else return order_key(srow[i]);
}

template <bool kStaged>
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const __grid_constant__ TopkArgs a) {
  extern __shared__ __align__(16) uint32_t keys[];
  __shared__ TopkSmem sm;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5;
  RowCtx c;
  c.row = blockIdx.x;
  c.n = a.lens[c.row];
  c.take = a.takes[c.row];
  const RowBounds rb = row_bounds(c.n, 64, a.window);
  c.sink = rb.sink;
  c.tail = rb.tail;
  c.L = static_cast<int>(min(static_cast<int64_t>(max(a.fine_lens[c.row], 0)), a.cols));
  float* srow = a.scores + c.row * a.score_stride;
  const bool select = c.L > a.topk;
  // staged path: bitmap of masked columns after the keys (words for take*64 columns)
  const int bm_words = kStaged ? static_cast<int>((min(static_cast<int64_t>(max(c.take, 0)) * 64, a.cols) + 31) / 32) : 0;
  uint32_t* bitmap = kStaged && select && a.mask ? keys + ((a.cols + 3) & ~int64_t(3)) : nullptr;
  const bool vec = (reinterpret_cast<uintptr_t>(srow) & 15) == 0;
  const int nv = (kStaged && select && vec) ? c.L >> 2 : 0;
  // 1. start the asynchronous copy of the row's scores into shared memory
  for (int v = tid; v < nv; v += nt) cp_async16(keys + 4 * v, srow + 4 * v);
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (bitmap)
    for (int w = tid; w < bm_words; w += nt) bitmap[w] = 0u;
  if (tid == 0) sm.nbnd = 0;
  __syncthreads();
  // 2. page ids of the selected ranks + boundary mask, overlapping the copy
  ranks_and_mask(a, c, srow, sm, bitmap);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  if (!select) {
    for (int t = tid; t < a.topk; t += nt) sm.rawbuf[t] = t < c.L ? t : -1;
    __syncthreads();
    emit_all<false>(a, c, sm, keys, srow);
  } else {
    if constexpr (kStaged) {
      // 3. floats -> order keys in place, masked columns -> -inf
      for (int i = tid; i < c.L; i += nt) {
        const float x = i < nv * 4 ? __uint_as_float(keys[i]) : srow[i];
        const bool masked = bitmap && i < bm_words * 32 && ((bitmap[i >> 5] >> (i & 31)) & 1u);
        keys[i] = masked ? kNegInfKey : order_key(x);
      }
      __syncthreads();
    }
    // ---- exact radix select of the T-th largest key --------------------------
    uint32_t prefix = 0, known = 0;
    int need = a.topk;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int b = tid; b < 256; b += nt) sm.hist[b] = 0;
      __syncthreads();
      const int iters = (c.L + nt - 1) / nt;
      for (int j = 0; j < iters; ++j) {
        const int i = j * nt + tid;
        int bin = -1;
        if (i < c.L) {
          const uint32_t k = key_at<kStaged>(keys, srow, i);
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
    // ---- place selected candidates in ascending index order -------------------
    const int chunk = (c.L + nt - 1) / nt;
    const int beg = min(tid * chunk, c.L), end = min(beg + chunk, c.L);
    int eq = 0, gt = 0;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = key_at<kStaged>(keys, srow, i);
      eq += k == thr;
      gt += k > thr;
    }
    int tot;
    const int eq_before = block_exclusive_scan(eq, sm.warp_tot, &tot);
    const int take_eq = min(max(need - eq_before, 0), eq);
    int pos = block_exclusive_scan(gt + take_eq, sm.warp_tot, &tot);
    int eq_seen = eq_before;
    for (int i = beg; i < end; ++i) {
      const uint32_t k = key_at<kStaged>(keys, srow, i);
      bool sel = k > thr;
      if (k == thr) {
        sel = eq_seen < need;
        ++eq_seen;
      }
      if (sel && pos < a.topk) sm.rawbuf[pos++] = i;
    }
    __syncthreads();
    emit_all<kStaged>(a, c, sm, keys, srow);
  }
  if (a.expansion_stride) {
    for (int64_t j = static_cast<int64_t>(a.topk) * 4 + tid; j < a.expansion_stride; j += nt)
      a.expanded[c.row * a.expansion_stride + j] = -1;
  }
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_topk(float* scores, int64_t score_stride, int64_t cols, const int32_t* fine_lens,
                        const int32_t* members, int64_t member_rows, const int32_t* rt,
                        const int32_t* nt, int64_t pages, const void* selected, int selected_is_i64,
                        int64_t take_stride, const int32_t* lens, const int32_t* takes,
                        int32_t* physical, int32_t* logical, int32_t* raw, int64_t topk,
                        int64_t window, int mask, int32_t* expanded, int64_t expansion_stride,
                        int physical_output, int bucket_from_rank, const int32_t* fine_table,
                        int64_t fine_table_cols, int direct_fine, int64_t batch, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(batch >= 0, "topk: negative batch");
  V1X_CHECK_ARG(topk > 0 && topk <= 2048, "Unsupported fused V1 TopK: topk=%lld", (long long)topk);
  V1X_CHECK_ARG(window >= 0 && window <= 4096, "Unsupported fused V1 TopK: window=%lld",
                (long long)window);
  V1X_CHECK_ARG(expansion_stride == 0 || expansion_stride == topk * 4 + 64,
                "Invalid expansion buffer");
  V1X_CHECK_ARG(!direct_fine || fine_table_cols >= take_stride, "Invalid direct fine table");
  V1X_CHECK_ARG(score_stride >= cols && cols >= 0, "topk: score stride < cols");
  V1X_CHECK_ARG(pages > 0 && take_stride >= 0 && member_rows > 0, "topk: bad table shapes");
  if (batch == 0) return V1X_OK;
  TopkArgs a{scores, score_stride, cols, fine_lens, members, member_rows, rt, nt, pages, selected,
             selected_is_i64, take_stride, lens, takes, physical, logical, raw,
             static_cast<int>(topk), static_cast<int>(window), mask, expanded, expansion_stride,
             physical_output, bucket_from_rank, fine_table, fine_table_cols, direct_fine};
  cudaStream_t s = as_stream(stream);
  V1X_CHECK_ARG(take_stride <= 65536, "topk: take stride too large");
  if (cols <= kTopkMaxSmemKeys) {
    const int64_t bm = (std::min<int64_t>(take_stride * 64, cols) + 31) / 32;
    const size_t smem = static_cast<size_t>(((cols + 3) & ~int64_t(3)) + bm + 1) * 4;
    if (smem > 48 * 1024) {
      static DeviceOnce once;
      if (once.first()) {
        cudaFuncSetAttribute(topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kTopkMaxSmemKeys * 4 + kTopkMaxSmemKeys / 8 + 64);
      }
    }
    topk_kernel<true><<<static_cast<unsigned>(batch), kTopkThreads, smem, s>>>(a);
  } else {
    topk_kernel<false><<<static_cast<unsigned>(batch), kTopkThreads, 0, s>>>(a);
  }
  return launch_status("v1x_topk");
}
