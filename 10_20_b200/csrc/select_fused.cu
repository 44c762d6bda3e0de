// The selection of one query row in one CTA, for sm_100a: query metadata,
// fused.route over the centre page maxima, FP8 fine scoring of the row's
// candidates on the tensor cores, the in-kernel boundary mask, the exact
// Top-T and the raw -> logical -> physical mapping.
//
// Reference sequence replaced (sglang/srt/layers/attention/v1_deepseek/
// runtime.py:446-611 with the fixed page budget of
// bench_v1_dynamic_budget_metadata.py:5-28): query_metadata
// (DS/kernels.py:568-591), fused.route (v1_query.cuh:7-49), fine_table_shared
// (DS/kernels.py:488-514), stage_tail_shared (:518-564), DeepGEMM fine logits
// over the fine pool (runtime.py:538-548, formula DS/kernels.py:310-313) and
// fused.topk (v1_query.cuh:62-153).  The outputs are those of that sequence;
// the fine logits never leave the SM.
//
// B200 design, one CTA of 256 threads per row:
//   * metadata and the shared-tail owner (tail_rows) from the row's length and
//     native page table;
//   * route: the row's page maxima (written by the centre scorer's epilogue) ->
//     the take best pages in the reference's stable order (a 12-bit histogram
//     finds the bin of the K-th key, the winners are ordered by counting);
//   * fine scoring: tiles of 128 keys = two 64-token pages, each moved by TMA
//     (128-byte swizzle) into a ring of shared-memory stages and contracted
//     with the row's q on the 5th-generation tensor cores (tcgen05.mma
//     kind::f8f6f4, E4M3 x E4M3 -> F32, accumulators in TMEM).  The sink and
//     tail candidates are read straight from the NATIVE pages that hold them --
//     there is no staging copy (the reference copies them into per-row fine
//     pool pages first); their loads are issued before the route, so they land
//     while the route runs.  The selected pages' tiles follow.
//   * epilogue (4 warps, one key per thread): tcgen05.ld of the H head columns,
//     ReLU, the weighted head sum, the key's scale, the boundary-bucket mask;
//     each score's order key lands in shared memory at its raw candidate
//     column and is counted in the Top-T histogram as it is written;
//   * Top-T over the shared-memory row (histogram bin, exact ranking of the
//     threshold bin, ties to the lower index), outputs in ascending raw order,
//     mapped through the staged members and the native page table.
// Warp roles during scoring: warp 1 TMEM owner and MMA issuer, warps 2-5
// epilogue, warp 0 and the warps past the epilogue (6-7) TMA producers -- warp 0
// alone issues the sink/tail tiles before the route, then each ring stage is fed
// by one producer warp in tile order (a stage fed by two warps could see a
// parity wait pass two phases behind); every warp takes part in the metadata,
// route and Top-T phases.  Every mbarrier wait is bounded (2 s): on expiry the CTA
// writes V1X_STATUS_TIMEOUT, lets what it issued retire, frees its TMEM and
// leaves the row's outputs unwritten.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "select.cuh"
#include "sm100.cuh"

namespace v1x {
namespace {

using namespace sm100;

constexpr int kSfMaxThreads = 512;
constexpr int kSfMaxWarps = kSfMaxThreads / 32;
constexpr int kProdWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;               // warps 2-5 (and 6-9: a second group with 512 threads)
constexpr int kSfAcc = 4;                  // TMEM accumulators in flight
constexpr int kMaxStages = 8;
constexpr int kMaxScaleSlots = 16;
constexpr int kMaxNativePages = 72;        // sink page + tail pages (window <= 4096)
constexpr int kSfMaxBin = 2048;            // threshold-bin keys ranked exactly
constexpr int kSfSmallBin = 96;
constexpr int kSfMaxBin2 = 256;

// Bytes of sf_topk's scratch for rows of max_cand candidates: the 16 KB
// candidate list, the selection bit flags, the sub-bin histogram and list.
__host__ __device__ constexpr int64_t sf_topk_scratch_bytes(int64_t max_cand) {
  return 16384 + (max_cand + 1023) / 1024 * 128 + 1024 + kSfMaxBin2 * 8;
}
constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // order_key(-inf)
constexpr uint64_t kSfWaitNs = 2000000000ull;
constexpr int kRankDirectSf = 256;

struct SfArgs {
  const int32_t* lens;
  const int32_t* budget;      // device word (fixed budget) or NULL: ratio rule num/den
  int num, den;
  const int32_t* nt;          // [B, pages] native page table
  const int32_t* rt;          // [B, pages] reordered page table
  int pages;
  const float* page_scores;   // [B, page_stride] max of each page's 8 centre logits
  int64_t page_stride;
  const float* w;             // [B, H]
  int H, N;                   // heads, MMA width (16 for one head)
  const int32_t* members;     // [member_rows, 64]
  int64_t member_rows, capacity;
  int topk, window, take_stride;
  int64_t fine_cols;          // fine-table columns
  int32_t *fine_lens, *takes, *dg_lens, *center_lens, *tail_rows;
  int32_t* selected;          // [B, take_stride]
  int32_t* fine_table;        // [B, fine_cols]
  int32_t *physical, *logical, *raw, *expanded;
  int64_t expansion_stride;
  float* scores_out;          // optional [B, score_stride]: the masked fine logits
  int64_t score_stride;
  int B, stages, scale_slots, n_items, base, max_cand;
  uint32_t tmem_cols;
  int32_t* status;
  // dynamic shared-memory offsets (bytes from the 1024-aligned base)
  int off_q, off_sring, off_w, off_sel, off_sh, off_tab, off_u;
};

struct SfShared {
  uint64_t full[kMaxStages], empty[kMaxStages];
  uint64_t sfull[kMaxScaleSlots], sempty[kMaxScaleSlots];
  uint64_t tfull[kSfAcc], tempty[kSfAcc];
  uint64_t qfull;
  uint32_t tmem_base;
  int abort, zero;
  // row metadata
  int n, take, sink, tail, L, tail_row, ntiles_nat, ntiles;
  int natp[kMaxNativePages];   // logical page numbers of the sink / tail pages
  // route / Top-T scratch
  int4 red[2 * kSfMaxWarps];
  int warp_tot[kSfMaxWarps + 1];
  int2 wcnt[kSfMaxWarps];      // per warp: threshold-bin candidates, then their offsets
  uint32_t wmin[kSfMaxWarps], wmax[kSfMaxWarps];
  int4 res, res2;
  int2 carry;
  int count, ncand, ncand2;
  uint32_t kmin, kmax, kmin2, kmax2;
};

__device__ __forceinline__ void sf_cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

__device__ __forceinline__ void sf_abort(SfShared& sh, int32_t* status) {
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
  if (status) atomicExch(status, V1X_STATUS_TIMEOUT);
}

// ---------------------------------------------------------------------------
// route of one row (v1_query.cuh:7-49) by the whole CTA: page keys from the
// page maxima, the want-th key's histogram bin, winners ordered by (key desc,
// blocked rank asc).  Writes selected[0:take_stride], the fine table, and the
// row's selected pages / boundary flags into shared memory.
// ---------------------------------------------------------------------------
template <int kThreads, int kPer>
__device__ void sf_route(const SfArgs& a, SfShared& sh, int64_t row, int* hist, unsigned long long* list,
                         int* spage, uint8_t* sbnd, const float* spsc, const int* rtrow) {
  constexpr int kWarps = kThreads / 32;
  const int tid = threadIdx.x, nt = kThreads;
  const int n = sh.n, take = sh.take;
  const int active = max(n - 1, 0) / 1024 * 16;
  int32_t* ftrow = a.fine_table + row * a.fine_cols;
  const int64_t base_ft = a.capacity + static_cast<int64_t>(sh.tail_row) * 68;
  for (int64_t j = take + tid; j < a.fine_cols; j += nt)
    ftrow[j] = static_cast<int32_t>(base_ft + min(j - take, int64_t(67)));
  auto set_rank = [&](int pos, int p) {
    if (pos < a.take_stride) a.selected[row * a.take_stride + pos] = p;
    if (pos < take) {
      const int page = p < a.pages ? rtrow[p] : -1;
      if (pos < a.fine_cols) ftrow[pos] = page;
      spage[pos] = page;
      const int bucket = (p / 16) * 1024;   // bucket of the rank (query_bucket_rank_mask)
      sbnd[pos] = (bucket < sh.sink || bucket + 1024 > sh.tail) ? 1 : 0;
    }
  };
  const int want = min(a.n_items, max(a.take_stride, take));
  if (take >= active || want <= 0) {
    if (take >= active)
      for (int i = tid; i < max(a.take_stride, take); i += nt) set_rank(i, i);
    __syncthreads();
    return;
  }
  if (tid == 0) sh.count = 0;
  const int act = min(active, a.pages);
  uint32_t kr[kPer];
  const int nv = a.n_items > tid ? (a.n_items - tid + nt - 1) / nt : 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = tid + j * nt;
    kr[j] = order_key(p < act ? spsc[p] : -CUDART_INF_F);
  }
  zero_hist<kThreads>(hist);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (j < nv) atomicAdd(&hist[bin_of(kr[j])], 1);
  __syncthreads();
  const TopBin tb = find_top_bin<kThreads>(want, hist, sh.warp_tot, &sh.res);
  uint32_t lo = static_cast<uint32_t>(tb.bin) << (32 - kBinBits);
  if (tb.above + tb.in > kRankDirectSf) {
    int gt = 0;
    lo = block_kth_largest<kWarps>(
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
        sh.red, &gt);
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (j < nv && kr[j] >= lo) {
      const int p = tid + j * nt;
      const uint32_t rank = static_cast<uint32_t>((p & 127) * a.base + (p >> 7));
      const int e = atomicAdd(&sh.count, 1);
      list[e] = (static_cast<unsigned long long>(kr[j]) << 32) | (0xFFFFFFFFu - rank);
    }
  }
  __syncthreads();
  const int m = sh.count;
  auto emit = [&](int pos, unsigned long long comp) {
    const int r = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(comp & 0xFFFFFFFFull));
    set_rank(pos, r / a.base + (r % a.base) * 128);
  };
  if (m <= kRankDirectSf) {
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
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Top-T of the row's keys in shared memory (order-preserving uint32 keys,
// kNegInfKey for -inf), (key desc, index asc); emit(pos, raw) for every output
// slot in ascending raw order.  hist: the keys' 12-bit histogram, already
// counted (the scoring epilogue adds each key as it writes it).  Every pass
// over the keys is blocked -- thread t owns the contiguous keys [t*per,
// (t+1)*per) -- so one block scan of per-thread counts places a thread's
// candidates and outputs in index order.  scratch: 16 KB candidate list + bit
// flags + 1 KB + the sub-bin list (the stage ring, free by now).
// ---------------------------------------------------------------------------
template <int kThreads, class Emit>
__device__ void sf_topk(SfShared& sh, const uint32_t* keys, const int* hist, int L, int T, uint8_t* scratch,
                        Emit emit) {
  constexpr int kWarps = kThreads / 32;
  const int tid = threadIdx.x, nt = kThreads, lane = tid & 31;
  if (L <= T) {
    for (int t = tid; t < T; t += nt) emit(t, t < L ? t : -1);
    return;
  }
  int2* cand = reinterpret_cast<int2*>(scratch);                                // 16 KB
  uint32_t* selbit = reinterpret_cast<uint32_t*>(scratch + 16384);              // L/32 words
  int* hist2 = reinterpret_cast<int*>(scratch + 16384 + ((L + 1023) / 1024) * 128);  // 256
  int2* cand2 = reinterpret_cast<int2*>(hist2 + 256);                           // kSfMaxBin2
  const int per = (L + nt - 1) / nt;
  const int i0 = min(tid * per, L), i1 = min(i0 + per, L);
  for (int wd = tid; wd < (L + 31) / 32; wd += nt) selbit[wd] = 0u;
  if (tid < 256) hist2[tid] = 0;
  if (tid == 0) {
    sh.ncand2 = 0;
    sh.kmin2 = 0xFFFFFFFFu;
    sh.kmax2 = 0u;
  }
  const TopBin tb = find_top_bin<kThreads>(T, hist, sh.warp_tot, &sh.res);   // (contains barriers)
  const bool keep = tb.in <= kSfMaxBin;
  {
    // the threshold bin's keys: this thread's count and key range, a block scan
    // of the counts, then each thread writes its candidates in index order
    int c = 0;
    uint32_t lo = 0xFFFFFFFFu, hi = 0u;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = keys[i];
      if (bin_of(k) == tb.bin) {
        ++c;
        lo = min(lo, k);
        hi = max(hi, k);
      }
    }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lane == 0) {
      sh.wmin[tid >> 5] = lo;
      sh.wmax[tid >> 5] = hi;
    }
    int tot;
    int b0 = block_exclusive_scan(c, sh.warp_tot, &tot);   // (barriers make wmin / wmax visible)
    if (tid == 0) {
      uint32_t mn = 0xFFFFFFFFu, mx = 0u;
      for (int w = 0; w < kWarps; ++w) {
        mn = min(mn, sh.wmin[w]);
        mx = max(mx, sh.wmax[w]);
      }
      sh.kmin = mn;
      sh.kmax = mx;
    }
    if (keep && c > 0)
      for (int i = i0; i < i1; ++i) {
        const uint32_t k = keys[i];
        if (bin_of(k) == tb.bin) cand[b0++] = make_int2(static_cast<int>(k), i);
      }
  }
  __syncthreads();
  bool by_bin = false, have_tie = false;
  uint32_t tie_thr = 0;
  int tie_need = 0;
  if (sh.kmin == sh.kmax) {
    tie_thr = sh.kmin;
    tie_need = T - tb.above;
    have_tie = true;
  } else if (keep) {
    by_bin = true;
    int need_bin = T - tb.above;
    const int2* rk = cand;
    int nres = tb.in;
    if (tb.in > kSfSmallBin) {
      for (int q = tid; q < tb.in; q += nt) atomicAdd(&hist2[(cand[q].x >> (24 - kBinBits)) & 255], 1);
      __syncthreads();
      if (tid < 32) {
        const int hb = 256 - lane * 8;
        int cc[8], sm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          cc[j] = hist2[hb - 8 + j];
          sm += cc[j];
        }
        int cum = warp_inclusive_scan(sm) - sm;
        if (cum < need_bin && cum + sm >= need_bin) {
#pragma unroll
          for (int j = 7; j >= 0; --j) {
            if (cum < need_bin && cum + cc[j] >= need_bin) sh.res2 = make_int4(hb - 8 + j, cum, cc[j], 0);
            cum += cc[j];
          }
        }
      }
      __syncthreads();
      const int4 r2 = sh.res2;
      if (r2.z <= kSfMaxBin2) {
        for (int q = tid; q < tb.in; q += nt) {
          const int2 me = cand[q];
          const int sub = (me.x >> (24 - kBinBits)) & 255;
          if (sub > r2.x) atomicOr(&selbit[me.y >> 5], 1u << (me.y & 31));
          else if (sub == r2.x) cand2[atomicAdd(&sh.ncand2, 1)] = me;
        }
        __syncthreads();
        need_bin -= r2.y;
        rk = cand2;
        nres = r2.z;
      } else {
        by_bin = false;
        uint32_t lo = 0xFFFFFFFFu, hi = 0u;
        for (int q = tid; q < tb.in; q += nt) {
          const uint32_t k = static_cast<uint32_t>(cand[q].x);
          if (((k >> (24 - kBinBits)) & 255) == static_cast<uint32_t>(r2.x)) {
            lo = min(lo, k);
            hi = max(hi, k);
          }
        }
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        if (lane == 0) {
          atomicMin(&sh.kmin2, lo);
          atomicMax(&sh.kmax2, hi);
        }
        __syncthreads();
        if (sh.kmin2 == sh.kmax2) {
          tie_thr = sh.kmin2;
          tie_need = need_bin - r2.y;
          have_tie = true;
        }
      }
    }
    if (by_bin) {
      for (int q = tid; q < nres; q += nt) {
        const int2 me = rk[q];
        const uint32_t k = static_cast<uint32_t>(me.x);
        int r = 0;
        for (int f = 0; f < nres; ++f) {
          const int2 o = rk[f];
          const uint32_t ko = static_cast<uint32_t>(o.x);
          r += (ko > k) | ((ko == k) & (o.y < me.y));
        }
        if (r < need_bin) atomicOr(&selbit[me.y >> 5], 1u << (me.y & 31));
      }
      __syncthreads();
    }
  }
  uint32_t thr = tie_thr;
  int need = tie_need;
  if (!by_bin && !have_tie) {
    int gt = 0;
    thr = block_kth_largest<kWarps>(
        T,
        [&](uint32_t c1, uint32_t c2, uint32_t c3, int& n1, int& n2, int& n3) {
          n1 = n2 = n3 = 0;
          for (int i = i0; i < i1; ++i) {
            const uint32_t k = keys[i];
            n1 += k >= c1;
            n2 += k >= c2;
            n3 += k >= c3;
          }
        },
        sh.red, &gt);
    need = T - gt;
  }
  // class of candidate i with key k: 1 = selected outright, 2 = tie of thr
  // (selected while fewer than `need` ties precede it), 0 = not selected
  auto klass = [&](int i, uint32_t k) -> int {
    if (by_bin) {
      const int b = bin_of(k);
      return (b > tb.bin || (b == tb.bin && ((selbit[i >> 5] >> (i & 31)) & 1u))) ? 1 : 0;
    }
    return k > thr ? 1 : (k == thr ? 2 : 0);
  };
  // this thread's (selected, tie) counts -> one block scan -> output slots; the
  // classes of a thread's first 32 keys are kept as bit masks between the two
  // passes
  int g = 0, e = 0;
  uint32_t m1 = 0u, m2 = 0u;
  for (int i = i0; i < i1; ++i) {
    const int kl = klass(i, keys[i]);
    g += kl == 1;
    e += kl == 2;
    if (i - i0 < 32) {
      m1 |= static_cast<uint32_t>(kl == 1) << (i - i0);
      m2 |= static_cast<uint32_t>(kl == 2) << (i - i0);
    }
  }
  long long tot;
  const long long packed = block_exclusive_scan((static_cast<long long>(g) << 32) | e,
                                                reinterpret_cast<long long*>(sh.red), &tot);
  int gt_lt = static_cast<int>(packed >> 32), eq_lt = static_cast<int>(packed & 0xFFFFFFFFll);
  for (int i = i0; i < i1; ++i) {
    const int j = i - i0;
    const int kl = j < 32 ? static_cast<int>(((m1 >> j) & 1u) | (((m2 >> j) & 1u) << 1)) : klass(i, keys[i]);
    if (kl == 1) emit(gt_lt + min(eq_lt, need), i);
    else if (kl == 2 && eq_lt < need) emit(gt_lt + eq_lt, i);
    gt_lt += kl == 1;
    eq_lt += kl == 2;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// kThreads: 256 as launched (one epilogue group; warps 6-7 join warp 0 as
// producers after the route); the code also serves 512 (two epilogue groups on
// alternate tiles, warps 10-15 producers).  kPer: route keys per thread
// (n_items / kThreads rounded up).
template <int kThreads, int kPer>
__global__ void __launch_bounds__(kThreads, kThreads >= 512 ? 1 : 2)
    select_fused_kernel(const __grid_constant__ CUtensorMap fine_map, const __grid_constant__ CUtensorMap fine_scales,
                        const __grid_constant__ CUtensorMap nat_map, const __grid_constant__ CUtensorMap nat_scales,
                        const __grid_constant__ CUtensorMap q_map, const __grid_constant__ SfArgs a) {
  constexpr int kGroups = kThreads >= 512 ? 2 : 1;       // epilogue groups
  constexpr int kHelper0 = kEpiWarp0 + 4 * kGroups;      // first warp idle during scoring
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = base;                                                  // stages x 16 KB
  uint8_t* qsm = base + a.off_q;                                           // N x 128 B
  float* sring = reinterpret_cast<float*>(base + a.off_sring);             // scale slots x 128
  float* wsm = reinterpret_cast<float*>(base + a.off_w);                   // H
  int* spage = reinterpret_cast<int*>(base + a.off_sel);                   // take_stride
  uint8_t* sbnd = reinterpret_cast<uint8_t*>(spage + a.take_stride);       // take_stride
  // the row's tables, copied at the start: page maxima, reordered and native pages
  float* spsc = reinterpret_cast<float*>(base + a.off_tab);
  int* srt = reinterpret_cast<int*>(spsc + a.pages);
  int* sntab = srt + a.pages;
  int* thist = reinterpret_cast<int*>(base + a.off_tab + ((a.pages * 12 + 15) & ~15));  // the keys' histogram
  uint8_t* uni = base + a.off_u;
  // route view of the union: histogram + winner list
  int* rhist = reinterpret_cast<int*>(uni);
  unsigned long long* rlist = reinterpret_cast<unsigned long long*>(uni + 16384);
  // row view of the union: scores (keys after the Top-T conversion) + members
  float* sc = reinterpret_cast<float*>(uni);
  int* memb = reinterpret_cast<int*>(uni + static_cast<size_t>(a.max_cand) * 4);
  SfShared& sh = *reinterpret_cast<SfShared*>(base + a.off_sh);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x;
  const int S = a.stages, SS = a.scale_slots;

  // ---- the row's tables: asynchronous copies, in flight during the set-up ---------
  {
    const float* ps = a.page_scores + row * a.page_stride;
    const int32_t* rt = a.rt + row * a.pages;
    const int32_t* ntr = a.nt + row * a.pages;
    const bool v16 = ((reinterpret_cast<uintptr_t>(ps) | reinterpret_cast<uintptr_t>(rt) |
                       reinterpret_cast<uintptr_t>(ntr)) & 15) == 0 && (a.pages & 3) == 0;
    if (v16) {
      for (int v = tid; v < a.pages / 4; v += kThreads) {
        sf_cp_async16(spsc + 4 * v, ps + 4 * v);
        sf_cp_async16(srt + 4 * v, rt + 4 * v);
        sf_cp_async16(sntab + 4 * v, ntr + 4 * v);
      }
    } else {
      for (int v = tid; v < a.pages; v += kThreads) {
        spsc[v] = ps[v];
        srt[v] = rt[v];
        sntab[v] = ntr[v];
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  // ---- set-up: barriers, TMEM, tensor-map prefetch -------------------------------
  if (tid == 0) {
    sh.abort = 0;
    sh.zero = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int r = 0; r < SS; ++r) {
      mbar_init(&sh.sfull[r], 1);
      mbar_init(&sh.sempty[r], 128);
    }
    for (int c = 0; c < kSfAcc; ++c) {
      mbar_init(&sh.tfull[c], 1);
      mbar_init(&sh.tempty[c], 128);
    }
    mbar_init(&sh.qfull, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sh.tmem_base, a.tmem_cols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp == kProdWarp && lane == 0) {
    tma_prefetch_desc(&fine_map);
    tma_prefetch_desc(&fine_scales);
    tma_prefetch_desc(&nat_map);
    tma_prefetch_desc(&nat_scales);
    tma_prefetch_desc(&q_map);
  }
  // ---- metadata (DS/kernels.py:568-591; fixed budget or ratio take rule) ---------
  const int n = a.lens[row];
  const int n0 = a.lens[0];
  const int built_pages = max(n - 1, 0) / 1024 * 16;
  int take;
  if (a.budget) {
    take = min(built_pages, *a.budget);
  } else {
    const int64_t r = (static_cast<int64_t>(built_pages) * a.num + a.den - 1) / a.den;
    take = static_cast<int>(min(static_cast<int64_t>(built_pages), max(r, static_cast<int64_t>((a.topk + 63) / 64))));
  }
  take = max(min(take, a.take_stride), 0);
  const RowBounds rb = row_bounds(n, 64, a.window);
  const int L = take * 64 + rb.sink + n - rb.tail;
  // shared-tail owner: row 0 when this row has row 0's length and the same native
  // pages at page 0 and pages tail/64 ... (up to 127 of them); row 0's entries
  // are read from global memory (every CTA reads the same ones), this row's from
  // its staged table
  int first = -1;
  const int tpage = tid == 0 ? 0 : rb.tail / 64 + tid - 1;
  const bool tvalid = tid < 128 && n > 0 && (tid == 0 || tpage < (n + 63) / 64) && tpage < a.pages;
  if (tvalid && n == n0) first = a.nt[tpage];
  if (tid < a.H) wsm[tid] = a.w[row * a.H + tid];
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const bool differs = tid < 128 && (tvalid ? sntab[tpage] : -1) != (tvalid ? first : -1);
  const int any_differs = __syncthreads_or(differs && n == n0);   // every thread takes part
  const bool share = n == n0 && !any_differs;
  if (tid == 0) {
    sh.n = n;
    sh.take = take;
    sh.sink = rb.sink;
    sh.tail = rb.tail;
    sh.L = L;
    sh.tail_row = share ? 0 : static_cast<int>(row);
    a.fine_lens[row] = L;
    a.takes[row] = take;
    a.dg_lens[row] = max(L, 1);
    a.center_lens[row] = max(built_pages * 8, 1);
    a.tail_rows[row] = share ? 0 : static_cast<int>(row);
    // native pages holding the sink [0, sink) and the tail [tail, n)
    int np = 0;
    if (rb.sink > 0) sh.natp[np++] = 0;
    if (n > rb.tail)
      for (int p = rb.tail / 64; p <= (n - 1) / 64 && np < kMaxNativePages; ++p)
        if (p != 0 || rb.sink == 0) sh.natp[np++] = p;
    sh.ntiles_nat = (np + 1) / 2;
    sh.ntiles = sh.ntiles_nat + (take + 1) / 2;
    for (int p = np; p < 2 * sh.ntiles_nat; ++p) sh.natp[p] = -1;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int ntiles = sh.ntiles, nnat = sh.ntiles_nat;
  const uint32_t q_bytes = static_cast<uint32_t>(a.N) * 128;

  // producer warp: one tile's loads (tile t: native pages first, then selected
  // ranks).  Lane 0 waits for the stage and arms the barriers; lanes 0-1 issue
  // the two page boxes and lanes 2-3 the two scale vectors, in parallel.
  auto issue = [&](int t) -> bool {
    const int s = t % S, r = t % SS;
    bool ok = true;
    if (lane == 0)
      ok = mbar_wait(&sh.empty[s], ((t / S) & 1) ^ 1, &sh.abort, kSfWaitNs) &&
           mbar_wait(&sh.sempty[r], ((t / SS) & 1) ^ 1, &sh.abort, kSfWaitNs);
    if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return false;
    const bool nat = t < nnat;
    int pg = -1;                              // lanes 0-1 and 2-3: page of half lane & 1
    if (lane < 4) {
      const int h = lane & 1;
      if (nat) {
        const int lp = sh.natp[2 * t + h];
        pg = (lp >= 0 && lp < a.pages) ? sntab[lp] : -1;
      } else {
        const int k = t - nnat;
        pg = 2 * k + h < sh.take ? spage[2 * k + h] : -1;
      }
    }
    const unsigned have = __ballot_sync(0xffffffffu, lane < 2 && pg >= 0);
    if (lane == 0) {
      const uint32_t halves = __popc(have);
      mbar_arrive_expect_tx(&sh.full[s], 8192u * halves);
      mbar_arrive_expect_tx(&sh.sfull[r], 256u * halves);
    }
    __syncwarp();
    if (lane < 4 && pg >= 0) {
      const int h = lane & 1;
      if (lane < 2) tma_load_3d(stages + s * 16384 + h * 8192, nat ? &nat_map : &fine_map, &sh.full[s], 0, 0, pg);
      else tma_load_2d(sring + r * 128 + h * 64, nat ? &nat_scales : &fine_scales, &sh.sfull[r], 0, pg);
    }
    return true;
  };

  // Producers: warp 0 and the warps idle during scoring.  Stage s is fed by
  // producer s % nprod only, in tile order, before and after the route: a
  // stage's next tile is issued by the warp that issued its previous one, so
  // the parity waits on its barriers can never see a phase two behind.
  const int pidx = warp == kProdWarp ? 0 : (warp >= kHelper0 ? 1 + warp - kHelper0 : -1);
  const int nprod = min(1 + kThreads / 32 - kHelper0, S);
  const auto mine = [&](int t) { return (t % S) % nprod == pidx; };
  const bool producer = pidx >= 0 && pidx < nprod;
  int last = -1;                             // the last tile this warp issued
  if (warp == kProdWarp && lane == 0) {
    mbar_arrive_expect_tx(&sh.qfull, q_bytes);
    tma_load_2d(qsm, &q_map, &sh.qfull, 0, static_cast<int>(row) * a.H);
  }
  // the sink / tail tiles do not depend on the route: their loads fly while it
  // runs (each producer issues those on its own stages)
  const int pre = min(nnat, min(S, SS));
  if (producer) {
    for (int t = 0; t < pre; ++t) {
      if (!mine(t)) continue;
      if (!issue(t)) {
        if (lane == 0) sf_abort(sh, a.status);
        break;
      }
      last = t;
    }
  }

  // ---- route (all threads) ----------------------------------------------------------
  sf_route<kThreads, kPer>(a, sh, row, rhist, rlist, spage, sbnd, spsc, srt);
  // (sf_route ends with a barrier: spage / sbnd are visible)

  if (warp == kProdWarp || warp >= kHelper0) {
    // producers after the route, on their own stages
    if (producer && !*reinterpret_cast<volatile int*>(&sh.abort)) {
      for (int t = pre; t < ntiles; ++t) {
        if (!mine(t)) continue;
        if (__shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&sh.abort), 0)) break;
        if (!issue(t)) {
          if (lane == 0) sf_abort(sh, a.status);
          break;
        }
        last = t;
      }
    }
    if (lane == 0 && *reinterpret_cast<volatile int*>(&sh.abort)) {  // let this warp's recent loads land
      for (int k = 0, it = last; k < S && it >= 0; --it) {
        if (!mine(it)) continue;
        mbar_wait(&sh.full[it % S], (it / S) & 1, &sh.zero, kSfWaitNs);
        mbar_wait(&sh.sfull[it % SS], (it / SS) & 1, &sh.zero, kSfWaitNs);
        ++k;
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc = idesc_e4m3_f32(128, a.N);
      int t = 0;
      if (!mbar_wait(&sh.qfull, 0, &sh.abort, kSfWaitNs)) {
        sf_abort(sh, a.status);
      } else {
        for (; t < ntiles; ++t) {
          const int s = t % S, acc = t % kSfAcc;
          if (!mbar_wait(&sh.tempty[acc], ((t / kSfAcc) & 1) ^ 1, &sh.abort, kSfWaitNs) ||
              !mbar_wait(&sh.full[s], (t / S) & 1, &sh.abort, kSfWaitNs)) {
            sf_abort(sh, a.status);
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + s * 16384);
          const uint32_t sb = smem_u32(qsm);
          const uint32_t d = tmem + static_cast<uint32_t>(acc * a.N);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f8(d, umma_desc_sw128(sa + 32 * k), umma_desc_sw128(sb + 32 * k), idesc, k > 0 ? 1u : 0u);
          umma_commit(&sh.empty[s]);
          umma_commit(&sh.tfull[acc]);
        }
      }
      if (*reinterpret_cast<volatile int*>(&sh.abort) && t > 0)
        mbar_wait(&sh.tfull[(t - 1) % kSfAcc], ((t - 1) / kSfAcc) & 1, &sh.zero, kSfWaitNs);
    }
  } else if (warp < kHelper0) {
    // ---- epilogue: members of the selected pages, then one key per thread; group
    // g takes tiles g, g + kGroups, ... ------------------------------------------------
    const int e = tid - 32 * kEpiWarp0;      // 0 .. 128 * kGroups - 1
    const int g = e >> 7;
    const int tk = sh.take, sink = sh.sink, tail = sh.tail;
    for (int rr = e; rr < tk; rr += 128 * kGroups) {
      const int page = spage[rr];
      if (page >= 0 && page < a.member_rows) {
        const int32_t* src = a.members + static_cast<int64_t>(page) * 64;
#pragma unroll
        for (int q = 0; q < 16; ++q) sf_cp_async16(memb + rr * 64 + 4 * q, src + 4 * q);
      } else {
        for (int q = 0; q < 64; ++q) memb[rr * 64 + q] = -1;
      }
    }
    // the Top-T histogram, counted as the keys are written
    for (int v = e; v < kBins / 4; v += 128 * kGroups) reinterpret_cast<int4*>(thist)[v] = make_int4(0, 0, 0, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_all;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"r"(128 * kGroups) : "memory");
    const int q4 = warp & 3;
    const int i = q4 * 32 + lane;            // key of the tile == TMEM lane
    const int h = i >> 6, slot = i & 63;
    float* gout = a.scores_out ? a.scores_out + row * a.score_stride : nullptr;
    for (int t = g; t < ntiles; t += kGroups) {
      const int acc = t % kSfAcc, r = t % SS;
      if (!mbar_wait(&sh.sfull[r], (t / SS) & 1, &sh.abort, kSfWaitNs) ||
          !mbar_wait(&sh.tfull[acc], (t / kSfAcc) & 1, &sh.abort, kSfWaitNs)) {
        sf_abort(sh, a.status);
        break;
      }
      const float scale = sring[r * 128 + i];
      tc_fence_after();
      const uint32_t ta = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(acc * a.N);
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      if (a.H == 1) {
        const float v0 = fmaxf(__uint_as_float(tmem_ld1(ta)), 0.0f);
        tmem_ld_wait();
        s0 = wsm[0] * v0;
      }
      for (int c0 = 0; a.H > 1 && c0 < a.H; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(ta + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(wsm + c0 + j);
          s0 = fmaf(w4.x, fmaxf(__uint_as_float(v[j]), 0.0f), s0);
          s1 = fmaf(w4.y, fmaxf(__uint_as_float(v[j + 1]), 0.0f), s1);
          s2 = fmaf(w4.z, fmaxf(__uint_as_float(v[j + 2]), 0.0f), s2);
          s3 = fmaf(w4.w, fmaxf(__uint_as_float(v[j + 3]), 0.0f), s3);
        }
      }
      tc_fence_before();
      mbar_arrive(&sh.tempty[acc]);
      mbar_arrive(&sh.sempty[r]);
      float score = ((s0 + s1) + (s2 + s3)) * scale;
      int col = -1;
      if (t < nnat) {
        const int lp = sh.natp[2 * t + h];
        if (lp >= 0 && lp < a.pages) {
          const int lg = lp * 64 + slot;
          // raw columns: [take*64 selected keys | sink | tail]
          if (lg < sink) col = tk * 64 + lg;
          else if (lg >= tail && lg < sh.n) col = tk * 64 + sink + lg - tail;
        }
      } else {
        const int rr = 2 * (t - nnat) + h;
        if (rr < tk) {
          col = rr * 64 + slot;
          if (spage[rr] < 0) {
            score = -CUDART_INF_F;            // no page behind this rank: no candidates
          } else if (sbnd[rr]) {
            const int lg = memb[col];
            if (lg < sink || lg >= tail) score = -CUDART_INF_F;
          }
        }
      }
      if (col >= 0) {
        const uint32_t key = order_key(score);
        reinterpret_cast<uint32_t*>(sc)[col] = key;
        atomicAdd(&thist[bin_of(key)], 1);
        if (gout) gout[col] = score;
      }
    }
  }
  __syncthreads();
  if (!*reinterpret_cast<volatile int*>(&sh.abort)) {
    // ---- Top-T + mapping (all threads) ------------------------------------------------
    const int Lr = sh.L, tk = sh.take, sink = sh.sink, tail = sh.tail, nn = sh.n;
    const uint32_t* keys = reinterpret_cast<const uint32_t*>(sc);   // order keys, written by the epilogue
    // the Top-T places each selected candidate's raw column at its output slot
    // in shared memory (after the Top-T scratch in the stage ring); then every
    // thread maps raw -> logical -> physical for consecutive slots, so the
    // mapping runs in parallel over the slots and the rows are written coalesced
    const int T = a.topk;
    int* orw = reinterpret_cast<int*>(stages + ((sf_topk_scratch_bytes(a.max_cand) + 15) & ~int64_t(15)));
    sf_topk<kThreads>(sh, keys, thist, Lr, T, stages, [&](int pos, int rawi) { orw[pos] = rawi; });
    __syncthreads();
    int32_t* gl = a.logical + row * T;
    int32_t* gp = a.physical + row * T;
    int32_t* gr = a.raw + row * T;
    int32_t* ex = a.expansion_stride ? a.expanded + row * a.expansion_stride : nullptr;
    for (int pos = tid; pos < T; pos += kThreads) {
      const int rawi = orw[pos];
      int lg = -1;
      if (rawi >= 0 && rawi < Lr && keys[rawi] != kNegInfKey) {
        if (rawi < tk * 64) {
          lg = memb[rawi];
        } else {
          const int off = rawi - tk * 64;
          lg = off < sink ? off : tail + off - sink;
        }
      }
      if (!(lg >= 0 && lg < nn)) lg = -1;
      int ph = -1;
      if (lg >= 0 && (lg >> 6) < a.pages) ph = sntab[lg >> 6] * 64 + (lg & 63);
      gl[pos] = lg;
      gp[pos] = ph;
      gr[pos] = rawi;
      if (ex) {
        const int b4 = lg * 4;
        reinterpret_cast<int4*>(ex)[pos] = lg < 0 ? make_int4(-1, -1, -1, -1) : make_int4(b4, b4 + 1, b4 + 2, b4 + 3);
      }
    }
    if (ex)
      for (int64_t j = static_cast<int64_t>(T) * 4 + tid; j < a.expansion_stride; j += kThreads) ex[j] = -1;
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 sf_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int sf_encode(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, CUtensorMapDataType type, int rank,
              const void* ptr, const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
              CUtensorMapSwizzle swz, const char* what) {
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(m, type, rank, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swz, swz == CU_TENSOR_MAP_SWIZZLE_NONE ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                                                                : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("select_fused: %s tensor map encode failed (%d)", what, static_cast<int>(r));
    return V1X_ERR_CUDA;
  }
  return V1X_OK;
}

int pool_maps(PFN_cuTensorMapEncodeTiled_v12000 enc, const uint8_t* pool, int64_t pages, CUtensorMap* keys,
              CUtensorMap* scales, const char* what) {
  const cuuint64_t kd[3] = {128, 64, static_cast<cuuint64_t>(pages)};
  const cuuint64_t ks[2] = {128, static_cast<cuuint64_t>(kPageBytes)};
  const cuuint32_t kb[3] = {128, 64, 1};
  if (int rc = sf_encode(enc, keys, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, pool, kd, ks, kb, CU_TENSOR_MAP_SWIZZLE_128B,
                         what))
    return rc;
  const cuuint64_t sd[2] = {64, static_cast<cuuint64_t>(pages)};
  const cuuint64_t ss[1] = {static_cast<cuuint64_t>(kPageBytes)};
  const cuuint32_t sb[2] = {64, 1};
  return sf_encode(enc, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, pool + kKeyBytes, sd, ss, sb,
                   CU_TENSOR_MAP_SWIZZLE_NONE, what);
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_select_fused(const uint8_t* q, const float* w, int64_t heads, const int32_t* lens,
                                const int32_t* budget, int64_t ratio_num, int64_t ratio_den,
                                const int32_t* native_table, const int32_t* reordered_table, int64_t pages,
                                const float* page_scores, int64_t page_stride, const uint8_t* fine,
                                int64_t fine_pages, const int32_t* members, int64_t member_rows,
                                const uint8_t* native, int64_t native_pages, int64_t capacity, int64_t topk,
                                int64_t window, int64_t take_stride, int64_t fine_cols, int32_t* fine_lens,
                                int32_t* takes, int32_t* dg_lens, int32_t* center_lens, int32_t* tail_rows,
                                int32_t* selected, int32_t* fine_table, int32_t* physical, int32_t* logical,
                                int32_t* raw, int32_t* expanded, int64_t expansion_stride, float* scores_out,
                                int64_t score_stride, int64_t batch, int32_t* status, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && batch <= (int64_t(1) << 30), "select_fused: bad batch");
  V1X_CHECK_ARG(heads == 1 || (heads % 32 == 0 && heads <= 128), "select_fused: heads must be 1 or 32/64/96/128");
  V1X_CHECK_ARG(topk > 0 && topk <= 2048, "select_fused: 0 < topk <= 2048");
  V1X_CHECK_ARG(window >= 0 && window <= 4096, "select_fused: 0 <= window <= 4096");
  V1X_CHECK_ARG(pages >= 64 && pages <= 4096, "select_fused: 64 <= pages <= 4096");
  V1X_CHECK_ARG(take_stride > 0 && take_stride <= pages && take_stride <= 128,
                "select_fused: 0 < take_stride <= min(pages, 128)");
  V1X_CHECK_ARG(fine_cols >= take_stride, "select_fused: fine table narrower than take_stride");
  V1X_CHECK_ARG(page_stride >= pages, "select_fused: page scores narrower than the page table");
  V1X_CHECK_ARG(budget != nullptr || (ratio_num > 0 && ratio_den > 0), "select_fused: budget or ratio");
  V1X_CHECK_ARG(expansion_stride == 0 || expansion_stride == topk * 4 + 64, "Invalid expansion buffer");
  V1X_CHECK_ARG(scores_out == nullptr || score_stride >= take_stride * 64 + 64 + std::max<int64_t>(window, 1024),
                "select_fused: kept-score rows too narrow");
  V1X_CHECK_ARG(fine_pages > 0 && native_pages > 0 && member_rows > 0 && capacity >= 0, "select_fused: empty pool");
  V1X_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(fine) |
                  reinterpret_cast<uintptr_t>(native) | reinterpret_cast<uintptr_t>(members)) & 15) == 0,
                "select_fused: q, pools and members must be 16-byte aligned");
  if (batch == 0) return V1X_OK;
  auto enc = sf_encode_fn();
  if (!enc) {
    set_error("select_fused: cuTensorMapEncodeTiled unavailable");
    return V1X_ERR_CUDA;
  }
  const int64_t n_mma = heads == 1 ? 16 : heads;
  CUtensorMap fine_map, fine_sc, nat_map, nat_sc, q_map;
  if (int rc = pool_maps(enc, fine, fine_pages, &fine_map, &fine_sc, "fine pool")) return rc;
  if (int rc = pool_maps(enc, native, native_pages, &nat_map, &nat_sc, "native pool")) return rc;
  {
    const cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(batch * heads)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(n_mma)};
    if (int rc = sf_encode(enc, &q_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B, "q"))
      return rc;
  }
  // route geometry of the reference (v1_query.cuh:175-177)
  int r_threads, r_items;
  if (pages <= 128) { r_threads = 64; r_items = 2; }
  else if (pages <= 256) { r_threads = 64; r_items = 4; }
  else if (pages <= 512) { r_threads = 64; r_items = 8; }
  else if (pages <= 1024) { r_threads = 128; r_items = 8; }
  else if (pages <= 2048) { r_threads = 128; r_items = 16; }
  else { r_threads = 128; r_items = 32; }
  const int n_items = r_threads * r_items;
  const int max_cand = static_cast<int>(take_stride * 64 + 64 + std::max<int64_t>(window, 1024));
  // 256 threads: three producer warps after the route keep the scoring fed,
  // and a CTA leaves room on its SM for an independent batch's gather CTAs
  // (512-thread CTAs took the whole register file for 3 us less latency per
  // row, and cut the throughput of batches in flight from 922K to 735K
  // queries/s)
  const int threads = 256;
  // shared memory plan: everything but the stage ring, then as many 16 KB
  // stages (4 to 8) as fit the CTA's share of the SM
  auto align = [](int64_t x, int64_t al) { return (x + al - 1) / al * al; };
  const int64_t route_bytes = 16384 + static_cast<int64_t>(n_items) * 8;
  const int64_t row_bytes = static_cast<int64_t>(max_cand) * 4 + take_stride * 64 * 4;
  // the Top-T scratch and the staged output slots share the stage ring
  const int64_t topk_scratch = ((sf_topk_scratch_bytes(max_cand) + 15) & ~int64_t(15)) + topk * 4;
  auto plan = [&](int stages, int64_t* offs) {   // offs: q, sring, w, sel, sh, tab, u; returns total bytes
    int64_t off = static_cast<int64_t>(stages) * 16384;
    offs[0] = off;
    off = align(off + n_mma * 128, 1024);
    offs[1] = off;
    off += static_cast<int64_t>(2 * stages) * 512;
    offs[2] = off;
    off = align(off + heads * 4, 16);
    offs[3] = off;
    off = align(off + take_stride * 5, 16);
    offs[4] = off;
    off = align(off + static_cast<int64_t>(sizeof(SfShared)), 16);
    offs[5] = off;
    off = align(align(off + pages * 12, 16) + 4 * kBins, 16);
    offs[6] = off;
    off += std::max(route_bytes, row_bytes);
    return off + 1024;
  };
  // two CTAs per SM when they fit (one head, many rows), else one
  const int64_t budget_bytes = heads == 1 ? 113 * 1024 : 227 * 1024;
  // one head: three stages, so that two CTAs share an SM; else six (eight gave
  // the same row latency, but a CTA of 219 KB of shared memory leaves its SM
  // almost no L1 for an independent batch's gather running beside it: 832K
  // against 930K queries/s with batches in flight)
  int stages = heads == 1 ? 3 : 6;
  int64_t offs[7];
  while (stages > 4 && plan(stages, offs) > budget_bytes) --stages;
  const int64_t total = plan(stages, offs);
  if (total > 227 * 1024 || topk_scratch > static_cast<int64_t>(stages) * 16384) {
    set_error("select_fused: shared memory %lld too large (pages %lld, window %lld)", (long long)total,
              (long long)pages, (long long)window);
    return V1X_ERR_UNSUPPORTED;
  }
  const size_t smem = static_cast<size_t>(total);
  const int scale_slots = 2 * stages;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(kSfAcc * n_mma)) cols <<= 1;
  SfArgs args{lens, budget, static_cast<int>(ratio_num), static_cast<int>(ratio_den), native_table,
              reordered_table, static_cast<int>(pages), page_scores, page_stride, w, static_cast<int>(heads),
              static_cast<int>(n_mma), members, member_rows, capacity, static_cast<int>(topk),
              static_cast<int>(window), static_cast<int>(take_stride), fine_cols, fine_lens, takes, dg_lens,
              center_lens, tail_rows, selected, fine_table, physical, logical, raw, expanded, expansion_stride,
              scores_out, score_stride, static_cast<int>(batch), stages, scale_slots, n_items, n_items / 128,
              max_cand, cols, status, static_cast<int>(offs[0]), static_cast<int>(offs[1]),
              static_cast<int>(offs[2]), static_cast<int>(offs[3]), static_cast<int>(offs[4]),
              static_cast<int>(offs[5]), static_cast<int>(offs[6])};
  static DeviceOnce once;
  once.run([] {
    cudaFuncSetAttribute(select_fused_kernel<256, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(select_fused_kernel<256, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  const dim3 grid(static_cast<unsigned>(batch)), block(threads);
  cudaStream_t s = as_stream(stream);
  if (n_items <= 2 * 256)
    launch_kernel(select_fused_kernel<256, 2>, grid, block, smem, s, fine_map, fine_sc, nat_map, nat_sc, q_map, args);
  else
    launch_kernel(select_fused_kernel<256, 16>, grid, block, smem, s, fine_map, fine_sc, nat_map, nat_sc, q_map, args);
  return launch_status("v1x_select_fused");
}
