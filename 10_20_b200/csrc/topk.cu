// fused.topk for sm_100a: in-place boundary mask + exact Top-T selection +
// raw -> logical -> physical mapping (+ optional x4 expansion), one CTA per row.
//
// Reference behaviour: sglang/kernels/jit/csrc/deepseek_v4/v1_query.cuh:62-153
// (kernel) and :181-220 (host checks).  Selection semantics: the T largest of
// scores[row, :fine_lens[row]] ordered by (value desc, index asc) -- exact ties at
// the boundary go to the lower index, where the reference falls back to
// shared-memory atomic order (topk_impl.cuh:400-401).  Outputs are written in
// ascending raw-index order (the reference leaves the order unspecified).
//
// Design (one CTA of 512 threads per row):
//   1. cp.async copies of the row's scores, its native-table row and the 64
//      members of every selected rank's page into shared memory, overlapping
//      the dependent selected -> rt loads that find those pages;
//   2. one pass turns the scores into order-preserving keys and applies the
//      boundary-bucket mask (global -inf write + key) from the staged members;
//   3. the exact T-th key comes from the bitwise search of select.cuh;
//   4. warp ballots + one scan over (slice, warp) counts give every selected
//      candidate its output slot in index order, and the selecting thread maps
//      raw -> logical -> physical from shared memory and stores the outputs.
// Rows whose scores do not fit in shared memory read them from global memory
// at every step (same results, slower).
#include <algorithm>

#include "common.cuh"
#include "select.cuh"

namespace v1x {
namespace {

constexpr int kTopkThreads = 512;
constexpr int kTopkMaxSmemKeys = 48 * 1024;  // 192 KB of staged keys per CTA
constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // order_key(-inf)
constexpr int kStageTake = 128;    // ranks whose 64 members are staged (32 KB)
constexpr int kStageNt = 4096;     // native-table entries staged (16 KB)
constexpr int kRegKeys = 16;       // keys per thread kept in registers (cols <= 8192)
constexpr int kMaskQueue = 256;
constexpr int kMaxBin = 2048;      // threshold-bin keys resolved exactly (else bitwise search)
constexpr int kSmallBin = 96;      // bins up to this size are ranked pairwise directly
constexpr int kMaxBin2 = 256;      // second-level bin size limit

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
  // shared-memory staging plan (staged modes): word offsets in the dynamic area
  int stage_take, stage_nt, memb_off, ntab_off;
  // page-table transform mode (TopK-v2's transform): out = page_table[row,
  // raw >> page_bits] << page_bits | (raw & page mask), through original_ids
  // when given; no mask and no V1 mapping
  const int32_t* page_table;
  int64_t table_stride;
  int page_bits;
  const int32_t* original_ids;
  int transform;
  // unstaged mode: words of the selection bitmap in the dynamic shared memory
  // (0: the bitwise threshold search over the row in global memory)
  int sel_words;
};

struct RowCtx {
  int64_t row;
  int n, take, sink, tail, L;
};

// Per-CTA geometry.  512 threads: rows of up to 48K staged keys.  256 threads
// (mode 2 only, rows of up to 4096 keys): a quarter of the shared memory, so four
// CTAs fit an SM when a batch has many more rows than SMs.
template <int kThreads>
struct TopkShape {
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kMaxKeys = kThreads >= 512 ? kTopkMaxSmemKeys : 4096;  // staged keys per CTA
  static constexpr int kRankCache = kMaxKeys / 64;    // ranks whose page ids live in smem
  static constexpr int kMaxSlices = kMaxKeys / kThreads;
};

template <int kThreads>
struct TopkSmem {
  using Shape = TopkShape<kThreads>;
  static constexpr int kRankCache = Shape::kRankCache;
  static constexpr int kWarps = Shape::kWarps;
  int pgc[kRankCache];              // page of rank r used for the mapping
  int rpg[kRankCache];              // reordered page of rank r used for the mask
  uint8_t bflag[kRankCache];        // rank r < take is a boundary bucket
  union {
    struct {
      int hist[kBins];              // coarse histogram (selection step 1)
      int2 bnd[kMaskQueue];         // boundary queue of the unstaged mode
    } h;
    struct {
      int2 cand[kMaxBin];           // keys + indices of the threshold bin
      int2 cnt[Shape::kMaxSlices * kWarps];  // per (slice, warp) counts, then their scan
    } c;
  } u;
  uint32_t selbit[Shape::kMaxKeys / 32];  // threshold-bin keys that are selected
  int hist2[256];                   // second level over the threshold bin
  int2 cand2[kMaxBin2];
  int warp_tot[kWarps + 1];
  int4 red[2 * kWarps];
  int4 res, res2;
  int2 carry;
  int nbnd, ncand, ncand2;
  uint32_t kmin, kmax, kmin2, kmax2;  // key range of the threshold bin / sub-bin
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gsrc)
               : "memory");
}

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

// Members of the boundary bucket page `page` outside [sink, tail) -> -inf in
// global memory (VQ:94-103); unstaged mode only.
__device__ __forceinline__ void mask_page(const TopkArgs& a, const RowCtx& c, float* srow, int r, int64_t page,
                                          int lane_lo, int lane_step) {
  for (int off = lane_lo; off < 64; off += lane_step) {
    const int lg = a.members[page * 64 + off];
    const int64_t col = static_cast<int64_t>(r) * 64 + off;
    if ((lg < c.sink || lg >= c.tail) && col < a.cols) srow[col] = -CUDART_INF_F;
  }
}

// Two CTAs per SM (register cap 64, a few spilled registers): with many rows
// (1024 single-head queries) the second resident CTA hides the first's latency
// chains, and with few rows it leaves room for an overlapping batch's gather.
// kMode 0: keys read from global memory at every use (rows too long for smem);
// 1: keys staged in shared memory; 2: staged and also held in registers
// (cols <= kRegKeys * 512).
// kThreads 256 (mode 2 only): four CTAs per SM for batches of many rows.
// Candidates i .. i + 3 of a row of L (the ones past L read as -inf), by one
// 16-byte load when `vec` (row 16-byte aligned, i a multiple of 4).
__device__ __forceinline__ float4 load4(const float* row, int i, int L, bool vec) {
  if (vec && i + 3 < L) return __ldcg(reinterpret_cast<const float4*>(row + i));
  float4 f = make_float4(-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F);
  if (i < L) f.x = __ldcg(row + i);
  if (i + 1 < L) f.y = __ldcg(row + i + 1);
  if (i + 2 < L) f.z = __ldcg(row + i + 2);
  if (i + 3 < L) f.w = __ldcg(row + i + 3);
  return f;
}

template <int kMode, int kThreads>
__global__ void __launch_bounds__(kThreads, kThreads >= 512 ? 2 : 4) topk_kernel(const __grid_constant__ TopkArgs a) {
  using Shape = TopkShape<kThreads>;
  constexpr int kTopkWarps = Shape::kWarps;
  constexpr int kRankCache = Shape::kRankCache;
  constexpr int kMaxSlices = Shape::kMaxSlices;
  constexpr bool kStaged = kMode > 0;
  extern __shared__ __align__(16) uint32_t dyn[];
  __shared__ TopkSmem<kThreads> sm;
  uint32_t* keys = dyn;
  // selection bitmap: the staged modes' static one, or the unstaged mode's
  // dynamic one (one bit per candidate)
  uint32_t* selbits = kStaged ? sm.selbit : dyn;
  const bool hist_path = kStaged || a.sel_words > 0;
  int* memb = reinterpret_cast<int*>(dyn) + a.memb_off;
  int* ntab = reinterpret_cast<int*>(dyn) + a.ntab_off;
  const int tid = threadIdx.x, nt = kThreads;
  const int lane = tid & 31, warp = tid >> 5;
  RowCtx c;
  c.row = blockIdx.x;
  // lengths and the native-table row (its copy overlaps the selection below)
  c.n = a.lens[c.row];
  const int Sn = kStaged ? static_cast<int>(min(min(a.pages, static_cast<int64_t>(a.stage_nt)),
                                                (static_cast<int64_t>(max(c.n, 0)) + 63) / 64))
                         : 0;
  const int32_t* ntrow = a.nt + c.row * a.pages;
  if (kStaged) {
    if ((reinterpret_cast<uintptr_t>(ntrow) & 15) == 0) {
      for (int v = tid; v < (Sn >> 2); v += nt) cp_async16(ntab + 4 * v, ntrow + 4 * v);
      for (int v = (Sn & ~3) + tid; v < Sn; v += nt) cp_async4(ntab + v, ntrow + v);
    } else {
      for (int v = tid; v < Sn; v += nt) cp_async4(ntab + v, ntrow + v);
    }
  }
  const int64_t rank0 = tid < a.take_stride ? load_index(a.selected, a.sel64, c.row * a.take_stride + tid) : -1;
  c.take = a.takes ? a.takes[c.row] : 0;
  const RowBounds rb = row_bounds(c.n, 64, a.window);
  c.sink = rb.sink;
  c.tail = rb.tail;
  c.L = static_cast<int>(min(static_cast<int64_t>(max(a.fine_lens[c.row], 0)), a.cols));
  float* srow = a.scores + c.row * a.score_stride;
  const bool select = c.L > a.topk;
  const int S = kStaged ? min(max(c.take, 0), a.stage_take) : 0;  // ranks with staged members

  // ---- 1. asynchronous copies into shared memory --------------------------------
  const int nv4 = (kStaged && (reinterpret_cast<uintptr_t>(srow) & 15) == 0) ? c.L >> 2 : 0;
  if (kStaged) {
    for (int v = tid; v < nv4; v += nt) cp_async16(keys + 4 * v, srow + 4 * v);
  } else {
    if (tid == 0) sm.nbnd = 0;
    __syncthreads();
  }
  // selected ranks -> pages; members of staged ranks; boundary flags
  for (int r = tid; r < c.take; r += nt) {
    int64_t rank = -1, rpage = -1;
    if (r < a.take_stride) rank = r == tid ? rank0 : load_index(a.selected, a.sel64, c.row * a.take_stride + r);
    const bool rank_ok = rank >= 0 && rank < a.pages;
    if (rank_ok) rpage = a.rt[c.row * a.pages + rank];
    const int64_t epage =
        a.direct_fine ? (r < a.fine_table_cols ? a.fine_table[c.row * a.fine_table_cols + r] : -1) : rpage;
    if (r < kRankCache) {
      sm.pgc[r] = static_cast<int>(epage);
      sm.rpg[r] = static_cast<int>(rpage);
    }
    if (r < S && epage >= 0 && epage < a.member_rows) {
      const int32_t* src = a.members + epage * 64;
#pragma unroll
      for (int q = 0; q < 16; ++q) cp_async16(memb + r * 64 + 4 * q, src + 4 * q);
    }
    bool boundary = false;
    if (a.mask && rank_ok && rpage >= 0 && rpage < a.member_rows) {
      const int bucket =
          a.bucket_from_rank ? static_cast<int>(rank / 16) * 1024 : (a.members[rpage * 64] / 1024) * 1024;
      boundary = bucket < c.sink || bucket + 1024 > c.tail;
    }
    if (kStaged) {
      // ranks >= kRankCache only own columns >= cols: nothing to mask there
      if (r < kRankCache) sm.bflag[r] = boundary ? 1 : 0;
    } else if (boundary) {
      const int k = atomicAdd(&sm.nbnd, 1);
      if (k < kMaskQueue) sm.u.h.bnd[k] = make_int2(r, static_cast<int>(rpage));
      else mask_page(a, c, srow, r, rpage, 0, 1);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // ---- 2. mask + keys -------------------------------------------------------------
  if (kStaged) {
    const int mcols = a.mask ? static_cast<int>(min(static_cast<int64_t>(max(c.take, 0)) * 64, a.cols)) : 0;
    const int hi = max(c.L, mcols);
    for (int i = tid; i < hi; i += nt) {
      bool masked = false;
      if (i < mcols) {
        const int r = i >> 6;
        if (sm.bflag[r]) {
          // the staged members are those of the mapping page; they are the mask
          // page's too unless a direct fine table points elsewhere
          const int lg = (r < S && sm.rpg[r] == sm.pgc[r]) ? memb[i]
                                                           : a.members[static_cast<int64_t>(sm.rpg[r]) * 64 + (i & 63)];
          masked = lg < c.sink || lg >= c.tail;
          if (masked) srow[i] = -CUDART_INF_F;
        }
      }
      if (i < c.L) keys[i] = masked ? kNegInfKey : order_key(i < nv4 * 4 ? __uint_as_float(keys[i]) : srow[i]);
    }
  } else {
    const int nb = min(sm.nbnd, kMaskQueue);
    for (int k = warp; k < nb; k += kTopkWarps) mask_page(a, c, srow, sm.u.h.bnd[k].x, sm.u.h.bnd[k].y, lane, 32);
  }
  __syncthreads();

  // ---- mapping epilogue for one output slot (VQ:121-148) ----------------------------
  auto emit = [&](int pos, int raw) {
    if (a.transform) {
      int32_t o = -1;
      if (raw >= 0) {
        const int32_t idx = (a.page_table[c.row * a.table_stride + (raw >> a.page_bits)] << a.page_bits) |
                            (raw & ((1 << a.page_bits) - 1));
        o = a.original_ids ? a.original_ids[idx] : idx;
      }
      a.physical[c.row * a.topk + pos] = o;
      if (a.raw) a.raw[c.row * a.topk + pos] = raw;
      return;
    }
    bool live = false;
    if (raw >= 0 && raw < c.L) live = kStaged ? keys[raw] != kNegInfKey : srow[raw] != -CUDART_INF_F;
    int lg = -1;
    if (live) {
      if (raw < c.take * 64) {
        const int r = raw >> 6;
        const int64_t page = r < kRankCache ? sm.pgc[r] : page_of_rank(a, c, r);
        if (page >= 0 && page < a.member_rows) lg = r < S ? memb[raw] : a.members[page * 64 + (raw & 63)];
      } else {
        const int off = raw - c.take * 64;
        lg = off < c.sink ? off : c.tail + off - c.sink;
      }
    }
    if (!(lg >= 0 && lg < c.n)) lg = -1;
    const int64_t dst = c.row * a.topk + pos;
    a.logical[dst] = lg;
    if (a.physical_output) {
      int ph = -1;
      if (lg >= 0) {
        const int p = lg >> 6;
        if (p < a.pages) ph = (p < Sn ? ntab[p] : ntrow[p]) * 64 + (lg & 63);
      }
      a.physical[dst] = ph;
      a.raw[dst] = raw;
    }
    if (a.expansion_stride) {
      const int b = lg * 4;
      reinterpret_cast<int4*>(a.expanded + c.row * a.expansion_stride)[pos] =
          lg < 0 ? make_int4(-1, -1, -1, -1) : make_int4(b, b + 1, b + 2, b + 3);
    }
  };

  if (!select) {
    for (int t = tid; t < a.topk; t += nt) emit(t, t < c.L ? t : -1);
  } else {
    // ---- 3. selection ---------------------------------------------------------------
    const int nsl = (c.L + nt - 1) / nt;  // slices of nt consecutive candidates
    uint32_t kr[kMode == 2 ? kRegKeys : 1];
    if constexpr (kMode == 2) {
#pragma unroll
      for (int j = 0; j < kRegKeys; ++j) {
        const int i = j * nt + tid;
        kr[j] = i < c.L ? keys[i] : 0u;
      }
    }
    auto key_of = [&](int j) -> uint32_t {  // this thread's key of slice j (i < L)
      const int i = j * nt + tid;
      if constexpr (kMode == 0) return order_key(srow[i]);
      else return keys[i];
    };
    // one 12-bit histogram pass finds the bin of the T-th key; the bin's keys
    // are ranked exactly by (key desc, index asc) and the selected ones flagged.
    // The unstaged mode with a bitmap reads the row twice (histogram, then the
    // bin's keys and the keys above it, which it flags too) and places from the
    // bitmap alone.  Rows whose bin holds more than kMaxBin keys (mass ties)
    // and the unstaged mode without a bitmap take the bitwise search instead.
    // unstaged mode: 16-byte loads when the row is aligned (row strides are
    // multiples of 4 floats)
    const bool vec4 = (reinterpret_cast<uintptr_t>(srow) & 15) == 0;
    bool by_bin = false, have_tie = false;
    uint32_t tie_thr = 0;
    int tie_need = 0;
    TopBin tb{0, 0, 0};
    if (hist_path) {
      int* hist = sm.u.h.hist;
      zero_hist<kThreads>(hist);
      for (int w = tid; w < (c.L + 31) / 32; w += nt) selbits[w] = 0u;
      if (tid < 256) sm.hist2[tid] = 0;
      if (tid == 0) {
        sm.ncand = 0;
        sm.ncand2 = 0;
        sm.kmin = sm.kmin2 = 0xFFFFFFFFu;
        sm.kmax = sm.kmax2 = 0u;
      }
      __syncthreads();
      if constexpr (kMode == 2) {
#pragma unroll
        for (int j = 0; j < kRegKeys; ++j)
          if (j * nt + tid < c.L) atomicAdd(&hist[bin_of(kr[j])], 1);
      } else if constexpr (kMode == 0) {
        // the row streams from global memory: a warp takes 128 consecutive
        // candidates at a time (four per lane), four such groups in flight
        for (int g0 = warp; g0 * 128 < c.L; g0 += 4 * kTopkWarps) {
          float4 f[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) f[q] = load4(srow, (g0 + q * kTopkWarps) * 128 + lane * 4, c.L, vec4);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = (g0 + q * kTopkWarps) * 128 + lane * 4;
            const float x[4] = {f[q].x, f[q].y, f[q].z, f[q].w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (i + u < c.L) atomicAdd(&hist[bin_of(order_key(x[u]))], 1);
          }
        }
      } else {
        for (int i = tid; i < c.L; i += nt) atomicAdd(&hist[bin_of(keys[i])], 1);
      }
      __syncthreads();
      tb = find_top_bin<kThreads>(a.topk, hist, sm.warp_tot, &sm.res);
      // the histogram is dead: the candidate list reuses its storage.  The bin's
      // key range is tracked while compacting it: a bin of one repeated value
      // (ReLU zeros of single-head scores, for instance) needs no ranking -- its
      // ties are taken by lowest index.
      int2* cand = sm.u.c.cand;
      const bool keep = tb.in <= kMaxBin;
      {
        const uint32_t ltm = lanemask_lt();
        auto append = [&](int j, uint32_t k) {
          const bool m = j * nt + tid < c.L && bin_of(k) == tb.bin;
          const unsigned bal = __ballot_sync(0xffffffffu, m);
          if (bal == 0u) return;
          const uint32_t lo = __reduce_min_sync(0xffffffffu, m ? k : 0xFFFFFFFFu);
          const uint32_t hi = __reduce_max_sync(0xffffffffu, m ? k : 0u);
          int base = 0;
          if (lane == 0) {
            atomicMin(&sm.kmin, lo);
            atomicMax(&sm.kmax, hi);
            if (keep) base = atomicAdd(&sm.ncand, __popc(bal));
          }
          base = __shfl_sync(0xffffffffu, base, 0);
          if (keep && m) cand[base + __popc(bal & ltm)] = make_int2(static_cast<int>(k), j * nt + tid);
        };
        if constexpr (kMode == 2) {
#pragma unroll
          for (int j = 0; j < kRegKeys; ++j)
            if (j < nsl) append(j, kr[j]);
        } else if constexpr (kMode == 0) {
          // the second pass over the row, 128 candidates per warp step as in the
          // histogram: the keys above the bin are flagged in the bitmap (lanes
          // 8w .. 8w + 7 hold word w's 32 bits as nibbles, OR-ed by shuffles),
          // the bin's keys are listed one by one (a few hundred per row)
          for (int g0 = warp; g0 * 128 < c.L; g0 += 2 * kTopkWarps) {
            float4 f[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) f[q] = load4(srow, (g0 + q * kTopkWarps) * 128 + lane * 4, c.L, vec4);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int i = (g0 + q * kTopkWarps) * 128 + lane * 4;
              const float x[4] = {f[q].x, f[q].y, f[q].z, f[q].w};
              uint32_t nib = 0;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                if (i + u >= c.L) continue;
                const uint32_t k = order_key(x[u]);
                const int b = bin_of(k);
                if (b > tb.bin) nib |= 1u << u;
                if (b == tb.bin) {
                  atomicMin(&sm.kmin, k);
                  atomicMax(&sm.kmax, k);
                  if (keep) cand[atomicAdd(&sm.ncand, 1)] = make_int2(static_cast<int>(k), i + u);
                }
              }
              uint32_t word = nib << (4 * (lane & 7));
              word |= __shfl_xor_sync(0xffffffffu, word, 1);
              word |= __shfl_xor_sync(0xffffffffu, word, 2);
              word |= __shfl_xor_sync(0xffffffffu, word, 4);
              const int w = (i - 4 * (lane & 7)) >> 5;  // the word of lanes 8w' .. 8w' + 7
              if ((lane & 7) == 0 && w * 32 < c.L) selbits[w] = word;
            }
          }
        } else {
          for (int j = 0; j < nsl; ++j) append(j, j * nt + tid < c.L ? key_of(j) : 0u);
        }
      }
      __syncthreads();
      if (sm.kmin == sm.kmax) {
        tie_thr = sm.kmin;
        tie_need = a.topk - tb.above;
        have_tie = true;
      } else if (keep) {
        by_bin = true;
        int need_bin = a.topk - tb.above;
        const int2* rk = cand;
        int nres = tb.in;
        if (tb.in > kSmallBin) {
          // second level: the next 8 key bits of the bin's keys
          for (int q = tid; q < tb.in; q += nt) atomicAdd(&sm.hist2[(cand[q].x >> (24 - kBinBits)) & 255], 1);
          __syncthreads();
          if (warp == 0) {
            const int hi = 256 - lane * 8;  // lane owns sub-bins [hi - 8, hi), descending
            int cc[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              cc[j] = sm.hist2[hi - 8 + j];
              s += cc[j];
            }
            int cum = warp_inclusive_scan(s) - s;
            if (cum < need_bin && cum + s >= need_bin) {
#pragma unroll
              for (int j = 7; j >= 0; --j) {
                if (cum < need_bin && cum + cc[j] >= need_bin) sm.res2 = make_int4(hi - 8 + j, cum, cc[j], 0);
                cum += cc[j];
              }
            }
          }
          __syncthreads();
          const int4 r2 = sm.res2;
          if (r2.z <= kMaxBin2) {
            for (int q = tid; q < tb.in; q += nt) {
              const int2 me = cand[q];
              const int sub = (me.x >> (24 - kBinBits)) & 255;
              if (sub > r2.x) atomicOr(&selbits[me.y >> 5], 1u << (me.y & 31));
              else if (sub == r2.x) sm.cand2[atomicAdd(&sm.ncand2, 1)] = me;
            }
            __syncthreads();
            need_bin -= r2.y;
            rk = sm.cand2;
            nres = r2.z;
          } else {
            // a crowded sub-bin: one repeated value takes the tie path, anything
            // else the bitwise search
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
              atomicMin(&sm.kmin2, lo);
              atomicMax(&sm.kmax2, hi);
            }
            __syncthreads();
            if (sm.kmin2 == sm.kmax2) {
              tie_thr = sm.kmin2;
              tie_need = need_bin - r2.y;
              have_tie = true;
            }
          }
        }
        if (by_bin) {
          // exact rank among the remaining keys by (key desc, index asc)
          for (int q = tid; q < nres; q += nt) {
            const int2 me = rk[q];
            const uint32_t k = static_cast<uint32_t>(me.x);
            int r = 0;
            for (int f = 0; f < nres; ++f) {
              const int2 o = rk[f];
              const uint32_t ko = static_cast<uint32_t>(o.x);
              r += (ko > k) | ((ko == k) & (o.y < me.y));
            }
            if (r < need_bin) atomicOr(&selbits[me.y >> 5], 1u << (me.y & 31));
          }
          __syncthreads();
        }
      }
    }
    uint32_t thr = tie_thr;
    int need = tie_need;
    if (!by_bin && !have_tie) {
      int gt = 0;
      thr = block_kth_largest<kTopkWarps>(
          a.topk,
          [&](uint32_t c1, uint32_t c2, uint32_t c3, int& n1, int& n2, int& n3) {
            n1 = n2 = n3 = 0;
            if constexpr (kMode == 2) {
#pragma unroll
              for (int j = 0; j < kRegKeys; ++j) {
                if (j * nt + tid < c.L) {
                  n1 += kr[j] >= c1;
                  n2 += kr[j] >= c2;
                  n3 += kr[j] >= c3;
                }
              }
            } else {
              for (int i = tid; i < c.L; i += nt) {
                const uint32_t k = kMode == 1 ? keys[i] : order_key(srow[i]);
                n1 += k >= c1;
                n2 += k >= c2;
                n3 += k >= c3;
              }
            }
          },
          sm.red, &gt);
      need = a.topk - gt;  // ties of thr that are selected (lowest indices)
    }
    // class of candidate i with key k: 1 = selected outright, 2 = tie of thr
    // (selected while fewer than `need` ties precede it), 0 = not selected
    auto klass = [&](int i, uint32_t k) -> int {
      if (i >= c.L) return 0;
      if (by_bin) {
        const int b = bin_of(k);
        return (b > tb.bin || (b == tb.bin && ((selbits[i >> 5] >> (i & 31)) & 1u))) ? 1 : 0;
      }
      return k > thr ? 1 : (k == thr ? 2 : 0);
    };
    // ---- 4. output slot of every selected candidate, in index order ----------------
    // (selected, tie) counts per (slice, warp) -> exclusive scan -> slot =
    // selected before it + min(ties before it, need).  Chunks of kMaxSlices
    // slices (more than one only in the unstaged mode) carry their totals.
    const uint32_t lt = lanemask_lt();
    int2* cnt = sm.u.c.cnt;
    auto count_slice = [&](int j, int jc, uint32_t k) {
      const int kl = klass(j * nt + tid, k);
      const unsigned gb = __ballot_sync(0xffffffffu, kl == 1);
      const unsigned eb = __ballot_sync(0xffffffffu, kl == 2);
      if (lane == 0) cnt[jc * kTopkWarps + warp] = make_int2(__popc(gb), __popc(eb));
    };
    auto place_slice = [&](int j, int jc, uint32_t k) {
      const int i = j * nt + tid;
      const int kl = klass(i, k);
      const unsigned gb = __ballot_sync(0xffffffffu, kl == 1);
      const unsigned eb = __ballot_sync(0xffffffffu, kl == 2);
      const int2 base = cnt[jc * kTopkWarps + warp];
      const int gt_lt = base.x + __popc(gb & lt);
      const int eq_lt = base.y + __popc(eb & lt);
      if (kl == 1 || (kl == 2 && eq_lt < need)) emit(gt_lt + min(eq_lt, need), i);
    };
    auto scan_counts = [&](int E, int2 carry) {
      if (warp == 0) {
        const int ch = (E + 31) / 32;
        const int beg = min(lane * ch, E), end = min(beg + ch, E);
        int sg = 0, se = 0;
        for (int q = beg; q < end; ++q) {
          sg += cnt[q].x;
          se += cnt[q].y;
        }
        const int ig = warp_inclusive_scan(sg), ie = warp_inclusive_scan(se);
        int rg = carry.x + ig - sg, re = carry.y + ie - se;
        for (int q = beg; q < end; ++q) {
          const int2 v = cnt[q];
          cnt[q] = make_int2(rg, re);
          rg += v.x;
          re += v.y;
        }
        if (lane == 31) sm.carry = make_int2(carry.x + ig, carry.y + ie);
      }
    };
    if (kMode == 0 && by_bin) {
      // the bitmap holds every pick: a thread takes consecutive bitmap words,
      // their counts are scanned, and the set bits are emitted in index order
      const int nw = (c.L + 31) / 32;
      const int per = (nw + nt - 1) / nt;
      const int w0 = min(tid * per, nw), w1 = min(w0 + per, nw);
      int cnt = 0;
      for (int w = w0; w < w1; ++w) cnt += __popc(selbits[w]);
      int total;
      int pos = block_exclusive_scan(cnt, sm.warp_tot, &total);
      for (int w = w0; w < w1; ++w) {
        uint32_t bits = selbits[w];
        while (bits) {
          const int b = __ffs(bits) - 1;
          bits &= bits - 1;
          if (pos < a.topk) emit(pos, w * 32 + b);
          ++pos;
        }
      }
    } else if constexpr (kMode == 2) {
      // rolled loops over the staged keys: the unrolled mapping epilogue would be
      // kRegKeys copies of a long code path
#pragma unroll 1
      for (int j = 0; j < nsl; ++j) count_slice(j, j, j * nt + tid < c.L ? keys[j * nt + tid] : 0u);
      __syncthreads();
      scan_counts(nsl * kTopkWarps, make_int2(0, 0));
      __syncthreads();
#pragma unroll 1
      for (int j = 0; j < nsl; ++j) place_slice(j, j, j * nt + tid < c.L ? keys[j * nt + tid] : 0u);
    } else {
      int2 carry = make_int2(0, 0);
      for (int j0 = 0; j0 < nsl; j0 += kMaxSlices) {
        const int jn = min(nsl - j0, kMaxSlices);
        for (int jc = 0; jc < jn; ++jc)
          count_slice(j0 + jc, jc, (j0 + jc) * nt + tid < c.L ? key_of(j0 + jc) : 0u);
        __syncthreads();
        scan_counts(jn * kTopkWarps, carry);
        __syncthreads();
        for (int jc = 0; jc < jn; ++jc)
          place_slice(j0 + jc, jc, (j0 + jc) * nt + tid < c.L ? key_of(j0 + jc) : 0u);
        carry = sm.carry;
        __syncthreads();
      }
    }
  }
  if (a.expansion_stride) {
    for (int64_t j = static_cast<int64_t>(a.topk) * 4 + tid; j < a.expansion_stride; j += nt)
      a.expanded[c.row * a.expansion_stride + j] = -1;
  }
}

}  // namespace
}  // namespace v1x

namespace v1x {
namespace {
int topk_launch(TopkArgs a, int64_t cols, int64_t batch, int64_t stake0, int64_t snt0, cudaStream_t s,
                const char* what);
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
             physical_output, bucket_from_rank, fine_table, fine_table_cols, direct_fine,
             0, 0, 0, 0, nullptr, 0, 0, nullptr, 0, 0};
  V1X_CHECK_ARG(take_stride <= 65536, "topk: take stride too large");
  const int64_t rank_bound = direct_fine ? fine_table_cols : take_stride;
  const int64_t stake0 =
      (reinterpret_cast<uintptr_t>(members) & 15) == 0 ? std::min<int64_t>(rank_bound, kStageTake) : 0;
  const int64_t snt0 = std::min<int64_t>(pages, kStageNt);
  return topk_launch(a, cols, batch, stake0, snt0, as_stream(stream), "v1x_topk");
}

namespace v1x {
namespace {

// Launches topk_kernel for `batch` rows of `cols` columns: the shared-memory plan
// (keys | staged members | staged native-table row, up to stake0 ranks and snt0
// entries) picks the CTA shape and the staged or unstaged mode.
int topk_launch(TopkArgs a, int64_t cols, int64_t batch, int64_t stake0, int64_t snt0, cudaStream_t s,
                const char* what) {
  // dynamic shared memory of the staged modes: keys | staged members | staged
  // native-table row; rows whose keys alone do not fit take the unstaged mode
  const int64_t cols_pad = (cols + 3) & ~int64_t(3);
  const dim3 grid(static_cast<unsigned>(batch));
  // Many more rows than SMs (1024 single-head queries): 256-thread CTAs, four
  // per SM, when the row's keys fit their registers and a quarter of an SM's
  // shared memory.  Otherwise 512 threads, two per SM.
  if (batch > 2 * static_cast<int64_t>(num_sms()) && cols <= kRegKeys * 256 &&
      cols <= TopkShape<256>::kMaxKeys) {
    const int64_t limit4 = 228 * 1024 / 4 - static_cast<int64_t>(sizeof(TopkSmem<256>)) - 1024;
    int64_t stake = stake0, snt = snt0;
    auto bytes = [&] { return (cols_pad + stake * 64 + snt) * 4; };
    if (bytes() > limit4) snt = 0;
    if (bytes() > limit4) stake = 0;
    if (bytes() <= limit4) {
      a.stage_take = static_cast<int>(stake);
      a.stage_nt = static_cast<int>(snt);
      a.memb_off = static_cast<int>(cols_pad);
      a.ntab_off = static_cast<int>(cols_pad + stake * 64);
      static DeviceOnce once4;
      once4.run([&] {
        cudaFuncSetAttribute(topk_kernel<2, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(limit4));
      });
      launch_kernel(topk_kernel<2, 256>, grid, dim3(256), static_cast<size_t>(bytes()), s, a);
      return launch_status(what);
    }
  }
  const int64_t limit = 227 * 1024 - static_cast<int64_t>(sizeof(TopkSmem<kTopkThreads>)) - 1024;
  if (cols <= kTopkMaxSmemKeys && cols_pad * 4 <= limit) {
    int64_t stake = stake0, snt = snt0;
    auto bytes = [&] { return (cols_pad + stake * 64 + snt) * 4; };
    if (bytes() > limit) snt = 0;
    if (bytes() > limit) stake = 0;
    a.stage_take = static_cast<int>(stake);
    a.stage_nt = static_cast<int>(snt);
    a.memb_off = static_cast<int>(cols_pad);
    a.ntab_off = static_cast<int>(cols_pad + stake * 64);
    static DeviceOnce once;
    once.run([&] {
      cudaFuncSetAttribute(topk_kernel<1, kTopkThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(limit));
      cudaFuncSetAttribute(topk_kernel<2, kTopkThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(limit));
    });
    if (cols <= kRegKeys * kTopkThreads)
      launch_kernel(topk_kernel<2, kTopkThreads>, grid, dim3(kTopkThreads), static_cast<size_t>(bytes()), s, a);
    else
      launch_kernel(topk_kernel<1, kTopkThreads>, grid, dim3(kTopkThreads), static_cast<size_t>(bytes()), s, a);
  } else {
    a.stage_take = a.stage_nt = a.memb_off = a.ntab_off = 0;
    // the selection bitmap (one bit per column) in the dynamic shared memory
    const int64_t words = (cols + 31) / 32;
    a.sel_words = words * 4 <= limit ? static_cast<int>(words) : 0;
    static DeviceOnce once0;
    once0.run([&] {
      cudaFuncSetAttribute(topk_kernel<0, kTopkThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(limit));
    });
    launch_kernel(topk_kernel<0, kTopkThreads>, grid, dim3(kTopkThreads), static_cast<size_t>(a.sel_words) * 4, s,
                  a);
  }
  return launch_status(what);
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_topk_transform(const float* scores, int64_t score_stride, int64_t cols, const int32_t* seq_lens,
                                  const int32_t* page_table, int64_t table_stride, int64_t page_size,
                                  const int32_t* original_ids, int32_t* out, int32_t* raw, int64_t topk,
                                  int64_t batch, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(batch >= 0 && cols >= 0 && score_stride >= cols, "topk_transform: bad score geometry");
  V1X_CHECK_ARG(topk > 0 && topk <= 2048, "topk must be in (0, 2048]");
  V1X_CHECK_ARG(score_stride % 4 == 0, "score_stride must be a multiple of 4 (16-byte vectorized load)");
  V1X_CHECK_ARG(page_size > 0 && (page_size & (page_size - 1)) == 0 && page_size <= (1 << 20),
                "page_size must be power of 2");
  V1X_CHECK_ARG(table_stride >= 0, "topk_transform: bad page-table stride");
  if (batch == 0) return V1X_OK;
  V1X_CHECK_ARG(scores && seq_lens && page_table && out, "topk_transform: a required buffer is NULL");
  int page_bits = 0;
  while ((int64_t(1) << page_bits) < page_size) ++page_bits;
  TopkArgs a{const_cast<float*>(scores), score_stride, cols, seq_lens, nullptr, 0, nullptr, nullptr, 0, nullptr,
             0, 0, seq_lens, nullptr, out, nullptr, raw, static_cast<int>(topk), 0, 0, nullptr, 0, 0, 0,
             nullptr, 0, 0, 0, 0, 0, 0, page_table, table_stride, page_bits, original_ids, 1};
  return topk_launch(a, cols, batch, 0, 0, as_stream(stream), "v1x_topk_transform");
}
