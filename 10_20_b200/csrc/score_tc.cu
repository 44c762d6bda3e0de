// Tensor-core FP8 paged scoring for sm_100a (tcgen05, TMA, TMEM).
//
//   out[b, j] = sum_h w[b,h] * relu(q[b,h,:] . k_j) * scale_j      (j < len[b])
//
// Same contract as the SIMT path in score.cu (DeepGEMM fp8_paged_mqa_logits as
// called at sglang/srt/layers/attention/v1_deepseek/runtime.py:434-444 and
// :538-548; formula of kernels.py:310-313).  With many index heads the score is
// a dense contraction -- 64 heads x 128 dims per key is ~124 FLOP per key byte --
// so it runs on the 5th-generation tensor cores:
//
//   tile = 128 keys (two 64-token pages) of one row; D[128 x H] = K[128 x 128] .
//   Q[H x 128]^T with tcgen05.mma kind::f8f6f4 (E4M3 x E4M3 -> F32), four K=32
//   steps, accumulator in TMEM (four accumulators in flight).
//
// One head (2 FLOP per key byte) also runs here: the per-key dot products are
// what bounds a CUDA-core scorer (~90 instructions per 16 key bytes), and on
// the tensor cores they cost nothing.  The MMA takes its smallest N, 16: the q
// box is the row's query and the next 15 rows' (zero past the batch), and the
// epilogue reads only column 0 of the accumulator.
//
// Warp roles in a persistent CTA (352 threads, two CTAs per SM; one head: 224
// threads, a single epilogue group):
//   warps 0-1  TMA producers (alternate tiles): two 8 KB page boxes (3-D tensor
//              map over the packed pool, 128-byte swizzle) and the two pages'
//              256-byte scale vectors.  Several issuing warps are needed: one
//              warp sustains only ~4 TMA operations per microsecond.
//   warp 2     TMEM owner + single-thread MMA issuer; loads the row's q tile
//              (H x 128) when the row changes; commits release the smem stage
//              and publish the accumulator.
//   warps 3-10 two epilogue groups (alternate tiles; one head: warps 3-6,
//              one group): tcgen05.ld of the
//              accumulator (one key per thread), ReLU, weighted head sum with
//              the head weights staged in smem, per-key scale, coalesced store.
// Each CTA owns a contiguous range of tiles (row, 128-key block), computed from
// a per-row tile prefix over the device lengths, so q and the head weights
// change only at row boundaries.  Every mbarrier wait is bounded (2 s); on
// timeout the CTA records V1X_STATUS_TIMEOUT, lets what it issued retire and
// frees its TMEM before exiting.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace v1x {
namespace {

using namespace sm100;

constexpr int kProducers = 2;                      // TMA issuing warps
constexpr int kMmaWarp = kProducers;
constexpr int kEpiWarp0 = kProducers + 1;          // first epilogue warp
constexpr int kTcThreads = 32 * (kProducers + 1 + 16);  // four epilogue groups (the most)
template <int kGroups>
constexpr int tc_threads() { return 32 * (kProducers + 1 + 4 * kGroups); }
constexpr int kTcStages = 4;      // key smem stages (2 pages each)
constexpr int kScaleSlots = 8;    // per-tile key scales (2 x 256 B), consumed by the epilogues
constexpr int kQSlots = 2;        // per-row q tiles
constexpr int kMaxAcc = 4;        // TMEM accumulators (epilogue group = accumulator & 1)
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kMaxTcRows = 8192;
constexpr int64_t kMaxWRows = 8;  // head-weight rows staged in shared memory per CTA

struct TcArgs {
  const int32_t* lens;
  const int32_t* table;
  int64_t table_stride;
  const float* w;
  float* out;
  int64_t out_stride, max_len;
  float* page_max;
  int64_t page_stride;
  int B, H, N, relu, clean, w_rows, lens_kind;  // N: MMA width (H, or 16 for one head)
  uint32_t tmem_cols;
  int32_t* status;
  // grouped mode: a virtual row is group_rows query rows of four heads each
  // (H = N = 4 * group_rows columns), scored against one shared key table; the
  // logit of query row r for key j goes to gout[r, colmap[page(j), r] * 64 +
  // j % 64] (or gout[r, j] without a column map), rows >= real_rows dropped.
  // colmap is page-major: [colmap_pages, colmap_stride >= virtual rows x group_rows]
  const int32_t* colmap;
  int64_t colmap_stride, colmap_pages;
  const uint8_t* key_valid;  // grouped mode without a column map: key j's logits are -inf where 0
  // grouped mode with a column map: mask_scores fused (NA/kernels.py:47-59,
  // without its dedup columns) -- row r's logit of a key is -inf when the key's
  // logical token l = mask_map[page * 64 + slot] is < 0 or > mask_pos[r]
  const int32_t* mask_map;
  const int32_t* mask_pos;
  // flat keys (fp8_mqa_logits): key j at j * 128 of a flat array, its scale in
  // a flat array; no page table (tile t holds keys 128t .. 128t + 127); rows'
  // logits outside [win_lo[r], win_hi[r]) are -inf
  int flat;
  const int32_t* win_lo;
  const int32_t* win_hi;
  float* gout;
  int64_t gout_stride;
  int real_rows, group_rows;
};

struct TcShared {
  uint64_t full[kTcStages], empty[kTcStages];
  uint64_t sfull[kScaleSlots], sempty[kScaleSlots];
  uint64_t qfull[kQSlots], qempty[kQSlots];
  uint64_t tfull[kMaxAcc], tempty[kMaxAcc];
  uint32_t tmem_base;
  int abort;
  int zero;  // always 0: lets drain waits ignore the abort flag
  int total, per;
  int warp_tot[kTcThreads / 32 + 1];
};

__device__ __forceinline__ int locate_row(const int* prefix, int B, int T) {
  int lo = 0, hi = B;  // prefix[lo] <= T < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= T) lo = mid;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ void raise_abort(TcShared& sh, int32_t* status) {
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
  if (status) atomicExch(status, V1X_STATUS_TIMEOUT);
}

__device__ __forceinline__ int64_t row_eff(const TcArgs& a, int b) {
  return a.lens ? min(score_len(a.lens[b], a.lens_kind), a.max_len) : a.max_len;  // no lengths: every row max_len
}

__device__ __forceinline__ int tiles_of(const TcArgs& a, int b) {
  const int64_t eff = row_eff(a, b);
  return eff > 0 ? static_cast<int>((eff + 127) / 128) : 0;
}

// Walks a CTA's contiguous tile range as (row, tile-in-row) without searching per tile.
struct TileCursor {
  int T, b, t, B;
  __device__ void start(const int* prefix, int nrows, int T0) {
    B = nrows;
    T = T0;
    b = locate_row(prefix, B, T0);
    t = T0 - prefix[b];
  }
  __device__ void next(const int* prefix) {
    ++T;
    ++t;
    while (b + 1 < B && T >= prefix[b + 1]) {  // skip rows without tiles
      ++b;
      t = 0;
    }
  }
  __device__ void advance(const int* prefix, int k) {
    for (int i = 0; i < k; ++i) next(prefix);
  }
};

// kGroups epilogue groups of four warps: two for many heads (a key's H columns
// take a while to reduce), one for a single head, whose epilogue is one TMEM
// column per key -- that CTA has 224 threads and at most 97 registers each, so
// two of them leave an SM room for another batch's top-k or route CTA.
template <int kGroups, bool kGrouped = false>
__global__ void __launch_bounds__(tc_threads<kGroups>(), kGroups == 4 ? 1 : (kGroups == 2 ? 2 : 3))
    score_tc_kernel(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ CUtensorMap q_map,
                    const __grid_constant__ CUtensorMap scale_map, const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t q_bytes = static_cast<uint32_t>(a.N) * 128;
  uint8_t* stages = base;                                               // kTcStages x 16 KB (A operand)
  uint8_t* qring = stages + kTcStages * 16384;                          // kQSlots x H*128 (B operand)
  float* sring = reinterpret_cast<float*>(qring + kQSlots * q_bytes);   // kScaleSlots x 128 scales
  float* wsm = sring + kScaleSlots * 128;                               // head weights of this CTA's rows
  TcShared& sh = *reinterpret_cast<TcShared*>(
      (reinterpret_cast<uintptr_t>(wsm + a.w_rows * a.H) + 15) & ~uintptr_t(15));  // 16-byte aligned
  int* prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(&sh) + sizeof(TcShared));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- barriers, TMEM, tensor-map prefetch, then the per-row tile prefix ---------
  if (tid == 0) {
    sh.abort = 0;
    sh.zero = 0;
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int r = 0; r < kScaleSlots; ++r) {
      mbar_init(&sh.sfull[r], 1);
      mbar_init(&sh.sempty[r], 128);
    }
    for (int r = 0; r < kQSlots; ++r) {
      mbar_init(&sh.qfull[r], 1);
      mbar_init(&sh.qempty[r], 1);
    }
    for (int c = 0; c < kMaxAcc; ++c) {
      mbar_init(&sh.tfull[c], 1);
      mbar_init(&sh.tempty[c], 128);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sh.tmem_base, a.tmem_cols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&pool_map);
    tma_prefetch_desc(&q_map);
    tma_prefetch_desc(&scale_map);
  }
  {
    constexpr int kThreads = tc_threads<kGroups>();
    const int chunk = (a.B + kThreads - 1) / kThreads;
    const int beg = min(tid * chunk, a.B), end = min(beg + chunk, a.B);
    int local = 0;
    for (int b = beg; b < end; ++b) local += tiles_of(a, b);
    int tot;
    int run = block_exclusive_scan(local, sh.warp_tot, &tot);
    for (int b = beg; b < end; ++b) {
      prefix[b] = run;
      run += tiles_of(a, b);
    }
    if (tid == 0) {
      prefix[a.B] = tot;
      sh.total = tot;
      sh.per = (tot + gridDim.x - 1) / gridDim.x;
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int T0 = min(static_cast<int>(blockIdx.x) * sh.per, sh.total);
  const int T1 = min(T0 + sh.per, sh.total);
  const int ntiles = T1 - T0;
  // head weights of the rows this CTA's tiles belong to, staged once
  const int b_first = ntiles > 0 ? locate_row(prefix, a.B, T0) : 0;
  const int b_last = ntiles > 0 ? locate_row(prefix, a.B, T1 - 1) : -1;
  const bool w_staged = b_last - b_first + 1 <= a.w_rows;

  if (warp < kProducers) {
    // ---------------- TMA producers: warp p issues tiles p, p + kProducers, ... ----------------
    if (lane == 0) {
      int last_it = -1;
      TileCursor cur;
      if (warp < ntiles) {
        cur.start(prefix, a.B, T0);
        cur.advance(prefix, warp);
      }
      for (int it = warp; it < ntiles; it += kProducers) {
        const int b = cur.b, t = cur.t;
        const int64_t eff = row_eff(a, b);
        const int p0 = a.flat ? 2 * t : a.table[b * a.table_stride + 2 * t];
        const int p1 = (static_cast<int64_t>(2 * t + 1) * 64 < eff) ? (a.flat ? 2 * t + 1 : a.table[b * a.table_stride + 2 * t + 1])
                                                                     : p0;
        const int s = it % kTcStages, r = it % kScaleSlots;
        if (!mbar_wait(&sh.empty[s], ((it / kTcStages) & 1) ^ 1, &sh.abort, kWaitLimitNs) ||
            !mbar_wait(&sh.sempty[r], ((it / kScaleSlots) & 1) ^ 1, &sh.abort, kWaitLimitNs)) {
          raise_abort(sh, a.status);
          break;
        }
        mbar_arrive_expect_tx(&sh.full[s], 16384);
        mbar_arrive_expect_tx(&sh.sfull[r], 512);
        if (a.flat) {  // 64-key boxes of the flat arrays (zero-filled past the last key)
          tma_load_2d(stages + s * 16384, &pool_map, &sh.full[s], 0, 64 * p0);
          tma_load_2d(stages + s * 16384 + 8192, &pool_map, &sh.full[s], 0, 64 * p1);
          tma_load_1d(sring + r * 128, &scale_map, &sh.sfull[r], 64 * p0);
          tma_load_1d(sring + r * 128 + 64, &scale_map, &sh.sfull[r], 64 * p1);
        } else {
          tma_load_3d(stages + s * 16384, &pool_map, &sh.full[s], 0, 0, p0);
          tma_load_3d(stages + s * 16384 + 8192, &pool_map, &sh.full[s], 0, 0, p1);
          tma_load_2d(sring + r * 128, &scale_map, &sh.sfull[r], 0, p0);
          tma_load_2d(sring + r * 128 + 64, &scale_map, &sh.sfull[r], 0, p1);
        }
        last_it = it;
        cur.advance(prefix, kProducers);
      }
      if (*reinterpret_cast<volatile int*>(&sh.abort)) {  // let this warp's recent loads land
        for (int k = 0, it = last_it; k < 4 && it >= 0; ++k, it -= kProducers) {
          mbar_wait(&sh.full[it % kTcStages], (it / kTcStages) & 1, &sh.zero, kWaitLimitNs);
          mbar_wait(&sh.sfull[it % kScaleSlots], (it / kScaleSlots) & 1, &sh.zero, kWaitLimitNs);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer (also loads q at row changes) ----------------
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc = idesc_e4m3_f32(128, a.N);
      TileCursor cur;
      cur.start(prefix, a.B, T0);
      int q_rows = 0, cur_b = -1, it = 0;
      bool q_pending = false;
      for (; it < ntiles; ++it) {
        const int s = it % kTcStages, acc = it % kMaxAcc;
        if (cur.b != cur_b) {
          if (cur_b >= 0) umma_commit(&sh.qempty[(q_rows - 1) % kQSlots]);  // previous row's q is free
          const int qs = q_rows % kQSlots;
          if (!mbar_wait(&sh.qempty[qs], ((q_rows / kQSlots) & 1) ^ 1, &sh.abort, kWaitLimitNs)) {
            raise_abort(sh, a.status);
            break;
          }
          mbar_arrive_expect_tx(&sh.qfull[qs], q_bytes);
          tma_load_2d(qring + qs * q_bytes, &q_map, &sh.qfull[qs], 0, cur.b * a.H);
          q_pending = true;
          if (!mbar_wait(&sh.qfull[qs], (q_rows / kQSlots) & 1, &sh.abort, kWaitLimitNs)) {
            raise_abort(sh, a.status);
            break;
          }
          q_pending = false;
          cur_b = cur.b;
          ++q_rows;
        }
        if (!mbar_wait(&sh.tempty[acc], ((it / kMaxAcc) & 1) ^ 1, &sh.abort, kWaitLimitNs) ||
            !mbar_wait(&sh.full[s], (it / kTcStages) & 1, &sh.abort, kWaitLimitNs)) {
          raise_abort(sh, a.status);
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(stages + s * 16384);
        const uint32_t sb = smem_u32(qring + ((q_rows - 1) % kQSlots) * q_bytes);
        const uint32_t d = tmem + static_cast<uint32_t>(acc * a.N);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f8(d, umma_desc_sw128(sa + 32 * k), umma_desc_sw128(sb + 32 * k), idesc, k > 0 ? 1u : 0u);
        umma_commit(&sh.empty[s]);
        umma_commit(&sh.tfull[acc]);
        cur.next(prefix);
      }
      if (*reinterpret_cast<volatile int*>(&sh.abort)) {  // let issued copies and MMAs retire
        if (q_pending) mbar_wait(&sh.qfull[q_rows % kQSlots], (q_rows / kQSlots) & 1, &sh.zero, kWaitLimitNs);
        if (it > 0) mbar_wait(&sh.tfull[(it - 1) % kMaxAcc], ((it - 1) / kMaxAcc) & 1, &sh.zero, kWaitLimitNs);
      }
    }
  } else {
    // ---------------- epilogue: group g = 0 (warps 3-6) / 1 (warps 7-10), alternate tiles ----------------
    const int g = (warp - kEpiWarp0) >> 2;
    const int q4 = warp & 3;                      // TMEM lane quarter this warp may access
    const int i = q4 * 32 + lane;                 // key of the 128-key tile == TMEM lane
    // the epilogue warps alone stage the head weights (off the producers' path)
    if (w_staged)
      for (int e = tid - 32 * kEpiWarp0; e < (b_last - b_first + 1) * a.H; e += 128 * kGroups)
        wsm[e] = a.w[static_cast<int64_t>(b_first) * a.H + e];
    asm volatile("bar.sync 1, %0;" ::"r"(128 * kGroups) : "memory");
    TileCursor cur;
    if (ntiles > g) {
      cur.start(prefix, a.B, T0);
      cur.advance(prefix, g);
    }
    for (int it = g; it < ntiles; it += kGroups) {
      const int acc = it % kMaxAcc, r = it % kScaleSlots;
      const int b = cur.b;
      const int64_t eff = row_eff(a, b);
      const int64_t key = static_cast<int64_t>(cur.t) * 128 + i;
      const float* wr = w_staged ? wsm + (b - b_first) * a.H : a.w + static_cast<int64_t>(b) * a.H;
      // grouped mode: the tile's row and page values, loaded before the waits
      // so that their latency overlaps the MMA.  The warp's 32 keys lie in one
      // page: lane l fetches query row b * G + l's column of it (and its
      // position / window), handed to the other lanes by shuffles below
      bool live = false, valid = true;
      int cm_lane = -1, pos_lane = 0, logical = 0, lo_lane = 0, hi_lane = 0;
      if constexpr (kGrouped) {
        live = key < eff;
        valid = !(a.key_valid && live) || a.key_valid[key] != 0;
        if (a.win_lo && lane < a.group_rows && b * a.group_rows + lane < a.real_rows) {
          lo_lane = a.win_lo[b * a.group_rows + lane];
          hi_lane = a.win_hi[b * a.group_rows + lane];
        }
        if (a.colmap) {
          const int64_t key0 = static_cast<int64_t>(cur.t) * 128 + q4 * 32;
          const int64_t wpage = key0 < eff ? a.table[b * a.table_stride + (key0 >> 6)] : -1;
          if (wpage >= 0 && wpage < a.colmap_pages && lane < a.group_rows) {
            cm_lane = a.colmap[wpage * a.colmap_stride + static_cast<int64_t>(b) * a.group_rows + lane];
            if (a.mask_map && b * a.group_rows + lane < a.real_rows) pos_lane = a.mask_pos[b * a.group_rows + lane];
          }
          if (a.mask_map && wpage >= 0 && wpage < a.colmap_pages) logical = a.mask_map[wpage * 64 + (key & 63)];
        }
      }
      if (!mbar_wait(&sh.sfull[r], (it / kScaleSlots) & 1, &sh.abort, kWaitLimitNs) ||
          !mbar_wait(&sh.tfull[acc], (it / kMaxAcc) & 1, &sh.abort, kWaitLimitNs)) {
        raise_abort(sh, a.status);
        break;
      }
      const float scale = sring[r * 128 + i];
      tc_fence_after();
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
      const uint32_t ta = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(acc * a.N);
      if constexpr (kGrouped) {
        // four heads per query row: columns 4g..4g+3 are row b * G + g; the
        // head sum keeps the per-row epilogue's order (four partial sums, one
        // head each, then (s0 + s1) + (s2 + s3)), so the logits are those of
        // the per-row path with the heads padded by zero weights
        const int row0 = b * a.group_rows;
        const int kcol = static_cast<int>(key & 63);
        const bool store_ok = live && (!a.key_valid || valid);
        float* const out0 = a.gout + static_cast<int64_t>(row0) * a.gout_stride;
        for (int c0 = 0; c0 < a.N; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(ta + c0, v);
          tmem_ld_wait();
#pragma unroll
          for (int g4 = 0; g4 < 32; g4 += 4) {
            const int rl = (c0 + g4) >> 2;  // row of the group
            const int cm = __shfl_sync(0xffffffffu, cm_lane, rl);
            const int pos = __shfl_sync(0xffffffffu, pos_lane, rl);
            const int wlo = __shfl_sync(0xffffffffu, lo_lane, rl), whi = __shfl_sync(0xffffffffu, hi_lane, rl);
            if (a.colmap && cm < 0) continue;  // the row does not name this page (warp-uniform)
            if (row0 + rl >= a.real_rows) continue;
            const float4 w4 = *reinterpret_cast<const float4*>(wr + c0 + g4);
            float v0 = __uint_as_float(v[g4]), v1 = __uint_as_float(v[g4 + 1]);
            float v2 = __uint_as_float(v[g4 + 2]), v3 = __uint_as_float(v[g4 + 3]);
            if (a.relu) {
              v0 = fmaxf(v0, 0.0f);
              v1 = fmaxf(v1, 0.0f);
              v2 = fmaxf(v2, 0.0f);
              v3 = fmaxf(v3, 0.0f);
            }
            const float sum = (fmaf(w4.x, v0, 0.0f) + fmaf(w4.y, v1, 0.0f)) +
                              (fmaf(w4.z, v2, 0.0f) + fmaf(w4.w, v3, 0.0f));
            if (live) {
              const int64_t col = a.colmap ? static_cast<int64_t>(cm * 64 + kcol) : key;
              const bool masked = (a.mask_map && (logical < 0 || logical > pos)) ||
                                  (a.win_lo && (key < wlo || key >= whi));
              out0[rl * a.gout_stride + col] = store_ok && !masked ? sum * scale : -CUDART_INF_F;
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&sh.tempty[acc]);
        mbar_arrive(&sh.sempty[r]);
        cur.advance(prefix, kGroups);
        continue;
      }
      if (a.H == 1) {  // column 0 only: the other 15 belong to the next rows' queries
        float v0 = __uint_as_float(tmem_ld1(ta));
        tmem_ld_wait();
        if (a.relu) v0 = fmaxf(v0, 0.0f);
        s0 = fmaf(wr[0], v0, s0);
      }
      for (int c0 = 0; a.H > 1 && c0 < a.H; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(ta + c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 w4 = *reinterpret_cast<const float4*>(wr + c0 + j);
          float v0 = __uint_as_float(v[j]), v1 = __uint_as_float(v[j + 1]);
          float v2 = __uint_as_float(v[j + 2]), v3 = __uint_as_float(v[j + 3]);
          if (a.relu) {
            v0 = fmaxf(v0, 0.0f);
            v1 = fmaxf(v1, 0.0f);
            v2 = fmaxf(v2, 0.0f);
            v3 = fmaxf(v3, 0.0f);
          }
          s0 = fmaf(w4.x, v0, s0);
          s1 = fmaf(w4.y, v1, s1);
          s2 = fmaf(w4.z, v2, s2);
          s3 = fmaf(w4.w, v3, s3);
        }
      }
      tc_fence_before();
      mbar_arrive(&sh.tempty[acc]);
      mbar_arrive(&sh.sempty[r]);
      const float sum = (s0 + s1) + (s2 + s3);
      const float score = key < eff ? sum * scale : -CUDART_INF_F;
      if (a.out && key < a.max_len && (key < eff || a.clean)) a.out[b * a.out_stride + key] = score;
      if (a.page_max) {
        float m = score;
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        if ((lane & 7) == 0 && key < a.max_len) a.page_max[b * a.page_stride + (key >> 3)] = m;
      }
      cur.advance(prefix, kGroups);
    }
    // columns past the last tile: -inf logits (clean) and -inf page maxima (always)
    const int e = tid - 32 * kEpiWarp0;   // 0 .. 128 * kGroups - 1 across the groups
    for (int b = blockIdx.x; b < a.B; b += gridDim.x) {
      const int64_t eff = row_eff(a, b);
      const int64_t start = eff > 0 ? (eff + 127) / 128 * 128 : 0;
      if (a.clean && a.out)
        for (int64_t j = start + e; j < a.max_len; j += 128 * kGroups) a.out[b * a.out_stride + j] = -CUDART_INF_F;
      if (a.page_max)
        for (int64_t gg = start / 8 + e; gg < (a.max_len + 7) / 8; gg += 128 * kGroups)
          a.page_max[b * a.page_stride + gg] = -CUDART_INF_F;
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, a.tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

int encode(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* m, CUtensorMapDataType type, int rank, const void* ptr,
           const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
           const char* what) {
  const cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(m, type, rank, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swz, swz == CU_TENSOR_MAP_SWIZZLE_NONE ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                                                                : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("score_fp8: %s tensor map encode failed (%d)", what, static_cast<int>(r));
    return V1X_ERR_CUDA;
  }
  return V1X_OK;
}

struct GroupedOut {
  const int32_t* colmap;
  int64_t colmap_stride, colmap_pages;
  const uint8_t* key_valid;
  const int32_t* mask_map;
  const int32_t* mask_pos;
  float* out;
  int64_t out_stride;
  int64_t real_rows, group_rows;
  const float* flat_scale;  // flat keys: `pool` is k [flat_keys, 128], flat_scale [flat_keys]
  int64_t flat_keys;
  const int32_t* win_lo;
  const int32_t* win_hi;
};

int score_tc_launch(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                    const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                    float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int lens_kind,
                    int64_t batch, int32_t* status, cudaStream_t stream, const GroupedOut* grp,
                    int64_t max_ctas = 0);

}  // namespace

// Launch the tensor-core scorer; returns V1X_ERR_UNSUPPORTED if the shape is not covered.
int score_fp8_tc(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                 const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                 float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int lens_kind,
                 int64_t batch, int32_t* status, cudaStream_t stream, int64_t max_ctas) {
  return score_tc_launch(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                         page_stride, heads, relu, clean, lens_kind, batch, status, stream, nullptr, max_ctas);
}

// Grouped mode: `vrows` virtual rows of group_rows query rows x 4 heads.
int score_fp8_tc_grouped(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages,
                         const int32_t* lens, const int32_t* table, int64_t table_stride, int64_t max_len,
                         const int32_t* colmap, int64_t colmap_stride, int64_t colmap_pages,
                         const uint8_t* key_valid, const int32_t* mask_map, const int32_t* mask_pos, float* out,
                         int64_t out_stride, int64_t group_rows, int64_t real_rows, int relu, int64_t vrows,
                         int32_t* status, cudaStream_t stream) {
  const GroupedOut g{colmap, colmap_stride, colmap_pages, key_valid, mask_map, mask_pos, out,
                     out_stride, real_rows, group_rows, nullptr, 0, nullptr, nullptr};
  return score_tc_launch(q, w, pool, pool_pages, lens, table, table_stride, nullptr, 0, max_len, nullptr, 0,
                         4 * group_rows, relu, 0, 0, vrows, status, stream, &g);
}

// Grouped mode over flat keys (fp8_mqa_logits): out[r, j] for j < keys, -inf
// outside [win_lo[r], win_hi[r]).
int mqa_tc_grouped(const uint8_t* q, const float* w, const uint8_t* k, const float* k_scale, int64_t keys,
                   const int32_t* win_lo, const int32_t* win_hi, float* out, int64_t out_stride, int64_t group_rows,
                   int64_t real_rows, int relu, int64_t vrows, int32_t* status, cudaStream_t stream) {
  const GroupedOut g{nullptr, 0,          0,          nullptr, nullptr, nullptr, out,
                     out_stride, real_rows, group_rows, k_scale, keys,   win_lo,  win_hi};
  return score_tc_launch(q, w, k, (keys + 63) / 64, nullptr, nullptr, 0, nullptr, 0, keys, nullptr, 0,
                         4 * group_rows, relu, 0, 0, vrows, status, stream, &g);
}

namespace {
int score_tc_launch(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                    const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                    float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int lens_kind,
                    int64_t batch, int32_t* status, cudaStream_t stream, const GroupedOut* grp,
                    int64_t max_ctas) {
  if ((heads != 1 && heads % 32 != 0) || heads > 128 || batch > kMaxTcRows || pool_pages >= (int64_t(1) << 31)) {
    set_error("score_fp8 (tensor core): heads must be 1 or a multiple of 32 <= 128 and batch <= %d", kMaxTcRows);
    return V1X_ERR_UNSUPPORTED;
  }
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(w)) & 15) != 0) {
    set_error("score_fp8 (tensor core): q and w must be 16-byte aligned");
    return V1X_ERR_INVALID;
  }
  auto enc = encode_fn();
  if (!enc) {
    set_error("score_fp8: cuTensorMapEncodeTiled unavailable");
    return V1X_ERR_CUDA;
  }
  const int64_t n_mma = heads == 1 ? 16 : heads;
  CUtensorMap pool_map, q_map, scale_map;
  const bool flat = grp && grp->flat_scale;
  if (flat) {
    // flat keys: {128 bytes, keys}, 64 keys per box; scales: {keys}, 64 per box
    const cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(grp->flat_keys)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {128, 64};
    if (int rc = encode(enc, &pool_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, pool, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, "flat keys"))
      return rc;
    const cuuint64_t sdims[1] = {static_cast<cuuint64_t>(grp->flat_keys)};
    const cuuint64_t sstrides[1] = {4};
    const cuuint32_t sbox[1] = {64};
    if (int rc = encode(enc, &scale_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 1, grp->flat_scale, sdims, sstrides, sbox,
                        CU_TENSOR_MAP_SWIZZLE_NONE, "flat scales"))
      return rc;
  } else {
    // keys: {128 bytes, 64 tokens, pages}, one page per box, 128-byte swizzle
    const cuuint64_t dims[3] = {128, 64, static_cast<cuuint64_t>(pool_pages)};
    const cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(kPageBytes)};
    const cuuint32_t box[3] = {128, 64, 1};
    if (int rc = encode(enc, &pool_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, pool, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, "pool"))
      return rc;
    // the 64 fp32 scales of each page: 256 contiguous bytes at page + 8192
    const cuuint64_t sdims[2] = {64, static_cast<cuuint64_t>(pool_pages)};
    const cuuint64_t sstrides[1] = {static_cast<cuuint64_t>(kPageBytes)};
    const cuuint32_t sbox[2] = {64, 1};
    if (int rc = encode(enc, &scale_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, pool + kKeyBytes, sdims, sstrides, sbox,
                        CU_TENSOR_MAP_SWIZZLE_NONE, "scale"))
      return rc;
  }
  {
    // q: {128 bytes, batch*heads rows}, one row's H heads per box (one head:
    // 16 rows from the row's own, zero-filled past the batch)
    const cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(batch * heads)};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(n_mma)};
    if (int rc = encode(enc, &q_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, "q"))
      return rc;
  }
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(kMaxAcc * n_mma)) cols <<= 1;
  const int64_t max_tiles = batch * ((max_len + 127) / 128);
  const int64_t sms = num_sms();
  // head-weight rows staged per CTA: a range of ceil(total/grid) tiles touches at
  // most that many rows plus one; at most kMaxWRows are staged (a CTA whose range
  // spans more rows reads the weights from global memory)
  auto plan = [&](int64_t grid, int64_t& w_rows) {
    w_rows = std::min<int64_t>({batch, (std::max<int64_t>(max_tiles, 1) + grid - 1) / grid + 1, kMaxWRows});
    return static_cast<size_t>(1024 + kTcStages * 16384 + kQSlots * n_mma * 128 + kScaleSlots * 512 +
                               w_rows * heads * 4 + sizeof(TcShared) + (batch + 1) * 4 + 16);
  };
  int64_t grid = std::min<int64_t>(sms * 2, std::max<int64_t>(max_tiles, 1)), w_rows = 0;
  size_t smem = plan(grid, w_rows);
  if (cols > 256 || smem > 113 * 1024) {  // two CTAs per SM need <= 256 TMEM columns and <= 113 KB each
    grid = std::min<int64_t>(sms, std::max<int64_t>(max_tiles, 1));
    smem = plan(grid, w_rows);
  }
  if (max_ctas > 0 && grid > max_ctas) {  // the caller's cap (small batches of many in flight)
    grid = max_ctas;
    smem = plan(grid, w_rows);
  }
  if (smem > 227 * 1024) {
    set_error("score_fp8 (tensor core): shared memory %zu too large", smem);
    return V1X_ERR_UNSUPPORTED;
  }
  TcArgs args{lens, table, table_stride, w, out, out_stride, max_len, page_max, page_stride,
              static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(n_mma), relu, clean,
              static_cast<int>(w_rows), lens_kind,
              cols, status, nullptr, 0, 0, nullptr, nullptr, nullptr, 0, nullptr, nullptr, nullptr, 0, 0, 0};
  static DeviceOnce once;
  once.run([] {
    cudaFuncSetAttribute(score_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(score_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(score_tc_kernel<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (grp) {
    args.colmap = grp->colmap;
    args.colmap_stride = grp->colmap_stride;
    args.colmap_pages = grp->colmap_pages;
    args.key_valid = grp->key_valid;
    args.mask_map = grp->mask_map;
    args.mask_pos = grp->mask_pos;
    args.flat = flat ? 1 : 0;
    args.win_lo = grp->win_lo;
    args.win_hi = grp->win_hi;
    args.gout = grp->out;
    args.gout_stride = grp->out_stride;
    args.real_rows = static_cast<int>(grp->real_rows);
    args.group_rows = static_cast<int>(grp->group_rows);
    launch_kernel(score_tc_kernel<4, true>, dim3(static_cast<unsigned>(grid)), dim3(tc_threads<4>()), smem, stream,
                  pool_map, q_map, scale_map, args);
  } else if (heads == 1)
    launch_kernel(score_tc_kernel<1>, dim3(static_cast<unsigned>(grid)), dim3(tc_threads<1>()), smem, stream,
                  pool_map, q_map, scale_map, args);
  else
    launch_kernel(score_tc_kernel<2>, dim3(static_cast<unsigned>(grid)), dim3(tc_threads<2>()), smem, stream,
                  pool_map, q_map, scale_map, args);
  return launch_status("v1x_score_fp8 (tensor core)");
}
}  // namespace

}  // namespace v1x
