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
//   steps, accumulator in TMEM (two accumulators, ping-pong).
//
// Warp roles in a persistent CTA (192 threads):
//   warp 0    TMA producer: per tile, two 8 KB page boxes (3-D tensor map over
//             the packed pool, 128-byte swizzle) + the row's 64x128 q box.
//   warp 1    TMEM owner + single-thread MMA issuer; commits release the smem
//             stage and publish the accumulator.
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (one key per thread),
//             ReLU, weighted head sum, per-key scale, coalesced store.
// Tiles (row, 128-key block) are enumerated from a per-row prefix computed in
// shared memory from the device lengths and dealt round-robin to the CTAs.
// Every mbarrier wait is bounded (2 s); on timeout the CTA records
// V1X_STATUS_TIMEOUT, drains what it issued and frees its TMEM before exiting.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

namespace v1x {
namespace {

using namespace sm100;

constexpr int kTcThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-5 / 6-9 two epilogue groups
constexpr int kTcStages = 4;      // key smem stages (2 pages each)
constexpr int kScaleSlots = 8;    // per-tile key scales (2 x 256 B), consumed by the epilogues
constexpr int kQSlots = 2;        // per-row q tiles
constexpr int kMaxAcc = 4;        // TMEM accumulators (epilogue group = acc & 1)
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr int kMaxTcRows = 8192;

struct TcArgs {
  const int32_t* lens;
  const int32_t* table;
  int64_t table_stride;
  const float* w;
  float* out;
  int64_t out_stride, max_len;
  float* page_max;
  int64_t page_stride;
  int B, H, relu, clean;
  uint32_t tmem_cols;
  int32_t* status;
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
  return min(static_cast<int64_t>(a.lens[b]), a.max_len);
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
};

__global__ void __launch_bounds__(kTcThreads, 1)
    score_tc_kernel(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ CUtensorMap q_map,
                    const __grid_constant__ CUtensorMap scale_map, const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t q_bytes = static_cast<uint32_t>(a.H) * 128;
  uint8_t* stages = base;                                    // kTcStages x 16 KB (A operand)
  uint8_t* qring = stages + kTcStages * 16384;               // kQSlots x H*128 (B operand)
  float* sring = reinterpret_cast<float*>(qring + kQSlots * q_bytes);   // kScaleSlots x 128
  TcShared& sh = *reinterpret_cast<TcShared*>(sring + kScaleSlots * 128);
  int* prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(&sh) + sizeof(TcShared));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- per-row tile prefix and this CTA's contiguous tile range ---------------
  {
    const int chunk = (a.B + kTcThreads - 1) / kTcThreads;
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
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, a.tmem_cols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&pool_map);
    tma_prefetch_desc(&q_map);
    tma_prefetch_desc(&scale_map);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int T0 = min(static_cast<int>(blockIdx.x) * sh.per, sh.total);
  const int T1 = min(T0 + sh.per, sh.total);
  const int ntiles = T1 - T0;

  if (warp == 0) {
    // ---------------- TMA producer: lanes resolve 32 tiles' pages at once; lanes 0-3 issue ----------------
    int issued_keys = 0, issued_scales = 0, q_rows = 0, cur_b = -1;
    bool stop = false;
    for (int c = 0; c < ntiles && !stop; c += 32) {
      int bl = 0, p0l = 0, p1l = 0;
      if (c + lane < ntiles) {
        const int T = T0 + c + lane;
        bl = locate_row(prefix, a.B, T);
        const int t = T - prefix[bl];
        const int64_t eff = row_eff(a, bl);
        p0l = a.table[bl * a.table_stride + 2 * t];
        p1l = (static_cast<int64_t>(2 * t + 1) * 64 < eff) ? a.table[bl * a.table_stride + 2 * t + 1] : p0l;
      }
      const int n = min(32, ntiles - c);
      for (int j = 0; j < n; ++j) {
        const int it = c + j;
        const int b = __shfl_sync(0xffffffffu, bl, j);
        const int p0 = __shfl_sync(0xffffffffu, p0l, j);
        const int p1 = __shfl_sync(0xffffffffu, p1l, j);
        const int s = it % kTcStages, r = it % kScaleSlots;
        int ok = 1;
        if (lane == 0) {
          if (b != cur_b) {  // new row: its q tile into the next q slot
            const int qs = q_rows % kQSlots;
            ok = mbar_wait(&sh.qempty[qs], ((q_rows / kQSlots) & 1) ^ 1, &sh.abort, kWaitLimitNs);
            if (ok) {
              mbar_arrive_expect_tx(&sh.qfull[qs], q_bytes);
              tma_load_2d(qring + qs * q_bytes, &q_map, &sh.qfull[qs], 0, b * a.H);
            }
          }
          ok = ok && mbar_wait(&sh.empty[s], ((it / kTcStages) & 1) ^ 1, &sh.abort, kWaitLimitNs);
          ok = ok && mbar_wait(&sh.sempty[r], ((it / kScaleSlots) & 1) ^ 1, &sh.abort, kWaitLimitNs);
          if (ok) {
            mbar_arrive_expect_tx(&sh.full[s], 16384);
            mbar_arrive_expect_tx(&sh.sfull[r], 512);
          } else {
            raise_abort(sh, a.status);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
        if (b != cur_b) {
          cur_b = b;
          ++q_rows;
        }
        // four TMA issues in parallel, one per lane
        if (lane == 0) tma_load_3d(stages + s * 16384, &pool_map, &sh.full[s], 0, 0, p0);
        else if (lane == 1) tma_load_3d(stages + s * 16384 + 8192, &pool_map, &sh.full[s], 0, 0, p1);
        else if (lane == 2) tma_load_2d(sring + r * 128, &scale_map, &sh.sfull[r], 0, p0);
        else if (lane == 3) tma_load_2d(sring + r * 128 + 64, &scale_map, &sh.sfull[r], 0, p1);
        ++issued_keys;
        ++issued_scales;
        __syncwarp();
      }
    }
    if (lane == 0 && *reinterpret_cast<volatile int*>(&sh.abort)) {  // drain what was issued
      for (int k = max(0, issued_keys - kTcStages); k < issued_keys; ++k)
        mbar_wait(&sh.full[k % kTcStages], (k / kTcStages) & 1, &sh.zero, kWaitLimitNs);
      for (int k = max(0, issued_scales - kScaleSlots); k < issued_scales; ++k)
        mbar_wait(&sh.sfull[k % kScaleSlots], (k / kScaleSlots) & 1, &sh.zero, kWaitLimitNs);
      for (int k = max(0, q_rows - kQSlots); k < q_rows; ++k)
        mbar_wait(&sh.qfull[k % kQSlots], (k / kQSlots) & 1, &sh.zero, kWaitLimitNs);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      const uint32_t idesc = idesc_e4m3_f32(128, a.H);
      TileCursor cur;
      cur.start(prefix, a.B, T0);
      int q_rows = 0, cur_b = -1, it = 0;
      for (; it < ntiles; ++it) {
        const int s = it % kTcStages, acc = it % kMaxAcc;
        if (cur.b != cur_b) {
          if (cur_b >= 0) umma_commit(&sh.qempty[(q_rows - 1) % kQSlots]);  // previous row's q is free
          const int qs = q_rows % kQSlots;
          if (!mbar_wait(&sh.qfull[qs], (q_rows / kQSlots) & 1, &sh.abort, kWaitLimitNs)) { raise_abort(sh, a.status); break; }
          cur_b = cur.b;
          ++q_rows;
        }
        if (!mbar_wait(&sh.tempty[acc], ((it / kMaxAcc) & 1) ^ 1, &sh.abort, kWaitLimitNs)) { raise_abort(sh, a.status); break; }
        if (!mbar_wait(&sh.full[s], (it / kTcStages) & 1, &sh.abort, kWaitLimitNs)) { raise_abort(sh, a.status); break; }
        tc_fence_after();
        const uint32_t sa = smem_u32(stages + s * 16384);
        const uint32_t sb = smem_u32(qring + ((q_rows - 1) % kQSlots) * q_bytes);
        const uint32_t d = tmem + static_cast<uint32_t>(acc * a.H);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f8(d, umma_desc_sw128(sa + 32 * k), umma_desc_sw128(sb + 32 * k), idesc, k > 0 ? 1u : 0u);
        umma_commit(&sh.empty[s]);
        umma_commit(&sh.tfull[acc]);
        cur.next(prefix);
      }
      if (*reinterpret_cast<volatile int*>(&sh.abort) && it > 0) {  // let issued MMAs retire
        const int k = it - 1;
        mbar_wait(&sh.tfull[k % kMaxAcc], (k / kMaxAcc) & 1, &sh.zero, kWaitLimitNs);
      }
    }
  } else {
    // ---------------- epilogue: group g = 0 (warps 2-5) / 1 (warps 6-9), alternate tiles ----------------
    const int g = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int i = q4 * 32 + lane;                 // row of the 128-key tile == TMEM lane
    TileCursor cur;
    if (ntiles > g) {
      cur.start(prefix, a.B, T0);
      if (g) cur.next(prefix);
    }
    for (int it = g; it < ntiles; it += 2) {
      const int acc = it % kMaxAcc, r = it % kScaleSlots;
      const int b = cur.b;
      const int64_t eff = row_eff(a, b);
      const int64_t key = static_cast<int64_t>(cur.t) * 128 + i;
      const float* wg = a.w + static_cast<int64_t>(b) * a.H;   // L1-resident: a CTA's tiles share rows
      if (!mbar_wait(&sh.sfull[r], (it / kScaleSlots) & 1, &sh.abort, kWaitLimitNs)) { raise_abort(sh, a.status); break; }
      const float scale = sring[r * 128 + i];
      if (!mbar_wait(&sh.tfull[acc], (it / kMaxAcc) & 1, &sh.abort, kWaitLimitNs)) { raise_abort(sh, a.status); break; }
      tc_fence_after();
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
      for (int c0 = 0; c0 < a.H; c0 += 64) {
        uint32_t v[64];
        const uint32_t ta = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(acc * a.H + c0);
        tmem_ld32(ta, *reinterpret_cast<uint32_t(*)[32]>(v));
        if (c0 + 32 < a.H) tmem_ld32(ta + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tmem_ld_wait();
        const int ncol = min(64, a.H - c0);
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
          if (j < ncol) {
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(wg + c0 + j));
            float v0 = __uint_as_float(v[j]), v1 = __uint_as_float(v[j + 1]);
            float v2 = __uint_as_float(v[j + 2]), v3 = __uint_as_float(v[j + 3]);
            if (a.relu) {
              v0 = fmaxf(v0, 0.0f); v1 = fmaxf(v1, 0.0f); v2 = fmaxf(v2, 0.0f); v3 = fmaxf(v3, 0.0f);
            }
            s0 = fmaf(w4.x, v0, s0);
            s1 = fmaf(w4.y, v1, s1);
            s2 = fmaf(w4.z, v2, s2);
            s3 = fmaf(w4.w, v3, s3);
          }
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
      cur.next(prefix);
      cur.next(prefix);
    }
    // columns past the last tile: -inf logits (clean) and -inf page maxima (always)
    const int e = tid - 64;   // 0..255 across both groups
    for (int b = blockIdx.x; b < a.B; b += gridDim.x) {
      const int64_t eff = row_eff(a, b);
      const int64_t start = eff > 0 ? (eff + 127) / 128 * 128 : 0;
      if (a.clean && a.out)
        for (int64_t j = start + e; j < a.max_len; j += 256) a.out[b * a.out_stride + j] = -CUDART_INF_F;
      if (a.page_max)
        for (int64_t gg = start / 8 + e; gg < (a.max_len + 7) / 8; gg += 256)
          a.page_max[b * a.page_stride + gg] = -CUDART_INF_F;
    }
  }
  __syncthreads();
  if (warp == 1) {
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

}  // namespace

// Launch the tensor-core scorer; returns V1X_ERR_UNSUPPORTED if the shape is not covered.
int score_fp8_tc(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                 const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                 float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int64_t batch,
                 int32_t* status, cudaStream_t stream) {
  if (heads % 32 != 0 || heads > 128 || batch > kMaxTcRows || pool_pages >= (int64_t(1) << 31)) {
    set_error("score_fp8 (tensor core): heads must be a multiple of 32 <= 128 and batch <= %d", kMaxTcRows);
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
  CUtensorMap pool_map, q_map, scale_map;
  {
    cuuint64_t dims[3] = {128, 64, static_cast<cuuint64_t>(pool_pages)};
    cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(kPageBytes)};
    cuuint32_t box[3] = {128, 64, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&pool_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(pool), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("score_fp8: pool tensor map encode failed (%d)", static_cast<int>(r));
      return V1X_ERR_CUDA;
    }
  }
  {
    cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(batch * heads)};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, static_cast<cuuint32_t>(heads)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&q_map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("score_fp8: q tensor map encode failed (%d)", static_cast<int>(r));
      return V1X_ERR_CUDA;
    }
  }
  {
    // the 64 fp32 scales of each page: 256 contiguous bytes at page + 8192
    cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(pool_pages)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kPageBytes)};
    cuuint32_t box[2] = {64, 1};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&scale_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<uint8_t*>(pool) + kKeyBytes, dims,
                     strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("score_fp8: scale tensor map encode failed (%d)", static_cast<int>(r));
      return V1X_ERR_CUDA;
    }
  }
  const int nacc = kMaxAcc;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(nacc * heads)) cols <<= 1;
  if (cols > 512) {
    set_error("score_fp8 (tensor core): heads > 128 not supported");
    return V1X_ERR_UNSUPPORTED;
  }
  TcArgs args{lens, table, table_stride, w, out, out_stride, max_len, page_max, page_stride,
              static_cast<int>(batch), static_cast<int>(heads), relu, clean, cols, status};
  const size_t smem = 1024 + kTcStages * 16384 + kQSlots * heads * 128 + kScaleSlots * 512 + sizeof(TcShared) +
                      (batch + 1) * 4 + 16;
  static DeviceOnce once;
  if (once.first())
    cudaFuncSetAttribute(score_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (smem > 227 * 1024) {
    set_error("score_fp8 (tensor core): shared memory %zu too large", smem);
    return V1X_ERR_UNSUPPORTED;
  }
  const int64_t max_tiles = batch * ((max_len + 127) / 128);
  const int per_sm = (cols <= 256 && smem <= 113 * 1024) ? 2 : 1;  // TMEM and smem both allow two
  int64_t grid = static_cast<int64_t>(num_sms()) * per_sm;
  if (grid > max_tiles) grid = max_tiles > 0 ? max_tiles : 1;
  score_tc_kernel<<<static_cast<unsigned>(grid), kTcThreads, smem, stream>>>(pool_map, q_map, scale_map, args);
  return launch_status("v1x_score_fp8 (tensor core)");
}

}  // namespace v1x
