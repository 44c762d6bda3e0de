// FP8 paged scoring for sm_100a: out[b, j] = sum_h w[b,h] * relu(q[b,h,:] . k_j) * s_j.
//
// Reference contract: DeepGEMM fp8_paged_mqa_logits as called at
// sglang/srt/layers/attention/v1_deepseek/runtime.py:434-444 (centres) and
// :538-548 (fine candidates); the formula is the reference's own restatement in
// kernels.py:310-313 (fine) / :210-213 (coarse), pinned against DeepGEMM at
// experiments/fine_pool_shared_20261021/test_and_bench.py:37-41.
//
// This file holds the SIMT path: one thread per key, 16-byte loads of the
// key's 128 FP8 bytes, exact e4m3 -> fp32 conversion, and a FIXED fp32
// evaluation order (per head d = 0..127 with fma -- every e4m3 x e4m3 product
// is exact in fp32 -- then acc += w_h * relu with separately rounded multiply
// and add, then * scale) so the result is bit-identical to the CPU oracle.
// It is the path for few heads (the single-head config is 2 FLOP/byte).
#include <cuda_fp8.h>

#include "common.cuh"

namespace v1x {
namespace {

constexpr int kScoreThreads = 128;
constexpr int kSimtMaxHeads = 64;

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
};

__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// kHeads: 1 compiles the single-head case (a 512-byte query in shared memory and
// a register budget for eight resident CTAs per SM); 0 takes the head count from
// the arguments (up to kSimtMaxHeads).  The arithmetic per key is the same.
template <int kHeads>
__global__ void __launch_bounds__(kScoreThreads, kHeads == 1 ? 8 : 1)
    score_simt_kernel(const __grid_constant__ ScoreArgs a) {
  __shared__ __align__(16) float qs[(kHeads ? kHeads : kSimtMaxHeads) * 128];
  __shared__ float ws[kHeads ? kHeads : kSimtMaxHeads];
  const int64_t b = blockIdx.x;
  const int H = kHeads ? kHeads : a.heads;
  for (int i = threadIdx.x; i < H * 64; i += blockDim.x) {
    const uint16_t two = reinterpret_cast<const uint16_t*>(a.q + b * H * 128)[i];
    const float2 f = e4m3x2_to_float2(two);
    qs[2 * i] = f.x;
    qs[2 * i + 1] = f.y;
  }
  for (int h = threadIdx.x; h < H; h += blockDim.x) ws[h] = a.w[b * H + h];
  __syncthreads();
  // Grid-stride over the row's blocks of 128 keys: the query is staged once per
  // CTA, and the next block's key bytes are loaded while the current block is
  // evaluated (two keys' loads in flight per thread).
  const int64_t n = score_len(a.lens[b], a.lens_kind);
  const int64_t lim = min(n, a.max_len);   // keys j < lim are scored
  const int64_t step = static_cast<int64_t>(gridDim.y) * blockDim.x;
  auto load_key = [&](int64_t j, uint4 (&kw)[8], float& scale) {
    if (j < lim) {
      const int64_t page = a.table[b * a.table_stride + j / 64];
      const uint8_t* kp = a.pool + page * kPageBytes + (j % 64) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) kw[c] = reinterpret_cast<const uint4*>(kp)[c];
      scale = reinterpret_cast<const float*>(a.pool + page * kPageBytes)[kScaleWord + j % 64];
    }
  };
  uint4 cur[8], nxt[8];
  float cur_scale = 0.0f, nxt_scale = 0.0f;
  int64_t j = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  load_key(j, cur, cur_scale);
  for (; j - threadIdx.x < a.max_len; j += step) {
    load_key(j + step, nxt, nxt_scale);
    float result = -CUDART_INF_F;
    if (j < lim) {
      float acc = 0.0f;
      for (int h = 0; h < H; ++h) {
        const float4* qh = reinterpret_cast<const float4*>(qs + h * 128);
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t w4[4] = {cur[c].x, cur[c].y, cur[c].z, cur[c].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float2 lo = e4m3x2_to_float2(static_cast<uint16_t>(w4[u] & 0xFFFFu));
            const float2 hi = e4m3x2_to_float2(static_cast<uint16_t>(w4[u] >> 16));
            const float4 qq = qh[c * 4 + u];
            dot = __fmaf_rn(qq.x, lo.x, dot);
            dot = __fmaf_rn(qq.y, lo.y, dot);
            dot = __fmaf_rn(qq.z, hi.x, dot);
            dot = __fmaf_rn(qq.w, hi.y, dot);
          }
        }
        const float r = a.relu ? (dot > 0.0f ? dot : 0.0f) : dot;
        acc = __fadd_rn(acc, __fmul_rn(ws[h], r));
      }
      result = __fmul_rn(acc, cur_scale);
    }
    if (a.page_max) {  // max over each group of 8 consecutive keys (lanes 8k..8k+7)
      float m = result;
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      if ((threadIdx.x & 7) == 0 && j < a.max_len) a.page_max[b * a.page_stride + j / 8] = m;
    }
    if (j < a.max_len && a.out && (j < n || a.clean)) a.out[b * a.out_stride + j] = result;
#pragma unroll
    for (int c = 0; c < 8; ++c) cur[c] = nxt[c];
    cur_scale = nxt_scale;
  }
}

}  // namespace

int score_fp8_tc(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                 const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                 float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int lens_kind,
                 int64_t batch, int32_t* status, cudaStream_t stream);

namespace {
int score_dispatch(const uint8_t* q, const float* w, const uint8_t* pool, int64_t pool_pages, const int32_t* lens,
                   const int32_t* table, int64_t table_stride, float* out, int64_t out_stride, int64_t max_len,
                   float* page_max, int64_t page_stride, int64_t heads, int relu, int clean, int impl,
                   int lens_kind, int32_t* status, int64_t batch, void* stream) {
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
  const bool tc = impl == 2 || (impl == 0 && heads % 32 == 0 && heads <= 128);
  if (tc)
    return score_fp8_tc(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                        page_stride, heads, relu, clean, lens_kind, batch, status, as_stream(stream));
  if (heads > kSimtMaxHeads) {
    set_error("score_fp8: the SIMT path takes heads <= %d", kSimtMaxHeads);
    return V1X_ERR_UNSUPPORTED;
  }
  ScoreArgs a{q, w, pool, lens, table, table_stride, out, out_stride, max_len, page_max, page_stride,
              static_cast<int>(heads), relu, clean, lens_kind};
  const int64_t blocks = (max_len + kScoreThreads - 1) / kScoreThreads;
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(blocks < 8 ? blocks : 8));
  if (heads == 1) launch_kernel(score_simt_kernel<1>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  else launch_kernel(score_simt_kernel<0>, grid, dim3(kScoreThreads), 0, as_stream(stream), a);
  return launch_status("v1x_score_fp8");
}
}  // namespace
}  // namespace v1x

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
                                int lens_kind, int32_t* status, int64_t batch, void* stream) {
  return v1x::score_dispatch(q, w, pool, pool_pages, lens, table, table_stride, out, out_stride, max_len, page_max,
                             page_stride, heads, relu, clean, impl, lens_kind, status, batch, stream);
}
