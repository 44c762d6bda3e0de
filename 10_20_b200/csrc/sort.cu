// _sort for sm_100a: stable descending sort of fixed-size score segments.
//
// Reference behaviour: sglang/srt/layers/attention/v1_native/fused_grouping.py:64-76.
// Segment (g, h) is S[h*4096 + g*N + i], i < N.  A score equal to zero becomes
// +0 (:69); the key (ordered(score) << 32) | (0xFFFFFFFF - i) is sorted descending
// (:70-74) -- score desc, position asc -- and O[... + i] = P[... + pos_i].  All
// keys are unique, so any correct sort of them is bit-identical: one CTA sorts
// one segment with a shared-memory bitonic network.
#include "common.cuh"

namespace v1x {
namespace {

__device__ __forceinline__ unsigned long long sort_key(float s, int i) {
  if (s == 0.0f) s = 0.0f;
  const uint32_t b = __float_as_uint(s);
  const uint32_t o = b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
  return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
}

__global__ void __launch_bounds__(1024) sort_kernel(const int32_t* __restrict__ P,
                                                    int32_t* __restrict__ O,
                                                    const float* __restrict__ S,
                                                    const int32_t* __restrict__ flag, int N) {
  extern __shared__ unsigned long long list[];
  if (*flag >= 0) return;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * 4096 + static_cast<int64_t>(blockIdx.x) * N;
  for (int i = threadIdx.x; i < N; i += blockDim.x) list[i] = sort_key(S[base + i], i);
  bitonic_sort_desc(list, N);
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int pos = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(list[i] & 0xFFFFFFFFull));
    O[base + i] = P[base + pos];
  }
}

// Per-segment descending group offsets of integer keys (an extension).
__global__ void group_offsets_kernel(const float* __restrict__ S, int32_t* __restrict__ offs,
                                     int N, int groups, int key_range) {
  extern __shared__ int hist[];
  __shared__ int warp_tot[33];
  const int g = blockIdx.x, h = blockIdx.y;
  const int64_t base = static_cast<int64_t>(h) * 4096 + static_cast<int64_t>(g) * N;
  for (int k = threadIdx.x; k < key_range; k += blockDim.x) hist[k] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const float s = S[base + i];
    const int k = static_cast<int>(s);
    if (s >= 0.0f && k < key_range && static_cast<float>(k) == s) atomicAdd(&hist[k], 1);
  }
  __syncthreads();
  // offs[j] = sum of hist[key_range-1-t] for t < j  (descending exclusive prefix)
  const int chunk = (key_range + blockDim.x - 1) / blockDim.x;
  const int beg = min(static_cast<int>(threadIdx.x) * chunk, key_range);
  const int end = min(beg + chunk, key_range);
  int local = 0;
  for (int j = beg; j < end; ++j) local += hist[key_range - 1 - j];
  int tot;
  int run = block_exclusive_scan(local, warp_tot, &tot);
  int32_t* out = offs + (static_cast<int64_t>(h) * groups + g) * (key_range + 1);
  for (int j = beg; j < end; ++j) {
    out[j] = run;
    run += hist[key_range - 1 - j];
  }
  if (threadIdx.x == 0) out[key_range] = tot;
}

}  // namespace
}  // namespace v1x

extern "C" int v1x_sort_segments(const int32_t* P, int32_t* O, const float* S, const int32_t* flag,
                                 int64_t N, int64_t groups, int64_t heads, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(N >= 2 && N <= 4096 && (N & (N - 1)) == 0, "_sort: N must be a power of two in [2, 4096]");
  V1X_CHECK_ARG(groups >= 0 && heads >= 0 && groups * N <= 4096, "_sort: groups*N exceeds 4096");
  if (groups == 0 || heads == 0) return V1X_OK;
  const int threads = static_cast<int>(N / 2 < 1024 ? (N / 2 < 32 ? 32 : N / 2) : 1024);
  const size_t smem = static_cast<size_t>(N) * 8;
  static DeviceOnce once;
  if (once.first())
    cudaFuncSetAttribute(sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 4096 * 8);
  sort_kernel<<<dim3(static_cast<unsigned>(groups), static_cast<unsigned>(heads)), threads, smem,
                as_stream(stream)>>>(P, O, S, flag, static_cast<int>(N));
  return launch_status("v1x_sort_segments");
}

extern "C" int v1x_group_offsets(const float* S, int32_t* offsets, int64_t N, int64_t groups,
                                 int64_t heads, int64_t key_range, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(N >= 1 && N <= 4096 && groups >= 0 && heads >= 0 && groups * N <= 4096,
                "group_offsets: bad segment geometry");
  V1X_CHECK_ARG(key_range >= 1 && key_range <= 12288, "group_offsets: key_range in [1, 12288]");
  if (groups == 0 || heads == 0) return V1X_OK;
  group_offsets_kernel<<<dim3(static_cast<unsigned>(groups), static_cast<unsigned>(heads)), 1024,
                         static_cast<size_t>(key_range) * 4, as_stream(stream)>>>(
      S, offsets, static_cast<int>(N), static_cast<int>(groups), static_cast<int>(key_range));
  return launch_status("v1x_group_offsets");
}
