// _sort for sm_100a: stable descending sort of fixed-size score segments.
//
// Reference behaviour: sglang/srt/layers/attention/v1_native/fused_grouping.py:64-76.
// Segment (g, h) is S[h*4096 + g*N + i], i < N.  A score equal to zero becomes
// +0 (:69); the key (ordered(score) << 32) | (0xFFFFFFFF - i) is sorted descending
// (:70-74) -- score desc, position asc -- and O[... + i] = P[... + pos_i].  All
// keys are unique, so any correct sort of them is bit-identical.
//
// Segments of up to 256 records: one thread per record, several segments per
// 256-thread CTA.  A record's output slot is its rank -- the number of records
// of its segment with a larger ordered score, plus those with an equal score at
// a lower position -- counted over the segment's keys in shared memory, and the
// record's P value is stored straight to that slot.  The flag, scores and P
// values are loaded together, so a launch costs one memory round trip.
// Segments of 512..4096 records: one CTA per segment, a stable block radix sort
// (CUB's header-only BlockRadixSort compiled into this kernel) of the 32-bit
// ordered scores carrying the records' P values: descending, and stable, so
// equal scores keep ascending positions -- the reference's composite key order.
// A shared-memory bitonic network of all log2(N)*(log2(N)+1)/2 stages remains
// for scores or outputs that are not 16-byte aligned.
#include <cub/block/block_radix_sort.cuh>

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
  int* sP = reinterpret_cast<int*>(list + N);  // the segment's P values, for the final permutation
  // the flag, the scores and P are loaded together (no dependent round trips)
  const int f = *flag;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * 4096 + static_cast<int64_t>(blockIdx.x) * N;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    list[i] = sort_key(S[base + i], i);
    sP[i] = P[base + i];
  }
  if (f >= 0) return;
  bitonic_sort_desc(list, N);
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int pos = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(list[i] & 0xFFFFFFFFull));
    O[base + i] = sP[pos];
  }
}

__device__ __forceinline__ uint32_t ordered_score(float s) {
  if (s == 0.0f) s = 0.0f;  // -0 -> +0 (:69)
  const uint32_t b = __float_as_uint(s);
  return b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}

// Segments of N <= 256 records by rank counting: a record's output slot is the
// number of records of its segment with a greater key, plus the equal keys
// before it (the stable order).  T threads share one record, each counting over
// N / T of the segment's keys, and a CTA of 256 threads takes R = 256 / T
// consecutive records -- so the 4096 records of a head row spread over 4096 / R
// CTAs (up to a few per SM) instead of the 4096 / 256 that one thread per record
// would give.  The CTA stages the keys of every segment it touches: its own R
// records when R >= N, else the whole segment its records lie in.
template <int N, int T>
__global__ void __launch_bounds__(256) sort_rank_kernel(const int32_t* __restrict__ P, int32_t* __restrict__ O,
                                                        const float* __restrict__ S,
                                                        const int32_t* __restrict__ flag, int records) {
  static_assert(N >= 2 && N <= 1024 && (N & (N - 1)) == 0, "segment size");
  static_assert(T >= 1 && T <= 32 && (T & (T - 1)) == 0 && T <= N, "threads per record");
  constexpr int R = 256 / T;            // records per CTA
  constexpr int C = N / T;              // keys compared per thread
  constexpr int K = R >= N ? R : N;     // keys staged per CTA
  __shared__ __align__(16) uint32_t skey[K];
  const int t = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.y) * 4096;
  const int base = blockIdx.x * R;                  // first record of the CTA
  const int kbase = R >= N ? base : base / N * N;   // first staged key
  // flag, scores and P in one round trip
  const int f = *flag;
#pragma unroll
  for (int y = t; y < K; y += 256) {
    const int x = kbase + y;
    skey[y] = x < records ? ordered_score(S[row + x]) : 0u;
  }
  const int r = t / T, part = t % T;
  const int rec = base + r;
  const bool live = rec < records;
  const int pv = live && part == 0 ? P[row + rec] : 0;
  __syncthreads();
  if (f >= 0) return;
  const int li = rec - kbase;           // the record's staged key
  const int sb = li / N * N;            // its segment's first staged key
  const int i = li - sb;                // its position in the segment
  const uint32_t k = skey[li];
  const uint32_t* keys = skey + sb + part * C;
  const int u0 = part * C;
  int rank = 0;
  if constexpr (C >= 4) {
#pragma unroll
    for (int u = 0; u < C; u += 4) {
      const uint4 v = *reinterpret_cast<const uint4*>(keys + u);
      const int j = u0 + u;
      rank += (v.x > k) + (v.y > k) + (v.z > k) + (v.w > k);
      rank += (v.x == k && j < i) + (v.y == k && j + 1 < i) + (v.z == k && j + 2 < i) + (v.w == k && j + 3 < i);
    }
  } else {
#pragma unroll
    for (int u = 0; u < C; ++u) rank += (keys[u] > k) + (keys[u] == k && u0 + u < i);
  }
#pragma unroll
  for (int o = T / 2; o >= 1; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
  if (live && part == 0) O[row + rec - i + rank] = pv;
}

struct LastValid {  // scan operator: the most recent valid (>= 0) value
  __device__ __forceinline__ int operator()(int a, int b) const { return b >= 0 ? b : a; }
};

// kThreads x kItems == N.  Thread t loads and stores records t*kItems + [0, kItems)
// (contiguous per thread), the blocked arrangement BlockRadixSort works in.  S and
// O must be 16-byte aligned when kItems % 4 == 0 (the host checks).
//
// Only the key bits that differ within the segment are sorted: bits equal in every
// key cannot change the order, and score keys usually share their high bits (group
// ids 0..4095 as floats differ in ~19 of 32), which saves radix passes.
//
// kOffsets: also write the segment's descending group offsets (v1x_group_offsets
// semantics) from the sorted keys: offs[j] = number of records whose score is an
// integer key in [0, key_range) greater than key_range-1-j.  In sorted order the
// valid keys appear descending; a record whose key v starts a run writes offs[j]
// for every threshold between v and the previous valid key, with the count of
// valid records before it -- every entry is written exactly once, no atomics.
template <int kThreads, int kItems, bool kOffsets>
__global__ void __launch_bounds__(kThreads) sort_radix_kernel(const int32_t* __restrict__ P,
                                                              int32_t* __restrict__ O,
                                                              const float* __restrict__ S,
                                                              const int32_t* __restrict__ flag,
                                                              int32_t* __restrict__ offs, int groups,
                                                              int key_range) {
  using Sorter = cub::BlockRadixSort<uint32_t, kThreads, kItems, int>;
  using Scan = cub::BlockScan<int, kThreads>;
  __shared__ union {
    typename Sorter::TempStorage sort;
    typename Scan::TempStorage scan;
  } temp;
  __shared__ uint32_t red_and[kThreads / 32], red_or[kThreads / 32];
  __shared__ int red_min[kThreads / 32];
  constexpr int N = kThreads * kItems;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * 4096 + static_cast<int64_t>(blockIdx.x) * N;
  const int i0 = threadIdx.x * kItems;
  // the flag, the scores and the P values (the sort's payload) in one round trip
  const int f = *flag;
  float s[kItems];
  int pv[kItems];
  if constexpr (kItems % 4 == 0) {   // 16-byte loads: segments start at multiples of N records
#pragma unroll
    for (int k = 0; k < kItems; k += 4) {
      const float4 v = *reinterpret_cast<const float4*>(S + base + i0 + k);
      s[k] = v.x;
      s[k + 1] = v.y;
      s[k + 2] = v.z;
      s[k + 3] = v.w;
      const int4 q = *reinterpret_cast<const int4*>(P + base + i0 + k);
      pv[k] = q.x;
      pv[k + 1] = q.y;
      pv[k + 2] = q.z;
      pv[k + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      s[k] = S[base + i0 + k];
      pv[k] = P[base + i0 + k];
    }
  }
  if (f >= 0) return;
  // Integer scores (group ids carried as floats): when every score of the segment
  // is an integer of magnitude <= 2^24, v - min is an order-preserving key (-0 and
  // +0 both map to 0, as the ordered key folds them) spanning far fewer bits than
  // the float bit patterns (12 instead of ~19 for ids 0..4095), so fewer passes.
  bool ints = true;
  int imin = 0x7FFFFFFF;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const bool is_int = fabsf(s[k]) <= 16777216.0f && s[k] == truncf(s[k]);  // false for NaN / inf
    ints = ints && is_int;
    if (is_int) imin = min(imin, static_cast<int>(s[k]));
  }
  ints = __syncthreads_and(ints) != 0;
  if (ints) {
    imin = __reduce_min_sync(0xffffffffu, imin);
    if ((threadIdx.x & 31) == 0) red_min[threadIdx.x >> 5] = imin;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) imin = min(imin, red_min[w]);
  }
  uint32_t key[kItems];
  uint32_t kand = 0xFFFFFFFFu, kor = 0u;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    key[k] = ints ? static_cast<uint32_t>(static_cast<int>(s[k]) - imin) : ordered_score(s[k]);
    kand &= key[k];
    kor |= key[k];
  }
  kand = __reduce_and_sync(0xffffffffu, kand);
  kor = __reduce_or_sync(0xffffffffu, kor);
  if ((threadIdx.x & 31) == 0) {
    red_and[threadIdx.x >> 5] = kand;
    red_or[threadIdx.x >> 5] = kor;
  }
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    kand &= red_and[w];
    kor |= red_or[w];
  }
  const uint32_t diff = kand ^ kor;   // bits that differ between some keys
  if (diff != 0u) {                   // all keys equal: the stable order is the identity
    const int begin = __ffs(diff) - 1, end = 32 - __clz(diff);
    Sorter(temp.sort).SortDescending(key, pv, begin, end);
  }
  if constexpr (kItems % 4 == 0) {
#pragma unroll
    for (int k = 0; k < kItems; k += 4)
      *reinterpret_cast<int4*>(O + base + i0 + k) = make_int4(pv[k], pv[k + 1], pv[k + 2], pv[k + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < kItems; ++k) O[base + i0 + k] = pv[k];
  }
  if constexpr (kOffsets) {
    // sorted keys back to scores; -1 marks records outside the integer key range
    int v[kItems];
    int nvalid = 0, last = -1;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      if (ints) {
        const int ki = static_cast<int>(key[k]) + imin;
        v[k] = ki >= 0 && ki < key_range ? ki : -1;
        nvalid += v[k] >= 0;
        if (v[k] >= 0) last = v[k];
        continue;
      }
      const uint32_t b = (key[k] & 0x80000000u) ? (key[k] ^ 0x80000000u) : ~key[k];
      const float x = __uint_as_float(b);
      const int ki = static_cast<int>(x);
      v[k] = (x >= 0.0f && ki < key_range && static_cast<float>(ki) == x) ? ki : -1;
      nvalid += v[k] >= 0;
      if (v[k] >= 0) last = v[k];
    }
    __syncthreads();  // the sort's shared storage is reused by the scans
    int before, prev, total;
    Scan(temp.scan).ExclusiveSum(nvalid, before, total);
    __syncthreads();
    Scan(temp.scan).ExclusiveScan(last, prev, -1, LastValid());
    int32_t* out = offs + (static_cast<int64_t>(blockIdx.y) * groups + blockIdx.x) * (key_range + 1);
    int cnt = before;
    int hi = prev >= 0 ? prev : key_range;  // previous valid key (key_range: none yet)
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      if (v[k] < 0) continue;
      if (v[k] != hi)   // first record of key v[k]: thresholds u in [v, hi) see cnt keys above
        for (int u = v[k]; u < hi; ++u) out[key_range - 1 - u] = cnt;
      hi = v[k];
      ++cnt;
    }
    if (threadIdx.x == kThreads - 1) {   // thresholds below the smallest valid key: all of them
      const int lo = total > 0 ? hi : key_range;
      for (int u = -1; u < lo; ++u) out[key_range - 1 - u] = total;
    }
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
  const dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(heads));
  cudaStream_t s = as_stream(stream);
  const bool al = ((reinterpret_cast<uintptr_t>(S) | reinterpret_cast<uintptr_t>(O)) & 15) == 0;
  const int g = static_cast<int>(groups);
  const int recs = static_cast<int>(groups * N);
  auto rank_grid = [&](int t) {   // 256 / t records per CTA
    const int r = 256 / t;
    return dim3(static_cast<unsigned>((recs + r - 1) / r), static_cast<unsigned>(heads));
  };
#define V1X_RANK(n, t) \
  case n: sort_rank_kernel<n, t><<<rank_grid(t), 256, 0, s>>>(P, O, S, flag, recs); return launch_status("v1x_sort_segments");
  switch (N) {   // records of up to 256 per segment: rank counting, any alignment
    V1X_RANK(256, 32)
    V1X_RANK(128, 8)
    V1X_RANK(64, 8)
    V1X_RANK(32, 4)
    V1X_RANK(16, 2)
    V1X_RANK(8, 1)
    V1X_RANK(4, 1)
    V1X_RANK(2, 1)
#undef V1X_RANK
    default: break;
  }
  const bool alp = al && (reinterpret_cast<uintptr_t>(P) & 15) == 0;
  switch (alp ? N : 0) {
    case 4096: sort_radix_kernel<512, 8, false><<<grid, 512, 0, s>>>(P, O, S, flag, nullptr, 0, 0); break;
    case 2048: sort_radix_kernel<256, 8, false><<<grid, 256, 0, s>>>(P, O, S, flag, nullptr, 0, 0); break;
    case 1024: sort_radix_kernel<128, 8, false><<<grid, 128, 0, s>>>(P, O, S, flag, nullptr, 0, 0); break;
    case 512: sort_radix_kernel<64, 8, false><<<grid, 64, 0, s>>>(P, O, S, flag, nullptr, 0, 0); break;
    default: {  // unaligned scores, P or output
      const int threads = static_cast<int>(N / 2 < 1024 ? (N / 2 < 32 ? 32 : N / 2) : 1024);
      sort_kernel<<<grid, threads, static_cast<size_t>(N) * 12, s>>>(P, O, S, flag, static_cast<int>(N));
    }
  }
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

extern "C" int v1x_sort_segments_grouped(const int32_t* P, int32_t* O, const float* S, const int32_t* flag,
                                         int32_t* offsets, int64_t N, int64_t groups, int64_t heads,
                                         int64_t key_range, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(N == 4096 || N == 2048 || N == 1024 || N == 512 || N == 256,
                "sort_segments_grouped: N must be a power of two in [256, 4096]");
  V1X_CHECK_ARG(groups >= 0 && heads >= 0 && groups * N <= 4096, "sort_segments_grouped: groups*N exceeds 4096");
  V1X_CHECK_ARG(key_range >= 1 && key_range <= (1 << 20), "sort_segments_grouped: key_range in [1, 2^20]");
  V1X_CHECK_ARG(((reinterpret_cast<uintptr_t>(S) | reinterpret_cast<uintptr_t>(O) |
                  reinterpret_cast<uintptr_t>(P)) & 15) == 0,
                "sort_segments_grouped: S, P and O must be 16-byte aligned");
  if (groups == 0 || heads == 0) return V1X_OK;
  const dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(heads));
  cudaStream_t s = as_stream(stream);
  const int g = static_cast<int>(groups), kr = static_cast<int>(key_range);
  switch (N) {
    case 4096: sort_radix_kernel<512, 8, true><<<grid, 512, 0, s>>>(P, O, S, flag, offsets, g, kr); break;
    case 2048: sort_radix_kernel<256, 8, true><<<grid, 256, 0, s>>>(P, O, S, flag, offsets, g, kr); break;
    case 1024: sort_radix_kernel<128, 8, true><<<grid, 128, 0, s>>>(P, O, S, flag, offsets, g, kr); break;
    case 512: sort_radix_kernel<64, 8, true><<<grid, 64, 0, s>>>(P, O, S, flag, offsets, g, kr); break;
    default: sort_radix_kernel<32, 8, true><<<grid, 32, 0, s>>>(P, O, S, flag, offsets, g, kr); break;
  }
  return launch_status("v1x_sort_segments_grouped");
}
