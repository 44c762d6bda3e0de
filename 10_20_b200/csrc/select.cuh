// Block-wide exact order-statistic search on order-preserving uint32 keys.
//
// The K-th largest key is built two bits at a time from the most significant
// end: for the three candidates v|1<<b, v|2<<b, v|3<<b every thread counts its
// keys >= each candidate, the warps reduce with redux.sync and one barrier makes
// the per-warp sums visible (double-buffered, so a single barrier per step).
// Sixteen steps give the exact key; the count of keys strictly above it falls
// out of the same steps.  Cost is independent of the key distribution (no
// histogram atomics, no per-digit contention), which matters for clustered
// float scores where a radix pass puts most keys into one or two bins.
#pragma once

#include "common.cuh"

namespace v1x {

// count3(c1, c2, c3, n1, n2, n3): this thread's number of keys >= c1, c2, c3
// (c1 < c2 < c3).  `red` is shared scratch of 2 * kWarps int4.  Every thread of
// the block must call this with the same K (1 <= K <= number of keys).  Returns
// the K-th largest key; *gt_out receives the number of keys strictly above it,
// so the top K holds all of those plus K - *gt_out keys equal to it.
template <int kWarps, class Count3>
__device__ __forceinline__ uint32_t block_kth_largest(int K, Count3 count3, int4* red, int* gt_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t v = 0;
  int above = 0;  // keys >= the lowest rejected candidate (== keys > v at the end)
#pragma unroll 1
  for (int b = 30, step = 0; b >= 0; b -= 2, ++step) {
    const uint32_t c1 = v | (1u << b), c2 = v | (2u << b), c3 = v | (3u << b);
    int n1, n2, n3;
    count3(c1, c2, c3, n1, n2, n3);
    n1 = __reduce_add_sync(0xffffffffu, n1);
    n2 = __reduce_add_sync(0xffffffffu, n2);
    n3 = __reduce_add_sync(0xffffffffu, n3);
    int4* buf = red + (step & 1) * kWarps;
    if (lane == 0) buf[warp] = make_int4(n1, n2, n3, 0);
    __syncthreads();
    int s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int4 x = buf[w];
      s1 += x.x;
      s2 += x.y;
      s3 += x.z;
    }
    if (s3 >= K) {
      v = c3;
    } else if (s2 >= K) {
      v = c2;
      above = s3;
    } else if (s1 >= K) {
      v = c1;
      above = s2;
    } else {
      above = s1;
    }
  }
  *gt_out = above;
  return v;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace v1x

namespace v1x {

// One-pass coarse selection: histogram of the top kBinBits bits of every key,
// then the bin holding the K-th largest key.  The caller resolves only that
// bin's keys (typically a few dozen to a few hundred) exactly.
constexpr int kBinBits = 12;
constexpr int kBins = 1 << kBinBits;

struct TopBin {
  int bin;    // bin of the K-th largest key
  int above;  // keys in higher bins (< K)
  int in;     // keys in that bin (above + in >= K)
};

__device__ __forceinline__ int bin_of(uint32_t key) { return static_cast<int>(key >> (32 - kBinBits)); }

// Zeroes the histogram (kBins ints, 16-byte aligned) -- call, then __syncthreads().
template <int kThreads>
__device__ __forceinline__ void zero_hist(int* hist) {
  for (int i = threadIdx.x; i < kBins / 4; i += kThreads) reinterpret_cast<int4*>(hist)[i] = make_int4(0, 0, 0, 0);
}

// After every thread has added its keys with atomicAdd(&hist[bin_of(k)], 1) and
// a __syncthreads(): the bin of the K-th largest key.  `warp_tot` is scratch of
// kThreads/32 + 1 ints, `res` an int4 slot.  Contains __syncthreads().
template <int kThreads>
__device__ __forceinline__ TopBin find_top_bin(int K, const int* hist, int* warp_tot, int4* res) {
  constexpr int kPer = kBins / kThreads;  // bins per thread, descending bin order
  static_assert(kPer % 4 == 0, "bins per thread must be a multiple of 4");
  const int hi = kBins - threadIdx.x * kPer;  // this thread owns bins [hi - kPer, hi)
  int c[kPer];
  int s = 0;
#pragma unroll
  for (int q = 0; q < kPer / 4; ++q) {
    const int4 v = reinterpret_cast<const int4*>(hist + hi - kPer)[q];
    c[4 * q] = v.x;
    c[4 * q + 1] = v.y;
    c[4 * q + 2] = v.z;
    c[4 * q + 3] = v.w;
    s += v.x + v.y + v.z + v.w;
  }
  int tot;
  int cum = block_exclusive_scan(s, warp_tot, &tot);
  if (cum < K && cum + s >= K) {
#pragma unroll
    for (int j = kPer - 1; j >= 0; --j) {
      if (cum < K && cum + c[j] >= K) *res = make_int4(hi - kPer + j, cum, c[j], 0);
      cum += c[j];
    }
  }
  __syncthreads();
  const int4 r = *res;
  return TopBin{r.x, r.y, r.z};
}

}  // namespace v1x
