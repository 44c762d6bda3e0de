// Shared helpers for the v1x kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <math_constants.h>

#include <mutex>
#include <utility>

#include "../../include/v1x.h"

namespace v1x {

// ---- host-side error reporting --------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define V1X_CHECK_ARG(cond, ...)            \
  do {                                      \
    if (!(cond)) {                          \
      ::v1x::set_error(__VA_ARGS__);        \
      return V1X_ERR_INVALID;               \
    }                                       \
  } while (0)

// Report the result of the launches just issued.
int launch_status(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();

// Per-device one-off host set-up (function attributes).  run(f) calls f once
// per device, the current one, under std::call_once: a thread that arrives
// while another runs the set-up waits for it to finish, so no launch can
// precede its kernel's attributes.
struct DeviceOnce {
  static constexpr int kMaxDevices = 64;
  std::once_flag flags[kMaxDevices];
  template <typename F>
  void run(F&& f) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
      f();  // no usable device index: set up every time (idempotent attributes)
      return;
    }
    std::call_once(flags[dev], std::forward<F>(f));
  }
};

// ---- launches ------------------------------------------------------------------
// Scheduling priority of a launch: the latency-bound selection kernels are
// launched at the device's greatest priority so that, when another batch's
// bandwidth-bound gather runs beside them, their CTAs are placed first as SM
// slots free up; the gather keeps the default (lowest) priority.
//
// Programmatic dependent launch (a kernel starting while its predecessor drains)
// was measured and is not used: it saved ~4 us per step with one batch at a
// time, but with independent batches in flight the early-launched CTAs sat
// resident waiting for their predecessor and held the SM slots the other
// batch's gather needed (159 vs 167 us per step without it).
enum class LaunchPriority { kHigh, kDefault };
int greatest_priority();

template <typename... KArgs, typename... Args>
inline void launch_kernel_prio(LaunchPriority prio, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = prio == LaunchPriority::kHigh ? greatest_priority() : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
inline void launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args... args) {
  launch_kernel_prio(LaunchPriority::kHigh, kernel, grid, block, smem, stream, args...);
}

// ---- device helpers ---------------------------------------------------------
constexpr int kPageBytes = 8448;
constexpr int kKeyBytes = 8192;
constexpr int kScaleWord = 2048;   // float index of token 0's scale within a page
constexpr int kPageWords = 2112;   // floats per page

// Order-preserving uint32 key of a float (descending sort on the key == descending
// sort on the value).  -0.0 is folded onto +0.0, matching CUB's radix key rule that
// the reference route inherits through BlockRadixSort.
__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t b = __float_as_uint(x);
  uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return k == 0x7FFFFFFFu ? 0x80000000u : k;
}

__device__ __forceinline__ int64_t load_index(const void* p, int is64, int64_t i) {
  return is64 ? static_cast<const int64_t*>(p)[i] : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// Scoring lengths: kind 0 = the lengths as given; kind 1 = the centre count of
// a token length n, max(8 * built pages, 1) with built pages = (n-1)//1024*16
// (center_lens of DS/kernels.py:589).
__device__ __forceinline__ int64_t score_len(int n, int kind) {
  if (kind == 1) return max(static_cast<int64_t>(max(n - 1, 0) / 1024) * 16 * 8, int64_t(1));
  return n;
}

// Row bounds shared by every stage (DS/kernels.py:242-243, VQ:69-70).
struct RowBounds {
  int sink, tail;
};
__device__ __forceinline__ RowBounds row_bounds(int n, int sink_cfg, int window) {
  int sink = min(sink_cfg, n);
  int built = max(n - 1, 0) / 1024 * 1024;
  int tail = max(sink, min(built, max(sink, n - window)));
  return {sink, tail};
}

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide exclusive scan of one value per thread.  `warp_tot` is shared
// scratch of at least blockDim.x/32 + 1 entries.  Returns the exclusive prefix;
// *total receives the block total.  Contains __syncthreads().
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* warp_tot, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  T inc = warp_inclusive_scan(v);
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T t = lane < nw ? warp_tot[lane] : T(0);
    T ti = warp_inclusive_scan(t);
    if (lane < nw) warp_tot[lane] = ti - t;
    if (lane == 31) warp_tot[nw] = ti;
  }
  __syncthreads();
  T r = warp_tot[warp] + inc - v;
  *total = warp_tot[nw];
  __syncthreads();
  return r;
}

// In-place descending bitonic sort of m (a power of two) unique 64-bit keys in
// shared memory by the whole block.  Starts and ends with __syncthreads().
__device__ __forceinline__ void bitonic_sort_desc(unsigned long long* list, int m) {
  const int tid = threadIdx.x, nt = blockDim.x;
  __syncthreads();
  for (int k = 2; k <= m; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < m; i += nt) {
        const int ij = i ^ j;
        if (ij > i) {
          const unsigned long long x = list[i], y = list[ij];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            list[i] = y;
            list[ij] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace v1x
