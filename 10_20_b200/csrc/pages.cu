// Paged-KV page lifecycle for sm_100a: fingerprint -> match_pages -> allocate ->
// publish -> release, one 16-page (1K-token) bucket per call.
//
// Reference behaviour: sglang/srt/layers/attention/v1_deepseek/kernels.py:57-179.
//  - fingerprint (:57-69): two wrapping int64 sums over a page's 8448 bytes and
//    64 members; integer sums are order-free, so the block reduction is exact.
//  - match_pages (:72-113): the LOWEST live page j whose hashes, bytes and
//    members all equal the tmp page's.  The reference scans all CAP slots in one
//    program per page; here the whole GPU sweeps the CAP hash/refcount arrays
//    once for all tmp pages, a warp confirms each hash hit byte-for-byte, and
//    atomicMin keeps the lowest confirmed j -- the same answer for any CAP.
//  - allocate (:116-131): fresh pages pop FREE[count-1-rank]; where the
//    reference device_asserts on an exhausted arena, this kernel writes
//    V1X_STATUS_ARENA_EXHAUSTED to a status word and changes nothing.
//  - publish (:134-167), release (:170-179): as the reference, vectorised.
#include <climits>

#include "common.cuh"

namespace v1x {
namespace {

constexpr int kMaxMatchPages = 32;

__global__ void __launch_bounds__(256) fingerprint_kernel(const uint8_t* __restrict__ tmp,
                                                          const int32_t* __restrict__ map,
                                                          const int32_t* __restrict__ meta,
                                                          int64_t* __restrict__ hash) {
  if (meta[2] == 0) return;
  const int64_t p = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(tmp + p * kPageBytes);
  uint64_t a = 0, b = 0;
  for (int c = threadIdx.x; c < kPageBytes / 16; c += blockDim.x) {
    const uint4 v = src[c];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const uint64_t x = (w[q >> 2] >> (8 * (q & 3))) & 0xFFu;
      const uint64_t i = static_cast<uint64_t>(c) * 16 + q;
      a += x * (i + 1);
      b += x * ((i + 7) * 1000003ull);
    }
  }
  if (threadIdx.x < 64) {
    const uint64_t m = static_cast<uint64_t>(static_cast<int64_t>(map[p * 64 + threadIdx.x]));
    a += m * 104729ull;
    b += m * (static_cast<uint64_t>(threadIdx.x) + 1) * 65537ull;
  }
  a = warp_sum(a);
  b = warp_sum(b);
  __shared__ uint64_t sa[8], sb[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sa[warp] = a;
    sb[warp] = b;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t ta = 0, tb = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      ta += sa[w];
      tb += sb[w];
    }
    hash[p * 2] = static_cast<int64_t>(ta);
    hash[p * 2 + 1] = static_cast<int64_t>(tb);
  }
}

__global__ void match_init_kernel(const int32_t* __restrict__ meta, int32_t* __restrict__ match,
                                  int n_pages) {
  if (meta[2] == 0) return;
  if (threadIdx.x < n_pages) match[threadIdx.x] = INT_MAX;
}

__global__ void match_final_kernel(const int32_t* __restrict__ meta, int32_t* __restrict__ match,
                                   int n_pages) {
  if (meta[2] == 0) return;
  if (threadIdx.x < n_pages && match[threadIdx.x] == INT_MAX) match[threadIdx.x] = -1;
}

__global__ void __launch_bounds__(256) match_scan_kernel(
    const uint8_t* __restrict__ tmp, const int32_t* __restrict__ map,
    const int64_t* __restrict__ hash, const int32_t* __restrict__ meta,
    const uint8_t* __restrict__ fine, const int32_t* __restrict__ members,
    const int64_t* __restrict__ hashes, const int32_t* __restrict__ refs,
    int32_t* __restrict__ match, int64_t cap, int n_pages) {
  if (meta[2] == 0) return;
  __shared__ int64_t h0[kMaxMatchPages], h1[kMaxMatchPages];
  if (threadIdx.x < n_pages) {
    h0[threadIdx.x] = hash[threadIdx.x * 2];
    h1[threadIdx.x] = hash[threadIdx.x * 2 + 1];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int64_t base = gw * 32; base < cap; base += warps * 32) {
    const int64_t j = base + lane;
    uint32_t pm = 0;
    if (j < cap && refs[j] > 0) {
      const int64_t a = hashes[j * 2], b = hashes[j * 2 + 1];
      for (int p = 0; p < n_pages; ++p) pm |= (a == h0[p] && b == h1[p]) ? (1u << p) : 0u;
    }
    unsigned hits = __ballot_sync(0xffffffffu, pm != 0);
    while (hits) {
      const int src = __ffs(hits) - 1;
      hits &= hits - 1;
      const int64_t jc = base + src;
      uint32_t pmask = __shfl_sync(0xffffffffu, pm, src);
      while (pmask) {
        const int p = __ffs(pmask) - 1;
        pmask &= pmask - 1;
        // warp-wide exact comparison of 8448 bytes and 64 members
        const uint4* x = reinterpret_cast<const uint4*>(tmp + static_cast<int64_t>(p) * kPageBytes);
        const uint4* y = reinterpret_cast<const uint4*>(fine + jc * kPageBytes);
        bool diff = false;
        for (int c = lane; c < kPageBytes / 16; c += 32) {
          const uint4 u = x[c], v = y[c];
          diff |= (u.x != v.x) | (u.y != v.y) | (u.z != v.z) | (u.w != v.w);
        }
        diff |= map[p * 64 + lane] != members[jc * 64 + lane];
        diff |= map[p * 64 + lane + 32] != members[jc * 64 + lane + 32];
        if (!__any_sync(0xffffffffu, diff) && lane == 0) atomicMin(&match[p], static_cast<int32_t>(jc));
      }
    }
  }
}

__global__ void allocate_kernel(const int32_t* __restrict__ meta, const int32_t* __restrict__ match,
                                int32_t* __restrict__ free_stack, int32_t* __restrict__ count,
                                int32_t* __restrict__ refs, int32_t* __restrict__ tables,
                                uint8_t* __restrict__ new_flags, int32_t* __restrict__ status) {
  if (meta[2] == 0) return;
  const int lane = threadIdx.x;
  int dst = lane < 16 ? match[lane] : 0;
  const bool fresh = lane < 16 && dst < 0;
  const unsigned fm = __ballot_sync(0xffffffffu, fresh);
  const int rank = __popc(fm & ((1u << lane) - 1u));
  const int needed = __popc(fm);
  const int cnt = *count;
  if (cnt < needed) {
    if (lane == 0 && status) *status = V1X_STATUS_ARENA_EXHAUSTED;
    return;
  }
  if (lane < 16) {
    if (fresh) dst = free_stack[cnt - 1 - rank];
    atomicAdd(&refs[dst], 1);
    tables[static_cast<int64_t>(meta[1]) * 16 + lane] = dst;
    new_flags[lane] = fresh ? 1 : 0;
  }
  __syncwarp();
  if (lane == 0) *count = cnt - needed;
}

__global__ void __launch_bounds__(256) publish_kernel(
    const uint8_t* __restrict__ tmp, const uint8_t* __restrict__ tc, const float* __restrict__ tcs,
    const int32_t* __restrict__ map, const int64_t* __restrict__ hash,
    const int32_t* __restrict__ meta, const int32_t* __restrict__ tables,
    const uint8_t* __restrict__ new_flags, uint8_t* __restrict__ fine, uint8_t* __restrict__ centers,
    float* __restrict__ cs, int32_t* __restrict__ members, int64_t* __restrict__ hashes) {
  if (meta[2] == 0) return;
  const int p = blockIdx.x;
  const int64_t lease = meta[1];
  if (new_flags[p]) {
    const int64_t dst = tables[lease * 16 + p];
    const uint4* src = reinterpret_cast<const uint4*>(tmp + static_cast<int64_t>(p) * kPageBytes);
    uint4* out = reinterpret_cast<uint4*>(fine + dst * kPageBytes);
    for (int c = threadIdx.x; c < kPageBytes / 16; c += blockDim.x) out[c] = src[c];
    if (threadIdx.x < 64) members[dst * 64 + threadIdx.x] = map[p * 64 + threadIdx.x];
    if (threadIdx.x < 2) hashes[dst * 2 + threadIdx.x] = hash[p * 2 + threadIdx.x];
  }
  // the bucket's 8 centres of page p: 8 x 128 bytes + 8 scales, to slot lease*128 + p*8 + g
  if (threadIdx.x < 64) {
    const int g = threadIdx.x >> 3, part = threadIdx.x & 7;
    const int64_t sc = p * 8 + g, dc = lease * 128 + sc;
    const uint4 v = reinterpret_cast<const uint4*>(tc + (sc / 64) * kPageBytes + (sc % 64) * 128)[part];
    reinterpret_cast<uint4*>(centers + (dc / 64) * kPageBytes + (dc % 64) * 128)[part] = v;
    if (part == 0) cs[(dc / 64) * kPageWords + kScaleWord + dc % 64] = tcs[(sc / 64) * kPageWords + kScaleWord + sc % 64];
  }
}

__global__ void release_kernel(const int32_t* __restrict__ table, int32_t* __restrict__ refs,
                               int32_t* __restrict__ free_stack, int32_t* __restrict__ count) {
  const int lane = threadIdx.x;
  int page = 0;
  bool dead = false;
  if (lane < 16) {
    page = table[lane];
    dead = atomicSub(&refs[page], 1) == 1;
  }
  const unsigned dm = __ballot_sync(0xffffffffu, dead);
  const int rank = __popc(dm & ((1u << lane) - 1u));
  int base = 0;
  if (lane == 0) base = atomicAdd(count, __popc(dm));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (dead) free_stack[base + rank] = page;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace v1x

extern "C" int v1x_fingerprint(const uint8_t* tmp, const int32_t* map, const int32_t* meta,
                               int64_t* hash, int64_t n_pages, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(n_pages >= 0 && aligned16(tmp), "fingerprint: tmp must be 16-byte aligned");
  if (n_pages == 0) return V1X_OK;
  fingerprint_kernel<<<static_cast<unsigned>(n_pages), 256, 0, as_stream(stream)>>>(tmp, map, meta, hash);
  return launch_status("v1x_fingerprint");
}

extern "C" int v1x_match_pages(const uint8_t* tmp, const int32_t* map, const int64_t* hash,
                               const int32_t* meta, const uint8_t* fine, const int32_t* members,
                               const int64_t* hashes, const int32_t* refs, int32_t* match,
                               int64_t cap, int64_t n_pages, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(n_pages >= 0 && n_pages <= kMaxMatchPages, "match_pages: at most 32 pages per call");
  V1X_CHECK_ARG(cap >= 0 && cap < INT_MAX, "match_pages: bad capacity");
  V1X_CHECK_ARG(aligned16(tmp) && aligned16(fine), "match_pages: page pools must be 16-byte aligned");
  if (n_pages == 0) return V1X_OK;
  cudaStream_t s = as_stream(stream);
  const int np = static_cast<int>(n_pages);
  match_init_kernel<<<1, 32, 0, s>>>(meta, match, np);
  int64_t blocks = (cap + 255) / 256;
  const int64_t maxb = static_cast<int64_t>(num_sms()) * 4;
  if (blocks > maxb) blocks = maxb;
  if (blocks < 1) blocks = 1;
  match_scan_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(tmp, map, hash, meta, fine, members,
                                                                  hashes, refs, match, cap, np);
  match_final_kernel<<<1, 32, 0, s>>>(meta, match, np);
  return launch_status("v1x_match_pages");
}

extern "C" int v1x_allocate(const int32_t* meta, const int32_t* match, int32_t* free_stack,
                            int32_t* count, int32_t* refs, int32_t* tables, uint8_t* new_flags,
                            int32_t* status, void* stream) {
  using namespace v1x;
  clear_error();
  allocate_kernel<<<1, 32, 0, as_stream(stream)>>>(meta, match, free_stack, count, refs, tables,
                                                   new_flags, status);
  return launch_status("v1x_allocate");
}

extern "C" int v1x_publish(const uint8_t* tmp, const uint8_t* tc_bytes, const float* tc_scales,
                           const int32_t* map, const int64_t* hash, const int32_t* meta,
                           const int32_t* tables, const uint8_t* new_flags, uint8_t* fine,
                           uint8_t* centers, float* center_scales, int32_t* members,
                           int64_t* hashes, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(aligned16(tmp) && aligned16(fine) && aligned16(tc_bytes) && aligned16(centers),
                "publish: page pools must be 16-byte aligned");
  publish_kernel<<<16, 256, 0, as_stream(stream)>>>(tmp, tc_bytes, tc_scales, map, hash, meta, tables,
                                                    new_flags, fine, centers, center_scales, members,
                                                    hashes);
  return launch_status("v1x_publish");
}

extern "C" int v1x_release(const int32_t* table, int32_t* refs, int32_t* free_stack, int32_t* count,
                           void* stream) {
  using namespace v1x;
  clear_error();
  release_kernel<<<1, 32, 0, as_stream(stream)>>>(table, refs, free_stack, count);
  return launch_status("v1x_release");
}
