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
//    V1X_STATUS_ARENA_EXHAUSTED to a status word and changes nothing in the
//    arena; the lease's table row reads -1 (no page).  The status is sticky:
//    later allocations on the same word abort as well until the host clears
//    it, as nothing runs after the reference's trap.  release skips -1 entries.
//  - publish (:134-167), release (:170-179): as the reference, vectorised.
//
// Batched prepare (extension): the buckets of one or more prepares, in the
// reference's canonical order, in five launches per call instead of six per
// bucket -- fingerprints of every page (the call's meta records arrive in the
// launch parameters and are written to the work array on the way); ONE whole-GPU sweep of the arena that lists the
// live pages whose fingerprint equals a batch page's (a shared-memory hash
// table of the batch's fingerprints: one probe per live arena page), and the
// batch pages with an equal fingerprint in an earlier bucket; one warp per
// listed pair comparing bytes and members, keeping the lowest live match and
// the earliest equal batch page; one CTA (a thread per batch page) that makes
// the reference's allocate decisions in closed form (decide_kernel) --
// a page with no live match takes the slot of its earliest equal batch page,
// fresh pages pop the free stack as allocate does -- and one publish over all
// buckets.
// The answers equal the sequential per-bucket calls: refcounts only grow during
// a prepare, so a page live at the start stays live; a page content is live at
// most once (a second copy would have matched the first -- given that a
// bucket's own 16 pages are distinct, their members being disjoint token
// positions); and a page that is not live at the start can only match a page
// published inside the batch.  (The CPU test suite restates this algorithm in
// numpy and compares it with the per-bucket sequence on randomised calls.)
#include <algorithm>
#include <climits>

#include <cstring>

#include "common.cuh"

namespace v1x {
namespace {

constexpr int kMaxMatchPages = 32;
constexpr uint8_t kAborted = 2;  // new-page flag of a bucket whose allocation failed

// Where bucket b of a call reads its tmp pages, members and centre pages:
// source bucket src[b] of the pools (the identity when src is NULL; the host
// checks the ids).
struct BucketSrc {
  const int32_t* src;
  __device__ __forceinline__ int64_t bucket(int64_t b) const { return src ? src[b] : b; }
  __device__ __forceinline__ int64_t page(int64_t p) const { return src ? bucket(p >> 4) * 16 + (p & 15) : p; }
};

// pages_per_meta: pages sharing one meta record of meta_stride ints (16 and 4
// for a bucket batch; all pages and 3 for the single-bucket call); match, when
// given, is reset to "no match" (and first, the batch's earliest-equal page,
// to "none"; counters, the batch's pair counters and flags, to 0).
__device__ __forceinline__ void fingerprint_page(const uint8_t* __restrict__ tmp, const int32_t* __restrict__ map,
                                                 const int32_t* __restrict__ meta, int64_t* __restrict__ hash,
                                                 int64_t pages_per_meta, int meta_stride, int32_t* __restrict__ match,
                                                 int32_t* __restrict__ first, int32_t* __restrict__ counters,
                                                 const BucketSrc& bs) {
  const int64_t p = blockIdx.x;
  if (match && threadIdx.x == 0) match[p] = INT_MAX;
  if (first && threadIdx.x == 0) first[p] = INT_MAX;
  if (counters && p == 0 && threadIdx.x < 4) counters[threadIdx.x] = 0;
  if (meta[(p / pages_per_meta) * meta_stride + 2] == 0) return;
  const int64_t sp = bs.page(p);
  const uint4* src = reinterpret_cast<const uint4*>(tmp + sp * kPageBytes);
  // byte i = 16c + j of the page (j < 16): x_i * (i + 1) = x_i * 16c + x_i * (j + 1),
  // so per 16-byte chunk two byte dot products (dp4a) give sum x and sum x*(j+1);
  // sum x_i*(i+7) = sum x_i*(i+1) + 6 * sum x_i.  Partial sums stay in 32 bits
  // (a thread's chunks sum to < 2^32), the totals wrap in 64 bits as the
  // reference's int64 sums do.
  uint32_t s1 = 0, s0 = 0;
  for (int c = threadIdx.x; c < kPageBytes / 16; c += blockDim.x) {
    const uint4 v = src[c];
    uint32_t lo = 0, cs = 0;
    lo = __dp4a(v.x, 0x04030201u, lo);
    lo = __dp4a(v.y, 0x08070605u, lo);
    lo = __dp4a(v.z, 0x0C0B0A09u, lo);
    lo = __dp4a(v.w, 0x100F0E0Du, lo);
    cs = __dp4a(v.x, 0x01010101u, cs);
    cs = __dp4a(v.y, 0x01010101u, cs);
    cs = __dp4a(v.z, 0x01010101u, cs);
    cs = __dp4a(v.w, 0x01010101u, cs);
    s1 += lo + cs * static_cast<uint32_t>(16 * c);
    s0 += cs;
  }
  uint64_t a = s1;
  uint64_t b = (static_cast<uint64_t>(s1) + 6ull * s0) * 1000003ull;
  if (threadIdx.x < 64) {
    const uint64_t m = static_cast<uint64_t>(static_cast<int64_t>(map[sp * 64 + threadIdx.x]));
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

__global__ void __launch_bounds__(256) fingerprint_kernel(const uint8_t* __restrict__ tmp,
                                                          const int32_t* __restrict__ map,
                                                          const int32_t* __restrict__ meta,
                                                          int64_t* __restrict__ hash, int64_t pages_per_meta,
                                                          int meta_stride, int32_t* __restrict__ match,
                                                          int32_t* __restrict__ first,
                                                          int32_t* __restrict__ counters) {
  fingerprint_page(tmp, map, meta, hash, pages_per_meta, meta_stride, match, first, counters, BucketSrc{nullptr});
}

// The batched call's meta records (and source ids) travel in the launch
// parameters: the fingerprints read them there, and CTA 0 also writes them to
// the work array, where the later kernels of the call read them.
constexpr int kMetaInts = 64 * 5;   // 64 buckets: 4-int meta records, then the source ids
struct MetaBlock {
  int32_t v[kMetaInts];
};

__global__ void __launch_bounds__(256) fingerprint_batch_kernel(const uint8_t* __restrict__ tmp,
                                                                const int32_t* __restrict__ map,
                                                                const __grid_constant__ MetaBlock mb, int n_meta,
                                                                int has_src, int32_t* __restrict__ meta_dst,
                                                                int64_t* __restrict__ hash,
                                                                int32_t* __restrict__ match,
                                                                int32_t* __restrict__ first,
                                                                int32_t* __restrict__ counters) {
  const int nb = n_meta / 4;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < n_meta + (has_src ? nb : 0); i += blockDim.x) meta_dst[i] = mb.v[i];
  fingerprint_page(tmp, map, mb.v, hash, 16, 4, match, first, counters, BucketSrc{has_src ? mb.v + n_meta : nullptr});
}

// Warp-wide exact comparison of two pages: 8448 bytes and 64 members.
__device__ __forceinline__ bool warp_pages_equal(const uint8_t* x, const int32_t* xm, const uint8_t* y,
                                                 const int32_t* ym) {
  const int lane = threadIdx.x & 31;
  const uint4* a = reinterpret_cast<const uint4*>(x);
  const uint4* b = reinterpret_cast<const uint4*>(y);
  bool diff = false;
  for (int c = lane; c < kPageBytes / 16; c += 32) {
    const uint4 u = a[c], v = b[c];
    diff |= (u.x != v.x) | (u.y != v.y) | (u.z != v.z) | (u.w != v.w);
  }
  diff |= xm[lane] != ym[lane];
  diff |= xm[lane + 32] != ym[lane + 32];
  return !__any_sync(0xffffffffu, diff);
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
        const bool eq = warp_pages_equal(tmp + static_cast<int64_t>(p) * kPageBytes, map + p * 64,
                                         fine + jc * kPageBytes, members + jc * 64);
        if (eq && lane == 0) atomicMin(&match[p], static_cast<int32_t>(jc));
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
  // An exhaustion is sticky: once the status word holds it, every later
  // allocation on that word aborts too (the reference traps at the first one),
  // until the host reads and clears it.
  const bool sticky = status != nullptr && *status == V1X_STATUS_ARENA_EXHAUSTED;
  if (cnt < needed || sticky) {
    // nothing in the arena changes; the flags tell publish that the bucket was
    // not allocated, and the lease's table row reads -1 (no page), so a later
    // release of the lease touches no refcount
    if (lane < 16) {
      new_flags[lane] = kAborted;
      tables[static_cast<int64_t>(meta[1]) * 16 + lane] = -1;
    }
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
    float* __restrict__ cs, int32_t* __restrict__ members, int64_t* __restrict__ hashes, int meta_stride,
    const BucketSrc bs) {
  // block = (bucket, page): the single-bucket call launches 16 blocks
  const int64_t b = blockIdx.x / 16;
  const int p = blockIdx.x % 16;
  meta += b * meta_stride;
  if (meta[2] == 0) return;
  const int64_t sb = bs.bucket(b);
  tmp += sb * 16 * kPageBytes;
  tc += sb * 2 * kPageBytes;
  tcs += sb * 2 * kPageWords;
  map += sb * 16 * 64;
  hash += b * 16 * 2;
  new_flags += b * 16;
  if (new_flags[p] == kAborted) return;  // allocation failed: the bucket changes nothing
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
    dead = page >= 0 && atomicSub(&refs[page], 1) == 1;  // -1: a lease whose allocation aborted
  }
  const unsigned dm = __ballot_sync(0xffffffffu, dead);
  const int rank = __popc(dm & ((1u << lane) - 1u));
  int base = 0;
  if (lane == 0) base = atomicAdd(count, __popc(dm));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (dead) free_stack[base + rank] = page;
}

// ---------------------------------------------------------------------------
// Batched prepare: buckets of one or more prepares in one pass (see the header)
// ---------------------------------------------------------------------------
constexpr int kBatchBuckets = 64;                 // buckets per call
constexpr int kBatchPages = kBatchBuckets * 16;   // pages per call
constexpr int kQTable = 2 * kBatchPages;          // hash-table slots (load <= 1/2)
constexpr uint32_t kQMask = kQTable - 1;
constexpr int kBatchMeta = 4;                     // per bucket: token start, lease, active, state row
constexpr int kPairCap = 4 * kBatchPages;         // hash-equal pairs kept per list
// work ints: counters and flags, arena pairs, batch pairs, earliest equal page
constexpr int kWorkHead = 4;
static_assert(kMetaInts == kBatchBuckets * (kBatchMeta + 1), "meta records, then source ids");
constexpr int kWorkMeta = kWorkHead + 4 * kPairCap + kBatchPages;
constexpr int kWorkInts = kWorkMeta + kMetaInts;
static_assert(kWorkInts == V1X_PREPARE_WORK_INTS, "v1x.h states the work size");
constexpr int kFlagArenaOverflow = 1;
constexpr int32_t kFirstNone = INT_MAX, kFirstCollision = -2;  // values of BatchWork::first

struct BatchWork {
  int32_t* head;     // [0] arena pairs, [1] batch pairs, [2] overflow flags
  int2* arena;       // (arena page j, batch page q) with equal fingerprints
  int2* batch;       // (q', q): q' the lowest earlier-bucket batch page with q's fingerprint
  int32_t* first;    // q' if its bytes equal q's; kFirstNone; kFirstCollision (search in decide)
  __device__ explicit BatchWork(int32_t* w)
      : head(w),
        arena(reinterpret_cast<int2*>(w + kWorkHead)),
        batch(reinterpret_cast<int2*>(w + kWorkHead) + kPairCap),
        first(w + kWorkHead + 4 * kPairCap) {}
};

__device__ __forceinline__ uint32_t fp_slot(int64_t h0, int64_t h1) {
  uint64_t x = static_cast<uint64_t>(h0) * 0x9E3779B97F4A7C15ull ^ static_cast<uint64_t>(h1);
  x ^= x >> 29;
  return static_cast<uint32_t>(x >> 32) & kQMask;
}

// Inserts page q (entry q + 1; 0 = empty) by linear probing.
__device__ __forceinline__ void fp_insert(int32_t* table, uint32_t slot, int q) {
  while (atomicCAS(&table[slot], 0, q + 1) != 0) slot = (slot + 1) & kQMask;
}

// Shared-memory hash table of the batch's active pages, in every CTA.
struct QueryTable {
  int64_t h0[kBatchPages], h1[kBatchPages];
  int32_t slot[kQTable];
};

__device__ void build_query_table(QueryTable& t, const int64_t* hash, const int32_t* meta, int nq) {
  for (int i = threadIdx.x; i < kQTable; i += blockDim.x) t.slot[i] = 0;
  for (int q = threadIdx.x; q < nq; q += blockDim.x) {
    t.h0[q] = hash[2 * q];
    t.h1[q] = hash[2 * q + 1];
  }
  __syncthreads();
  for (int q = threadIdx.x; q < nq; q += blockDim.x)
    if (meta[(q / 16) * kBatchMeta + 2] != 0) fp_insert(t.slot, fp_slot(t.h0[q], t.h1[q]), q);
  __syncthreads();
}

// Next batch page after `slot` on the probe chain with fingerprint (a, b), or
// -1 at the end of the chain (slot becomes -1 too).
__device__ __forceinline__ int next_equal(const QueryTable& t, int& slot, int64_t a, int64_t b) {
  while (slot >= 0) {
    const int e = t.slot[slot];
    if (e == 0) {
      slot = -1;
      return -1;
    }
    slot = static_cast<int>((slot + 1) & kQMask);
    if (t.h0[e - 1] == a && t.h1[e - 1] == b) return e - 1;
  }
  return -1;
}

// The arena sweep with every hash hit confirmed by the warp that found it (the
// exact path when the pair list overflows).
__device__ void sweep_inline(const QueryTable& t, const uint8_t* tmp, const int32_t* map, const BucketSrc& bs,
                             const uint8_t* fine, const int32_t* members, const int64_t* hashes, const int32_t* refs,
                             int32_t* match, int64_t cap) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int64_t base = gw * 32; base < cap; base += warps * 32) {
    const int64_t j = base + lane;
    int64_t a = 0, b = 0;
    int slot = -1;
    if (j < cap && refs[j] > 0) {
      a = hashes[j * 2];
      b = hashes[j * 2 + 1];
      slot = static_cast<int>(fp_slot(a, b));
    }
    while (true) {
      const int cand = next_equal(t, slot, a, b);
      unsigned todo = __ballot_sync(0xffffffffu, cand >= 0);
      if (!todo) break;
      while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        const int q = __shfl_sync(0xffffffffu, cand, src);
        const int64_t jc = base + src;
        const int64_t sq = bs.page(q);
        const bool eq = warp_pages_equal(tmp + sq * kPageBytes, map + sq * 64, fine + jc * kPageBytes,
                                         members + jc * 64);
        if (eq && lane == 0) atomicMin(&match[q], static_cast<int32_t>(jc));
      }
    }
  }
}

// Hash-equal pairs: every live arena page whose fingerprint equals a batch
// page's, and for every batch page the lowest page of an earlier bucket with
// the same fingerprint (one pair per page, whatever the number of copies).  No
// bytes are compared here; confirm_kernel does that in parallel.
__global__ void __launch_bounds__(1024) match_batch_kernel(const int64_t* __restrict__ hash,
                                                          const int32_t* __restrict__ meta,
                                                          const int64_t* __restrict__ hashes,
                                                          const int32_t* __restrict__ refs, int64_t cap, int nq,
                                                          int32_t* __restrict__ work) {
  __shared__ QueryTable t;
  BatchWork w(work);
  build_query_table(t, hash, meta, nq);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t j = tid; j < cap; j += stride) {
    if (refs[j] <= 0) continue;
    const int64_t a = hashes[j * 2], b = hashes[j * 2 + 1];
    int slot = static_cast<int>(fp_slot(a, b));
    for (int q = next_equal(t, slot, a, b); q >= 0; q = next_equal(t, slot, a, b)) {
      const int k = atomicAdd(&w.head[0], 1);
      if (k < kPairCap) w.arena[k] = make_int2(static_cast<int>(j), q);
      else atomicOr(&w.head[2], kFlagArenaOverflow);
    }
  }
  for (int64_t q = tid; q < nq; q += stride) {
    if (meta[(q / 16) * kBatchMeta + 2] == 0) continue;
    const int64_t a = t.h0[q], b = t.h1[q];
    int slot = static_cast<int>(fp_slot(a, b));
    int lowest = INT_MAX;
    for (int p = next_equal(t, slot, a, b); p >= 0; p = next_equal(t, slot, a, b))
      if (p / 16 < q / 16) lowest = min(lowest, p);  // earlier buckets only
    if (lowest != INT_MAX) w.batch[atomicAdd(&w.head[1], 1)] = make_int2(lowest, static_cast<int>(q));
  }
}

// One warp per pair compares the bytes and members: the lowest confirmed arena
// page is the live match; a batch page whose lowest equal-fingerprint earlier
// page has equal bytes takes it as its earliest equal page, and one whose bytes
// differ (a fingerprint collision) is left to decide_kernel's exact search.  If
// the arena list overflowed, the sweep runs again with inline confirmation
// instead (exact, slower).
__global__ void __launch_bounds__(256) confirm_kernel(const uint8_t* __restrict__ tmp, const int32_t* __restrict__ map,
                                                      const int64_t* __restrict__ hash, const int32_t* __restrict__ meta,
                                                      const uint8_t* __restrict__ fine,
                                                      const int32_t* __restrict__ members,
                                                      const int64_t* __restrict__ hashes,
                                                      const int32_t* __restrict__ refs, int32_t* __restrict__ match,
                                                      int64_t cap, int nq, int32_t* __restrict__ work,
                                                      const BucketSrc bs) {
  BatchWork w(work);
  const int flags = w.head[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int na = min(w.head[0], kPairCap), nb = min(w.head[1], kPairCap);
  if (flags & kFlagArenaOverflow) {
    __shared__ QueryTable t;
    build_query_table(t, hash, meta, nq);
    sweep_inline(t, tmp, map, bs, fine, members, hashes, refs, match, cap);
  } else {
    for (int64_t k = gw; k < na; k += warps) {
      const int2 pr = w.arena[k];
      const int64_t sy = bs.page(pr.y);
      const bool eq = warp_pages_equal(tmp + sy * kPageBytes, map + sy * 64,
                                       fine + static_cast<int64_t>(pr.x) * kPageBytes, members + pr.x * 64);
      if (eq && lane == 0) atomicMin(&match[pr.y], pr.x);
    }
  }
  for (int64_t k = gw; k < nb; k += warps) {
    const int2 pr = w.batch[k];
    const int64_t sy = bs.page(pr.y), sx = bs.page(pr.x);
    const bool eq = warp_pages_equal(tmp + sy * kPageBytes, map + sy * 64, tmp + sx * kPageBytes, map + sx * 64);
    if (lane == 0) w.first[pr.y] = eq ? pr.x : kFirstCollision;
  }
}

// The allocate decisions of every bucket of the call, one CTA of 1024 threads
// (one per batch page).  The reference decides bucket after bucket; the same
// answers come from closed forms:
//   * a page is FRESH iff it has no live match and no page of an earlier
//     bucket of the call has equal bytes and members -- the earliest such page
//     is BatchWork::first (its lowest equal-fingerprint page when that one's
//     bytes are equal; after a fingerprint collision a warp searches the
//     earlier pages here);
//   * that earliest equal page is itself fresh (an equal page with a live
//     match would have given this page the same match; an earlier equal page
//     would be earlier still), so the page takes its slot;
//   * bucket b's fresh pages pop FREE[count-1-off_b-rank], off_b the fresh
//     pages of the active buckets before b (a scan over the buckets), rank the
//     page's place among its bucket's fresh pages;
//   * the first bucket whose fresh pages exceed the free pages left writes
//     V1X_STATUS_ARENA_EXHAUSTED; it and every later bucket change nothing
//     (flags = aborted, lease table rows = -1); a status word that already
//     holds the exhaustion aborts every bucket of the call.
// Then refcounts (atomic adds: several pages may share a slot), lease tables,
// new-page flags and, with state_tables, the request's page-table row (state
// row from the meta record) and centre-table row, as the driver's copies of the
// lease tables do after each reference Build.
struct StateRows {
  int32_t* tables;
  int64_t table_stride;
  int32_t* centers;
  int64_t center_stride;
  const int32_t* center_pages;
};

constexpr int kDecideThreads = kBatchPages;   // 1024: one thread per batch page

__global__ void __launch_bounds__(kDecideThreads) decide_kernel(
    const uint8_t* __restrict__ tmp, const int32_t* __restrict__ map, const int64_t* __restrict__ hash,
    const int32_t* __restrict__ meta, const int32_t* __restrict__ match, int nb, const int32_t* __restrict__ free_stack,
    int32_t* __restrict__ count, int32_t* __restrict__ refs, int32_t* __restrict__ tables,
    uint8_t* __restrict__ new_flags, int32_t* __restrict__ status, const StateRows rows,
    const int32_t* __restrict__ work, const BucketSrc bs) {
  __shared__ int64_t sh0[kBatchPages], sh1[kBatchPages];
  __shared__ int32_t ssrc[kBatchPages];      // earliest equal page of an earlier bucket, or -1
  __shared__ int32_t sfree[kBatchPages];     // sfree[i] = FREE[count0 - 1 - i]
  __shared__ uint32_t sfresh[kBatchBuckets]; // per bucket: lane mask of its fresh pages
  __shared__ int32_t soff[kBatchBuckets + 1];
  __shared__ int32_t scoll[kBatchPages];     // pages left to the collision search
  __shared__ int ncoll, abort_from;
  const BatchWork w(const_cast<int32_t*>(work));
  const int q = threadIdx.x, lane = q & 31;
  const int nq = nb * 16;
  const int b = q >> 4;
  const int cnt0 = *count;
  const bool sticky = status != nullptr && *status == V1X_STATUS_ARENA_EXHAUSTED;
  const bool in = q < nq;
  const bool active = in && meta[b * kBatchMeta + 2] != 0;
  int m = -1, f = kFirstNone;
  if (in) {
    sh0[q] = hash[2 * q];
    sh1[q] = hash[2 * q + 1];
    const int mq = match[q];
    m = mq != INT_MAX ? mq : -1;
    f = w.first[q];
  }
  for (int i = q; i < min(nq, cnt0); i += kDecideThreads) sfree[i] = free_stack[cnt0 - 1 - i];
  if (q == 0) ncoll = 0;
  __syncthreads();
  int src = -1;
  if (active && m < 0) {
    if (f >= 0 && f != kFirstNone) src = f;
    else if (f == kFirstCollision) scoll[atomicAdd(&ncoll, 1)] = q;
  }
  if (in) ssrc[q] = src;
  __syncthreads();
  // after a fingerprint collision: the earliest page of an earlier bucket with
  // equal bytes and members (one warp per such page; rare)
  for (int k = q >> 5; k < ncoll; k += kDecideThreads / 32) {
    const int qc = scoll[k];
    const int lim = (qc >> 4) << 4;           // pages of earlier buckets
    int found = -1;
    for (int p0 = 0; p0 < lim && found < 0; p0 += 32) {
      const int p = p0 + lane;
      const bool cand = p < lim && meta[(p >> 4) * kBatchMeta + 2] != 0 && sh0[p] == sh0[qc] && sh1[p] == sh1[qc];
      unsigned todo = __ballot_sync(0xffffffffu, cand);
      while (todo && found < 0) {
        const int pc = p0 + __ffs(todo) - 1;
        todo &= todo - 1;
        const int64_t sq = bs.page(qc), sc = bs.page(pc);
        if (warp_pages_equal(tmp + sq * kPageBytes, map + sq * 64, tmp + sc * kPageBytes, map + sc * 64))
          found = pc;
      }
    }
    if (lane == 0) ssrc[qc] = found;
  }
  __syncthreads();
  // fresh pages, per bucket
  const bool fresh = active && m < 0 && ssrc[q] < 0;
  const unsigned bal = __ballot_sync(0xffffffffu, fresh);
  const uint32_t mine = (bal >> (q & 16)) & 0xFFFFu;   // this half-warp's bucket
  if ((q & 15) == 0 && b < kBatchBuckets) sfresh[b] = b < nb ? mine : 0u;
  __syncthreads();
  // exclusive scan of the buckets' fresh counts and the first exhausted bucket
  if (q < 32) {
    int c0 = 0, c1 = 0;
    const int b0 = 2 * q, b1 = 2 * q + 1;
    if (b0 < nb) c0 = __popc(sfresh[b0]);
    if (b1 < nb) c1 = __popc(sfresh[b1]);
    const int inc = warp_inclusive_scan(c0 + c1);
    const int o0 = inc - c0 - c1, o1 = o0 + c0;
    soff[b0] = o0;
    soff[b1] = o1;
    if (q == 31) soff[kBatchBuckets] = inc;
    // bucket bb aborts when its fresh pages exceed what the buckets before it left
    const bool x0 = b0 < nb && cnt0 - o0 < c0, x1 = b1 < nb && cnt0 - o1 < c1;
    const int first_ab = __reduce_min_sync(0xffffffffu, x0 ? b0 : (x1 ? b1 : nb));
    if (q == 0) abort_from = sticky ? 0 : first_ab;
  }
  __syncthreads();
  const int ab = abort_from;
  if (active) {
    const int64_t lease = meta[b * kBatchMeta + 1];
    if (b >= ab) {
      new_flags[q] = kAborted;
      tables[lease * 16 + (q & 15)] = -1;
    } else {
      int dst;
      if (m >= 0) {
        dst = m;
      } else {
        // this page's, or its earliest equal page's, place on the free stack
        const int p = fresh ? q : ssrc[q];
        const int pb = p >> 4;
        dst = sfree[soff[pb] + __popc(sfresh[pb] & ((1u << (p & 15)) - 1u))];
      }
      atomicAdd(&refs[dst], 1);
      tables[lease * 16 + (q & 15)] = dst;
      new_flags[q] = fresh ? 1 : 0;
      if (rows.tables) {
        const int64_t bucket = meta[b * kBatchMeta] / 1024;
        const int64_t srow = meta[b * kBatchMeta + 3];
        rows.tables[srow * rows.table_stride + bucket * 16 + (q & 15)] = dst;
        if ((q & 15) < 2)
          rows.centers[srow * rows.center_stride + bucket * 2 + (q & 15)] =
              rows.center_pages[lease * 2 + (q & 15)];
      }
    }
  }
  if (q == 0) {
    if (ab < nb && status && !sticky) *status = V1X_STATUS_ARENA_EXHAUSTED;
    *count = cnt0 - soff[min(ab, nb) == nb ? kBatchBuckets : ab];
  }
}

// Releases of several requests in order, one CTA.  A request's pages are
// distinct (its buckets cover disjoint token positions and a page's members are
// part of its identity), so all of a request's leases are decremented at once;
// the pages that reach zero are pushed in (lease, lane) order -- the order of
// the reference's per-lease release calls -- by a block scan.  Requests follow
// one another, since different requests may share pages.
constexpr int kReleaseThreads = 1024;

__global__ void __launch_bounds__(kReleaseThreads) release_many_kernel(
    const int32_t* __restrict__ tables, const int32_t* __restrict__ leases, const int32_t* __restrict__ offsets,
    int requests, int32_t* __restrict__ refs, int32_t* __restrict__ free_stack, int32_t* __restrict__ count) {
  __shared__ int warp_tot[kReleaseThreads / 32 + 1];
  int cnt = *count;
  for (int r = 0; r < requests; ++r) {
    const int64_t o0 = static_cast<int64_t>(offsets[r]) * 16, o1 = static_cast<int64_t>(offsets[r + 1]) * 16;
    for (int64_t c = o0; c < o1; c += kReleaseThreads) {
      const int64_t i = c + threadIdx.x;
      int page = 0, dead = 0;
      if (i < o1) {
        page = tables[static_cast<int64_t>(leases[i / 16]) * 16 + i % 16];
        dead = page >= 0 && atomicSub(&refs[page], 1) == 1;  // -1: an aborted lease
      }
      int total;
      const int rank = block_exclusive_scan(dead, warp_tot, &total);
      if (dead) free_stack[cnt + rank] = page;
      cnt += total;
    }
  }
  if (threadIdx.x == 0) *count = cnt;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Host-side offsets into the work array (as BatchWork on the device).
struct BatchWorkHost {
  int32_t* head;
  int32_t* first;
  explicit BatchWorkHost(int32_t* w) : head(w), first(w + kWorkHead + 4 * kPairCap) {}
};

}  // namespace
}  // namespace v1x

extern "C" int v1x_fingerprint(const uint8_t* tmp, const int32_t* map, const int32_t* meta,
                               int64_t* hash, int64_t n_pages, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(n_pages >= 0 && aligned16(tmp), "fingerprint: tmp must be 16-byte aligned");
  if (n_pages == 0) return V1X_OK;
  fingerprint_kernel<<<static_cast<unsigned>(n_pages), 256, 0, as_stream(stream)>>>(tmp, map, meta, hash, n_pages, 3,
                                                                                 nullptr, nullptr, nullptr);
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
                                                    hashes, 3, BucketSrc{nullptr});
  return launch_status("v1x_publish");
}

extern "C" int v1x_release(const int32_t* table, int32_t* refs, int32_t* free_stack, int32_t* count,
                           void* stream) {
  using namespace v1x;
  clear_error();
  release_kernel<<<1, 32, 0, as_stream(stream)>>>(table, refs, free_stack, count);
  return launch_status("v1x_release");
}

extern "C" int v1x_prepare_buckets(const uint8_t* tmp, const uint8_t* tc_bytes, const float* tc_scales,
                                   const int32_t* map, const int32_t* meta_host, const int32_t* src_host,
                                   int64_t src_buckets, int64_t buckets, int64_t* hash,
                                   int32_t* match, uint8_t* new_flags, uint8_t* fine, uint8_t* centers,
                                   float* center_scales, int32_t* members, int64_t* hashes, int32_t* refs,
                                   int32_t* free_stack, int32_t* count, int32_t* tables,
                                   const int32_t* center_pages, int32_t* state_tables, int64_t state_table_stride,
                                   int32_t* state_centers, int64_t state_center_stride, int64_t cap,
                                   int32_t* work, int32_t* status, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(buckets >= 0 && buckets <= kBatchBuckets, "prepare_buckets: at most %d buckets per call",
                kBatchBuckets);
  V1X_CHECK_ARG(tmp && tc_bytes && tc_scales && map && meta_host && hash && match && new_flags && fine && centers &&
                    center_scales && members && hashes && refs && free_stack && count && tables,
                "prepare_buckets: a required buffer is NULL");
  V1X_CHECK_ARG(cap > 0 && cap < INT_MAX, "prepare_buckets: bad capacity");
  V1X_CHECK_ARG(!src_host || (src_buckets > 0 && src_buckets < INT_MAX),
                "prepare_buckets: src needs src_buckets > 0");
  V1X_CHECK_ARG(aligned16(tmp) && aligned16(fine) && aligned16(tc_bytes) && aligned16(centers),
                "prepare_buckets: page pools must be 16-byte aligned");
  V1X_CHECK_ARG(!state_tables || (state_centers && center_pages && state_table_stride >= 16 &&
                                  state_center_stride >= 2),
                "prepare_buckets: state rows need both tables, the centre pages and their strides");
  if (buckets == 0) return V1X_OK;
  V1X_CHECK_ARG(work != nullptr, "prepare_buckets: work (V1X_PREPARE_WORK_INTS ints) is required");
  // the host meta records and source ids, into the launch parameters
  MetaBlock mb;
  const int nm = static_cast<int>(buckets) * kBatchMeta;
  std::memcpy(mb.v, meta_host, sizeof(int32_t) * nm);
  if (src_host) {
    for (int64_t b = 0; b < buckets; ++b)
      V1X_CHECK_ARG(src_host[b] >= 0 && src_host[b] < src_buckets,
                    "prepare_buckets: source id %d of bucket %lld outside [0, %lld)", src_host[b],
                    static_cast<long long>(b), static_cast<long long>(src_buckets));
    std::memcpy(mb.v + nm, src_host, sizeof(int32_t) * buckets);
  }
  cudaStream_t s = as_stream(stream);
  const int nq = static_cast<int>(buckets) * 16;
  BatchWorkHost wh(work);
  int32_t* meta = work + kWorkMeta;
  const BucketSrc bs{src_host ? meta + nm : nullptr};
  fingerprint_batch_kernel<<<nq, 256, 0, s>>>(tmp, map, mb, nm, src_host ? 1 : 0, meta, hash, match, wh.first,
                                              wh.head);
  int64_t blocks = (cap + 255) / 256;
  const int64_t maxb = static_cast<int64_t>(num_sms()) * 4;
  if (blocks > maxb) blocks = maxb;
  // the sweep: one 1024-thread CTA per SM, each builds the call's fingerprint
  // table in shared memory (one insert per thread) and sweeps its share of the arena
  const int64_t sweep_blocks = std::min<int64_t>((cap + 1023) / 1024, num_sms());
  match_batch_kernel<<<static_cast<unsigned>(sweep_blocks), 1024, 0, s>>>(hash, meta, hashes, refs, cap, nq, work);
  confirm_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(tmp, map, hash, meta, fine, members, hashes, refs,
                                                                match, cap, nq, work, bs);
  const StateRows rows{state_tables, state_table_stride, state_centers, state_center_stride, center_pages};
  decide_kernel<<<1, kDecideThreads, 0, s>>>(tmp, map, hash, meta, match, static_cast<int>(buckets), free_stack,
                                           count, refs, tables, new_flags, status, rows, work, bs);
  publish_kernel<<<nq, 256, 0, s>>>(tmp, tc_bytes, tc_scales, map, hash, meta, tables, new_flags, fine, centers,
                                    center_scales, members, hashes, kBatchMeta, bs);
  return launch_status("v1x_prepare_buckets");
}

extern "C" int v1x_release_many(const int32_t* tables, const int32_t* leases, const int32_t* offsets,
                                int64_t requests, int32_t* refs, int32_t* free_stack, int32_t* count,
                                void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(requests >= 0 && requests < INT_MAX, "release_many: bad request count");
  V1X_CHECK_ARG(requests == 0 || (tables && leases && offsets && refs && free_stack && count),
                "release_many: a required buffer is NULL");
  if (requests == 0) return V1X_OK;
  release_many_kernel<<<1, kReleaseThreads, 0, as_stream(stream)>>>(tables, leases, offsets,
                                                                    static_cast<int>(requests), refs, free_stack,
                                                                    count);
  return launch_status("v1x_release_many");
}
