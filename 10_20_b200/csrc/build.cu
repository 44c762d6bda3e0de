// Index build of 1024-token buckets for sm_100a: initialize -> balanced
// bisection grouping -> assemble.
//
// Reference: sglang/srt/layers/attention/v1_deepseek/runtime.py:170-233
// (Build.compute's first stages), v1_deepseek/kernels.py:9-54 (initialize,
// assemble) and v1_native/fused_grouping.py:27-76 (_init, _dots, _anchor,
// _sort).  The reference runs one bucket as 1 + 7 x 6 + 1 dependent launches
// (initialize; per level n = 1024 .. 16 three _dots, two _anchor and one _sort;
// assemble).
//
// Here one thread-block cluster of 8 CTAs x 1024 threads builds one bucket in a
// single launch (many buckets per launch, one cluster each).  CTA r owns
// positions (and, at initialisation, tokens) [128r, 128r + 128); eight lanes
// share a position and keep its member's unit vector in registers for the three
// dot modes of a level.  The unit vectors live in the bucket's workspace (L2).
// Levels whose groups span CTAs (n = 1024, 512, 256) send the argmin partials,
// the sort keys and the next permutation straight into the shared memory of the
// group's CTAs (distributed shared memory) behind hardware cluster barriers; from
// n = 128 down a group lies inside one CTA, whose members' vectors are copied
// into shared memory once, and the levels run with block barriers only.  There
// is no spin-wait anywhere.
//
// Fixed fp32 evaluation order (the one the reference's kernels produce in the
// Triton interpreter, whose tl.sum is numpy's pairwise float32 sum): a 128-term
// sum is eight strided accumulators r_j = p[j] + p[8+j] + ... + p[120+j] (lane j
// of the eight), combined ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) by the xor-1/2/4
// butterfly; products and sums are separately rounded (no fma contraction, as
// the reference's enable_fp_fusion=False); sqrt and division are IEEE.  A
// centre's mean adds its 8 members in order.  The centre scale is the smallest
// power of two >= max|mean| / 448 (exactly; the reference's exp2(ceil(log2()))
// can land one power lower a few ulps above a power of two).
#include <atomic>
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace v1x {
namespace {

constexpr int kBuildCtas = 8;          // cluster size: one bucket
constexpr int kBuildThreads = 1024;    // 128 positions x 8 lanes
constexpr int kSlice = 128;            // positions per CTA
constexpr int kBucket = 1024;          // tokens per bucket
constexpr int kWarps = kBuildThreads / 32;

// per-bucket workspace: the bucket's unit vectors, lane-major (512 KB, read by
// every CTA of the cluster from L2)
constexpr int64_t kWorkBytes = int64_t(kBucket) * 128 * 4;

struct BuildArgs {
  const uint8_t* native;
  int64_t native_pages;
  const int32_t* source;   // [buckets, 16] native page of each bucket page
  const int32_t* starts;   // [buckets] first logical token of the bucket
  uint8_t* tmp;            // [buckets, 16, 8448]
  uint8_t* centers;        // [buckets, 2, 8448]
  int32_t* mapping;        // [buckets, 16, 64]
  int32_t* perm;           // [buckets, 1024] final member order (optional)
  uint8_t* work;           // [buckets, kWorkBytes]
  int32_t* status;
};

struct BuildSmem {
  // levels <= 128: unit vectors of the slice's members (lane-major rows);
  // assemble: the dequantised rows of the CTA's positions
  float xs[kSlice][128];
  unsigned long long keys[kBucket];      // sort keys of the current group
  int pg[2][kSlice];                     // levels >= 256: member at each of the CTA's positions
  int ploc[2][kSlice];                   // levels <= 128: xs row at each position
  int tok[kSlice];                       // member of each xs row
  int4 part[2][kBuildCtas];              // MODE 0/1 argmin partials: (value bits, position, member)
  float wv[kWarps];
  int wp[kWarps];
  int wt[kWarps];
  float gv[kWarps];
  int gp[kWarps];
  float cmax[16][2];
};

__device__ __forceinline__ float e4m3_to_f32(uint32_t byte) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(byte), __NV_E4M3);
  return __half2float(__half(h));
}

// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) over the eight lanes of a position
__device__ __forceinline__ float lanes8_sum(float r) {
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
  return r;
}

// lane j's 16 values of a lane-major workspace row (16 contiguous floats)
__device__ __forceinline__ void load_row16(const float* __restrict__ src, float (&x)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src) + c);
    x[4 * c] = v.x;
    x[4 * c + 1] = v.y;
    x[4 * c + 2] = v.z;
    x[4 * c + 3] = v.w;
  }
}

// Shared-memory rows are chunk-major: lane j's chunk c (values 4c..4c+3) sits at
// float4 index c*8 + j, so the eight lanes of a position read eight distinct
// bank groups in every load.
__device__ __forceinline__ void load_srow16(const float* row, int j, float (&x)[16]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 v = reinterpret_cast<const float4*>(row)[c * 8 + j];
    x[4 * c] = v.x;
    x[4 * c + 1] = v.y;
    x[4 * c + 2] = v.z;
    x[4 * c + 3] = v.w;
  }
}

// lane j of 8: r_j = x[0]*y[0] + x[1]*y[1] + ... (dims j, j+8, ...), then the butterfly
__device__ __forceinline__ float dot_regs(const float (&x)[16], const float (&y)[16]) {
  float r = __fmul_rn(x[0], y[0]);
#pragma unroll
  for (int i = 1; i < 16; ++i) r = __fadd_rn(r, __fmul_rn(x[i], y[i]));
  return lanes8_sum(r);
}

__device__ __forceinline__ bool argmin_better(float v1, int p1, float v2, int p2) {
  return v1 < v2 || (v1 == v2 && p1 < p2);
}

// (v, p) reduced over the 4 positions of a warp (lanes 8 apart)
__device__ __forceinline__ void warp_argmin4(float& v, int& p) {
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int op = __shfl_xor_sync(0xffffffffu, p, o);
    if (argmin_better(ov, op, v, p)) {
      v = ov;
      p = op;
    }
  }
}

// Argmin of every group of n consecutive positions of the CTA (n in 16..128);
// returns the winning position of the calling thread's group.  Two barriers.
__device__ int cta_group_argmin(float v, int p, int n, BuildSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  warp_argmin4(v, p);
  if (lane == 0) {
    sm.wv[warp] = v;
    sm.wp[warp] = p;
  }
  __syncthreads();
  if (warp == 0) {
    float gv = sm.wv[lane];
    int gp = sm.wp[lane];
    const int gw = n / 4;  // warps per group
    for (int o = gw / 2; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
      const int op = __shfl_xor_sync(0xffffffffu, gp, o);
      if (argmin_better(ov, op, gv, gp)) {
        gv = ov;
        gp = op;
      }
    }
    sm.gv[lane] = gv;
    sm.gp[lane] = gp;
  }
  __syncthreads();
  return sm.gp[warp];
}

__device__ __forceinline__ unsigned long long sort_key(float s, int k) {
  return (static_cast<unsigned long long>(order_key(s)) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(k));
}

// number of keys[0..n) greater than `mine`, split over the position's 8 lanes
__device__ __forceinline__ int rank_in_group(const unsigned long long* keys, int n, unsigned long long mine, int j) {
  int c = 0;
  for (int k = j; k < n; k += 8) c += keys[k] > mine;
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  return c;
}

// Dequantised token row, lane j's 16 values x[i] = K[8i + j] * scale.
__device__ __forceinline__ bool load_token_lane(const BuildArgs& a, const int32_t* src_pages, int t, int j,
                                                float (&x)[16]) {
  const int64_t page = src_pages[t >> 6];
  const bool ok = page >= 0 && page < a.native_pages;
  if (!ok) {
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = 0.0f;
    return false;
  }
  const uint8_t* row = a.native + page * kPageBytes + (t & 63) * 128;
  const float scale = reinterpret_cast<const float*>(a.native + page * kPageBytes)[kScaleWord + (t & 63)];
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // bytes 16c..16c+15 = dims 16c + b: dim 8i+j for i = 2c, 2c+1
    const uint4 w = reinterpret_cast<const uint4*>(row)[c];
    const unsigned long long lo = (static_cast<unsigned long long>(w.y) << 32) | w.x;
    const unsigned long long hi = (static_cast<unsigned long long>(w.w) << 32) | w.z;
    x[2 * c] = __fmul_rn(e4m3_to_f32(static_cast<uint32_t>(lo >> (8 * j)) & 0xFFu), scale);
    x[2 * c + 1] = __fmul_rn(e4m3_to_f32(static_cast<uint32_t>(hi >> (8 * j)) & 0xFFu), scale);
  }
  return true;
}

__device__ __forceinline__ float pow2_ceil(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x007FFFFFu) == 0 ? v : __uint_as_float(((b >> 23) + 1u) << 23);
}

// assemble of the CTA's 128 positions = bucket pages 2r, 2r+1 and centres
// 16r .. 16r+15 (DS/kernels.py:32-54).  `ids` = the CTA's final member slice.
__device__ void assemble_slice(const BuildArgs& a, const int32_t* src_pages, int start, const int* ids, int r,
                               uint8_t* tmp, uint8_t* centers, int32_t* mapping, BuildSmem& sm) {
  const int tid = threadIdx.x, q = tid >> 3, j = tid & 7;
  const int pos = r * kSlice + q;  // bucket position = tmp page * 64 + row
  const int src = ids[q] & (kBucket - 1);
  const int64_t page = src_pages[src >> 6];
  const bool ok = page >= 0 && page < a.native_pages;
  uint8_t* dst = tmp + static_cast<int64_t>(pos >> 6) * kPageBytes;
  uint4 w = make_uint4(0, 0, 0, 0);
  float scale = 0.0f;
  if (ok) {
    w = reinterpret_cast<const uint4*>(a.native + page * kPageBytes + (src & 63) * 128)[j];
    scale = reinterpret_cast<const float*>(a.native + page * kPageBytes)[kScaleWord + (src & 63)];
  }
  reinterpret_cast<uint4*>(dst + (pos & 63) * 128)[j] = w;
  if (j == 0) {
    reinterpret_cast<float*>(dst)[kScaleWord + (pos & 63)] = scale;
    mapping[pos] = start + src;
  }
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int b = 0; b < 4; ++b)
      sm.xs[q][16 * j + 4 * u + b] = __fmul_rn(e4m3_to_f32((ws[u] >> (8 * b)) & 0xFFu), scale);
  __syncthreads();
  // centre c (16 per CTA): 64 threads, dims d and d + 64
  const int c = tid >> 6, d = tid & 63;
  float mean[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float acc = sm.xs[8 * c][d + 64 * h];
#pragma unroll
    for (int m = 1; m < 8; ++m) acc = __fadd_rn(acc, sm.xs[8 * c + m][d + 64 * h]);
    mean[h] = __fdiv_rn(acc, 8.0f);
  }
  float vmax = fmaxf(fabsf(mean[0]), fabsf(mean[1]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
  if ((tid & 31) == 0) sm.cmax[c][(tid >> 5) & 1] = vmax;
  __syncthreads();
  vmax = fmaxf(fmaxf(sm.cmax[c][0], sm.cmax[c][1]), 1.0e-4f);
  const float cs = pow2_ceil(__fdiv_rn(vmax, 448.0f));
  const int cg_ = r * 16 + c;  // centre index within the bucket
  uint8_t* cp = centers + static_cast<int64_t>(cg_ >> 6) * kPageBytes;
#pragma unroll
  for (int h = 0; h < 2; ++h)
    cp[(cg_ & 63) * 128 + d + 64 * h] =
        static_cast<uint8_t>(__nv_cvt_float_to_fp8(__fdiv_rn(mean[h], cs), __NV_SATFINITE, __NV_E4M3));
  if (d == 0) reinterpret_cast<float*>(cp)[kScaleWord + (cg_ & 63)] = cs;
}

__global__ void __cluster_dims__(kBuildCtas, 1, 1) __launch_bounds__(kBuildThreads, 1)
    build_bucket_kernel(const __grid_constant__ BuildArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BuildSmem& sm = *reinterpret_cast<BuildSmem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int r = static_cast<int>(cluster.block_rank());
  const int64_t bk = blockIdx.y;
  const int tid = threadIdx.x, q = tid >> 3, j = tid & 7;
  const int lane = tid & 31, warp = tid >> 5;
  const int32_t* src_pages = a.source + bk * 16;
  float* unit = reinterpret_cast<float*>(a.work + bk * kWorkBytes);
  const int pos = r * kSlice + q;
  // member ids index the workspace: kept in [0, 1024) by construction, masked
  // so that no value can address outside it
  constexpr int kIdMask = kBucket - 1;

  // ---- initialize (DS/kernels.py:9-29): unit vectors, lane-major, identity order
  {
    float x[16];
    if (!load_token_lane(a, src_pages, pos, j, x) && j == 0 && a.status) atomicExch(a.status, V1X_STATUS_BAD_PAGE);
    float ss = __fmul_rn(x[0], x[0]);
#pragma unroll
    for (int i = 1; i < 16; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    const float m = fmaxf(__fsqrt_rn(lanes8_sum(ss)), 1.0e-12f);
    float4* u = reinterpret_cast<float4*>(unit + static_cast<int64_t>(pos) * 128 + j * 16);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      u[c] = make_float4(__fdiv_rn(x[4 * c], m), __fdiv_rn(x[4 * c + 1], m), __fdiv_rn(x[4 * c + 2], m),
                         __fdiv_rn(x[4 * c + 3], m));
    if (j == 0) sm.pg[0][q] = pos;
  }
  cluster.sync();

  // ---- levels whose groups span CTAs: n = 1024, 512, 256.  Vectors come from the
  // L2 workspace; argmin partials, sort keys and the next order go straight into
  // the shared memory of the group's CTAs, behind cluster barriers.
  int cur = 0;
  for (int n = kBucket; n > kSlice; n >>= 1, cur ^= 1) {
    const int g0 = pos / n * n, c0 = g0 / kSlice, m = n / kSlice;  // the group's CTAs: c0 .. c0+m-1
    const int t = sm.pg[cur][q] & kIdMask;
    float x[16], y[16];
    load_row16(unit + static_cast<int64_t>(t) * 128 + j * 16, x);
    int anchor = *cluster.map_shared_rank(&sm.pg[cur][0], c0) & kIdMask;  // MODE 0: the group's first member
    float s1 = 0.0f;
    for (int mode = 0; mode < 3; ++mode) {
      load_row16(unit + static_cast<int64_t>(anchor) * 128 + j * 16, y);
      float s = dot_regs(x, y);
      if (mode == 2) {
        s = __fsub_rn(s, s1);
        if (j < m) *cluster.map_shared_rank(&sm.keys[pos - g0], c0 + j) = sort_key(s, pos - g0);
        break;
      }
      s1 = s;
      // argmin over the CTA's positions (all in one group), sent to the group's CTAs
      float v = s;
      int p = pos;
      int tk = t;
#pragma unroll
      for (int o = 8; o <= 16; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int op = __shfl_xor_sync(0xffffffffu, p, o);
        const int ot = __shfl_xor_sync(0xffffffffu, tk, o);
        if (argmin_better(ov, op, v, p)) {
          v = ov;
          p = op;
          tk = ot;
        }
      }
      if (lane == 0) {
        sm.wv[warp] = v;
        sm.wp[warp] = p;
        sm.wt[warp] = tk;
      }
      __syncthreads();
      if (warp == 0) {
        float gv = sm.wv[lane];
        int gp = sm.wp[lane], gt = sm.wt[lane];
        for (int o = 16; o >= 1; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
          const int op = __shfl_xor_sync(0xffffffffu, gp, o);
          const int ot = __shfl_xor_sync(0xffffffffu, gt, o);
          if (argmin_better(ov, op, gv, gp)) {
            gv = ov;
            gp = op;
            gt = ot;
          }
        }
        if (lane < m) *cluster.map_shared_rank(&sm.part[mode][r], c0 + lane) = make_int4(__float_as_int(gv), gp, gt, 0);
      }
      cluster.sync();
      int4 best = sm.part[mode][c0];
      for (int c = c0 + 1; c < c0 + m; ++c) {
        const int4 e = sm.part[mode][c];
        if (argmin_better(__int_as_float(e.x), e.y, __int_as_float(best.x), best.y)) best = e;
      }
      anchor = best.z & kIdMask;  // b after MODE 0, a after MODE 1
    }
    cluster.sync();  // the group's keys are complete in every CTA of the group
    // stable descending sort of the group's margins (NA/fused_grouping.py:64-76)
    const int rank = rank_in_group(sm.keys, n, sm.keys[pos - g0], j);
    const int dest = g0 + rank;
    if (j == 0) *cluster.map_shared_rank(&sm.pg[cur ^ 1][dest % kSlice], dest / kSlice) = t;
    cluster.sync();
  }

  // ---- levels inside one CTA: n = 128 .. 16.  The slice's member vectors are
  // copied into shared memory once; positions then hold xs rows.
  {
    const int t = sm.pg[cur][q] & kIdMask;
    float x[16];
    load_row16(unit + static_cast<int64_t>(t) * 128 + j * 16, x);
#pragma unroll
    for (int c = 0; c < 4; ++c)
      reinterpret_cast<float4*>(sm.xs[q])[c * 8 + j] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
    if (j == 0) {
      sm.tok[q] = t;
      sm.ploc[0][q] = q;
    }
  }
  __syncthreads();
  int lc = 0;
  for (int n = kSlice; n >= 16; n >>= 1, lc ^= 1) {
    const int g0 = q / n * n;
    const int row = sm.ploc[lc][q];
    float x[16], y[16];
    load_srow16(sm.xs[row], j, x);
    int anchor = sm.ploc[lc][g0];
    float s1 = 0.0f, s = 0.0f;
    for (int mode = 0; mode < 3; ++mode) {
      load_srow16(sm.xs[anchor], j, y);
      s = dot_regs(x, y);
      if (mode == 2) {
        s = __fsub_rn(s, s1);
        break;
      }
      s1 = s;
      anchor = sm.ploc[lc][cta_group_argmin(s, q, n, sm)];
    }
    if (j == 0) sm.keys[q] = sort_key(s, q - g0);
    __syncthreads();
    const int rank = rank_in_group(sm.keys + g0, n, sm.keys[q], j);
    if (j == 0) sm.ploc[lc ^ 1][g0 + rank] = row;
    __syncthreads();
  }
  if (j == 0) {
    const int member = sm.tok[sm.ploc[lc][q]];
    sm.pg[0][q] = member;
    if (a.perm) a.perm[bk * kBucket + pos] = member;
  }
  __syncthreads();

  // ---- assemble (DS/kernels.py:32-54)
  assemble_slice(a, src_pages, a.starts[bk], sm.pg[0], r, a.tmp + bk * 16 * kPageBytes,
                 a.centers + bk * 2 * kPageBytes, a.mapping + bk * kBucket, sm);
}

// ---------------------------------------------------------------------------
// The reference's single ops, for drop-in use and op-level parity.
// ---------------------------------------------------------------------------

// initialize (DS/kernels.py:9-29): natural [1024, 128] unit rows, PERM = 0..1023,
// FLAG = active ? -1 : 0.  Thread = (token, lane of 8).
__global__ void __launch_bounds__(256) initialize_kernel(const uint8_t* __restrict__ native, int64_t native_pages,
                                                         const int32_t* __restrict__ table,
                                                         const int32_t* __restrict__ meta, float* __restrict__ unit,
                                                         int32_t* __restrict__ perm, int32_t* __restrict__ flag,
                                                         int32_t* status) {
  const int active = meta[2];
  if (blockIdx.x == 0 && threadIdx.x == 0) *flag = active != 0 ? -1 : 0;
  if (!active) return;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 3, j = threadIdx.x & 7;
  BuildArgs a{};
  a.native = native;
  a.native_pages = native_pages;
  float x[16];
  if (!load_token_lane(a, table, t, j, x) && j == 0 && status) atomicExch(status, V1X_STATUS_BAD_PAGE);
  float ss = __fmul_rn(x[0], x[0]);
#pragma unroll
  for (int i = 1; i < 16; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  const float m = fmaxf(__fsqrt_rn(lanes8_sum(ss)), 1.0e-12f);
#pragma unroll
  for (int i = 0; i < 16; ++i) unit[static_cast<int64_t>(t) * 128 + 8 * i + j] = __fdiv_rn(x[i], m);
  if (j == 0) perm[t] = t;
}

// _init (NA/fused_grouping.py:27-37): U[h*4096 + i] = normalize(K[REQ[START+i], h])
// for the 4096 positions of head h, P[h*4096 + i] = START + i.  kind 0 = bf16 K, 1 = f32.
__global__ void __launch_bounds__(256) group_init_kernel(const void* __restrict__ k, int kind,
                                                         const int32_t* __restrict__ req, float* __restrict__ u,
                                                         int32_t* __restrict__ p, const int32_t* __restrict__ flag,
                                                         int64_t start, int64_t ks0, int64_t ks1) {
  if (*flag >= 0) return;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 3, j = threadIdx.x & 7;
  const int64_t h = blockIdx.y;
  const int64_t slot = req[start + i];
  float x[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int64_t off = slot * ks0 + h * ks1 + 8 * e + j;
    x[e] = kind == 0 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(k)[off])
                     : reinterpret_cast<const float*>(k)[off];
  }
  float ss = __fmul_rn(x[0], x[0]);
#pragma unroll
  for (int e = 1; e < 16; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
  const float m = fmaxf(__fsqrt_rn(lanes8_sum(ss)), 1.0e-12f);
#pragma unroll
  for (int e = 0; e < 16; ++e) u[(h * 4096 + i) * 128 + 8 * e + j] = __fdiv_rn(x[e], m);
  if (j == 0) p[h * 4096 + i] = static_cast<int32_t>(start + i);
}

// _dots (NA/fused_grouping.py:39-54), natural [heads, 4096, 128] unit rows.
__global__ void __launch_bounds__(256) group_dots_kernel(const float* __restrict__ u, const int32_t* __restrict__ p,
                                                         const int32_t* __restrict__ anc, float* __restrict__ s,
                                                         const int32_t* __restrict__ flag, int n, int64_t start,
                                                         int mode, int count) {
  if (*flag >= 0) return;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 3, j = threadIdx.x & 7;
  if (i >= count) return;  // whole 8-lane groups leave together
  const int64_t h = blockIdx.y;
  const int group = i / n;
  const int64_t id = p[h * 4096 + i] - start;
  const int64_t an = (mode == 0 ? p[h * 4096 + static_cast<int64_t>(group) * n] : anc[(h * 256 + group) * 2 + (mode - 1)]) - start;
  const float* x = u + (h * 4096 + id) * 128;
  const float* y = u + (h * 4096 + an) * 128;
  float r = __fmul_rn(x[j], y[j]);
#pragma unroll
  for (int e = 1; e < 16; ++e) r = __fadd_rn(r, __fmul_rn(x[8 * e + j], y[8 * e + j]));
  r = lanes8_sum(r);
  if (j == 0) s[h * 4096 + i] = mode == 2 ? __fsub_rn(r, s[h * 4096 + i]) : r;
}

// _anchor (NA/fused_grouping.py:56-63): one CTA per (group, head).
__global__ void __launch_bounds__(256) group_anchor_kernel(const int32_t* __restrict__ p, int32_t* __restrict__ anc,
                                                           const float* __restrict__ s,
                                                           const int32_t* __restrict__ flag, int n, int slot) {
  if (*flag >= 0) return;
  __shared__ float wv[8];
  __shared__ int wp[8];
  const int64_t h = blockIdx.y, g = blockIdx.x;
  const float* row = s + h * 4096 + g * n;
  float v = 0.0f;
  int pidx = -1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = row[i];
    if (pidx < 0 || argmin_better(x, i, v, pidx)) {
      v = x;
      pidx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int op = __shfl_xor_sync(0xffffffffu, pidx, o);
    if (op >= 0 && (pidx < 0 || argmin_better(ov, op, v, pidx))) {
      v = ov;
      pidx = op;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    wv[threadIdx.x >> 5] = v;
    wp[threadIdx.x >> 5] = pidx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (wp[w] >= 0 && (pidx < 0 || argmin_better(wv[w], wp[w], v, pidx))) {
        v = wv[w];
        pidx = wp[w];
      }
    anc[(h * 256 + g) * 2 + slot] = p[h * 4096 + g * n + pidx];
  }
}

// assemble (DS/kernels.py:32-54) of one bucket: one CTA per pair of pages.
__global__ void __launch_bounds__(kBuildThreads) assemble_kernel(const __grid_constant__ BuildArgs a,
                                                                 const int32_t* __restrict__ meta,
                                                                 const int32_t* __restrict__ ids) {
  if (!meta[2]) return;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BuildSmem& sm = *reinterpret_cast<BuildSmem*>(smem_raw);
  const int r = blockIdx.x;
  if (threadIdx.x < kSlice) sm.ploc[0][threadIdx.x] = ids[r * kSlice + threadIdx.x];
  __syncthreads();
  assemble_slice(a, a.source, meta[0], sm.ploc[0], r, a.tmp, a.centers, a.mapping, sm);
}

void set_smem_attr(const void* fn) {
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(BuildSmem)));
}

}  // namespace
}  // namespace v1x

extern "C" int64_t v1x_build_workspace_bytes(int64_t buckets) { return buckets < 0 ? 0 : buckets * v1x::kWorkBytes; }

extern "C" int v1x_build_buckets(const uint8_t* native, int64_t native_pages, const int32_t* source,
                                 const int32_t* starts, uint8_t* tmp, uint8_t* centers, int32_t* mapping,
                                 int32_t* perm, void* work, int32_t* status, int64_t buckets, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(buckets >= 0 && buckets <= 65535, "build_buckets: buckets must be in [0, 65535]");
  V1X_CHECK_ARG(native_pages > 0, "build_buckets: empty native pool");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(native) & 15) == 0 && (reinterpret_cast<uintptr_t>(tmp) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(work) & 15) == 0,
                "build_buckets: native, tmp and work must be 16-byte aligned");
  if (buckets == 0) return V1X_OK;
  static DeviceOnce once;
  once.run([] { set_smem_attr(reinterpret_cast<const void*>(build_bucket_kernel)); });
  BuildArgs a{native, native_pages, source, starts, tmp, centers, mapping, perm, static_cast<uint8_t*>(work), status};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kBuildCtas, static_cast<unsigned>(buckets));
  cfg.blockDim = dim3(kBuildThreads);
  cfg.dynamicSmemBytes = sizeof(BuildSmem);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = greatest_priority();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, build_bucket_kernel, a);
  return launch_status("v1x_build_buckets");
}

// ---------------------------------------------------------------------------
// No-allocation entry point: the same build with its workspace in a fixed
// array inside the library instead of a caller-supplied buffer.
// ---------------------------------------------------------------------------
namespace v1x {
namespace {
constexpr int kNoAllocBuckets = 8;  // 8 x 512 KB = 4 MB of device memory
}  // namespace
static __device__ __align__(256) uint8_t g_build_scratch[kNoAllocBuckets * kWorkBytes];
}  // namespace v1x

extern "C" int v1x_build_buckets_noalloc(const uint8_t* native, int64_t native_pages, const int32_t* source,
                                         const int32_t* starts, uint8_t* tmp, uint8_t* centers, int32_t* mapping,
                                         int32_t* perm, int32_t* status, int64_t buckets, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(buckets >= 0 && buckets <= kNoAllocBuckets,
                "build_buckets_noalloc: at most %d buckets per call (got %lld); split the call, or use "
                "v1x_build_buckets with a caller-supplied workspace",
                kNoAllocBuckets, (long long)buckets);
  V1X_CHECK_ARG(native_pages > 0, "build_buckets_noalloc: empty native pool");
  V1X_CHECK_ARG((reinterpret_cast<uintptr_t>(native) & 15) == 0 && (reinterpret_cast<uintptr_t>(tmp) & 15) == 0,
                "build_buckets_noalloc: native and tmp must be 16-byte aligned");
  if (buckets == 0) return V1X_OK;
  // The scratch array's address on the current device, looked up once per
  // device with that device current.  Host code may not pass the array's name
  // to a kernel: on the host it names a stand-in, not device memory.  The
  // per-device slots are atomics, so first calls from several host threads do
  // not race; a failed lookup leaves the slot empty and is retried next call.
  static std::atomic<void*> scratch[DeviceOnce::kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= DeviceOnce::kMaxDevices) {
    set_error("build_buckets_noalloc: no current device (%s)", cudaGetErrorString(e));
    return V1X_ERR_CUDA;
  }
  void* work = scratch[dev].load(std::memory_order_acquire);
  if (work == nullptr) {
    e = cudaGetSymbolAddress(&work, g_build_scratch);
    if (e != cudaSuccess || work == nullptr) {
      set_error("build_buckets_noalloc: scratch lookup failed (%s)", cudaGetErrorString(e));
      return V1X_ERR_CUDA;
    }
    scratch[dev].store(work, std::memory_order_release);  // every thread finds the same address
  }
  static DeviceOnce once;
  once.run([] { set_smem_attr(reinterpret_cast<const void*>(build_bucket_kernel)); });
  BuildArgs a{native, native_pages, source, starts, tmp, centers, mapping, perm, static_cast<uint8_t*>(work),
              status};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kBuildCtas, static_cast<unsigned>(buckets));
  cfg.blockDim = dim3(kBuildThreads);
  cfg.dynamicSmemBytes = sizeof(BuildSmem);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributePriority;
  attr[0].val.priority = greatest_priority();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, build_bucket_kernel, a);
  return launch_status("v1x_build_buckets_noalloc");
}

extern "C" int v1x_initialize(const uint8_t* native, int64_t native_pages, const int32_t* table,
                              const int32_t* meta, float* unit, int32_t* perm, int32_t* flag, int32_t* status,
                              void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(native_pages > 0 && (reinterpret_cast<uintptr_t>(native) & 15) == 0,
                "initialize: native pool must be non-empty and 16-byte aligned");
  initialize_kernel<<<kBucket * 8 / 256, 256, 0, as_stream(stream)>>>(native, native_pages, table, meta, unit, perm,
                                                                     flag, status);
  return launch_status("v1x_initialize");
}

extern "C" int v1x_group_init(const void* k, int k_is_f32, const int32_t* req, float* u, int32_t* p,
                              const int32_t* flag, int64_t start, int64_t ks0, int64_t ks1, int64_t heads,
                              void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(heads >= 1 && heads <= 65535 && start >= 0, "_init: bad heads / start");
  group_init_kernel<<<dim3(4096 * 8 / 256, static_cast<unsigned>(heads)), 256, 0, as_stream(stream)>>>(
      k, k_is_f32 ? 1 : 0, req, u, p, flag, start, ks0, ks1);
  return launch_status("v1x_group_init");
}

extern "C" int v1x_group_dots(const float* u, const int32_t* p, const int32_t* anchor, float* s,
                              const int32_t* flag, int64_t n, int64_t start, int mode, int64_t count,
                              int64_t heads, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(mode >= 0 && mode <= 2, "_dots: MODE must be 0, 1 or 2");
  V1X_CHECK_ARG(n >= 1 && count >= 4 && count <= 4096 && count % n == 0 && count % 4 == 0 && heads >= 1 &&
                    heads <= 65535,
                "_dots: bad group geometry");
  V1X_CHECK_ARG(count / n <= 256 || mode == 0, "_dots: at most 256 groups carry anchors");
  const unsigned blocks = static_cast<unsigned>((count * 8 + 255) / 256);
  group_dots_kernel<<<dim3(blocks, static_cast<unsigned>(heads)), 256, 0, as_stream(stream)>>>(
      u, p, anchor, s, flag, static_cast<int>(n), start, mode, static_cast<int>(count));
  return launch_status("v1x_group_dots");
}

extern "C" int v1x_group_anchor(const int32_t* p, int32_t* anchor, const float* s, const int32_t* flag, int64_t n,
                                int slot, int64_t count, int64_t heads, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(slot == 0 || slot == 1, "_anchor: SLOT must be 0 or 1");
  V1X_CHECK_ARG(n >= 1 && count >= n && count <= 4096 && count % n == 0 && count / n <= 256 && heads >= 1 &&
                    heads <= 65535,
                "_anchor: bad group geometry");
  group_anchor_kernel<<<dim3(static_cast<unsigned>(count / n), static_cast<unsigned>(heads)), 256, 0,
                        as_stream(stream)>>>(p, anchor, s, flag, static_cast<int>(n), slot);
  return launch_status("v1x_group_anchor");
}

extern "C" int v1x_assemble(const uint8_t* native, int64_t native_pages, const int32_t* table, const int32_t* meta,
                            const int32_t* ids, uint8_t* tmp, uint8_t* centers, int32_t* mapping, void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(native_pages > 0 && (reinterpret_cast<uintptr_t>(native) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(tmp) & 15) == 0,
                "assemble: native and tmp must be 16-byte aligned");
  static DeviceOnce once;
  once.run([] { set_smem_attr(reinterpret_cast<const void*>(assemble_kernel)); });
  BuildArgs a{native, native_pages, table, nullptr, tmp, centers, mapping, nullptr, nullptr, nullptr};
  assemble_kernel<<<kBucket / kSlice, kBuildThreads, sizeof(BuildSmem), as_stream(stream)>>>(a, meta, ids);
  return launch_status("v1x_assemble");
}
