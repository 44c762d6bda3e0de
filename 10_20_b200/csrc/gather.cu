// _gather_slots for sm_100a: copy the selected K/V slot rows into contiguous
// workspace rows.
//
// Reference behaviour: sglang/srt/layers/attention/v1_native/kernels.py:62-77
// (kernel) and :102-111 (GatherWorkspace.gather).  Output row t = (q, j) gets
// K[REQ[ids[q, j]], HEAD, :] (and V), or zeros when the id is negative.  The
// reference fixes D = 128; any D is accepted here (D = 576 for the MLA latent).
//
// Design: a pure HBM copy.  Rows of 72 or 16 16-byte chunks (the 576-wide
// latent, 128-wide heads) take gather_rows_kernel (a warp per group of rows,
// chunk counts known at compile time); other 16-byte-aligned rows take the
// general vector path (consecutive threads own consecutive chunks of the flat
// output, 4 loads in flight per thread); anything else the scalar path.  Loads
// bypass L1 and stores are marked evict-first so the streamed output does not
// flush the slot index out of L2.
#include "common.cuh"

namespace v1x {
namespace {

struct GatherArgs {
  const unsigned char* k;
  const unsigned char* v;
  const int32_t* req;
  const int32_t* ids;
  unsigned char* kg;
  unsigned char* vg;
  int64_t rows, top, head, ks0, ks1, ks2, vs0, vs1, vs2, ids_stride, dim, elem;
};

__device__ __forceinline__ int64_t slot_of(const GatherArgs& a, int64_t t) {
  const int64_t q = t / a.top, j = t - q * a.top;
  const int32_t id = a.ids[q * a.ids_stride + j];
  if (id < 0) return -1;
  return a.req ? static_cast<int64_t>(a.req[id]) : static_cast<int64_t>(id);
}

constexpr int kUnroll = 4;

template <bool kHasV>
__global__ void __launch_bounds__(256) gather_vec_kernel(const __grid_constant__ GatherArgs a) {
  const int64_t cpr = a.dim * a.elem / 16;  // 16-byte chunks per row
  const int64_t total = a.rows * a.top * cpr;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t kb = a.head * a.ks1 * a.elem, vb = a.head * a.vs1 * a.elem;
  for (int64_t c0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c0 < total;
       c0 += stride * kUnroll) {
    uint4 kv[kUnroll], vv[kUnroll];
    int64_t cc[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t c = c0 + u * stride;
      cc[u] = c;
      kv[u] = make_uint4(0, 0, 0, 0);
      vv[u] = make_uint4(0, 0, 0, 0);
      if (c < total) {
        const int64_t t = c / cpr, part = c - t * cpr;
        const int64_t s = slot_of(a, t);
        if (s >= 0) {
          kv[u] = __ldcs(reinterpret_cast<const uint4*>(a.k + s * a.ks0 * a.elem + kb) + part);
          if (kHasV) vv[u] = __ldcs(reinterpret_cast<const uint4*>(a.v + s * a.vs0 * a.elem + vb) + part);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (cc[u] < total) {
        __stcs(reinterpret_cast<uint4*>(a.kg) + cc[u], kv[u]);
        if (kHasV) __stcs(reinterpret_cast<uint4*>(a.vg) + cc[u], vv[u]);
      }
    }
  }
}

// Rows of a compile-time number of 16-byte chunks (kCpr: 72 for the 576-wide
// bf16 latent, 16 for 128-wide bf16 heads): a warp copies kR consecutive output
// rows at a time.  The row -> slot lookups are done once per row by kR lanes and
// broadcast with shuffles, the (row, chunk) split of a lane's flat index is a
// division by a constant, and every lane keeps kPer 16-byte loads in flight
// (kCpr * kR is a multiple of 32, so no lane idles).  Per chunk this is a handful
// of instructions -- the general path above spends a 64-bit division per chunk,
// which at ~37M chunks per decode step is as long as the copy itself.
// Single-output gathers (K only, the MMA latent) are capped at 64 registers so
// that four 256-thread CTAs fit an SM: 32 warps of 9 loads in flight instead of
// 24 (89% -> 93% of HBM on the 1024 x 2048-slot gather); with V as well the
// cap would spill, so those keep the default.
template <int kCpr, int kR, bool kHasV>
__global__ void __launch_bounds__(256, kHasV ? 1 : 4) gather_rows_kernel(const __grid_constant__ GatherArgs a) {
  static_assert((kCpr * kR) % 32 == 0, "a row group must fill the warp's lanes");
  constexpr int kPer = kCpr * kR / 32;
  const int lane = threadIdx.x & 31;
  const int64_t nrows = a.rows * a.top;
  const int64_t ngroups = (nrows + kR - 1) / kR;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const unsigned char* kbase = a.k + a.head * a.ks1 * a.elem;
  const unsigned char* vbase = kHasV ? a.v + a.head * a.vs1 * a.elem : nullptr;
  const int64_t krow = a.ks0 * a.elem, vrow = kHasV ? a.vs0 * a.elem : 0;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < ngroups;
       g += nwarps) {
    const int64_t t0 = g * kR;
    int64_t my_slot = -1;
    if (lane < kR && t0 + lane < nrows) my_slot = slot_of(a, t0 + lane);
    uint4 kv[kPer], vv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int f = lane + 32 * i;
      const int r = f / kCpr, c = f - r * kCpr;
      const int64_t s = __shfl_sync(0xffffffffu, my_slot, r);
      kv[i] = make_uint4(0, 0, 0, 0);
      if (kHasV) vv[i] = make_uint4(0, 0, 0, 0);
      if (s >= 0) {
        kv[i] = __ldcs(reinterpret_cast<const uint4*>(kbase + s * krow) + c);
        if (kHasV) vv[i] = __ldcs(reinterpret_cast<const uint4*>(vbase + s * vrow) + c);
      }
    }
    // output rows are contiguous: the group's chunks are one coalesced span
    uint4* ko = reinterpret_cast<uint4*>(a.kg) + t0 * kCpr;
    uint4* vo = kHasV ? reinterpret_cast<uint4*>(a.vg) + t0 * kCpr : nullptr;
    const int64_t limit = (nrows - t0) * kCpr;  // chunks left in the output
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int f = lane + 32 * i;
      if (f < limit) {
        __stcs(ko + f, kv[i]);
        if (kHasV) __stcs(vo + f, vv[i]);
      }
    }
  }
}

template <typename T>
__global__ void gather_scalar_kernel(const __grid_constant__ GatherArgs a) {
  const int64_t total = a.rows * a.top * a.dim;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const T* k = reinterpret_cast<const T*>(a.k);
  const T* v = reinterpret_cast<const T*>(a.v);
  T* kg = reinterpret_cast<T*>(a.kg);
  T* vg = reinterpret_cast<T*>(a.vg);
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += stride) {
    const int64_t t = e / a.dim, d = e - t * a.dim;
    const int64_t s = slot_of(a, t);
    T x = T(0), y = T(0);
    if (s >= 0) {
      x = k[s * a.ks0 + a.head * a.ks1 + d * a.ks2];
      if (v) y = v[s * a.vs0 + a.head * a.vs1 + d * a.vs2];
    }
    kg[e] = x;
    if (vg) vg[e] = y;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace v1x

extern "C" int v1x_gather_slots(const void* k, const void* v, const int32_t* req, const int32_t* ids,
                                void* kg, void* vg, int64_t rows, int64_t top, int64_t head,
                                int64_t ks0, int64_t ks1, int64_t ks2, int64_t vs0, int64_t vs1,
                                int64_t vs2, int64_t ids_stride, int64_t dim, int64_t elem_bytes,
                                void* stream) {
  using namespace v1x;
  clear_error();
  V1X_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4, "gather: element size 1, 2 or 4");
  V1X_CHECK_ARG(rows >= 0 && top >= 0 && dim > 0 && head >= 0, "gather: bad geometry");
  V1X_CHECK_ARG((v == nullptr) == (vg == nullptr), "gather: v and vg must both be given or both NULL");
  if (rows == 0 || top == 0) return V1X_OK;
  GatherArgs a{static_cast<const unsigned char*>(k), static_cast<const unsigned char*>(v), req, ids,
               static_cast<unsigned char*>(kg), static_cast<unsigned char*>(vg), rows, top, head, ks0,
               ks1, ks2, vs0, vs1, vs2, ids_stride, dim, elem_bytes};
  const bool hv = v != nullptr;
  bool vec = ks2 == 1 && (dim * elem_bytes) % 16 == 0 && (ks0 * elem_bytes) % 16 == 0 &&
             (ks1 * elem_bytes) % 16 == 0 && al16(k) && al16(kg);
  if (hv) vec = vec && vs2 == 1 && (vs0 * elem_bytes) % 16 == 0 && (vs1 * elem_bytes) % 16 == 0 && al16(v) && al16(vg);
  cudaStream_t s = as_stream(stream);
  const int64_t sms = num_sms();
  const int64_t cpr = vec ? dim * elem_bytes / 16 : 0;
  if (vec && (cpr == 72 || cpr == 16)) {
    const int64_t groups = (rows * top + (cpr == 72 ? 4 : 8) - 1) / (cpr == 72 ? 4 : 8);
    int64_t blocks = (groups + 7) / 8;
    blocks = blocks < sms * 16 ? blocks : sms * 16;
    const dim3 grid(static_cast<unsigned>(blocks)), block(256);
    if (cpr == 72) {
      if (hv) launch_kernel_prio(LaunchPriority::kDefault, gather_rows_kernel<72, 4, true>, grid, block, 0, s, a);
      else launch_kernel_prio(LaunchPriority::kDefault, gather_rows_kernel<72, 4, false>, grid, block, 0, s, a);
    } else {
      if (hv) launch_kernel_prio(LaunchPriority::kDefault, gather_rows_kernel<16, 8, true>, grid, block, 0, s, a);
      else launch_kernel_prio(LaunchPriority::kDefault, gather_rows_kernel<16, 8, false>, grid, block, 0, s, a);
    }
  } else if (vec) {
    const int64_t total = rows * top * dim * elem_bytes / 16;
    int64_t blocks = (total + 256 * kUnroll - 1) / (256 * kUnroll);
    blocks = blocks < sms * 16 ? blocks : sms * 16;
    if (hv) launch_kernel_prio(LaunchPriority::kDefault, gather_vec_kernel<true>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
    else launch_kernel_prio(LaunchPriority::kDefault, gather_vec_kernel<false>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
  } else {
    const int64_t total = rows * top * dim;
    int64_t blocks = (total + 255) / 256;
    blocks = blocks < sms * 32 ? blocks : sms * 32;
    if (elem_bytes == 1) launch_kernel_prio(LaunchPriority::kDefault, gather_scalar_kernel<uint8_t>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
    else if (elem_bytes == 2) launch_kernel_prio(LaunchPriority::kDefault, gather_scalar_kernel<uint16_t>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
    else launch_kernel_prio(LaunchPriority::kDefault, gather_scalar_kernel<uint32_t>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, a);
  }
  return launch_status("v1x_gather_slots");
}
