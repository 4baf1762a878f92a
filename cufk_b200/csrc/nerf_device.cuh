// Device-side building blocks of the sm_100a NeRF chain kernels.
//
// Layout conventions used by every kernel in this library:
//   * one CTA reconstructs one chain; its W warps own consecutive runs of K steps per lane
//     (lane-major: thread t owns steps [t*K, t*K + K)), K odd so that the lanes' shared-memory
//     strides (3K words) hit 32 distinct banks;
//   * a chain's per-atom data lives in shared memory as "slots": atom a owns the three words
//     X[3a..3a+2].  Inputs are scattered into the slot of the atom they place (length L[i] ->
//     X[3(i+1)], angle A[i] -> X[3(i+2)+1], dihedral D[i] -> X[3(i+3)+2]), so that step s reads
//     its (L[s+2], A[s+1], D[s]) from slot s+3 and can overwrite it in place with its result:
//     the xyz of atom s+3 in the forward, the three parameter gradients in the backward.  The slot
//     array then has exactly the layout of the (N, 3) output row.
//
// Reference behaviour restated here (paths relative to the cufk project root):
//   * local transform R rows [(-c,-s,0), (sC,-cC,-S), (sS,-cS,C)], t = l R[:,0]
//     (src/cufk/csrc/affine.cuh:36-51), applied as P <- P Rx(phi) Mz(theta) which is the same
//     product written as two plane rotations;
//   * affine compose (R1,t1)(R2,t2) = (R1 R2, t1 + R1 t2) (affine.cuh:53-58);
//   * first frame (src/cufk/csrc/block.cu:113-148, frame_utils.cuh:17-31).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "nerf_math.cuh"

namespace cufkb {

constexpr int kWarp = 32;
constexpr int kMaxWarps = 8;

// ------------------------------------------------------------------------------------------
// element types: 16-bit storage computes in float, float in float, double in double
// ------------------------------------------------------------------------------------------
template <typename T>
struct ComputeOf {
  using type = float;
};
template <>
struct ComputeOf<double> {
  using type = double;
};

template <typename R, typename T>
__device__ __forceinline__ R to_r(T x) {
  if constexpr (std::is_same_v<T, __half>) {
    return static_cast<R>(__half2float(x));
  } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    return static_cast<R>(__bfloat162float(x));
  } else {
    return static_cast<R>(x);
  }
}

template <typename T, typename R>
__device__ __forceinline__ T from_r(R x) {
  if constexpr (std::is_same_v<T, __half>) {
    return __float2half_rn(static_cast<float>(x));
  } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    return __float2bfloat16_rn(static_cast<float>(x));
  } else {
    return static_cast<T>(x);
  }
}

// Angles of real chains take the short reduction of nerf_math.cuh; anything beyond its range (or
// NaN/inf) takes the CUDA library routine.  float64 always uses the library routine.
__device__ __forceinline__ void sin_cos(float x, float& s, float& c) {
  if (fabsf(x) <= kSinCosFastRange) {
    sincos_fast(x, s, c);
  } else {
    sincosf(x, &s, &c);
  }
}
__device__ __forceinline__ void sin_cos(double x, double& s, double& c) { sincos(x, &s, &c); }
__device__ __forceinline__ float sqrt_r(float x) { return sqrtf(x); }
__device__ __forceinline__ double sqrt_r(double x) { return sqrt(x); }
__device__ __forceinline__ float max_r(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double max_r(double a, double b) { return fmax(a, b); }
__device__ __forceinline__ float abs_r(float a) { return fabsf(a); }
__device__ __forceinline__ double abs_r(double a) { return fabs(a); }

// ------------------------------------------------------------------------------------------
// async copies (sm_80+ LDGSTS for scattered elements, sm_90+ bulk copy engine for stores)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int Bytes>
__device__ __forceinline__ void cp_async(void* smem_dst, const void* gmem_src) {
  static_assert(Bytes == 4 || Bytes == 8 || Bytes == 16);
  if constexpr (Bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "n"(Bytes)
                 : "memory");
  }
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// One bulk (TMA engine) store of a 16-byte aligned, 16-byte multiple range from shared memory.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gmem_dst), "r"(smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}

// Waits until every committed bulk store has finished READING shared memory (the CTA may then
// exit or reuse the buffer; the global writes complete on their own).
__device__ __forceinline__ void bulk_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }

// Copies a contiguous global range of `count` elements into shared memory so that the shared
// copy starts at `smem_base + (gaddr % 16)`: the 16-byte aligned interior moves in 16-byte
// LDGSTS chunks and the ragged ends element by element.  Returns the shared pointer of element 0.
template <typename T>
__device__ __forceinline__ T* stage_row_async(unsigned char* smem_base16, const T* gsrc, int count, int tid, int nthreads) {
  const uintptr_t g0 = reinterpret_cast<uintptr_t>(gsrc);
  T* dst = reinterpret_cast<T*>(smem_base16 + (g0 & 15u));
  const uintptr_t g1 = g0 + static_cast<uintptr_t>(count) * sizeof(T);
  const uintptr_t a0 = (g0 + 15u) & ~uintptr_t(15);
  const uintptr_t a1 = g1 & ~uintptr_t(15);
  if (a1 > a0) {
    const int head = static_cast<int>((a0 - g0) / sizeof(T));
    const int chunks = static_cast<int>((a1 - a0) / 16u);
    const int tail0 = static_cast<int>((a1 - g0) / sizeof(T));
    for (int c = tid; c < chunks; c += nthreads) {
      cp_async<16>(reinterpret_cast<unsigned char*>(dst + head) + 16 * c, reinterpret_cast<const unsigned char*>(a0) + 16 * c);
    }
    for (int i = tid; i < head; i += nthreads) dst[i] = gsrc[i];
    for (int i = tail0 + tid; i < count; i += nthreads) dst[i] = gsrc[i];
  } else {
    for (int i = tid; i < count; i += nthreads) dst[i] = gsrc[i];
  }
  return dst;
}

// Bytes of shared memory reserved for a row staged by stage_row_async.
__host__ __device__ constexpr size_t staged_row_bytes(size_t count, size_t elem) { return ((count * elem + 15) & ~size_t(15)) + 16; }

// Writes `count` elements of shared memory (laid out with the same address residue mod 16 as
// the destination) to global memory: one bulk store for the aligned interior, plain stores for the
// ragged ends.  Every thread of the CTA calls it after a barrier that follows the last shared
// write; `fence.proxy.async` orders those generic-proxy writes before the bulk engine reads them.
template <typename T>
__device__ __forceinline__ void store_row_bulk(T* gdst, const T* ssrc, int count, int tid, int nthreads) {
  const uintptr_t g0 = reinterpret_cast<uintptr_t>(gdst);
  const uintptr_t g1 = g0 + static_cast<uintptr_t>(count) * sizeof(T);
  const uintptr_t a0 = (g0 + 15u) & ~uintptr_t(15);
  const uintptr_t a1 = g1 & ~uintptr_t(15);
  if (a1 > a0) {
    const int head = static_cast<int>((a0 - g0) / sizeof(T));
    const int tail0 = static_cast<int>((a1 - g0) / sizeof(T));
    if (tid == 0) {
      bulk_store(reinterpret_cast<void*>(a0), ssrc + head, static_cast<uint32_t>(a1 - a0));
    }
    for (int i = tid; i < head; i += nthreads) gdst[i] = ssrc[i];
    for (int i = tail0 + tid; i < count; i += nthreads) gdst[i] = ssrc[i];
    if (tid == 0) bulk_store_wait_read();
  } else {
    for (int i = tid; i < count; i += nthreads) gdst[i] = ssrc[i];
  }
}

// ------------------------------------------------------------------------------------------
// affine frames in registers
// ------------------------------------------------------------------------------------------
template <typename R>
struct Affine {
  R m[9];  // row-major rotation
  R v[3];  // translation
};

template <typename R>
__device__ __forceinline__ Affine<R> affine_identity() {
  Affine<R> a;
#pragma unroll
  for (int i = 0; i < 9; ++i) a.m[i] = (i % 4 == 0) ? R(1) : R(0);
  a.v[0] = a.v[1] = a.v[2] = R(0);
  return a;
}

// (a.m, a.v)(b.m, b.v) = (a.m b.m, a.v + a.m b.v)
template <typename R>
__device__ __forceinline__ Affine<R> compose(const Affine<R>& a, const Affine<R>& b) {
  Affine<R> r;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      r.m[3 * i + j] = a.m[3 * i + 0] * b.m[0 + j] + a.m[3 * i + 1] * b.m[3 + j] + a.m[3 * i + 2] * b.m[6 + j];
    }
    r.v[i] = a.v[i] + a.m[3 * i + 0] * b.v[0] + a.m[3 * i + 1] * b.v[1] + a.m[3 * i + 2] * b.v[2];
  }
  return r;
}

// P <- P * L(l, theta, phi) with L = (Rx(phi) Mz(theta), l Rx(phi) Mz(theta) e_x):
//   Rx(phi) = [[1,0,0],[0,C,-S],[0,S,C]],  Mz(theta) = [[-c,-s,0],[s,-c,0],[0,0,1]].
// Their product is the reference's local rotation; the translation is l times the new first
// column, so one step costs 27 multiply-adds.
template <typename R>
__device__ __forceinline__ void advance(Affine<R>& P, R l, R s, R c, R S, R C) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const R c0 = P.m[3 * r + 0];
    const R c1 = P.m[3 * r + 1];
    const R c2 = P.m[3 * r + 2];
    const R y = C * c1 + S * c2;
    const R z = C * c2 - S * c1;
    const R x0 = s * y - c * c0;
    const R y0 = -(s * c0 + c * y);
    P.m[3 * r + 0] = x0;
    P.m[3 * r + 1] = y0;
    P.m[3 * r + 2] = z;
    P.v[r] += l * x0;
  }
}

template <typename R>
__device__ __forceinline__ R shfl_up_r(R x, int off) {
  return __shfl_up_sync(0xffffffffu, x, off);
}
template <typename R>
__device__ __forceinline__ R shfl_down_r(R x, int off) {
  return __shfl_down_sync(0xffffffffu, x, off);
}
template <typename R>
__device__ __forceinline__ R shfl_idx_r(R x, int src) {
  return __shfl_sync(0xffffffffu, x, src);
}

template <typename R>
__device__ __forceinline__ Affine<R> shfl_up_affine(const Affine<R>& a, int off) {
  Affine<R> r;
#pragma unroll
  for (int i = 0; i < 9; ++i) r.m[i] = shfl_up_r(a.m[i], off);
#pragma unroll
  for (int i = 0; i < 3; ++i) r.v[i] = shfl_up_r(a.v[i], off);
  return r;
}

// Exclusive prefix (product of the totals of all lower threads of the CTA) of each thread's
// affine total.  Warp level: Kogge-Stone over lanes; CTA level: warp totals through shared memory.
template <typename R>
__device__ __forceinline__ Affine<R> cta_exclusive_affine(const Affine<R>& total, Affine<R>* warp_totals, int nwarps) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  Affine<R> x = total;
#pragma unroll
  for (int off = 1; off < kWarp; off <<= 1) {
    const Affine<R> y = shfl_up_affine(x, off);
    if (lane >= off) x = compose(y, x);
  }
  Affine<R> excl = shfl_up_affine(x, 1);
  if (lane == 0) excl = affine_identity<R>();
  if (nwarps > 1) {
    if (lane == kWarp - 1) warp_totals[warp] = x;
    __syncthreads();
    if (warp > 0) {
      Affine<R> carry = warp_totals[0];
      for (int w = 1; w < warp; ++w) carry = compose(carry, warp_totals[w]);
      excl = compose(carry, excl);
    }
  }
  return excl;
}

// Exclusive suffix sum over the CTA's threads of an N-word additive payload (sum over all higher
// threads), warp level with shfl_down, CTA level through shared memory.
template <typename R, int Words>
__device__ __forceinline__ void cta_exclusive_suffix(const R (&val)[Words], R (&out)[Words], R* warp_sums, int nwarps) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  R x[Words];
#pragma unroll
  for (int i = 0; i < Words; ++i) x[i] = val[i];
#pragma unroll
  for (int off = 1; off < kWarp; off <<= 1) {
#pragma unroll
    for (int i = 0; i < Words; ++i) {
      const R y = shfl_down_r(x[i], off);
      if (lane + off < kWarp) x[i] += y;
    }
  }
#pragma unroll
  for (int i = 0; i < Words; ++i) {
    const R y = shfl_down_r(x[i], 1);
    out[i] = (lane == kWarp - 1) ? R(0) : y;
  }
  if (nwarps > 1) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < Words; ++i) warp_sums[warp * Words + i] = x[i];
    }
    __syncthreads();
    for (int w = warp + 1; w < nwarps; ++w) {
#pragma unroll
      for (int i = 0; i < Words; ++i) out[i] += warp_sums[w * Words + i];
    }
  }
}

// Sum over the CTA of one value per thread; the result is valid in thread 0.
template <typename R>
__device__ __forceinline__ R cta_sum_to_thread0(R x, R* warp_sums, int nwarps) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  if (nwarps > 1) {
    const int lane = threadIdx.x & (kWarp - 1);
    const int warp = threadIdx.x / kWarp;
    if (lane == 0) warp_sums[warp] = x;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < nwarps; ++w) x += warp_sums[w];
    }
  }
  return x;
}

// ------------------------------------------------------------------------------------------
// first frame of a chain (block.cu:113-148), computed in R by every thread
// ------------------------------------------------------------------------------------------
template <typename R>
struct FirstFrame {
  R p0[3], p1[3], p2[3];
  R dir0[3], turn0[3], dir1[3], normal[3];
  R F[9];  // row-major; columns are dir1, side = normal x dir1, normal
  R s0, c0;
};

template <typename R>
__device__ __forceinline__ R dot3(const R* a, const R* b) {
  return a[0] * b[0] + a[1] * b[1] + a[2] * b[2];
}

template <typename R>
__device__ __forceinline__ void cross3(const R* a, const R* b, R* out) {
  const R x = a[1] * b[2] - a[2] * b[1];
  const R y = a[2] * b[0] - a[0] * b[2];
  const R z = a[0] * b[1] - a[1] * b[0];
  out[0] = x;
  out[1] = y;
  out[2] = z;
}

// v / sqrt(max(|v|^2, eps)), eps = the float literal 1e-12f (frame_utils.cuh:7, 17-20)
template <typename R>
__device__ __forceinline__ void normalize3(R* v) {
  const R n2 = dot3(v, v);
  const R inv = R(1) / sqrt_r(max_r(n2, static_cast<R>(1.0e-12f)));
  v[0] *= inv;
  v[1] *= inv;
  v[2] *= inv;
}

template <typename R, typename T>
__device__ __forceinline__ void load_anchor(const T* p, R d0, R d1, R d2, R* out) {
  if (p == nullptr) {
    out[0] = d0;
    out[1] = d1;
    out[2] = d2;
  } else {
    out[0] = to_r<R>(p[0]);
    out[1] = to_r<R>(p[1]);
    out[2] = to_r<R>(p[2]);
  }
}

// Anchors may be null: the reference's defaults (0,0,0), (1,0,0), (0,0,1) (reconstruct.py:69-71).
template <typename R, typename T>
__device__ __forceinline__ FirstFrame<R> first_frame(R l0, R l1, R a0, const T* p0, const T* first_direction, const T* initial_normal) {
  FirstFrame<R> f;
  load_anchor<R>(p0, R(0), R(0), R(0), f.p0);
  load_anchor<R>(first_direction, R(1), R(0), R(0), f.dir0);
  normalize3(f.dir0);
#pragma unroll
  for (int i = 0; i < 3; ++i) f.p1[i] = f.p0[i] + l0 * f.dir0[i];
  R n0[3];
  load_anchor<R>(initial_normal, R(0), R(0), R(1), n0);
  const R proj = dot3(n0, f.dir0);
#pragma unroll
  for (int i = 0; i < 3; ++i) n0[i] -= proj * f.dir0[i];
  if (dot3(n0, n0) < static_cast<R>(1.0e-12f)) {
    // stable_perpendicular (frame_utils.cuh:22-31)
    R helper[3] = {R(1), R(0), R(0)};
    if (abs_r(f.dir0[0]) >= static_cast<R>(0.9)) {
      helper[0] = R(0);
      helper[1] = R(1);
    }
    cross3(f.dir0, helper, n0);
    normalize3(n0);
  } else {
    normalize3(n0);
  }
  cross3(n0, f.dir0, f.turn0);
  normalize3(f.turn0);
  sin_cos(a0, f.s0, f.c0);
#pragma unroll
  for (int i = 0; i < 3; ++i) f.dir1[i] = -f.c0 * f.dir0[i] + f.s0 * f.turn0[i];
#pragma unroll
  for (int i = 0; i < 3; ++i) f.p2[i] = f.p1[i] + l1 * f.dir1[i];
  cross3(f.dir0, f.dir1, f.normal);
  normalize3(f.normal);
  R side[3];
  cross3(f.normal, f.dir1, side);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    f.F[3 * i + 0] = f.dir1[i];
    f.F[3 * i + 1] = side[i];
    f.F[3 * i + 2] = f.normal[i];
  }
  return f;
}

// ------------------------------------------------------------------------------------------
// launch geometry shared by host and device
// ------------------------------------------------------------------------------------------
struct ChainGeometry {
  int points;  // N
  int steps;   // N - 3
  int items;   // K: steps per thread (odd)
};

}  // namespace cufkb
