// Device-side building blocks of the sm_100a NeRF chain kernels.
//
// Layout conventions used by every kernel in this library:
//   * one CTA reconstructs one chain; its W warps own consecutive runs of K steps per lane
//     (thread t owns steps [t*K, t*K + K)), K odd so that the lanes' shared-memory strides (3K words)
//     hit 32 distinct banks;
//   * a chain's per-atom data lives in shared memory as "slots": atom a owns the three words
//     X[3a..3a+2].  Inputs are scattered into the slot of the atom they place (length L[i] ->
//     X[3(i+1)], angle A[i] -> X[3(i+2)+1], dihedral D[i] -> X[3(i+3)+2]), so that step s reads
//     its (L[s+2], A[s+1], D[s]) from slot s+3 and can overwrite it in place with its result:
//     the xyz of atom s+3 in the forward, the three parameter gradients in the backward.  The slot
//     array then has exactly the layout of the (N, 3) output row;
//   * arithmetic runs on the compute type V (float for 32- and 16-bit storage, double for float64)
//     through explicit multiply-adds; the two angles of a step share one packed sm_100 f32x2
//     evaluation of their sine/cosine polynomials.
//
// Reference behaviour restated here (paths relative to the cufk project root):
//   * local transform R rows [(-c,-s,0), (sC,-cC,-S), (sS,-cS,C)], t = l R[:,0]
//     (src/cufk/csrc/affine.cuh:36-51), applied as P <- P Rx(phi) Mz(theta), the same product
//     written as two plane rotations;
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

// ------------------------------------------------------------------------------------------
// arithmetic on the compute type V = float | double
// ------------------------------------------------------------------------------------------
template <typename V>
struct Lanes;
template <>
struct Lanes<float> {
  using S = float;
  static constexpr int kCount = 1;
};
template <>
struct Lanes<double> {
  using S = double;
  static constexpr int kCount = 1;
};

__device__ __forceinline__ float vfma(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ double vfma(double a, double b, double c) { return fma(a, b, c); }
__device__ __forceinline__ float vmul(float a, float b) { return a * b; }
__device__ __forceinline__ double vmul(double a, double b) { return a * b; }
__device__ __forceinline__ float vadd(float a, float b) { return a + b; }
__device__ __forceinline__ double vadd(double a, double b) { return a + b; }
__device__ __forceinline__ float vneg(float a) { return -a; }
__device__ __forceinline__ double vneg(double a) { return -a; }
// 1/sqrt(x): the CUDA math library's rsqrtf (float) and rsqrt (double)
__device__ __forceinline__ float vrsqrt(float a) { return rsqrtf(a); }
__device__ __forceinline__ double vrsqrt(double a) { return rsqrt(a); }
// a - b
__device__ __forceinline__ float vsub(float a, float b) { return a - b; }
__device__ __forceinline__ double vsub(double a, double b) { return a - b; }

template <typename V>
__device__ __forceinline__ V splat(typename Lanes<V>::S x) {
  return x;
}

// 1 / sqrt(max(n2, 1e-12f)) (the clamp of normalized, frame_utils.cuh:17-20)
template <typename V>
__device__ __forceinline__ V vrecip_sqrt_clamped(V n2) {
  return V(1) / sqrt(n2 > static_cast<V>(1.0e-12f) ? n2 : static_cast<V>(1.0e-12f));
}

// sine and cosine of an angle pair (one step: bond angle and dihedral).  Float angles of real chains
// take the packed short reduction of nerf_math.cuh; anything beyond its range (or NaN/inf) takes
// the CUDA library routine for that step.  float64 always uses the library routine.
__device__ __forceinline__ bool fast_range(float x) { return fabsf(x) <= kSinCosFastRange; }

// Kept out of line: the library routine's large-argument reduction would otherwise sit inside every
// unrolled step of the hot loops and crowd the instruction cache.
__device__ __noinline__ float4 step_sincos_library(float th, float ph) {
  float4 r;
  sincosf(th, &r.x, &r.y);
  sincosf(ph, &r.z, &r.w);
  return r;
}

__device__ __forceinline__ void step_sincos(float th, float ph, float& st, float& ct, float& sp, float& cp) {
  if (fast_range(th) && fast_range(ph)) {
    float2 s, c;
    sincos_fast2(make_float2(th, ph), s, c);
    st = s.x;
    ct = c.x;
    sp = s.y;
    cp = c.y;
  } else {
    const float4 r = step_sincos_library(th, ph);
    st = r.x;
    ct = r.y;
    sp = r.z;
    cp = r.w;
  }
}

__device__ __forceinline__ void step_sincos(double th, double ph, double& st, double& ct, double& sp, double& cp) {
  sincos(th, &st, &ct);
  sincos(ph, &sp, &cp);
}

// ------------------------------------------------------------------------------------------
// async copies (sm_80+ LDGSTS for scattered elements, sm_90+ bulk copy engine for stores)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

template <int Bytes>
__device__ __forceinline__ void cp_async(void* smem_dst, const void* gmem_src) {
  static_assert(Bytes == 4 || Bytes == 8 || Bytes == 16);
  if constexpr (Bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "n"(Bytes) : "memory");
  }
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
// Waits until at most `Pending` of this thread's committed cp.async groups are still in flight.
template <int Pending>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(Pending) : "memory");
}


// Programmatic dependent launch.  The library launches small grids so that they may be scheduled
// while the previous kernel in the stream is still running; each kernel calls this first, before any
// global-memory access: griddepcontrol.wait returns once the previous grid has completed and its
// writes are visible (the ordering of a plain launch; a no-op when the launch did not allow the
// overlap), and launch_dependents then lets the next kernel in the stream be scheduled once every
// CTA of this grid has started.  The saving is the launch latency between dependent kernels.
__device__ __forceinline__ void enter_after_previous_grid() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// One bulk (TMA engine) store of a 16-byte aligned, 16-byte multiple range from shared memory.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(gmem_dst), "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}

// Waits until every committed bulk store of this thread has finished READING shared memory (the
// CTA may then exit or reuse the buffer; the global writes complete on their own).
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
    unsigned char* d = reinterpret_cast<unsigned char*>(dst + head);
    const unsigned char* s = reinterpret_cast<const unsigned char*>(a0);
#pragma unroll 4
    for (int c = tid; c < chunks; c += nthreads) cp_async<16>(d + 16 * c, s + 16 * c);
    for (int i = tid; i < head; i += nthreads) dst[i] = gsrc[i];
    for (int i = tail0 + tid; i < count; i += nthreads) dst[i] = gsrc[i];
  } else {
    for (int i = tid; i < count; i += nthreads) dst[i] = gsrc[i];
  }
  return dst;
}

// Bytes of shared memory reserved for a row staged by stage_row_async.
__host__ __device__ constexpr size_t staged_row_bytes(size_t count, size_t elem) { return ((count * elem + 15) & ~size_t(15)) + 16; }

// Writes `count` elements of shared memory (laid out with the same address residue mod 16 as the
// destination) to global memory: one bulk store for the aligned interior, issued by `issuer`, plain
// stores for the ragged ends.  Every thread of the CTA calls it after a barrier that follows the last
// shared write; `fence.proxy.async` orders those generic-proxy writes before the bulk engine reads.
template <typename T>
__device__ __forceinline__ void store_row_bulk(T* gdst, const T* ssrc, int count, int tid, int nthreads, int issuer) {
  const uintptr_t g0 = reinterpret_cast<uintptr_t>(gdst);
  const uintptr_t g1 = g0 + static_cast<uintptr_t>(count) * sizeof(T);
  const uintptr_t a0 = (g0 + 15u) & ~uintptr_t(15);
  const uintptr_t a1 = g1 & ~uintptr_t(15);
  if (a1 > a0) {
    const int head = static_cast<int>((a0 - g0) / sizeof(T));
    const int tail0 = static_cast<int>((a1 - g0) / sizeof(T));
    if (tid == issuer) bulk_store(reinterpret_cast<void*>(a0), ssrc + head, static_cast<uint32_t>(a1 - a0));
    for (int i = tid; i < head; i += nthreads) gdst[i] = ssrc[i];
    for (int i = tail0 + tid; i < count; i += nthreads) gdst[i] = ssrc[i];
  } else {
    for (int i = tid; i < count; i += nthreads) gdst[i] = ssrc[i];
  }
}

// ------------------------------------------------------------------------------------------
// affine frames in registers
// ------------------------------------------------------------------------------------------
template <typename V>
struct Affine {
  V m[9];  // row-major rotation
  V v[3];  // translation
};

template <typename V>
__device__ __forceinline__ Affine<V> affine_identity() {
  using S = typename Lanes<V>::S;
  Affine<V> a;
#pragma unroll
  for (int i = 0; i < 9; ++i) a.m[i] = splat<V>((i % 4 == 0) ? S(1) : S(0));
  a.v[0] = a.v[1] = a.v[2] = splat<V>(S(0));
  return a;
}

// (a.m, a.v)(b.m, b.v) = (a.m b.m, a.v + a.m b.v)
template <typename V>
__device__ __forceinline__ Affine<V> compose(const Affine<V>& a, const Affine<V>& b) {
  Affine<V> r;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      r.m[3 * i + j] = vfma(a.m[3 * i + 2], b.m[6 + j], vfma(a.m[3 * i + 1], b.m[3 + j], vmul(a.m[3 * i + 0], b.m[0 + j])));
    }
    r.v[i] = vfma(a.m[3 * i + 2], b.v[2], vfma(a.m[3 * i + 1], b.v[1], vfma(a.m[3 * i + 0], b.v[0], a.v[i])));
  }
  return r;
}

// Precomputed per-step factors of the local transform: s, c of the bond angle and S, C of the
// dihedral, with the negations the multiply-adds below need.
template <typename V>
struct StepRot {
  V s, c, S, C, ns, nc, nS, l;
};

template <typename V>
__device__ __forceinline__ StepRot<V> step_rot(V l, V s, V c, V S, V C) {
  return {s, c, S, C, vneg(s), vneg(c), vneg(S), l};
}

// P <- P * L(l, theta, phi) with L = (Rx(phi) Mz(theta), l Rx(phi) Mz(theta) e_x):
//   Rx(phi) = [[1,0,0],[0,C,-S],[0,S,C]],  Mz(theta) = [[-c,-s,0],[s,-c,0],[0,0,1]].
// Their product is the reference's local rotation; the translation is l times the new first
// column, so one step costs 27 multiply-adds.
template <typename V>
__device__ __forceinline__ void advance(Affine<V>& P, const StepRot<V>& q) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const V c0 = P.m[3 * r + 0];
    const V c1 = P.m[3 * r + 1];
    const V c2 = P.m[3 * r + 2];
    const V y = vfma(q.S, c2, vmul(q.C, c1));       // C c1 + S c2
    const V z = vfma(q.nS, c1, vmul(q.C, c2));      // C c2 - S c1
    const V x0 = vfma(q.s, y, vmul(q.nc, c0));      // s y - c c0
    const V y0 = vfma(q.ns, c0, vmul(q.nc, y));     // -s c0 - c y
    P.m[3 * r + 0] = x0;
    P.m[3 * r + 1] = y0;
    P.m[3 * r + 2] = z;
    P.v[r] = vfma(q.l, x0, P.v[r]);
  }
}

__device__ __forceinline__ float shfl_up(float x, int off) { return __shfl_up_sync(0xffffffffu, x, off); }
__device__ __forceinline__ double shfl_up(double x, int off) { return __shfl_up_sync(0xffffffffu, x, off); }
__device__ __forceinline__ float shfl_down(float x, int off) { return __shfl_down_sync(0xffffffffu, x, off); }
__device__ __forceinline__ double shfl_down(double x, int off) { return __shfl_down_sync(0xffffffffu, x, off); }
__device__ __forceinline__ float shfl_xor(float x, int m) { return __shfl_xor_sync(0xffffffffu, x, m); }
__device__ __forceinline__ double shfl_xor(double x, int m) { return __shfl_xor_sync(0xffffffffu, x, m); }

template <typename V>
__device__ __forceinline__ Affine<V> shfl_up_affine(const Affine<V>& a, int off) {
  Affine<V> r;
#pragma unroll
  for (int i = 0; i < 9; ++i) r.m[i] = shfl_up(a.m[i], off);
#pragma unroll
  for (int i = 0; i < 3; ++i) r.v[i] = shfl_up(a.v[i], off);
  return r;
}

// Exclusive prefix (product of the totals of all lower threads of the CTA) of each thread's affine
// total.  Warp level: Kogge-Stone over lanes; CTA level: warp totals through shared memory.
template <typename V>
__device__ __forceinline__ Affine<V> cta_exclusive_affine(const Affine<V>& total, Affine<V>* warp_totals, int nwarps) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  Affine<V> x = total;
#pragma unroll
  for (int off = 1; off < kWarp; off <<= 1) {
    const Affine<V> y = shfl_up_affine(x, off);
    if (lane >= off) x = compose(y, x);
  }
  Affine<V> excl = shfl_up_affine(x, 1);
  if (lane == 0) excl = affine_identity<V>();
  if (nwarps > 1) {
    if (lane == kWarp - 1) warp_totals[warp] = x;
    __syncthreads();
    if (warp > 0) {
      Affine<V> carry = warp_totals[0];
      for (int w = 1; w < warp; ++w) carry = compose(carry, warp_totals[w]);
      excl = compose(carry, excl);
    }
  }
  return excl;
}

// Exclusive suffix sum over the CTA's threads of a `Words`-word additive payload (sum over all
// higher threads), warp level with shfl_down, CTA level through shared memory.
template <typename V, int Words>
__device__ __forceinline__ void cta_exclusive_suffix(const V (&val)[Words], V (&out)[Words], V* warp_sums, int nwarps) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  V x[Words];
#pragma unroll
  for (int i = 0; i < Words; ++i) x[i] = val[i];
#pragma unroll
  for (int off = 1; off < kWarp; off <<= 1) {
#pragma unroll
    for (int i = 0; i < Words; ++i) {
      const V y = shfl_down(x[i], off);
      if (lane + off < kWarp) x[i] = vadd(x[i], y);
    }
  }
#pragma unroll
  for (int i = 0; i < Words; ++i) {
    const V y = shfl_down(x[i], 1);
    out[i] = (lane == kWarp - 1) ? splat<V>(0) : y;
  }
  if (nwarps > 1) {
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < Words; ++i) warp_sums[warp * Words + i] = x[i];
    }
    __syncthreads();
    for (int w = warp + 1; w < nwarps; ++w) {
#pragma unroll
      for (int i = 0; i < Words; ++i) out[i] = vadd(out[i], warp_sums[w * Words + i]);
    }
  }
}

// Sum over the CTA of one value per thread; the result is valid in thread 0.
template <typename V>
__device__ __forceinline__ V cta_sum_to_thread0(V x, V* warp_sums, int nwarps) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) x = vadd(x, shfl_xor(x, off));
  if (nwarps > 1) {
    const int lane = threadIdx.x & (kWarp - 1);
    const int warp = threadIdx.x / kWarp;
    if (lane == 0) warp_sums[warp] = x;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < nwarps; ++w) x = vadd(x, warp_sums[w]);
    }
  }
  return x;
}

// ------------------------------------------------------------------------------------------
// vector helpers
// ------------------------------------------------------------------------------------------
template <typename V>
__device__ __forceinline__ V dot3(const V* a, const V* b) {
  return vfma(a[2], b[2], vfma(a[1], b[1], vmul(a[0], b[0])));
}

// a x b
template <typename V>
__device__ __forceinline__ void cross3(const V* a, const V* b, V* out) {
  const V x = vfma(a[1], b[2], vneg(vmul(a[2], b[1])));
  const V y = vfma(a[2], b[0], vneg(vmul(a[0], b[2])));
  const V z = vfma(a[0], b[1], vneg(vmul(a[1], b[0])));
  out[0] = x;
  out[1] = y;
  out[2] = z;
}

// ------------------------------------------------------------------------------------------
// first frame of a chain (block.cu:113-148)
// ------------------------------------------------------------------------------------------
// Anchor part, shared by every chain of a call: dir0 = normalized(first_direction) and
// turn0 = normalized(n0 x dir0) with n0 the initial normal made perpendicular to dir0 (or
// stable_perpendicular(dir0) when that vanishes, frame_utils.cuh:22-31).
template <typename S>
struct AnchorFrame {
  S p0[3], dir0[3], turn0[3];
};

template <typename S>
__device__ __forceinline__ void normalize3_s(S* v) {
  const S n2 = v[0] * v[0] + v[1] * v[1] + v[2] * v[2];
  const S inv = S(1) / sqrt(n2 > static_cast<S>(1.0e-12f) ? n2 : static_cast<S>(1.0e-12f));
  v[0] *= inv;
  v[1] *= inv;
  v[2] *= inv;
}

template <typename S>
__device__ __forceinline__ void cross3_s(const S* a, const S* b, S* out) {
  const S x = a[1] * b[2] - a[2] * b[1];
  const S y = a[2] * b[0] - a[0] * b[2];
  const S z = a[0] * b[1] - a[1] * b[0];
  out[0] = x;
  out[1] = y;
  out[2] = z;
}

// Anchors may be null: the reference's defaults (0,0,0), (1,0,0), (0,0,1) (reconstruct.py:69-71).
template <typename S, typename T>
__device__ __forceinline__ AnchorFrame<S> anchor_frame(const T* p0, const T* first_direction, const T* initial_normal) {
  AnchorFrame<S> a;
  if (p0 == nullptr && first_direction == nullptr && initial_normal == nullptr) {
    // the general computation below gives exactly these values for the default anchors
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      a.p0[i] = S(0);
      a.dir0[i] = S(i == 0);
      a.turn0[i] = S(i == 1);
    }
    return a;
  }
  S n0[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    a.p0[i] = p0 ? to_r<S>(p0[i]) : S(0);
    a.dir0[i] = first_direction ? to_r<S>(first_direction[i]) : S(i == 0);
    n0[i] = initial_normal ? to_r<S>(initial_normal[i]) : S(i == 2);
  }
  normalize3_s(a.dir0);
  const S proj = n0[0] * a.dir0[0] + n0[1] * a.dir0[1] + n0[2] * a.dir0[2];
#pragma unroll
  for (int i = 0; i < 3; ++i) n0[i] -= proj * a.dir0[i];
  if (n0[0] * n0[0] + n0[1] * n0[1] + n0[2] * n0[2] < static_cast<S>(1.0e-12f)) {
    S helper[3] = {S(1), S(0), S(0)};
    if ((a.dir0[0] < S(0) ? -a.dir0[0] : a.dir0[0]) >= static_cast<S>(0.9)) {
      helper[0] = S(0);
      helper[1] = S(1);
    }
    cross3_s(a.dir0, helper, n0);
  }
  normalize3_s(n0);
  cross3_s(n0, a.dir0, a.turn0);
  normalize3_s(a.turn0);
  return a;
}

// Chain part: p1, p2 and F = [dir1 | normal x dir1 | normal] (row-major).
template <typename V>
struct ChainFrame {
  V p1[3], p2[3], dir1[3], normal[3];
  V F[9];
  V s0, c0;
};

template <typename V>
__device__ __forceinline__ ChainFrame<V> chain_frame(const AnchorFrame<typename Lanes<V>::S>& a, V l0, V l1, V a0) {
  ChainFrame<V> f;
  V st, ct, sp, cp;
  step_sincos(a0, a0, st, ct, sp, cp);
  f.s0 = st;
  f.c0 = ct;
  V dir0[3], turn0[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    dir0[i] = splat<V>(a.dir0[i]);
    turn0[i] = splat<V>(a.turn0[i]);
    f.p1[i] = vfma(l0, dir0[i], splat<V>(a.p0[i]));
    f.dir1[i] = vfma(st, turn0[i], vmul(vneg(ct), dir0[i]));
  }
#pragma unroll
  for (int i = 0; i < 3; ++i) f.p2[i] = vfma(l1, f.dir1[i], f.p1[i]);
  cross3(dir0, f.dir1, f.normal);
  const V inv = vrecip_sqrt_clamped(dot3(f.normal, f.normal));
#pragma unroll
  for (int i = 0; i < 3; ++i) f.normal[i] = vmul(f.normal[i], inv);
  V side[3];
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
// A packed (ragged) batch: chain b's points are [offsets[b], offsets[b+1]) of the packed xyz of
// `total` points; offsets is null for a (B, N) batch.
struct PackedLayout {
  const int64_t* offsets = nullptr;
  int64_t total = 0;
};

struct ChainGeometry {
  int batch;   // B
  int points;  // N (a packed batch: the largest N of its chains)
  int steps;   // N - 3
  int items;   // K: steps per thread
  PackedLayout packed = {};
};

// Element offsets of one chain's rows in the (B, N-1), (B, N-2), (B, N-3) and (B, N, 3) arrays,
// or in their packed forms, where chain b with points [p, p + N_b) owns lengths [p - b, p - b +
// N_b - 1), angles [p - 2b, ...), dihedrals [p - 3b, ...) and xyz rows [p, p + N_b).
struct ChainRows {
  int points;  // N of this chain
  int64_t lengths, angles, dihedrals, xyz;
};

__host__ __device__ inline ChainRows rows_at(int64_t chain, int64_t first_point, int points) {
  return {points, first_point - chain, first_point - 2 * chain, first_point - 3 * chain, 3 * first_point};
}

// A packed chain gets points = 0 (the kernels leave it untouched) when its point count lies outside
// [4, geo.points] or when any of its four rows would reach outside its packed array: xyz
// [p, p + n) in [0, total), lengths [p - b, p - b + n - 1) in [0, total - B), angles
// [p - 2b, ...) in [0, total - 2B), dihedrals [p - 3b, ...) in [0, total - 3B).  So offsets that
// are not those of a packed layout cannot make a kernel read or write out of bounds.
// L2 prefetch (one request to the bulk-copy engine) of the 16-byte aligned interior of a global
// row.  A prefetch only warms L2, the GPU's point of coherence, so it is safe before the previous
// kernel has finished: a value that kernel writes afterwards is what the later loads see.
__device__ __forceinline__ void prefetch_row_l2(const void* p, size_t bytes) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15u) & ~uintptr_t(15);
  const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
  if (e > a) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(static_cast<uint32_t>(e - a)) : "memory");
}

__device__ __forceinline__ ChainRows chain_rows(const ChainGeometry& g, int64_t chain) {
  if (g.packed.offsets == nullptr) return rows_at(chain, chain * g.points, g.points);
  const int64_t p0 = g.packed.offsets[chain];
  const int64_t n = g.packed.offsets[chain + 1] - p0;
  const int64_t B = g.batch, total = g.packed.total;
  const bool inside = n >= 4 && n <= g.points && p0 - 3 * chain >= 0 && p0 + n <= total && p0 - chain + n - 1 <= total - B &&
                      p0 - 2 * chain + n - 2 <= total - 2 * B && p0 - 3 * chain + n - 3 <= total - 3 * B;
  return rows_at(chain, inside ? p0 : 0, inside ? static_cast<int>(n) : 0);
}

}  // namespace cufkb
