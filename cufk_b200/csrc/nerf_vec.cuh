// Vector-slot kernels of the block path:
//
//   block_forward_vec_kernel       <- src/cufk/csrc/block.cu:157-204  (xyz from lengths/angles/dihedrals;
//                                      float32, float64)
//   block_backward_xyz_vec_kernel     the gradients of block.cu:206-313 from the forward's xyz
//                                      (float32, float64)
//   block_backward_xyz32_kernel       the gradients of block.cu:206-313 for float16/bfloat16 from
//                                      the float32 positions block_forward_kernel writes beside xyz
//   torsion_backward_xyz_vec_kernel   the raw-pair gradients of torsion.cu:297-381 from the forward's
//                                      xyz (float32, float64)
//   torsion_backward_xyz32_kernel     the same for float16/bfloat16 from the torsion forward's float32
//                                      positions
//
// They compute what block_forward_kernel and block_backward_xyz_kernel compute, with fewer
// instructions per atom:
//   * a thread owns K consecutive atoms, K a multiple of G = 16 / sizeof(T) (4 float, 2 double), and
//     the atoms of every thread start on a 16-byte boundary of shared memory, so that each group of G
//     atom slots (3 G elements = 48 bytes) moves with three 16-byte shared loads or stores;
//   * the slot row keeps the residue mod 16 of the chain's row in global memory (the forward's
//     output row leaves in one bulk store), so the thread ranges are shifted by `delta` in [0, G)
//     atoms: thread u owns atoms [u K - delta, u K - delta + K).  Thread 0 then starts on 3 + delta
//     atoms that are not steps (atoms 0, 1, 2 and delta slots in front of the row), and the last
//     thread runs past atom N-1 into padding;
//   * those padding atoms are given inputs that cost no test in the loops.  Forward: zero inputs,
//     whose step (l = 0, theta = 0, phi = 0) is exactly the half turn diag(-1, -1, 1) about z, so
//     thread 0 reaches atom 3 with the exact frame diag(-1, -1, 1)^(3 + delta) and folds its inverse
//     (the same matrix) into its world carry.  Backward: positions on a right-angled zig-zag of the
//     adjacent bond length, with zero gradients, so the steps through them pass the accuracy tests
//     and, by telescoping, leave the running torque exactly where the first real step needs it;
//   * the forward folds the chain's base frame (F, p2) into thread 0's total before the affine scan,
//     so the exclusive prefix of every thread is already its world carry.
//
// One CTA holds C chains of W warps each (C > 1 only with W = 1, where a chain synchronises with
// __syncwarp alone).
#pragma once

#include "nerf_kernels.cuh"

namespace cufkb {

template <typename T>
struct VecSlots {
  static constexpr int kAtoms = 16 / static_cast<int>(sizeof(T));  // atoms per 48-byte group
  static constexpr int kElems = 3 * kAtoms;
};

// Bytes in front of a chain's slot row: up to 5 padding atoms (thread 0's shift plus the two atoms
// in front of it that the backward reads) of 12 (float) or 24 (double) bytes.
constexpr int kVecFrontPad = 80;

// Shared memory of one chain's slot row: front padding, the row residue, and N + K atoms (the last
// thread may own up to K - 1 atoms past N - 1).
__host__ __device__ inline size_t vec_row_bytes(int points, int items, size_t elem) {
  return kVecFrontPad + 16 + ((3 * elem * static_cast<size_t>(points + items) + 15) & ~size_t(15));
}

// Shift delta in [0, G) such that 3 sizeof(T) delta = residue (mod 16): then atom u K - delta of
// every thread starts on a 16-byte boundary (K is a multiple of G).
template <typename T>
__host__ __device__ inline int vec_delta(uintptr_t residue) {
  if constexpr (sizeof(T) == 4) {
    return static_cast<int>(((residue >> 2) * 3) & 3);
  } else {
    return static_cast<int>(residue >> 3);
  }
}

// 1/sqrt(x) for the xyz backward's bond and normal lengths: the approximate reciprocal square root
// instruction without denormal handling (its inputs are squared lengths that the accuracy tests
// bound far from zero; a chain where one underflows takes the recompute form), double the library
// routine.
__device__ __forceinline__ float bond_rsqrt(float x) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ double bond_rsqrt(double x) { return rsqrt(x); }

template <typename T>
struct SlotGroup {
  T v[VecSlots<T>::kElems];
};

__device__ __forceinline__ void load_group(const float* p, SlotGroup<float>& g) {
  const float4* q = reinterpret_cast<const float4*>(p);
  const float4 a = q[0], b = q[1], c = q[2];
  g.v[0] = a.x, g.v[1] = a.y, g.v[2] = a.z, g.v[3] = a.w;
  g.v[4] = b.x, g.v[5] = b.y, g.v[6] = b.z, g.v[7] = b.w;
  g.v[8] = c.x, g.v[9] = c.y, g.v[10] = c.z, g.v[11] = c.w;
}

__device__ __forceinline__ void store_group(float* p, const SlotGroup<float>& g) {
  float4* q = reinterpret_cast<float4*>(p);
  q[0] = make_float4(g.v[0], g.v[1], g.v[2], g.v[3]);
  q[1] = make_float4(g.v[4], g.v[5], g.v[6], g.v[7]);
  q[2] = make_float4(g.v[8], g.v[9], g.v[10], g.v[11]);
}

__device__ __forceinline__ void load_group(const double* p, SlotGroup<double>& g) {
  const double2* q = reinterpret_cast<const double2*>(p);
  const double2 a = q[0], b = q[1], c = q[2];
  g.v[0] = a.x, g.v[1] = a.y, g.v[2] = b.x, g.v[3] = b.y, g.v[4] = c.x, g.v[5] = c.y;
}

__device__ __forceinline__ void store_group(double* p, const SlotGroup<double>& g) {
  double2* q = reinterpret_cast<double2*>(p);
  q[0] = make_double2(g.v[0], g.v[1]);
  q[1] = make_double2(g.v[2], g.v[3]);
  q[2] = make_double2(g.v[4], g.v[5]);
}

// Barrier over the threads of one chain.
template <int W>
__device__ __forceinline__ void chain_sync() {
  if constexpr (W == 1) {
    __syncwarp();
  } else {
    __syncthreads();
  }
}

template <int W>
__device__ __forceinline__ bool chain_any(bool p) {
  if constexpr (W == 1) {
    return __any_sync(0xffffffffu, p) != 0;
  } else {
    return __syncthreads_or(p) != 0;
  }
}

// Sine/cosine of one step's two angles without the per-step range test: float takes the packed
// short reduction (the caller tracks the largest |angle| and redoes the thread on the library path
// when it exceeds kSinCosFastRange), double the library routine.
__device__ __forceinline__ void vec_sincos(float th, float ph, float& st, float& ct, float& sp, float& cp) {
  float2 s, c;
  sincos_fast2(make_float2(th, ph), s, c);
  st = s.x, ct = c.x, sp = s.y, cp = c.y;
}

__device__ __forceinline__ void vec_sincos(double th, double ph, double& st, double& ct, double& sp, double& cp) {
  sincos(th, &st, &ct);
  sincos(ph, &sp, &cp);
}

// Static shared memory per chain of the vector kernels: the base frame built by thread 0 and the
// warp totals / sums of the CTA scans.
template <typename V, int W>
struct VecChainShared {
  V frame[18];  // F (row-major 9), p2, p0, p1
  Affine<V> warp_totals[W > 1 ? W : 1];
  V warp_sums[W > 1 ? 6 * W : 1];
};

// --------------------------------------------------------------------------------------------
// forward
// --------------------------------------------------------------------------------------------
// Exclusive affine prefix over the threads of one chain (W warps).  `total` of thread 0 already
// holds the world frame, so the results are world carries; lane 0 of warp 0 gets `first`.
template <typename V, int W>
__device__ __forceinline__ Affine<V> chain_exclusive_affine(const Affine<V>& total, const Affine<V>& first, Affine<V>* warp_totals, int u) {
  const int lane = u & (kWarp - 1);
  Affine<V> x = total;
#pragma unroll
  for (int off = 1; off < kWarp; off <<= 1) {
    const Affine<V> y = shfl_up_affine(x, off);
    if (lane >= off) x = compose(y, x);
  }
  Affine<V> excl = shfl_up_affine(x, 1);
  if (lane == 0) excl = first;
  if constexpr (W > 1) {
    const int warp = u / kWarp;
    if (lane == kWarp - 1) warp_totals[warp] = x;
    __syncthreads();
    if (warp > 0) {
      Affine<V> carry = warp_totals[0];
      for (int w = 1; w < warp; ++w) carry = compose(carry, warp_totals[w]);
      excl = (lane == 0) ? carry : compose(carry, excl);
    }
  }
  return excl;
}

// One LDGSTS of `E` bytes from g + GOFF into shared address saddr + SOFF (both offsets immediates).
template <int E, int SOFF, int GOFF>
__device__ __forceinline__ void cp_async_at(uint32_t saddr, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0+%2], [%1+%3], %4;\n" ::"r"(saddr), "l"(g), "n"(SOFF), "n"(GOFF), "n"(E) : "memory");
}

// The three inputs of step s, L[s+2], A[s+1], D[s] (Lr, Ar, Dr point at the step-0 elements), into
// words 0..2 of slot s+3 (dst = slot 3), for every step s of thread u's stride-NT share.  Four
// steps per iteration with immediate offsets, so that a thread bumps its four base addresses once per
// twelve copies.
template <int E, int NT, int K>
__device__ __forceinline__ void scatter_unrolled(uint32_t sa, const char* l, const char* a, const char* d) {
  cp_async_at<E, 3 * K * NT * E + 0 * E, K * NT * E>(sa, l);
  cp_async_at<E, 3 * K * NT * E + 1 * E, K * NT * E>(sa, a);
  cp_async_at<E, 3 * K * NT * E + 2 * E, K * NT * E>(sa, d);
}

template <typename T, int NT>
__device__ __forceinline__ void scatter_step_inputs(T* dst, const T* Lr, const T* Ar, const T* Dr, int S, int u) {
  constexpr int E = static_cast<int>(sizeof(T));
  uint32_t sa = smem_u32(dst + 3 * u);
  const char* l = reinterpret_cast<const char*>(Lr + u);
  const char* a = reinterpret_cast<const char*>(Ar + u);
  const char* d = reinterpret_cast<const char*>(Dr + u);
  int s = u;
  for (; s + 3 * NT < S; s += 4 * NT) {
    scatter_unrolled<E, NT, 0>(sa, l, a, d);
    scatter_unrolled<E, NT, 1>(sa, l, a, d);
    scatter_unrolled<E, NT, 2>(sa, l, a, d);
    scatter_unrolled<E, NT, 3>(sa, l, a, d);
    sa += 12 * NT * E;
    l += 4 * NT * E;
    a += 4 * NT * E;
    d += 4 * NT * E;
  }
  for (; s < S; s += NT) {
    scatter_unrolled<E, NT, 0>(sa, l, a, d);
    sa += 3 * NT * E;
    l += NT * E;
    a += NT * E;
    d += NT * E;
  }
}

// The thread's sweep on the library sine/cosine, from global memory (its slots hold positions by
// now).  Runs only when an angle of the thread lies outside the short reduction's range.
template <typename T, typename V = typename ComputeOf<T>::type>
__device__ __noinline__ Affine<V> vec_forward_redo(const BlockArgs<T>& args, const ChainRows& rows, V* X, int a0, int K) {
  Affine<V> P = affine_identity<V>();
  const int N = rows.points;
  for (int k = 0; k < K; ++k) {
    const int a = a0 + k;
    V l = V(0), th = V(0), ph = V(0);
    if (a >= 3 && a < N) {
      l = to_r<V>(args.lengths[rows.lengths + a - 1]);
      th = to_r<V>(args.angles[rows.angles + a - 2]);
      ph = to_r<V>(args.dihedrals[rows.dihedrals + a - 3]);
    }
    V st, ct, sp, cp;
    sincos(th, &st, &ct);
    sincos(ph, &sp, &cp);
    advance(P, step_rot(l, st, ct, sp, cp));
    X[3 * a] = P.v[0];
    X[3 * a + 1] = P.v[1];
    X[3 * a + 2] = P.v[2];
  }
  return P;
}

// kPrefetch: the instantiation for launches that overlap the previous kernel ((B, N) batches); its
// chains' rows are asked of L2 before the grid dependency wait.  A separate instantiation because
// the prefetch code, even untaken, measured slower in large plain launches (config 1: 47.6 against
// 47.3 us per step).
template <typename T, int W, int C, bool kPrefetch = false>
__global__ void __launch_bounds__(kWarp* W* C) block_forward_vec_kernel(BlockArgs<T> args, T* __restrict__ xyz, ChainGeometry geo) {
  if constexpr (kPrefetch) {
    if (threadIdx.x % (kWarp * W) == 0) prefetch_input_rows(args, geo, int64_t(blockIdx.x) * C + threadIdx.x / (kWarp * W));
  }
  enter_after_previous_grid();
  static_assert(sizeof(T) >= 4, "vector slots hold 32- and 64-bit types");
  static_assert(C == 1 || W == 1, "several chains per CTA only with one warp per chain");
  using V = T;
  constexpr int G = VecSlots<T>::kAtoms;
  constexpr int NT = kWarp * W;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ VecChainShared<V, W> shared_chain[C];

  const int c = static_cast<int>(threadIdx.x) / NT;
  const int u = static_cast<int>(threadIdx.x) % NT;
  const int64_t chain = int64_t(blockIdx.x) * C + c;
  if (chain >= geo.batch) return;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the chain)
  VecChainShared<V, W>& sh = shared_chain[c];
  const int N = rows.points, K = geo.items;
  T* out = xyz + rows.xyz;
  const uintptr_t residue = reinterpret_cast<uintptr_t>(out) & 15u;
  const int delta = vec_delta<T>(residue);
  unsigned char* region = smem + static_cast<size_t>(c) * vec_row_bytes(geo.points, K, sizeof(T));
  T* X = reinterpret_cast<T*>(region + kVecFrontPad + residue);
  const int live = (N + delta + K - 1) / K;  // threads that own atoms
  const int a0 = u * K - delta;

  // Stage: slot s+3 <- (L[s+2], A[s+1], D[s]) for every step s; slots of atoms that are not steps
  // (the front padding, atoms 0..2, the tail padding) get zeros.
  {
    scatter_step_inputs<T, NT>(X + 9, args.lengths + rows.lengths + 2, args.angles + rows.angles + 1, args.dihedrals + rows.dihedrals, N - 3, u);
    for (int i = u; i < 3 * (delta + 3); i += NT) X[i - 3 * delta] = T(0);
    const int tail_end = 3 * (live * K - delta);
    for (int i = 3 * N + u; i < tail_end; i += NT) X[i] = T(0);
  }
  if (u == 0) {
    // the base frame while the rows stage, with its first two columns negated when 3 + delta (the
    // number of half turns thread 0 takes before atom 3) is odd
    const AnchorFrame<V> af = anchor_frame<V>(args.p0, args.first_direction, args.initial_normal);
    const ChainFrame<V> ff = chain_frame_of<T, V>(args, af, rows);
    const bool flip = ((3 + delta) & 1) != 0;
#pragma unroll
    for (int i = 0; i < 9; ++i) sh.frame[i] = (flip && (i % 3) < 2) ? -ff.F[i] : ff.F[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      sh.frame[9 + i] = ff.p2[i];
      sh.frame[12 + i] = af.p0[i];
      sh.frame[15 + i] = ff.p1[i];
    }
  }
  cp_async_wait_all();
  chain_sync<W>();

  // Sweep: local prefix positions of the thread's atoms, in place; P ends as the thread's total.
  Affine<V> P = affine_identity<V>();
  if (u < live) {
    float amax = 0.0f;
    const int groups = K / G;
    T* p = X + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, p += 3 * G) {
      SlotGroup<T> s;
      load_group(p, s);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V l = s.v[3 * j], th = s.v[3 * j + 1], ph = s.v[3 * j + 2];
        if constexpr (sizeof(T) == 4) amax = fmaxf(amax, fmaxf(fabsf(th), fabsf(ph)));
        V st, ct, sp, cp;
        vec_sincos(th, ph, st, ct, sp, cp);
        advance(P, step_rot(l, st, ct, sp, cp));
        s.v[3 * j] = P.v[0];
        s.v[3 * j + 1] = P.v[1];
        s.v[3 * j + 2] = P.v[2];
      }
      store_group(p, s);
    }
    if constexpr (sizeof(T) == 4) {
      if (!(amax <= kSinCosFastRange)) {
        P = vec_forward_redo<T>(args, rows, X, a0, K);
        // thread 0's redo starts from the identity at atom -delta too: same half turns as above
      }
    }
  }

  // World carries: thread 0 composes (F D, p2) in front of its total.
  Affine<V> first = affine_identity<V>();
  if (u == 0) {
#pragma unroll
    for (int i = 0; i < 9; ++i) first.m[i] = sh.frame[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) first.v[i] = sh.frame[9 + i];
    P = compose(first, P);
  }
  const Affine<V> Wc = chain_exclusive_affine<V, W>(P, first, sh.warp_totals, u);
  if (u < live) {
    const int groups = K / G;
    T* p = X + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, p += 3 * G) {
      SlotGroup<T> s;
      load_group(p, s);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V v0 = s.v[3 * j], v1 = s.v[3 * j + 1], v2 = s.v[3 * j + 2];
        s.v[3 * j] = vfma(Wc.m[2], v2, vfma(Wc.m[1], v1, vfma(Wc.m[0], v0, Wc.v[0])));
        s.v[3 * j + 1] = vfma(Wc.m[5], v2, vfma(Wc.m[4], v1, vfma(Wc.m[3], v0, Wc.v[1])));
        s.v[3 * j + 2] = vfma(Wc.m[8], v2, vfma(Wc.m[7], v1, vfma(Wc.m[6], v0, Wc.v[2])));
      }
      store_group(p, s);
    }
  }
  if (u == 0) {
    // atoms 0..2 (thread 0 wrote its carried padding positions there just above)
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      X[i] = sh.frame[12 + i];
      X[3 + i] = sh.frame[15 + i];
      X[6 + i] = sh.frame[9 + i];
    }
  }
  fence_proxy_async_smem();
  chain_sync<W>();
  store_row_bulk<T>(out, X, 3 * N, u, NT, 0);
  if (u == 0) bulk_store_wait_read();
}

// --------------------------------------------------------------------------------------------
// backward from xyz
// --------------------------------------------------------------------------------------------
// Positions of `count` padding atoms continuing a chain from atom `e` (position xe) away from its
// neighbour `xn`: a right-angled zig-zag x_{k+1} = x_k + L e1, x_{k+2} = x_{k+1} + L e2, ... with
// L = |xe - xn| and e1, e2 orthonormal and perpendicular to the bond b = (xe - xn) / L.  Every
// padding bond has the length of the adjacent real one and every angle through the padding is a
// right angle, so no padding step trips the short-bond or flat-angle tests.
template <typename V>
__device__ __forceinline__ void zigzag_padding(V* first_slot, int stride, int count, const V* xe, const V* xn) {
  V b[3] = {vsub(xe[0], xn[0]), vsub(xe[1], xn[1]), vsub(xe[2], xn[2])};
  const V L = sqrt(dot3(b, b));
  // the coordinate axis least aligned with b
  const V ax = fabs(b[0]), ay = fabs(b[1]), az = fabs(b[2]);
  V axis[3] = {V(0), V(0), V(0)};
  if (ax <= ay && ax <= az) {
    axis[0] = V(1);
  } else if (ay <= az) {
    axis[1] = V(1);
  } else {
    axis[2] = V(1);
  }
  V e1[3], e2[3];
  cross3(b, axis, e1);
  V n1 = sqrt(dot3(e1, e1));
  n1 = n1 > V(0) ? V(1) / n1 : V(0);
#pragma unroll
  for (int i = 0; i < 3; ++i) e1[i] = vmul(e1[i], n1);
  cross3(b, e1, e2);
  V n2 = sqrt(dot3(e2, e2));
  n2 = n2 > V(0) ? V(1) / n2 : V(0);
#pragma unroll
  for (int i = 0; i < 3; ++i) e2[i] = vmul(e2[i], n2);
  V x[3] = {xe[0], xe[1], xe[2]};
  for (int k = 0; k < count; ++k) {
    const V* e = (k & 1) ? e2 : e1;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      x[i] = vfma(L, e[i], x[i]);
      first_slot[stride * k + i] = x[i];
    }
  }
}

// Gradients of lengths[0], lengths[1] and angles[0] (write_first_frame_param_grads,
// block.cu:206-228) into slots 1 and 2 of the gradient row `out`, for an orthonormal base frame, in
// world coordinates with moments about p2: F3, M3 the force and moment suffix over atoms >= 3, g1
// and g2 the incoming gradients of atoms 1 and 2.
template <typename V>
__device__ __forceinline__ void first_frame_grads_world(V* out, const AnchorFrame<V>& af, const BackwardFrame<V>& bf, const V* g1, const V* g2, const V* F3,
                                                        const V* M3) {
  const ChainFrame<V>& ff = bf.ff;
  V grad_p2[3], d_dir[3], g12[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    d_dir[i] = vfma(ff.c0, V(af.turn0[i]), vmul(ff.s0, V(af.dir0[i])));
    grad_p2[i] = vadd(g2[i], F3[i]);
    g12[i] = vadd(g1[i], grad_p2[i]);
  }
  const V acc = vneg(vmul(bf.bv[0], dot3(ff.normal, M3)));
  const V dir0[3] = {af.dir0[0], af.dir0[1], af.dir0[2]};
  out[3] = dot3(g12, dir0);
  out[6] = dot3(grad_p2, ff.dir1);
  out[7] = vfma(bf.l1, dot3(grad_p2, d_dir), acc);
}

// Shared state of the xyz backward's chain beyond VecChainShared.
template <typename V>
struct VecBackwardShared {
  FirstFrame<V> first;
  V g12[6];  // incoming gradients of atoms 1 and 2
};

template <typename T, int W, bool kPrefetch = false>
__global__ void __launch_bounds__(kWarp* W)
    block_backward_xyz_vec_kernel(BlockArgs<T> args, const T* __restrict__ xyz, const T* __restrict__ grad_xyz, T* __restrict__ grad_lengths,
                                  T* __restrict__ grad_angles, T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  if constexpr (kPrefetch) {
    if (threadIdx.x == 0) prefetch_point_rows(xyz, grad_xyz, geo, blockIdx.x);  // as block_forward_vec_kernel's
  }
  enter_after_previous_grid();
  static_assert(sizeof(T) >= 4, "vector slots hold 32- and 64-bit types");
  using R = T;
  using V = T;
  constexpr int G = VecSlots<T>::kAtoms;
  constexpr int NT = kWarp * W;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ VecChainShared<V, W> sh;
  __shared__ VecBackwardShared<V> bsh;
  __shared__ CtaExchange<V> ex;  // the recompute form's scans

  const int u = static_cast<int>(threadIdx.x);
  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, K = geo.items;
  const T* xrow = xyz + rows.xyz;
  const T* grow = grad_xyz + rows.xyz;
  const uintptr_t residue = reinterpret_cast<uintptr_t>(xrow) & 15u;  // the host checked grad's equals it
  const int delta = vec_delta<T>(residue);
  const size_t row_bytes = vec_row_bytes(geo.points, K, sizeof(T));
  unsigned char* const xregion = smem;
  unsigned char* const gregion = smem + row_bytes;
  T* const X = reinterpret_cast<T*>(xregion + kVecFrontPad + residue);
  T* const Gd = reinterpret_cast<T*>(gregion + kVecFrontPad + residue);
  const int live = (N + delta + K - 1) / K;
  const int a0 = u * K - delta;
  const int pad_end = live * K - delta;  // atoms [N, pad_end) are tail padding

  stage_row_async(xregion + kVecFrontPad, xrow, 3 * N, u, NT);
  stage_row_async(gregion + kVecFrontPad, grow, 3 * N, u, NT);
  // zero gradients on the padding (front and tail)
  for (int i = u; i < 15; i += NT) Gd[i - 15] = T(0);
  for (int i = 3 * N + u; i < 3 * pad_end; i += NT) Gd[i] = T(0);
  if (u == 0) {
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const R l0 = to_r<R>(args.lengths[rows.lengths]);
    const R l1 = to_r<R>(args.lengths[rows.lengths + 1]);
    const R a0r = to_r<R>(args.angles[rows.angles]);
    bsh.first = FirstFrame<V>{af, backward_frame<V>(af, l0, l1, a0r)};
  }
  cp_async_wait_all();
  chain_sync<W>();

  const bool general = bsh.first.bf.general;  // uniform over the CTA
  bool redo = general;
  if (!redo) {
    // padding positions (thread 0: in front of atom 0, the last live thread: past atom N-1); atoms
    // 0..2's gradients are set aside and zeroed so that the sums start at atom 3
    if (u == 0) {
      zigzag_padding<V>(X - 3, -3, 5, X, X + 3);
#pragma unroll
      for (int i = 0; i < 6; ++i) bsh.g12[i] = Gd[3 + i];
#pragma unroll
      for (int i = 0; i < 9; ++i) Gd[i] = T(0);
    }
    if (u == live - 1 && pad_end > N) zigzag_padding<V>(X + 3 * N, 3, pad_end - N, X + 3 * (N - 1), X + 3 * (N - 2));
    const V o[3] = {X[6], X[7], X[8]};
    // pass 1: the thread's sums of g and (x - o) x g, and its largest |x|^2
    V gsum[3] = {V(0), V(0), V(0)};
    V msum[3] = {V(0), V(0), V(0)};
    V xmax2 = V(0);
    const int groups = K / G;
    if (u < live) {
      const T* px = X + 3 * a0;
      const T* pg = Gd + 3 * a0;
#pragma unroll 1
      for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
        SlotGroup<T> xs, gs;
        load_group(px, xs);
        load_group(pg, gs);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const V xw[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
          const V gg[3] = {gs.v[3 * j], gs.v[3 * j + 1], gs.v[3 * j + 2]};
          xmax2 = fmax(xmax2, dot3(xw, xw));
          const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
          V mx[3];
          cross3(x, gg, mx);
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            gsum[i] = vadd(gsum[i], gg[i]);
            msum[i] = vadd(msum[i], mx[i]);
          }
        }
      }
    }
    V Fs[3], Ms[3];
    {
      V mine[6] = {gsum[0], gsum[1], gsum[2], msum[0], msum[1], msum[2]};
      V after[6];
      cta_exclusive_suffix<V, 6>(mine, after, sh.warp_sums, W);
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        Fs[i] = vadd(after[i], gsum[i]);
        Ms[i] = vadd(after[3 + i], msum[i]);
      }
    }
    const V F3[3] = {Fs[0], Fs[1], Fs[2]};
    const V M3[3] = {Ms[0], Ms[1], Ms[2]};
    // pass 2: x2 = x_{a-1}, up = u_{a-2 -> a-1}, tau = sum_{j >= a} (x_j - x_{a-1}) x g_j, carried
    // from atom to atom as tau <- tau - (x_a - x_{a-1}) x F
    V dmin2 = V(1e30), wmin2 = V(1);
    if (u < live) {
      V x2[3], up[3], tau[3];
      {
        const T* q = X + 3 * (a0 - 2);
        const V x1[3] = {q[0], q[1], q[2]};
#pragma unroll
        for (int i = 0; i < 3; ++i) x2[i] = q[3 + i];
        const V d[3] = {vsub(x2[0], x1[0]), vsub(x2[1], x1[1]), vsub(x2[2], x1[2])};
        const V inv = bond_rsqrt(dot3(d, d));
#pragma unroll
        for (int i = 0; i < 3; ++i) up[i] = vmul(d[i], inv);
        const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
        V xf[3];
        cross3(xr, Fs, xf);
#pragma unroll
        for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
      }
      const T* px = X + 3 * a0;
      T* pg = Gd + 3 * a0;
#pragma unroll 1
      for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
        SlotGroup<T> xs, gs;
        load_group(px, xs);
        load_group(pg, gs);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const V x3[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
          const V d[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
          const V d2 = dot3(d, d);
          dmin2 = fmin(dmin2, d2);
          const V inv = bond_rsqrt(d2);
          const V uc[3] = {vmul(d[0], inv), vmul(d[1], inv), vmul(d[2], inv)};
          V w[3];
          cross3(up, uc, w);
          const V w2 = dot3(w, w);
          wmin2 = fmin(wmin2, w2);
          const V d_phi = dot3(up, tau);
          const V d_len = dot3(uc, Fs);
          const V d_theta = vneg(vmul(dot3(w, tau), bond_rsqrt(w2)));
          tau[0] = vfma(d[2], Fs[1], vfma(vneg(d[1]), Fs[2], tau[0]));
          tau[1] = vfma(d[0], Fs[2], vfma(vneg(d[2]), Fs[0], tau[1]));
          tau[2] = vfma(d[1], Fs[0], vfma(vneg(d[0]), Fs[1], tau[2]));
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            Fs[i] = vsub(Fs[i], gs.v[3 * j + i]);
            x2[i] = x3[i];
            up[i] = uc[i];
          }
          gs.v[3 * j] = d_len;
          gs.v[3 * j + 1] = d_theta;
          gs.v[3 * j + 2] = d_phi;
        }
        store_group(pg, gs);
      }
    }
    // Positions are accurate to ~1 ulp of |x|, so a bond direction from them is good to
    // ~ulp(|x|) / |d|: bonds shorter than 1e-3 |x|max, a plane normal with sin^2 < 1e-2 (and any
    // non-finite value: the comparisons fail) send the chain to the recompute form.
    const bool bad = u < live && !(dmin2 >= static_cast<V>(1e-6) * xmax2 && wmin2 >= static_cast<V>(1e-2));
    redo = chain_any<W>(bad);
    if (!redo && u == 0) first_frame_grads_world<V>(Gd, bsh.first.af, bsh.first.bf, bsh.g12, bsh.g12 + 3, F3, M3);
  }
  ChainViews<T> cv;
  cv.X = Gd;
  if (redo) {
    // the recompute form in the layout of block_backward_kernel: the grad row restaged (the fast
    // form wrote over it), the inputs scattered into the slots of the xyz region
    const AnchorFrame<V>& af = bsh.first.af;
    const BackwardFrame<V>& bf = bsh.first.bf;
    chain_sync<W>();
    cv.G = stage_row_async(gregion, grow, 3 * N, u, NT);
    stage_block_inputs<T>(cv, xregion, args, rows, 0, u, NT);
    cp_async_wait_all();
    chain_sync<W>();
    const int items = (N - 3 + NT - 1) / NT;
    const StepRange range = step_range(u, items, N - 3);
    auto step = [&](int s) {
      V l, th, ph, st, ct, sp, cp;
      block_step_inputs<T>(cv, s, l, th, ph);
      step_sincos(th, ph, st, ct, sp, cp);
      return step_rot(l, st, ct, sp, cp);
    };
    if (general) {
      block_backward_general<T, V>(cv, ex, af, bf, cv.G, range, W, step);
    } else {
      block_backward_recompute<true, T, V>(cv, ex, af, bf, cv.G, range, W, step);
    }
  }
  chain_sync<W>();
  write_block_grads<T>(cv, grad_lengths, grad_angles, grad_dihedrals, rows, u, NT);
}

// --------------------------------------------------------------------------------------------
// 16-bit backward from float32 positions
// --------------------------------------------------------------------------------------------
// The torsion xyz backward (torsion_backward_xyz_kernel's algorithm, the reference's own form
// torsion.cu:297-381 for the raw-pair gradients) in vector slots, as block_backward_xyz_vec_kernel
// runs the block one: positions and grad in two shifted slot rows, the sums of g and (x - o) x g
// per thread, the exclusive suffix scan, then one sweep giving d phi of each step, with the torque
// about the previous atom carried from step to step.  The raw row, staged beside them (reading it
// from global memory at the end instead measured 126 against 105 us at config 3), gives the chain
// rule to the (sin, cos) pairs.  Chains with a bond shorter than 1e-3 |x|max, or a pair below the
// norm clamp, take the recompute form in the same CTA.
template <typename T, int W>
__global__ void __launch_bounds__(kWarp* W)
    torsion_backward_xyz_vec_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                                    const T* __restrict__ xyz, const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride,
                                    ChainGeometry geo) {
  enter_after_previous_grid();
  static_assert(sizeof(T) >= 4, "vector slots hold 32- and 64-bit types");
  using R = T;
  using V = T;
  constexpr int G = VecSlots<T>::kAtoms;
  constexpr int NT = kWarp * W;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ VecChainShared<V, W> sh;
  __shared__ CtaExchange<V> ex;  // the recompute form's scans

  const int u = static_cast<int>(threadIdx.x);
  const int64_t chain = blockIdx.x;
  const int N = geo.points, St = geo.steps, K = geo.items;
  const T* raw = raw_pairs + chain * raw_stride;
  const T* xrow = xyz + chain * 3 * N;
  const T* grow = grad_xyz + chain * 3 * N;
  const uintptr_t residue = reinterpret_cast<uintptr_t>(xrow) & 15u;  // the host checked grad's equals it
  const int delta = vec_delta<T>(residue);
  const size_t row_bytes = vec_row_bytes(N, K, sizeof(T));
  unsigned char* const xregion = smem;
  unsigned char* const gregion = smem + row_bytes;
  unsigned char* const rregion = smem + 2 * row_bytes;
  T* const X = reinterpret_cast<T*>(xregion + kVecFrontPad + residue);
  T* const Gd = reinterpret_cast<T*>(gregion + kVecFrontPad + residue);
  const int live = (N + delta + K - 1) / K;
  const int a0 = u * K - delta;
  const int pad_end = live * K - delta;

  stage_row_async(xregion + kVecFrontPad, xrow, 3 * N, u, NT);
  stage_row_async(gregion + kVecFrontPad, grow, 3 * N, u, NT);
  const T* raw_s = stage_row_async(rregion, raw, 2 * St, u, NT);
  for (int i = u; i < 15; i += NT) Gd[i - 15] = T(0);
  for (int i = 3 * N + u; i < 3 * pad_end; i += NT) Gd[i] = T(0);
  cp_async_wait_all();
  chain_sync<W>();

  // padding positions (thread 0: in front of atom 0, the last live thread: past atom N-1); atoms
  // 0..2 carry no gradient (the base frame is fixed), so the sums start at atom 3
  if (u == 0) {
    zigzag_padding<V>(X - 3, -3, 5, X, X + 3);
#pragma unroll
    for (int i = 0; i < 9; ++i) Gd[i] = T(0);
  }
  if (u == live - 1 && pad_end > N) zigzag_padding<V>(X + 3 * N, 3, pad_end - N, X + 3 * (N - 1), X + 3 * (N - 2));
  const V o[3] = {X[6], X[7], X[8]};
  // pass 1: the thread's sums of g and (x - o) x g, and its largest |x|^2
  V gsum[3] = {V(0), V(0), V(0)};
  V msum[3] = {V(0), V(0), V(0)};
  V xmax2 = V(0);
  const int groups = K / G;
  if (u < live) {
    const T* px = X + 3 * a0;
    const T* pg = Gd + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
      SlotGroup<T> xs, gs;
      load_group(px, xs);
      load_group(pg, gs);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V xw[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
        const V gg[3] = {gs.v[3 * j], gs.v[3 * j + 1], gs.v[3 * j + 2]};
        xmax2 = fmax(xmax2, dot3(xw, xw));
        const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
        V mx[3];
        cross3(x, gg, mx);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          gsum[i] = vadd(gsum[i], gg[i]);
          msum[i] = vadd(msum[i], mx[i]);
        }
      }
    }
  }
  V Fs[3], Ms[3];
  {
    V mine[6] = {gsum[0], gsum[1], gsum[2], msum[0], msum[1], msum[2]};
    V after[6];
    cta_exclusive_suffix<V, 6>(mine, after, sh.warp_sums, W);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] = vadd(after[i], gsum[i]);
      Ms[i] = vadd(after[3 + i], msum[i]);
    }
  }
  // pass 2: at atom a, x1 = x_{a-2}, x2 = x_{a-1} and the torque about x2,
  // tau = sum_{j >= a} (x_j - x2) x g_j; d phi of step a-3 = (x2 - x1) . tau / |x2 - x1|; then
  // tau <- tau - (x_a - x2) x F and F <- F - g_a.  d phi goes to word 0 of slot a.
  V dmin2 = V(1e30);
  if (u < live) {
    V x1[3], x2[3], tau[3];
    {
      const T* q = X + 3 * (a0 - 2);
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        x1[i] = q[i];
        x2[i] = q[3 + i];
      }
      const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
      V xf[3];
      cross3(xr, Fs, xf);
#pragma unroll
      for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
    }
    const T* px = X + 3 * a0;
    T* pg = Gd + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
      SlotGroup<T> xs, gs;
      load_group(px, xs);
      load_group(pg, gs);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V x3[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
        const V d[3] = {vsub(x2[0], x1[0]), vsub(x2[1], x1[1]), vsub(x2[2], x1[2])};
        const V d2 = dot3(d, d);
        dmin2 = fmin(dmin2, d2);
        const V d_phi = vmul(dot3(d, tau), bond_rsqrt(d2));
        const V e[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
        tau[0] = vfma(e[2], Fs[1], vfma(vneg(e[1]), Fs[2], tau[0]));
        tau[1] = vfma(e[0], Fs[2], vfma(vneg(e[2]), Fs[0], tau[1]));
        tau[2] = vfma(e[1], Fs[0], vfma(vneg(e[0]), Fs[1], tau[2]));
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          Fs[i] = vsub(Fs[i], gs.v[3 * j + i]);
          x1[i] = x2[i];
          x2[i] = x3[i];
        }
        gs.v[3 * j] = d_phi;
      }
      store_group(pg, gs);
    }
  }
  // every bond a step uses is tested (the padding ones are sound); non-finite values fail it
  const bool bad = u < live && !(dmin2 >= static_cast<V>(1e-6) * xmax2);
  bool redo = chain_any<W>(bad);
  T* gr = grad_raw + chain * grad_stride;
  if (!redo) {
    // chain rule, one (sin, cos) pair per thread and iteration: d raw = d phi (c, -s) / n2 with
    // n2 = max(s^2 + c^2, clamp) (store_raw_pair_grad, torsion.cu:173-182); a pair below the norm
    // clamp is not a rotation, and the chain is redone below
    bool clamped = false;
#pragma unroll 4
    for (int k = u; k < St; k += NT) {
      const V rs = to_r<V>(raw_s[2 * k]);
      const V rc = to_r<V>(raw_s[2 * k + 1]);
      const V n2raw = vfma(rs, rs, vmul(rc, rc));
      clamped |= !(n2raw >= static_cast<V>(1.0e-8f * 1.0e-8f));
      const V rinv = torsion_rinv(torsion_norm2(rs, rc));
      const V scale = vmul(Gd[3 * (k + 3)], vmul(rinv, rinv));
      gr[2 * k] = from_r<T>(vmul(rc, scale));
      gr[2 * k + 1] = from_r<T>(vneg(vmul(rs, scale)));
    }
    redo = chain_any<W>(clamped);
  }
  if (redo) {
    // the recompute form, laid out as in torsion_backward_kernel
    chain_sync<W>();
    ChainViews<T> cv;
    cv.X = reinterpret_cast<R*>(xregion);
    scatter_pairs<T>(reinterpret_cast<T*>(cv.X), raw, St, u, NT);
    cv.G = stage_row_async(gregion, grow, 3 * N, u, NT);
    cp_async_wait_all();
    chain_sync<W>();
    const StepRange range = step_range(u, (St + NT - 1) / NT, St);
    torsion_backward_recompute<T, V, R, false>(cv, ex, consts, range, W);
    chain_sync<W>();
    write_pair_grads<T, R>(cv.X, gr, St, u, NT);
  }
}

// Shared memory of block_backward_xyz32_kernel: the float32 position row (vector slots) in a region
// that also fits the recompute form's float slots, then the 16-bit grad row with room for padding
// atoms on both sides.
template <typename T>
__host__ __device__ inline size_t xyz32_pos_region_bytes(int points, int items) {
  // the recompute form's float slots fit in the vector row (its input rows stay in global memory)
  const size_t vec = vec_row_bytes(points, items, sizeof(float));
  const size_t redo = slot_bytes(points, sizeof(float));
  return vec > redo ? vec : redo;
}
constexpr int kHalfFrontPad = 48;  // 5 padding atoms of 6 bytes, rounded up
template <typename T>
__host__ __device__ inline size_t xyz32_grad_region_bytes(int points, int items) {
  return kHalfFrontPad + 16 + ((3 * sizeof(T) * static_cast<size_t>(points + items) + 15) & ~size_t(15));
}

// d lengths/angles/dihedrals rows from gradient slots of the storage type (slot a holds
// d lengths[a-1], d angles[a-2], d dihedrals[a-3]).
template <typename T>
__device__ __forceinline__ void write_grad_slots(const T* X, T* grad_lengths, T* grad_angles, T* grad_dihedrals, const ChainRows& rows, int tid, int nthr) {
  const int N = rows.points;
  T* gl = grad_lengths + rows.lengths;
  T* ga = grad_angles + rows.angles;
  T* gd = grad_dihedrals + rows.dihedrals;
#pragma unroll 2
  for (int i = tid; i < N - 1; i += nthr) {
    const T* slot = X + 3 * i;
    gl[i] = slot[3];
    if (i < N - 2) ga[i] = slot[7];
    if (i < N - 3) gd[i] = slot[11];
  }
}

// The xyz-form backward of float16/bfloat16 chains from the float32 positions the 16-bit forward
// wrote beside its output (xyz32): a 16-bit position is too coarse for a bond direction, a float32
// one is what block_backward_xyz_vec_kernel reads in float32.  Positions sit in vector slots as
// there; the 16-bit grad row is staged as it is (16-byte copies), read element by element and
// overwritten in place by the three 16-bit gradients of each step.  Degenerate chains take the
// 16-bit recompute form (block_backward_kernel's code) in the same CTA.
template <typename T, int W>
__global__ void __launch_bounds__(kWarp* W)
    block_backward_xyz32_kernel(BlockArgs<T> args, const float* __restrict__ xyz32, const T* __restrict__ grad_xyz, T* __restrict__ grad_lengths,
                                T* __restrict__ grad_angles, T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  enter_after_previous_grid();
  static_assert(sizeof(T) == 2, "the float32-position backward serves the 16-bit types");
  using V = float;
  constexpr int G = VecSlots<float>::kAtoms;
  constexpr int NT = kWarp * W;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ VecChainShared<V, W> sh;
  __shared__ VecBackwardShared<V> bsh;
  __shared__ CtaExchange<V> ex;  // the recompute form's scans

  const int u = static_cast<int>(threadIdx.x);
  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, K = geo.items;
  const float* xrow = xyz32 + rows.xyz;
  const T* grow = grad_xyz + rows.xyz;
  const uintptr_t residue = reinterpret_cast<uintptr_t>(xrow) & 15u;
  const int delta = vec_delta<float>(residue);
  unsigned char* const xregion = smem;
  unsigned char* const gregion = smem + xyz32_pos_region_bytes<T>(geo.points, K);
  float* const X = reinterpret_cast<float*>(xregion + kVecFrontPad + residue);
  const int live = (N + delta + K - 1) / K;
  const int a0 = u * K - delta;
  const int pad_end = live * K - delta;

  stage_row_async(xregion + kVecFrontPad, xrow, 3 * N, u, NT);
  T* const Gh = stage_row_async(gregion + kHalfFrontPad, grow, 3 * N, u, NT);
  for (int i = u; i < 15; i += NT) Gh[i - 15] = from_r<T>(0.0f);
  for (int i = 3 * N + u; i < 3 * pad_end; i += NT) Gh[i] = from_r<T>(0.0f);
  if (u == 0) {
    const AnchorFrame<V> af = anchor_frame<V>(args.p0, args.first_direction, args.initial_normal);
    const V l0 = to_r<V>(args.lengths[rows.lengths]);
    const V l1 = to_r<V>(args.lengths[rows.lengths + 1]);
    const V a0r = to_r<V>(args.angles[rows.angles]);
    bsh.first = FirstFrame<V>{af, backward_frame<V>(af, l0, l1, a0r)};
  }
  cp_async_wait_all();
  chain_sync<W>();

  const bool general = bsh.first.bf.general;  // uniform over the CTA
  bool redo = general;
  if (!redo) {
    if (u == 0) {
      zigzag_padding<V>(X - 3, -3, 5, X, X + 3);
#pragma unroll
      for (int i = 0; i < 6; ++i) bsh.g12[i] = to_r<V>(Gh[3 + i]);
#pragma unroll
      for (int i = 0; i < 9; ++i) Gh[i] = from_r<T>(0.0f);
    }
    if (u == live - 1 && pad_end > N) zigzag_padding<V>(X + 3 * N, 3, pad_end - N, X + 3 * (N - 1), X + 3 * (N - 2));
    const V o[3] = {X[6], X[7], X[8]};
    V gsum[3] = {V(0), V(0), V(0)};
    V msum[3] = {V(0), V(0), V(0)};
    V xmax2 = V(0);
    const int groups = K / G;
    if (u < live) {
      const float* px = X + 3 * a0;
      const T* pg = Gh + 3 * a0;
#pragma unroll 1
      for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
        SlotGroup<float> xs;
        load_group(px, xs);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const V xw[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
          const V gg[3] = {to_r<V>(pg[3 * j]), to_r<V>(pg[3 * j + 1]), to_r<V>(pg[3 * j + 2])};
          xmax2 = fmax(xmax2, dot3(xw, xw));
          const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
          V mx[3];
          cross3(x, gg, mx);
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            gsum[i] = vadd(gsum[i], gg[i]);
            msum[i] = vadd(msum[i], mx[i]);
          }
        }
      }
    }
    V Fs[3], Ms[3];
    {
      V mine[6] = {gsum[0], gsum[1], gsum[2], msum[0], msum[1], msum[2]};
      V after[6];
      cta_exclusive_suffix<V, 6>(mine, after, sh.warp_sums, W);
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        Fs[i] = vadd(after[i], gsum[i]);
        Ms[i] = vadd(after[3 + i], msum[i]);
      }
    }
    const V F3[3] = {Fs[0], Fs[1], Fs[2]};
    const V M3[3] = {Ms[0], Ms[1], Ms[2]};
    V dmin2 = V(1e30), wmin2 = V(1);
    if (u < live) {
      V x2[3], up[3], tau[3];
      {
        const float* q = X + 3 * (a0 - 2);
        const V x1[3] = {q[0], q[1], q[2]};
#pragma unroll
        for (int i = 0; i < 3; ++i) x2[i] = q[3 + i];
        const V d[3] = {vsub(x2[0], x1[0]), vsub(x2[1], x1[1]), vsub(x2[2], x1[2])};
        const V inv = bond_rsqrt(dot3(d, d));
#pragma unroll
        for (int i = 0; i < 3; ++i) up[i] = vmul(d[i], inv);
        const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
        V xf[3];
        cross3(xr, Fs, xf);
#pragma unroll
        for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
      }
      const float* px = X + 3 * a0;
      T* pg = Gh + 3 * a0;
#pragma unroll 1
      for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
        SlotGroup<float> xs;
        load_group(px, xs);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const V x3[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
          const V gg[3] = {to_r<V>(pg[3 * j]), to_r<V>(pg[3 * j + 1]), to_r<V>(pg[3 * j + 2])};
          const V d[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
          const V d2 = dot3(d, d);
          dmin2 = fmin(dmin2, d2);
          const V inv = bond_rsqrt(d2);
          const V uc[3] = {vmul(d[0], inv), vmul(d[1], inv), vmul(d[2], inv)};
          V w[3];
          cross3(up, uc, w);
          const V w2 = dot3(w, w);
          wmin2 = fmin(wmin2, w2);
          const V d_phi = dot3(up, tau);
          const V d_len = dot3(uc, Fs);
          const V d_theta = vneg(vmul(dot3(w, tau), bond_rsqrt(w2)));
          tau[0] = vfma(d[2], Fs[1], vfma(vneg(d[1]), Fs[2], tau[0]));
          tau[1] = vfma(d[0], Fs[2], vfma(vneg(d[2]), Fs[0], tau[1]));
          tau[2] = vfma(d[1], Fs[0], vfma(vneg(d[0]), Fs[1], tau[2]));
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            Fs[i] = vsub(Fs[i], gg[i]);
            x2[i] = x3[i];
            up[i] = uc[i];
          }
          pg[3 * j] = from_r<T>(d_len);
          pg[3 * j + 1] = from_r<T>(d_theta);
          pg[3 * j + 2] = from_r<T>(d_phi);
        }
      }
    }
    const bool bad = u < live && !(dmin2 >= static_cast<V>(1e-6) * xmax2 && wmin2 >= static_cast<V>(1e-2));
    redo = chain_any<W>(bad);
    if (!redo && u == 0) {
      V out[8];
      first_frame_grads_world<V>(out, bsh.first.af, bsh.first.bf, bsh.g12, bsh.g12 + 3, F3, M3);
      Gh[3] = from_r<T>(out[3]);
      Gh[6] = from_r<T>(out[6]);
      Gh[7] = from_r<T>(out[7]);
    }
  }
  if (!redo) {
    chain_sync<W>();
    write_grad_slots<T>(Gh, grad_lengths, grad_angles, grad_dihedrals, rows, u, NT);
    return;
  }
  // the recompute form of block_backward_kernel: float slots in the position region, the 16-bit
  // input rows read from global memory (a rare path; staging them would cost every chain shared
  // memory), the grad row restaged (the fast form may have written over it)
  {
    ChainViews<T> cv;
    const AnchorFrame<V>& af = bsh.first.af;
    const BackwardFrame<V>& bf = bsh.first.bf;
    chain_sync<W>();
    cv.G = stage_row_async(gregion, grow, 3 * N, u, NT);
    cv.X = reinterpret_cast<float*>(xregion);
    cv.row[0] = args.lengths + rows.lengths;
    cv.row[1] = args.angles + rows.angles;
    cv.row[2] = args.dihedrals + rows.dihedrals;
    cp_async_wait_all();
    chain_sync<W>();
    const int items = (N - 3 + NT - 1) / NT;
    const StepRange range = step_range(u, items, N - 3);
    auto step = [&](int s) {
      V l, th, ph, st, ct, sp, cp;
      block_step_inputs<T>(cv, s, l, th, ph);
      step_sincos(th, ph, st, ct, sp, cp);
      return step_rot(l, st, ct, sp, cp);
    };
    if (general) {
      block_backward_general<T, V>(cv, ex, af, bf, cv.G, range, W, step);
    } else {
      block_backward_recompute<true, T, V>(cv, ex, af, bf, cv.G, range, W, step);
    }
    chain_sync<W>();
    write_block_grads<T>(cv, grad_lengths, grad_angles, grad_dihedrals, rows, u, NT);
  }
}

// Shared memory of torsion_backward_xyz32_kernel: float32 positions in a vector row that also fits
// the recompute form's float slots, the 16-bit grad row (xyz32_grad_region_bytes) and the 16-bit
// raw row.
template <typename T>
__host__ __device__ inline size_t torsion_xyz32_bytes(int points, int items) {
  const size_t vec = vec_row_bytes(points, items, sizeof(float));
  const size_t redo = slot_bytes(points, sizeof(float));
  return (vec > redo ? vec : redo) + (kHalfFrontPad + 16 + ((3 * sizeof(T) * static_cast<size_t>(points + items) + 15) & ~size_t(15))) +
         staged_row_bytes(size_t(2) * (points - 3), sizeof(T));
}

// The torsion xyz backward of float16/bfloat16 chains from the float32 positions the 16-bit
// torsion forward wrote beside its output: torsion_backward_xyz_vec_kernel's algorithm on float32
// positions in vector slots, with the 16-bit grad row staged as it is and read element by element.
// d phi stays in float (it is multiplied into both pair gradients): it goes over word 0 of the
// position slots, once every thread has read the two positions in front of its range.  Short bonds
// and clamped pairs take the recompute form (torsion_backward_kernel's) in the same CTA.
template <typename T, int W>
__global__ void __launch_bounds__(kWarp* W)
    torsion_backward_xyz32_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<float> consts, const float* __restrict__ xyz32,
                                  const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride, ChainGeometry geo) {
  enter_after_previous_grid();
  static_assert(sizeof(T) == 2, "the float32-position backward serves the 16-bit types");
  using R = float;
  using V = float;
  constexpr int G = VecSlots<float>::kAtoms;
  constexpr int NT = kWarp * W;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ VecChainShared<V, W> sh;
  __shared__ CtaExchange<V> ex;  // the recompute form's scans

  const int u = static_cast<int>(threadIdx.x);
  const int64_t chain = blockIdx.x;
  const int N = geo.points, St = geo.steps, K = geo.items;
  const T* raw = raw_pairs + chain * raw_stride;
  const float* xrow = xyz32 + chain * 3 * N;
  const T* grow = grad_xyz + chain * 3 * N;
  const uintptr_t residue = reinterpret_cast<uintptr_t>(xrow) & 15u;
  const int delta = vec_delta<float>(residue);
  const size_t vec = vec_row_bytes(N, K, sizeof(float));
  const size_t xbytes = vec > slot_bytes(N, sizeof(float)) ? vec : slot_bytes(N, sizeof(float));
  unsigned char* const xregion = smem;
  unsigned char* const gregion = smem + xbytes;
  unsigned char* const rregion = gregion + kHalfFrontPad + 16 + ((3 * sizeof(T) * static_cast<size_t>(N + K) + 15) & ~size_t(15));
  float* const X = reinterpret_cast<float*>(xregion + kVecFrontPad + residue);
  const int live = (N + delta + K - 1) / K;
  const int a0 = u * K - delta;
  const int pad_end = live * K - delta;

  stage_row_async(xregion + kVecFrontPad, xrow, 3 * N, u, NT);
  T* const Gh = stage_row_async(gregion + kHalfFrontPad, grow, 3 * N, u, NT);
  const T* raw_s = stage_row_async(rregion, raw, 2 * St, u, NT);
  for (int i = u; i < 15; i += NT) Gh[i - 15] = from_r<T>(0.0f);
  for (int i = 3 * N + u; i < 3 * pad_end; i += NT) Gh[i] = from_r<T>(0.0f);
  cp_async_wait_all();
  chain_sync<W>();

  if (u == 0) {
    zigzag_padding<V>(X - 3, -3, 5, X, X + 3);
#pragma unroll
    for (int i = 0; i < 9; ++i) Gh[i] = from_r<T>(0.0f);
  }
  if (u == live - 1 && pad_end > N) zigzag_padding<V>(X + 3 * N, 3, pad_end - N, X + 3 * (N - 1), X + 3 * (N - 2));
  const V o[3] = {X[6], X[7], X[8]};
  V gsum[3] = {V(0), V(0), V(0)};
  V msum[3] = {V(0), V(0), V(0)};
  V xmax2 = V(0);
  const int groups = K / G;
  if (u < live) {
    const float* px = X + 3 * a0;
    const T* pg = Gh + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
      SlotGroup<float> xs;
      load_group(px, xs);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V xw[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
        const V gg[3] = {to_r<V>(pg[3 * j]), to_r<V>(pg[3 * j + 1]), to_r<V>(pg[3 * j + 2])};
        xmax2 = fmax(xmax2, dot3(xw, xw));
        const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
        V mx[3];
        cross3(x, gg, mx);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          gsum[i] = vadd(gsum[i], gg[i]);
          msum[i] = vadd(msum[i], mx[i]);
        }
      }
    }
  }
  V Fs[3], Ms[3];
  {
    V mine[6] = {gsum[0], gsum[1], gsum[2], msum[0], msum[1], msum[2]};
    V after[6];
    cta_exclusive_suffix<V, 6>(mine, after, sh.warp_sums, W);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] = vadd(after[i], gsum[i]);
      Ms[i] = vadd(after[3 + i], msum[i]);
    }
  }
  V dmin2 = V(1e30);
  V x1[3], x2[3], tau[3];
  if (u < live) {
    const float* q = X + 3 * (a0 - 2);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      x1[i] = q[i];
      x2[i] = q[3 + i];
    }
    const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
    V xf[3];
    cross3(xr, Fs, xf);
#pragma unroll
    for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
  }
  chain_sync<W>();  // d phi goes over the position slots: every thread has read its two in front
  if (u < live) {
    float* px = X + 3 * a0;
    const T* pg = Gh + 3 * a0;
#pragma unroll 1
    for (int g = 0; g < groups; ++g, px += 3 * G, pg += 3 * G) {
      SlotGroup<float> xs;
      load_group(px, xs);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const V x3[3] = {xs.v[3 * j], xs.v[3 * j + 1], xs.v[3 * j + 2]};
        const V d[3] = {vsub(x2[0], x1[0]), vsub(x2[1], x1[1]), vsub(x2[2], x1[2])};
        const V d2 = dot3(d, d);
        dmin2 = fmin(dmin2, d2);
        const V d_phi = vmul(dot3(d, tau), bond_rsqrt(d2));
        const V e[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
        tau[0] = vfma(e[2], Fs[1], vfma(vneg(e[1]), Fs[2], tau[0]));
        tau[1] = vfma(e[0], Fs[2], vfma(vneg(e[2]), Fs[0], tau[1]));
        tau[2] = vfma(e[1], Fs[0], vfma(vneg(e[0]), Fs[1], tau[2]));
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          Fs[i] = vsub(Fs[i], to_r<V>(pg[3 * j + i]));
          x1[i] = x2[i];
          x2[i] = x3[i];
        }
        xs.v[3 * j] = d_phi;
      }
      store_group(px, xs);
    }
  }
  const bool bad = u < live && !(dmin2 >= static_cast<V>(1e-6) * xmax2);
  bool redo = chain_any<W>(bad);
  T* gr = grad_raw + chain * grad_stride;
  if (!redo) {
    // chain rule, one (sin, cos) pair per thread and iteration, as torsion_backward_xyz_vec_kernel
    bool clamped = false;
#pragma unroll 4
    for (int k = u; k < St; k += NT) {
      const V rs = to_r<V>(raw_s[2 * k]);
      const V rc = to_r<V>(raw_s[2 * k + 1]);
      const V n2raw = vfma(rs, rs, vmul(rc, rc));
      clamped |= !(n2raw >= 1.0e-8f * 1.0e-8f);
      const V rinv = torsion_rinv(torsion_norm2(rs, rc));
      const V scale = vmul(X[3 * (k + 3)], vmul(rinv, rinv));
      gr[2 * k] = from_r<T>(vmul(rc, scale));
      gr[2 * k + 1] = from_r<T>(vneg(vmul(rs, scale)));
    }
    redo = chain_any<W>(clamped);
  }
  if (redo) {
    // the recompute form of torsion_backward_kernel: float slots over the position region, the raw
    // row and the grad row as staged (the fast form wrote neither)
    chain_sync<W>();
    ChainViews<T> cv;
    cv.X = reinterpret_cast<R*>(xregion);
    cv.row[0] = raw_s;
    cv.G = Gh;
    const StepRange range = step_range(u, (St + NT - 1) / NT, St);
    torsion_backward_recompute<T, V, R, false>(cv, ex, consts, range, W);
    chain_sync<W>();
    write_pair_grads<T, R>(cv.X, gr, St, u, NT);
  }
}

}  // namespace cufkb
