// sm_100a kernels for the cufk reconstruction path.
//
// block_forward_kernel    <- src/cufk/csrc/block.cu:157-204   (xyz from lengths/angles/dihedrals)
// block_backward_kernel   <- src/cufk/csrc/block.cu:206-313   (d lengths/angles/dihedrals)
// torsion_forward_kernel  <- src/cufk/csrc/torsion.cu:254-295 (xyz from raw (sin, cos) pairs)
// torsion_backward_kernel <- src/cufk/csrc/torsion.cu:297-381 (d raw pairs)
//
// One CTA reconstructs kC chains (1, or 2 for float arithmetic: the two chains ride in the two
// halves of float2 lanes, so each multiply-add is one packed f32x2 instruction for both), with
// W = blockDim.x / 32 warps and K (odd) consecutive steps per thread.
//
// Forward: stage the chains' inputs into atom slots (LDGSTS), sweep each thread's K steps
// sequentially from the identity (the local prefix position written back into the slot), exclusive
// affine scan of the thread totals across the CTA, then x = p2 + F (C.v + C.m v) per slot in place
// and one bulk (TMA-engine) store per (N, 3) row.
//
// Backward (one kernel, nothing saved from the forward): the gradient of every parameter of
// step s follows from the force/moment suffix of the atoms it moves.  In base-frame coordinates
// (x~ = P.v, g~ = F^T g, P_s = L_0...L_s):
//   F_s = sum_{j >= s+3} g~_j,  M_s = sum_{j >= s+3} x~_j x g~_j,  tau_s = M_s - x~_{s+2} x F_s,
//   d dihedral[s]   =  P_{s-1}.col0 . tau_s   (rotation about the incoming bond)
//   d angle[s+1]    = -P_s.col2     . tau_s   (rotation about the frame normal)
//   d length[s+2]   =  P_s.col0     . F_s     (translation along the new bond)
// which is the derivative of the reference's forward for any base frame F; the first-frame
// terms (lengths[0..1], angles[0]) follow write_first_frame_param_grads (block.cu:206-228).
// Sweep 1 builds each thread's local prefix, its sum of g~ and the 3x3 moment matrix
// Q = sum p (x) g~ (p = local position), so that once the affine scan gives the thread's carry C
// the thread's moment total is C.v x G + axial(C.m Q) without revisiting its steps.  An exclusive
// suffix scan of (G, M) gives each thread the sums of all later threads; sweep 2 recomputes the
// prefix from C, walks the running suffix down and writes the gradients into the slots in place.
#pragma once

#include "nerf_device.cuh"

namespace cufkb {

template <typename T>
struct BlockArgs {
  const T* lengths;          // (B, N-1)
  const T* angles;           // (B, N-2)
  const T* dihedrals;        // (B, N-3)
  const T* p0;               // (3,) or null = (0, 0, 0)
  const T* first_direction;  // (3,) or null = (1, 0, 0)
  const T* initial_normal;   // (3,) or null = (0, 0, 1)
};

template <typename R>
struct TorsionConsts {
  R length[3];  // bond lengths by phase, rounded to float first (torsion.cu:43-47)
  R sin_a[3];   // sin/cos of the bond angles by phase (torsion.cu:49-53)
  R cos_a[3];
};

// Lane type of a CTA handling kC chains of compute type R.
template <typename R, int kC>
using LaneOf = std::conditional_t<kC == 2, float2, R>;

// Shared memory of one CTA beyond the dynamic slots: scan exchange between warps.
template <typename V>
struct CtaExchange {
  Affine<V> warp_totals[kMaxWarps];
  V warp_sums[kMaxWarps * 6];  // suffix scan of (force, moment)
  V warp_red[kMaxWarps];       // first-frame reduction (separate: warps may still read warp_sums)
};

// --------------------------------------------------------------------------------------------
// shared-memory layout: one region per chain of the CTA
// --------------------------------------------------------------------------------------------
// 4- and 8-byte types ("scatter"): [X slots, 3N elements of T, offset so that X has the residue of
//   the output row mod 16] [G staged grad row (backward)]
// 16-bit types: [X slots, 3N floats] [staged input rows (T)] [G staged grad row (backward)]
__host__ __device__ inline size_t slot_bytes(int points, size_t elem) { return staged_row_bytes(size_t(3) * points, elem); }

template <typename T>
__host__ __device__ inline size_t block_region_bytes(int points, bool backward) {
  using R = typename ComputeOf<T>::type;
  size_t bytes = slot_bytes(points, sizeof(R));
  if (sizeof(T) < 4) {
    bytes += staged_row_bytes(points - 1, sizeof(T)) + staged_row_bytes(points - 2, sizeof(T)) + staged_row_bytes(points - 3, sizeof(T));
  }
  if (backward) bytes += staged_row_bytes(size_t(3) * points, sizeof(T));
  return bytes;
}

template <typename T>
__host__ __device__ inline size_t torsion_region_bytes(int points, bool backward) {
  using R = typename ComputeOf<T>::type;
  size_t bytes = slot_bytes(points, sizeof(R));
  if (sizeof(T) < 4) bytes += staged_row_bytes(size_t(2) * (points - 3), sizeof(T));
  if (backward) bytes += staged_row_bytes(size_t(3) * points, sizeof(T));
  return bytes;
}

// Steps [first, first + count) of thread `tid` (count may be 0 for trailing threads).
struct StepRange {
  int first;
  int count;
};

__device__ __forceinline__ StepRange step_range(int tid, int K, int S) {
  const int first = tid * K;
  const int left = S - first;
  return {first, left < 0 ? 0 : (left < K ? left : K)};
}

// Per-chain shared-memory views of one CTA.
template <typename T, int kC>
struct ChainViews {
  using R = typename ComputeOf<T>::type;
  using V = LaneOf<R, kC>;
  R* X[kC];                   // atom slots
  const T* row[kC][3];        // staged input rows of 16-bit types (lengths/angles/dihedrals or raw pairs)
  T* G[kC];                   // staged gradient rows (backward)

  __device__ __forceinline__ V slot(int off) const {
    if constexpr (kC == 2) {
      return make_float2(X[0][off], X[1][off]);
    } else {
      return X[0][off];
    }
  }
  __device__ __forceinline__ void set_slot(int off, V v) const {
    if constexpr (kC == 2) {
      X[0][off] = v.x;
      X[1][off] = v.y;
    } else {
      X[0][off] = v;
    }
  }
  __device__ __forceinline__ V staged(int which, int i) const {
    if constexpr (kC == 2) {
      return make_float2(to_r<float>(row[0][which][i]), to_r<float>(row[1][which][i]));
    } else {
      return to_r<R>(row[0][which][i]);
    }
  }
  __device__ __forceinline__ V grad(int off) const {
    if constexpr (kC == 2) {
      return make_float2(to_r<float>(G[0][off]), to_r<float>(G[1][off]));
    } else {
      return to_r<R>(G[0][off]);
    }
  }
  __device__ __forceinline__ void set_grad(int off, V v) const {
    if constexpr (kC == 2) {
      G[0][off] = v.x;
      G[1][off] = v.y;
    } else {
      G[0][off] = v;
    }
  }
};

// Block path inputs of step s: (L[s+2], A[s+1], D[s]).
template <typename T, int kC>
__device__ __forceinline__ void block_step_inputs(const ChainViews<T, kC>& cv, int s, LaneOf<typename ComputeOf<T>::type, kC>& l,
                                                  LaneOf<typename ComputeOf<T>::type, kC>& th, LaneOf<typename ComputeOf<T>::type, kC>& ph) {
  if constexpr (sizeof(T) >= 4) {
    l = cv.slot(3 * (s + 3));
    th = cv.slot(3 * (s + 3) + 1);
    ph = cv.slot(3 * (s + 3) + 2);
  } else {
    l = cv.staged(0, s + 2);
    th = cv.staged(1, s + 1);
    ph = cv.staged(2, s);
  }
}

// Scatters one chain's block inputs into the slots with 4/8-byte LDGSTS.
template <typename T>
__device__ __forceinline__ void scatter_block_inputs(T* X, const T* Lr, const T* Ar, const T* Dr, int N, int tid, int nthr) {
  int i = tid;
#pragma unroll 4
  for (; i < N - 3; i += nthr) {
    T* slot = X + 3 * i;
    cp_async<sizeof(T)>(slot + 3, Lr + i);
    cp_async<sizeof(T)>(slot + 7, Ar + i);
    cp_async<sizeof(T)>(slot + 11, Dr + i);
  }
  if (i < N - 1) cp_async<sizeof(T)>(X + 3 * i + 3, Lr + i);
  if (i < N - 2) cp_async<sizeof(T)>(X + 3 * i + 7, Ar + i);
  i += nthr;
  if (i < N - 1) cp_async<sizeof(T)>(X + 3 * i + 3, Lr + i);
  if (i < N - 2) cp_async<sizeof(T)>(X + 3 * i + 7, Ar + i);
}

// x = p2 + F (C.v + C.m v) for every slot the thread owns (in place).
template <typename T, int kC, typename V>
__device__ __forceinline__ void apply_carry(const ChainViews<T, kC>& cv, const Affine<V>& carry, const V* F, const V* p2, StepRange r) {
  V G[9];
  V h[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      G[3 * i + j] = vfma(F[3 * i + 2], carry.m[6 + j], vfma(F[3 * i + 1], carry.m[3 + j], vmul(F[3 * i + 0], carry.m[0 + j])));
    }
    h[i] = vfma(F[3 * i + 2], carry.v[2], vfma(F[3 * i + 1], carry.v[1], vfma(F[3 * i + 0], carry.v[0], p2[i])));
  }
  int off = 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, off += 3) {
    const V v0 = cv.slot(off), v1 = cv.slot(off + 1), v2 = cv.slot(off + 2);
    cv.set_slot(off + 0, vfma(G[2], v2, vfma(G[1], v1, vfma(G[0], v0, h[0]))));
    cv.set_slot(off + 1, vfma(G[5], v2, vfma(G[4], v1, vfma(G[3], v0, h[1]))));
    cv.set_slot(off + 2, vfma(G[8], v2, vfma(G[7], v1, vfma(G[6], v0, h[2]))));
  }
}

// Sweep 1 of the forward: local prefix positions into the slots; returns the thread total.
template <typename T, int kC, typename V, typename StepFn>
__device__ __forceinline__ Affine<V> sweep_local_prefix(const ChainViews<T, kC>& cv, StepRange r, StepFn step) {
  Affine<V> P = affine_identity<V>();
  int off = 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, off += 3) {
    advance(P, step(r.first + k));
    cv.set_slot(off, P.v[0]);
    cv.set_slot(off + 1, P.v[1]);
    cv.set_slot(off + 2, P.v[2]);
  }
  return P;
}

// g~ = F^T g
template <typename V>
__device__ __forceinline__ void to_base(const V* F, V g0, V g1, V g2, V* out) {
  out[0] = vfma(F[6], g2, vfma(F[3], g1, vmul(F[0], g0)));
  out[1] = vfma(F[7], g2, vfma(F[4], g1, vmul(F[1], g0)));
  out[2] = vfma(F[8], g2, vfma(F[5], g1, vmul(F[2], g0)));
}

// Sweep 1 of the backward: thread total of the prefix, of g~ and of Q = sum p (x) g~.  When the
// staged gradient row is in the compute type, g~ replaces g in place for sweep 2.
template <typename T, int kC, typename V, typename StepFn>
__device__ __forceinline__ Affine<V> sweep_backward_totals(const ChainViews<T, kC>& cv, const V* F, StepRange r, StepFn step, V (&gsum)[3],
                                                          V (&Q)[9]) {
  using R = typename ComputeOf<T>::type;
  Affine<V> P = affine_identity<V>();
#pragma unroll
  for (int i = 0; i < 3; ++i) gsum[i] = splat<V>(0);
#pragma unroll
  for (int i = 0; i < 9; ++i) Q[i] = splat<V>(0);
  int off = 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, off += 3) {
    advance(P, step(r.first + k));
    V gt[3];
    to_base(F, cv.grad(off), cv.grad(off + 1), cv.grad(off + 2), gt);
    if constexpr (std::is_same_v<T, R>) {
      cv.set_grad(off, gt[0]);
      cv.set_grad(off + 1, gt[1]);
      cv.set_grad(off + 2, gt[2]);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) gsum[c] = vadd(gsum[c], gt[c]);
#pragma unroll
    for (int d = 0; d < 3; ++d) {
#pragma unroll
      for (int c = 0; c < 3; ++c) Q[3 * d + c] = vfma(P.v[d], gt[c], Q[3 * d + c]);
    }
  }
  return P;
}

// g~ of the atom at slot offset `off` in sweep 2 (stored by sweep 1 for the compute type).
template <typename T, int kC, typename V>
__device__ __forceinline__ void base_grad(const ChainViews<T, kC>& cv, int off, const V* F, V* gt) {
  using R = typename ComputeOf<T>::type;
  if constexpr (std::is_same_v<T, R>) {
    gt[0] = cv.grad(off);
    gt[1] = cv.grad(off + 1);
    gt[2] = cv.grad(off + 2);
  } else {
    to_base(F, cv.grad(off), cv.grad(off + 1), cv.grad(off + 2), gt);
  }
}

// Thread's moment total from its carry: C.v x G + axial(C.m Q).
template <typename V>
__device__ __forceinline__ void moment_total(const Affine<V>& C, const V (&gsum)[3], const V (&Q)[9], V* M) {
  V H[9];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) H[3 * i + j] = vfma(C.m[3 * i + 2], Q[6 + j], vfma(C.m[3 * i + 1], Q[3 + j], vmul(C.m[3 * i + 0], Q[0 + j])));
  }
  cross3(C.v, gsum, M);
  M[0] = vadd(M[0], vsub(H[5], H[7]));
  M[1] = vadd(M[1], vsub(H[6], H[2]));
  M[2] = vadd(M[2], vsub(H[1], H[3]));
}

// Suffix sums (force, moment) over all atoms from this thread's first step on.
template <typename V>
__device__ __forceinline__ void suffix_base(const Affine<V>& carry, const V (&gsum)[3], const V (&Q)[9], CtaExchange<V>& ex, int nwarps, V* Fs,
                                            V* Ms) {
  V mlane[3];
  moment_total<V>(carry, gsum, Q, mlane);
  V mine[6] = {gsum[0], gsum[1], gsum[2], mlane[0], mlane[1], mlane[2]};
  V after[6];
  cta_exclusive_suffix<V, 6>(mine, after, ex.warp_sums, nwarps);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    Fs[i] = vadd(after[i], gsum[i]);
    Ms[i] = vadd(after[3 + i], mlane[i]);
  }
}

// Per-chain row pointers of this CTA: chain c of the CTA is blockIdx.x * kC + c; a missing last
// chain (odd batch) aliases chain 0's rows for reading and writes nothing.
template <int kC>
__device__ __forceinline__ int64_t cta_chain(int c, int batch, bool& valid) {
  const int64_t idx = int64_t(blockIdx.x) * kC + c;
  valid = idx < batch;
  return valid ? idx : int64_t(blockIdx.x) * kC;
}

// --------------------------------------------------------------------------------------------
// block path
// --------------------------------------------------------------------------------------------
template <typename T, int kC>
__global__ void __launch_bounds__(kMaxWarps* kWarp) block_forward_kernel(BlockArgs<T> args, T* __restrict__ xyz, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  using S = R;
  using V = LaneOf<R, kC>;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const size_t region = block_region_bytes<T>(N, false);
  ChainViews<T, kC> cv;
  T* out[kC];
  bool valid[kC];
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t chain = cta_chain<kC>(c, geo.batch, valid[c]);
    const T* Lr = args.lengths + chain * (N - 1);
    const T* Ar = args.angles + chain * (N - 2);
    const T* Dr = args.dihedrals + chain * (N - 3);
    out[c] = xyz + chain * 3 * N;
    unsigned char* base = smem + c * region;
    if constexpr (kScatter) {
      cv.X[c] = reinterpret_cast<R*>(base + (reinterpret_cast<uintptr_t>(out[c]) & 15u));
      scatter_block_inputs<T>(reinterpret_cast<T*>(cv.X[c]), Lr, Ar, Dr, N, tid, nthr);
    } else {
      cv.X[c] = reinterpret_cast<R*>(base);
      unsigned char* p = base + slot_bytes(N, sizeof(R));
      cv.row[c][0] = stage_row_async(p, Lr, N - 1, tid, nthr);
      p += staged_row_bytes(N - 1, sizeof(T));
      cv.row[c][1] = stage_row_async(p, Ar, N - 2, tid, nthr);
      p += staged_row_bytes(N - 2, sizeof(T));
      cv.row[c][2] = stage_row_async(p, Dr, N - 3, tid, nthr);
    }
  }
  const AnchorFrame<S> af = anchor_frame<S>(args.p0, args.first_direction, args.initial_normal);
  cp_async_wait_all();
  __syncthreads();

  V F[9], p2[3];
  {
    V l0, l1, a0;
    if constexpr (kScatter) {
      l0 = cv.slot(3);
      l1 = cv.slot(6);
      a0 = cv.slot(7);
    } else {
      l0 = cv.staged(0, 0);
      l1 = cv.staged(0, 1);
      a0 = cv.staged(1, 0);
    }
    const ChainFrame<V> ff = chain_frame<V>(af, l0, l1, a0);
#pragma unroll
    for (int i = 0; i < 9; ++i) F[i] = ff.F[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) p2[i] = ff.p2[i];
    if constexpr (kScatter) __syncthreads();  // every thread has read l0, l1, a0 from atom slots 1, 2
    if (tid == 0) {
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        cv.set_slot(i, splat<V>(af.p0[i]));
        cv.set_slot(3 + i, ff.p1[i]);
        cv.set_slot(6 + i, ff.p2[i]);
      }
    }
  }

  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T, kC>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };

  const StepRange range = step_range(tid, K, St);
  const Affine<V> total = sweep_local_prefix<T, kC, V>(cv, range, step);
  const Affine<V> carry = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  apply_carry<T, kC, V>(cv, carry, F, p2, range);

  if constexpr (kScatter) {
    fence_proxy_async_smem();
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      if (valid[c]) store_row_bulk<T>(out[c], reinterpret_cast<const T*>(cv.X[c]), 3 * N, tid, nthr, c);
    }
    if (tid < kC) bulk_store_wait_read();
  } else {
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      if (!valid[c]) continue;
#pragma unroll 4
      for (int e = tid; e < 3 * N; e += nthr) out[c][e] = from_r<T>(cv.X[c][e]);
    }
  }
}

// Sweep 1 of the block backward in world coordinates (orthonormal base frame): thread total of the
// local prefix, of g and of Q = sum p (x) g with p the local position.
template <typename T, int kC, typename V, typename StepFn>
__device__ __forceinline__ Affine<V> sweep_backward_totals_world(const ChainViews<T, kC>& cv, StepRange r, StepFn step, V (&gsum)[3], V (&Q)[9]) {
  Affine<V> P = affine_identity<V>();
#pragma unroll
  for (int i = 0; i < 3; ++i) gsum[i] = splat<V>(0);
#pragma unroll
  for (int i = 0; i < 9; ++i) Q[i] = splat<V>(0);
  int off = 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, off += 3) {
    advance(P, step(r.first + k));
    const V g[3] = {cv.grad(off), cv.grad(off + 1), cv.grad(off + 2)};
#pragma unroll
    for (int c = 0; c < 3; ++c) gsum[c] = vadd(gsum[c], g[c]);
#pragma unroll
    for (int d = 0; d < 3; ++d) {
#pragma unroll
      for (int c = 0; c < 3; ++c) Q[3 * d + c] = vfma(P.v[d], g[c], Q[3 * d + c]);
    }
  }
  return P;
}

// Sweep 2 of the block backward: prefix from the carry, gradients from the running suffix.
// kWorld: carry, positions and gradients in world coordinates (orthonormal base frame).
// Otherwise base-frame coordinates with g~ = F^T g, plus the per-step first-frame term `acc`
// (sum_j (g~_j.av) x~_j[0] + (g~_j.bv) x~_j[1]) that a non-orthonormal frame needs.
template <bool kWorld, typename T, int kC, typename V, typename StepFn>
__device__ __forceinline__ V block_backward_sweep2(const ChainViews<T, kC>& cv, const V* F, const Affine<V>& carry, V* Fs, V* Ms, const V* av,
                                                   const V* bv, StepRange r, StepFn step) {
  Affine<V> P = carry;
  V acc = splat<V>(0);
  int off = 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, off += 3) {
    const V u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
    const V xp[3] = {P.v[0], P.v[1], P.v[2]};
    advance(P, step(r.first + k));
    V g[3];
    if constexpr (kWorld) {
      g[0] = cv.grad(off);
      g[1] = cv.grad(off + 1);
      g[2] = cv.grad(off + 2);
    } else {
      base_grad<T, kC, V>(cv, off, F, g);
    }
    // tau = Ms - xp x Fs
    V xf[3];
    cross3(xp, Fs, xf);
    const V tau[3] = {vsub(Ms[0], xf[0]), vsub(Ms[1], xf[1]), vsub(Ms[2], xf[2])};
    const V d_phi = vfma(u2, tau[2], vfma(u1, tau[1], vmul(u0, tau[0])));
    const V d_theta = vneg(vfma(P.m[8], tau[2], vfma(P.m[5], tau[1], vmul(P.m[2], tau[0]))));
    const V d_len = vfma(P.m[6], Fs[2], vfma(P.m[3], Fs[1], vmul(P.m[0], Fs[0])));
    V mx[3];
    cross3(P.v, g, mx);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] = vsub(Fs[i], g[i]);
      Ms[i] = vsub(Ms[i], mx[i]);
    }
    if constexpr (!kWorld) {
      acc = vfma(dot3(g, av), P.v[0], acc);
      acc = vfma(dot3(g, bv), P.v[1], acc);
    }
    cv.set_slot(off, d_len);
    cv.set_slot(off + 1, d_theta);
    cv.set_slot(off + 2, d_phi);
  }
  return acc;
}

// The body of the block backward after staging, for one coordinate choice (see sweep 2).
template <bool kWorld, typename T, int kC, typename V, typename StepFn>
__device__ __forceinline__ void block_backward_body(const ChainViews<T, kC>& cv, CtaExchange<V>& ex, const AnchorFrame<typename ComputeOf<T>::type>& af,
                                                    const ChainFrame<V>& ff, const V* av, const V* bv, V l1, const T* grad_xyz,
                                                    const int64_t* chain_of, int N, StepRange range, int nwarps, StepFn step) {
  using R = typename ComputeOf<T>::type;
  V gsum[3];
  V Q[9];
  Affine<V> carry;
  if constexpr (kWorld) {
    const Affine<V> total = sweep_backward_totals_world<T, kC, V>(cv, range, step, gsum, Q);
    Affine<V> base;  // the base frame (F, p2): world = base * chain-local prefix
#pragma unroll
    for (int i = 0; i < 9; ++i) base.m[i] = ff.F[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) base.v[i] = ff.p2[i];
    carry = compose(base, cta_exclusive_affine<V>(total, ex.warp_totals, nwarps));
  } else {
    const Affine<V> total = sweep_backward_totals<T, kC, V>(cv, ff.F, range, step, gsum, Q);
    carry = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  }
  V Fs[3], Ms[3];
  suffix_base<V>(carry, gsum, Q, ex, nwarps, Fs, Ms);
  // thread 0's suffix base covers every atom >= 3 (S_0 of the reference)
  const V F3[3] = {Fs[0], Fs[1], Fs[2]};
  const V M3[3] = {Ms[0], Ms[1], Ms[2]};
  V acc = block_backward_sweep2<kWorld, T, kC, V>(cv, ff.F, carry, Fs, Ms, av, bv, range, step);
  if constexpr (!kWorld) acc = cta_sum_to_thread0<V>(acc, ex.warp_red, nwarps);
  if (threadIdx.x == 0) {
    V g1[3], g2[3], grad_p2[3], d_dir[3], dir0[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      if constexpr (kC == 2) {
        g1[i] = make_float2(to_r<float>(grad_xyz[chain_of[0] * 3 * N + 3 + i]), to_r<float>(grad_xyz[chain_of[1] * 3 * N + 3 + i]));
        g2[i] = make_float2(to_r<float>(grad_xyz[chain_of[0] * 3 * N + 6 + i]), to_r<float>(grad_xyz[chain_of[1] * 3 * N + 6 + i]));
      } else {
        g1[i] = to_r<R>(grad_xyz[chain_of[0] * 3 * N + 3 + i]);
        g2[i] = to_r<R>(grad_xyz[chain_of[0] * 3 * N + 6 + i]);
      }
      dir0[i] = splat<V>(af.dir0[i]);
      d_dir[i] = vfma(ff.c0, splat<V>(af.turn0[i]), vmul(ff.s0, dir0[i]));
    }
    if constexpr (kWorld) {
      // sum_{j>=3} g_j is F3 in world coordinates; the z moment about p2 in base coordinates is
      // normal . (M3 - p2 x F3), and for an orthonormal frame the projection term is -bv[0] times it
      V pf[3];
      cross3(ff.p2, F3, pf);
      const V m_about_p2[3] = {vsub(M3[0], pf[0]), vsub(M3[1], pf[1]), vsub(M3[2], pf[2])};
      acc = vneg(vmul(bv[0], dot3(ff.normal, m_about_p2)));
#pragma unroll
      for (int i = 0; i < 3; ++i) grad_p2[i] = vadd(g2[i], F3[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 3; ++i) grad_p2[i] = vfma(ff.F[3 * i + 2], F3[2], vfma(ff.F[3 * i + 1], F3[1], vfma(ff.F[3 * i + 0], F3[0], g2[i])));
    }
    V g12[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) g12[i] = vadd(g1[i], grad_p2[i]);
    cv.set_slot(3, dot3(g12, dir0));
    cv.set_slot(6, dot3(grad_p2, ff.dir1));
    cv.set_slot(7, vfma(l1, dot3(grad_p2, d_dir), acc));
  }
}

template <typename T, int kC>
__global__ void __launch_bounds__(kMaxWarps* kWarp) block_backward_kernel(BlockArgs<T> args, const T* __restrict__ grad_xyz,
                                                                         T* __restrict__ grad_lengths, T* __restrict__ grad_angles,
                                                                         T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  using S = R;
  using V = LaneOf<R, kC>;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const size_t region = block_region_bytes<T>(N, true);
  ChainViews<T, kC> cv;
  int64_t chain_of[kC];
  bool valid[kC];
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t chain = cta_chain<kC>(c, geo.batch, valid[c]);
    chain_of[c] = chain;
    const T* Lr = args.lengths + chain * (N - 1);
    const T* Ar = args.angles + chain * (N - 2);
    const T* Dr = args.dihedrals + chain * (N - 3);
    unsigned char* p = smem + c * region;
    cv.X[c] = reinterpret_cast<R*>(p);
    p += slot_bytes(N, sizeof(R));
    if constexpr (kScatter) {
      scatter_block_inputs<T>(reinterpret_cast<T*>(cv.X[c]), Lr, Ar, Dr, N, tid, nthr);
    } else {
      cv.row[c][0] = stage_row_async(p, Lr, N - 1, tid, nthr);
      p += staged_row_bytes(N - 1, sizeof(T));
      cv.row[c][1] = stage_row_async(p, Ar, N - 2, tid, nthr);
      p += staged_row_bytes(N - 2, sizeof(T));
      cv.row[c][2] = stage_row_async(p, Dr, N - 3, tid, nthr);
      p += staged_row_bytes(N - 3, sizeof(T));
    }
    cv.G[c] = stage_row_async(p, grad_xyz + chain * 3 * N, 3 * N, tid, nthr);
  }
  const AnchorFrame<S> af = anchor_frame<S>(args.p0, args.first_direction, args.initial_normal);
  cp_async_wait_all();
  __syncthreads();

  V l0, l1, a0;
  if constexpr (kScatter) {
    l0 = cv.slot(3);
    l1 = cv.slot(6);
    a0 = cv.slot(7);
  } else {
    l0 = cv.staged(0, 0);
    l1 = cv.staged(0, 1);
    a0 = cv.staged(1, 0);
  }
  const ChainFrame<V> ff = chain_frame<V>(af, l0, l1, a0);
  // projections of write_first_frame_param_grads (block.cu:224-227) in base coordinates
  V av[3], bv[3];
  {
    V d_dir[3], d_side[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) d_dir[i] = vfma(ff.c0, splat<V>(af.turn0[i]), vmul(ff.s0, splat<V>(af.dir0[i])));
    cross3(ff.normal, d_dir, d_side);
    to_base(ff.F, d_dir[0], d_dir[1], d_dir[2], av);
    to_base(ff.F, d_side[0], d_side[1], d_side[2], bv);
  }
  // For an orthonormal right-handed F, av = -sigma e_y and bv = sigma e_x (sigma = sign sin a0): the
  // whole backward can then run in world coordinates.  Otherwise (degenerate anchors or a collinear
  // first angle) it runs in base coordinates with the reference's general first-frame term.
  bool general = false;
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const S tol = static_cast<S>(1e-5);
    const S a0_ = lane(av[0], c), a1_ = lane(av[1], c), a2_ = lane(av[2], c);
    const S b0_ = lane(bv[0], c), b1_ = lane(bv[1], c), b2_ = lane(bv[2], c);
    const S dev = fabs(a0_) + fabs(a2_) + fabs(b1_) + fabs(b2_) + fabs(a1_ + b0_);
    general = general || !(dev <= tol && fabs(b0_) >= static_cast<S>(0.5));
  }

  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T, kC>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };

  const StepRange range = step_range(tid, K, St);
  if (general) {
    block_backward_body<false, T, kC, V>(cv, ex, af, ff, av, bv, l1, grad_xyz, chain_of, N, range, nwarps, step);
  } else {
    block_backward_body<true, T, kC, V>(cv, ex, af, ff, av, bv, l1, grad_xyz, chain_of, N, range, nwarps, step);
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    if (!valid[c]) continue;
    const int64_t chain = chain_of[c];
    T* gl = grad_lengths + chain * (N - 1);
    T* ga = grad_angles + chain * (N - 2);
    T* gd = grad_dihedrals + chain * (N - 3);
    const R* X = cv.X[c];
#pragma unroll 2
    for (int i = tid; i < N - 1; i += nthr) {
      const R* slot = X + 3 * i;
      gl[i] = from_r<T>(slot[3]);
      if (i < N - 2) ga[i] = from_r<T>(slot[7]);
      if (i < N - 3) gd[i] = from_r<T>(slot[11]);
    }
  }
}

// --------------------------------------------------------------------------------------------
// torsion-only path
// --------------------------------------------------------------------------------------------

// Fixed base frame of the torsion path (make_default_base_frame, torsion.cu:149-166).
template <typename V, typename R>
__device__ __forceinline__ void torsion_base(const TorsionConsts<R>& c, V* F, V* p1, V* p2) {
  const R s = c.sin_a[0], co = c.cos_a[0];
  // columns dir1 = (-c, s, 0), side = (-s, -c, 0), normal = (0, 0, 1)
  const R f[9] = {-co, -s, R(0), s, -co, R(0), R(0), R(0), R(1)};
#pragma unroll
  for (int i = 0; i < 9; ++i) F[i] = splat<V>(f[i]);
  p1[0] = splat<V>(c.length[0]);
  p1[1] = splat<V>(R(0));
  p1[2] = splat<V>(R(0));
  p2[0] = splat<V>(c.length[0] - c.length[1] * co);
  p2[1] = splat<V>(c.length[1] * s);
  p2[2] = splat<V>(R(0));
}

// |(s, c)|^2 clamped below at 1e-8f * 1e-8f (clamped_pair_norm2, torsion.cu:119-123)
template <typename V>
__device__ __forceinline__ V torsion_norm2(V s, V c) {
  const V n2 = vfma(s, s, vmul(c, c));
  return lanewise(n2, [](auto x) {
    using S = decltype(x);
    const S eps2 = static_cast<S>(1.0e-8f * 1.0e-8f);
    return x < eps2 ? eps2 : x;
  });
}
// 1/sqrt(n2): rsqrtf in float (the reference builds this path with fast math), 1/sqrt in double
template <typename V>
__device__ __forceinline__ V torsion_rinv(V n2) {
  return lanewise(n2, [](auto x) {
    if constexpr (std::is_same_v<decltype(x), float>) {
      return rsqrtf(x);
    } else {
      return 1.0 / sqrt(x);
    }
  });
}

// step s uses length phase (s+2)%3 and angle phase (s+1)%3 (torsion.cu:67-73, 219-236)
template <typename R>
__device__ __forceinline__ void torsion_constants_for(const TorsionConsts<R>& c, int s, R& l, R& st, R& ct) {
  const int ph = s % 3;
  l = ph == 0 ? c.length[2] : (ph == 1 ? c.length[0] : c.length[1]);
  st = ph == 0 ? c.sin_a[1] : (ph == 1 ? c.sin_a[2] : c.sin_a[0]);
  ct = ph == 0 ? c.cos_a[1] : (ph == 1 ? c.cos_a[2] : c.cos_a[0]);
}

template <typename T>
__device__ __forceinline__ void scatter_pairs(T* X, const T* raw, int S, int tid, int nthr) {
#pragma unroll 4
  for (int e = tid; e < 2 * S; e += nthr) cp_async<sizeof(T)>(X + 3 * ((e >> 1) + 3) + 1 + (e & 1), raw + e);
}

template <typename T, int kC>
__device__ __forceinline__ void torsion_pair(const ChainViews<T, kC>& cv, int s, LaneOf<typename ComputeOf<T>::type, kC>& rs,
                                             LaneOf<typename ComputeOf<T>::type, kC>& rc) {
  if constexpr (sizeof(T) >= 4) {
    rs = cv.slot(3 * (s + 3) + 1);
    rc = cv.slot(3 * (s + 3) + 2);
  } else {
    rs = cv.staged(0, 2 * s);
    rc = cv.staged(0, 2 * s + 1);
  }
}

template <typename T, int kC>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_forward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                           T* __restrict__ xyz, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  using V = LaneOf<R, kC>;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const size_t region = torsion_region_bytes<T>(N, false);
  ChainViews<T, kC> cv;
  T* out[kC];
  bool valid[kC];
  V F[9], p1[3], p2[3];
  torsion_base<V, R>(consts, F, p1, p2);
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t chain = cta_chain<kC>(c, geo.batch, valid[c]);
    const T* raw = raw_pairs + chain * raw_stride;
    out[c] = xyz + chain * 3 * N;
    unsigned char* base = smem + c * region;
    if constexpr (kScatter) {
      cv.X[c] = reinterpret_cast<R*>(base + (reinterpret_cast<uintptr_t>(out[c]) & 15u));
      scatter_pairs<T>(reinterpret_cast<T*>(cv.X[c]), raw, St, tid, nthr);
    } else {
      cv.X[c] = reinterpret_cast<R*>(base);
      cv.row[c][0] = stage_row_async(base + slot_bytes(N, sizeof(R)), raw, 2 * St, tid, nthr);
    }
  }
  if (tid == 0) {  // atom slots 0..2 receive no input
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      cv.set_slot(i, splat<V>(R(0)));
      cv.set_slot(3 + i, p1[i]);
      cv.set_slot(6 + i, p2[i]);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  auto step = [&](int s) {
    V rs, rc;
    torsion_pair<T, kC>(cv, s, rs, rc);
    const V rinv = torsion_rinv(torsion_norm2(rs, rc));
    R l, st, ct;
    torsion_constants_for(consts, s, l, st, ct);
    return step_rot(splat<V>(l), splat<V>(st), splat<V>(ct), vmul(rs, rinv), vmul(rc, rinv));
  };

  const StepRange range = step_range(tid, K, St);
  const Affine<V> total = sweep_local_prefix<T, kC, V>(cv, range, step);
  const Affine<V> carry = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  apply_carry<T, kC, V>(cv, carry, F, p2, range);

  if constexpr (kScatter) {
    fence_proxy_async_smem();
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      if (valid[c]) store_row_bulk<T>(out[c], reinterpret_cast<const T*>(cv.X[c]), 3 * N, tid, nthr, c);
    }
    if (tid < kC) bulk_store_wait_read();
  } else {
    __syncthreads();
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      if (!valid[c]) continue;
#pragma unroll 4
      for (int e = tid; e < 3 * N; e += nthr) out[c][e] = from_r<T>(cv.X[c][e]);
    }
  }
}

template <typename T, int kC>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_backward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                            const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  using V = LaneOf<R, kC>;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const size_t region = torsion_region_bytes<T>(N, true);
  ChainViews<T, kC> cv;
  int64_t chain_of[kC];
  bool valid[kC];
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int64_t chain = cta_chain<kC>(c, geo.batch, valid[c]);
    chain_of[c] = chain;
    const T* raw = raw_pairs + chain * raw_stride;
    unsigned char* p = smem + c * region;
    cv.X[c] = reinterpret_cast<R*>(p);
    p += slot_bytes(N, sizeof(R));
    if constexpr (kScatter) {
      scatter_pairs<T>(reinterpret_cast<T*>(cv.X[c]), raw, St, tid, nthr);
    } else {
      cv.row[c][0] = stage_row_async(p, raw, 2 * St, tid, nthr);
      p += staged_row_bytes(size_t(2) * St, sizeof(T));
    }
    cv.G[c] = stage_row_async(p, grad_xyz + chain * 3 * N, 3 * N, tid, nthr);
  }
  V F[9], p1[3], p2[3];
  torsion_base<V, R>(consts, F, p1, p2);
  cp_async_wait_all();
  __syncthreads();

  auto step = [&](int s) {
    V rs, rc;
    torsion_pair<T, kC>(cv, s, rs, rc);
    const V rinv = torsion_rinv(torsion_norm2(rs, rc));
    R l, st, ct;
    torsion_constants_for(consts, s, l, st, ct);
    return step_rot(splat<V>(l), splat<V>(st), splat<V>(ct), vmul(rs, rinv), vmul(rc, rinv));
  };

  const StepRange range = step_range(tid, K, St);
  V gsum[3];
  V Q[9];
  const Affine<V> total = sweep_backward_totals<T, kC, V>(cv, F, range, step, gsum, Q);
  const Affine<V> carry = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  V Fs[3], Ms[3];
  suffix_base<V>(carry, gsum, Q, ex, nwarps, Fs, Ms);

  Affine<V> P = carry;
  int off = 3 * (range.first + 3);
#pragma unroll 2
  for (int k = 0; k < range.count; ++k, off += 3) {
    const int s = range.first + k;
    const V u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
    const V nxp[3] = {vneg(P.v[0]), vneg(P.v[1]), vneg(P.v[2])};
    V rs, rc;
    torsion_pair<T, kC>(cv, s, rs, rc);
    const V n2 = torsion_norm2(rs, rc);
    const V rinv = torsion_rinv(n2);
    R l, st, ct;
    torsion_constants_for(consts, s, l, st, ct);
    advance(P, step_rot(splat<V>(l), splat<V>(st), splat<V>(ct), vmul(rs, rinv), vmul(rc, rinv)));
    V gt[3];
    base_grad<T, kC, V>(cv, off, F, gt);
    V tau[3];
    tau[0] = vfma(nxp[1], Fs[2], vfma(vneg(nxp[2]), Fs[1], Ms[0]));
    tau[1] = vfma(nxp[2], Fs[0], vfma(vneg(nxp[0]), Fs[2], Ms[1]));
    tau[2] = vfma(nxp[0], Fs[1], vfma(vneg(nxp[1]), Fs[0], Ms[2]));
    const V d_phi = vfma(u2, tau[2], vfma(u1, tau[1], vmul(u0, tau[0])));
    V mx[3];
    cross3(P.v, gt, mx);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] = vsub(Fs[i], gt[i]);
      Ms[i] = vsub(Ms[i], mx[i]);
    }
    // raw-pair chain rule (torsion.cu:173-182): d raw = d phi * (c, -s) / n2
    const V scale = lanewise(n2, [](auto x) { return decltype(x)(1) / x; });
    const V g = vmul(d_phi, scale);
    cv.set_slot(off + 1, vmul(rc, g));
    cv.set_slot(off + 2, vneg(vmul(rs, g)));
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    if (!valid[c]) continue;
    T* gr = grad_raw + chain_of[c] * grad_stride;
    const R* X = cv.X[c];
#pragma unroll 4
    for (int e = tid; e < 2 * St; e += nthr) gr[e] = from_r<T>(X[3 * ((e >> 1) + 3) + 1 + (e & 1)]);
  }
}

}  // namespace cufkb
