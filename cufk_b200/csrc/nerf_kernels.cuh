// sm_100a kernels for the cufk reconstruction path.
//
// block_forward_kernel    <- src/cufk/csrc/block.cu:157-204   (xyz from lengths/angles/dihedrals)
// block_backward_kernel   <- src/cufk/csrc/block.cu:206-313   (d lengths/angles/dihedrals)
// torsion_forward_kernel  <- src/cufk/csrc/torsion.cu:254-295 (xyz from raw (sin, cos) pairs)
// torsion_backward_kernel <- src/cufk/csrc/torsion.cu:297-381 (d raw pairs)
//
// One CTA per chain, W = blockDim.x / 32 warps, K (odd) consecutive steps per thread.
//
// Forward: stage the chain's inputs into atom slots (LDGSTS), sweep each thread's K steps
// sequentially from the identity (27 multiply-adds per step, the local prefix position written back
// into the slot), exclusive affine scan of the thread totals across the CTA, then
// x = p2 + F (C.v + C.m v) per slot in place and one bulk (TMA-engine) store of the (N, 3) row.
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
// the thread's moment total is C.v x G + axial(C.m Q) without revisiting its steps.  An
// exclusive suffix scan of (G, M) gives each thread the sums of all later threads; sweep 2
// recomputes the prefix from C, walks the running suffix down and writes the gradients into the
// slots in place.
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

// Shared memory of one CTA beyond the dynamic slots: scan exchange between warps.
template <typename R>
struct CtaExchange {
  Affine<R> warp_totals[kMaxWarps];
  R warp_sums[kMaxWarps * 6];  // suffix scan of (force, moment)
  R warp_red[kMaxWarps];       // first-frame reduction (separate: warps may still read warp_sums)
};

// --------------------------------------------------------------------------------------------
// shared-memory layout of one chain
// --------------------------------------------------------------------------------------------
// 4- and 8-byte types ("scatter"): [X slots, 3N elements of T, offset so that X has the residue of
//   the output row mod 16] [G staged grad row (backward)]
// 16-bit types: [X slots, 3N floats] [staged input rows (T)] [G staged grad row (backward)]
__host__ __device__ inline size_t slot_bytes(int points, size_t elem) { return staged_row_bytes(size_t(3) * points, elem); }

template <typename T>
__host__ __device__ inline size_t block_smem_bytes(int points, bool backward) {
  using R = typename ComputeOf<T>::type;
  size_t bytes = slot_bytes(points, sizeof(R));
  if (sizeof(T) < 4) {
    bytes += staged_row_bytes(points - 1, sizeof(T)) + staged_row_bytes(points - 2, sizeof(T)) +
             staged_row_bytes(points - 3, sizeof(T));
  }
  if (backward) bytes += staged_row_bytes(size_t(3) * points, sizeof(T));
  return bytes;
}

template <typename T>
__host__ __device__ inline size_t torsion_smem_bytes(int points, bool backward) {
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

// --------------------------------------------------------------------------------------------
// pieces shared by the four kernels
// --------------------------------------------------------------------------------------------

// Scatters one chain's block inputs into the slots with 4/8-byte LDGSTS.
template <typename T>
__device__ __forceinline__ void scatter_block_inputs(T* X, const T* Lr, const T* Ar, const T* Dr, int N, int tid, int nthr) {
#pragma unroll 2
  for (int i = tid; i < N - 1; i += nthr) {
    T* slot = X + 3 * i;
    cp_async<sizeof(T)>(slot + 3, Lr + i);
    if (i < N - 2) cp_async<sizeof(T)>(slot + 7, Ar + i);
    if (i < N - 3) cp_async<sizeof(T)>(slot + 11, Dr + i);
  }
}

// x = p2 + F (C.v + C.m v) for every slot the thread owns (in place).
template <typename R>
__device__ __forceinline__ void apply_carry(R* X, const Affine<R>& carry, const R* F, const R* p2, StepRange r) {
  R G[9];
  R h[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      G[3 * i + j] = F[3 * i + 0] * carry.m[0 + j] + F[3 * i + 1] * carry.m[3 + j] + F[3 * i + 2] * carry.m[6 + j];
    }
    h[i] = p2[i] + F[3 * i + 0] * carry.v[0] + F[3 * i + 1] * carry.v[1] + F[3 * i + 2] * carry.v[2];
  }
  R* slot = X + 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, slot += 3) {
    const R v0 = slot[0], v1 = slot[1], v2 = slot[2];
    slot[0] = h[0] + G[0] * v0 + G[1] * v1 + G[2] * v2;
    slot[1] = h[1] + G[3] * v0 + G[4] * v1 + G[5] * v2;
    slot[2] = h[2] + G[6] * v0 + G[7] * v1 + G[8] * v2;
  }
}

template <typename R>
__device__ __forceinline__ void write_head_points(R* X, const R* p0, const R* p1, const R* p2) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    X[i] = p0[i];
    X[3 + i] = p1[i];
    X[6 + i] = p2[i];
  }
}

// Writes the slot array (3N values in R) to the output row.  Scatter types hold final T values
// with the row's residue mod 16, so the row leaves in one bulk store; 16-bit types convert.
template <typename T, typename R>
__device__ __forceinline__ void store_xyz_row(T* out, R* X, int points, int tid, int nthr) {
  if constexpr (sizeof(T) >= 4) {
    fence_proxy_async_smem();
    __syncthreads();
    store_row_bulk<T>(out, reinterpret_cast<const T*>(X), 3 * points, tid, nthr);
  } else {
    __syncthreads();
#pragma unroll 4
    for (int e = tid; e < 3 * points; e += nthr) out[e] = from_r<T>(X[e]);
  }
}

// Sweep 1 of the forward: local prefix positions into the slots; returns the thread total.
template <typename R, typename StepFn>
__device__ __forceinline__ Affine<R> sweep_local_prefix(R* X, StepRange r, StepFn step) {
  Affine<R> P = affine_identity<R>();
  R* slot = X + 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, slot += 3) {
    R l, st, ct, sp, cp;
    step(r.first + k, l, st, ct, sp, cp);
    advance(P, l, st, ct, sp, cp);
    slot[0] = P.v[0];
    slot[1] = P.v[1];
    slot[2] = P.v[2];
  }
  return P;
}

// g~ = F^T g
template <typename R>
__device__ __forceinline__ void to_base(const R* F, R g0, R g1, R g2, R* out) {
  out[0] = F[0] * g0 + F[3] * g1 + F[6] * g2;
  out[1] = F[1] * g0 + F[4] * g1 + F[7] * g2;
  out[2] = F[2] * g0 + F[5] * g1 + F[8] * g2;
}

// Sweep 1 of the backward: thread total of the prefix, of g~ and of Q = sum p (x) g~.  When the
// staged gradient row is in the compute type, g~ replaces g in place for sweep 2.
template <typename R, typename T, typename StepFn>
__device__ __forceinline__ Affine<R> sweep_backward_totals(T* Grow, const R* F, StepRange r, StepFn step, R (&gsum)[3], R (&Q)[9]) {
  Affine<R> P = affine_identity<R>();
#pragma unroll
  for (int i = 0; i < 3; ++i) gsum[i] = R(0);
#pragma unroll
  for (int i = 0; i < 9; ++i) Q[i] = R(0);
  T* g = Grow + 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, g += 3) {
    R l, st, ct, sp, cp;
    step(r.first + k, l, st, ct, sp, cp);
    advance(P, l, st, ct, sp, cp);
    R gt[3];
    to_base(F, to_r<R>(g[0]), to_r<R>(g[1]), to_r<R>(g[2]), gt);
    if constexpr (std::is_same_v<T, R>) {
      g[0] = gt[0];
      g[1] = gt[1];
      g[2] = gt[2];
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) gsum[c] += gt[c];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
#pragma unroll
      for (int c = 0; c < 3; ++c) Q[3 * d + c] += P.v[d] * gt[c];
    }
  }
  return P;
}

// g~ of atom slot `g` in sweep 2 (stored by sweep 1 for the compute type, recomputed otherwise).
template <typename R, typename T>
__device__ __forceinline__ void base_grad(const T* g, const R* F, R* gt) {
  if constexpr (std::is_same_v<T, R>) {
    gt[0] = g[0];
    gt[1] = g[1];
    gt[2] = g[2];
  } else {
    to_base(F, to_r<R>(g[0]), to_r<R>(g[1]), to_r<R>(g[2]), gt);
  }
}

// Thread's moment total from its carry: C.v x G + axial(C.m Q).
template <typename R>
__device__ __forceinline__ void moment_total(const Affine<R>& C, const R (&gsum)[3], const R (&Q)[9], R* M) {
  R H[9];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) H[3 * i + j] = C.m[3 * i + 0] * Q[0 + j] + C.m[3 * i + 1] * Q[3 + j] + C.m[3 * i + 2] * Q[6 + j];
  }
  cross3(C.v, gsum, M);
  M[0] += H[5] - H[7];
  M[1] += H[6] - H[2];
  M[2] += H[1] - H[3];
}

// Suffix sums (force, moment) over all atoms from this thread's first step on.
template <typename R>
__device__ __forceinline__ void suffix_base(const Affine<R>& carry, const R (&gsum)[3], const R (&Q)[9], CtaExchange<R>& ex, int nwarps,
                                            R* Fs, R* Ms) {
  R mlane[3];
  moment_total<R>(carry, gsum, Q, mlane);
  R mine[6] = {gsum[0], gsum[1], gsum[2], mlane[0], mlane[1], mlane[2]};
  R after[6];
  cta_exclusive_suffix<R, 6>(mine, after, ex.warp_sums, nwarps);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    Fs[i] = after[i] + gsum[i];
    Ms[i] = after[3 + i] + mlane[i];
  }
}

// --------------------------------------------------------------------------------------------
// block path
// --------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp) block_forward_kernel(BlockArgs<T> args, T* __restrict__ xyz, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<R> ex;

  const int N = geo.points, S = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* Lr = args.lengths + chain * (N - 1);
  const T* Ar = args.angles + chain * (N - 2);
  const T* Dr = args.dihedrals + chain * (N - 3);
  T* out = xyz + chain * 3 * N;

  R* X;
  const T* Ls = nullptr;
  const T* As = nullptr;
  const T* Ds = nullptr;
  if constexpr (kScatter) {
    X = reinterpret_cast<R*>(smem + (reinterpret_cast<uintptr_t>(out) & 15u));
    scatter_block_inputs<T>(reinterpret_cast<T*>(X), Lr, Ar, Dr, N, tid, nthr);
  } else {
    unsigned char* p = smem;
    X = reinterpret_cast<R*>(p);
    p += slot_bytes(N, sizeof(R));
    Ls = stage_row_async(p, Lr, N - 1, tid, nthr);
    p += staged_row_bytes(N - 1, sizeof(T));
    As = stage_row_async(p, Ar, N - 2, tid, nthr);
    p += staged_row_bytes(N - 2, sizeof(T));
    Ds = stage_row_async(p, Dr, N - 3, tid, nthr);
  }
  cp_async_wait_all();
  __syncthreads();

  R F[9], p2[3];
  {
    const R l0 = kScatter ? X[3] : to_r<R>(Ls[0]);
    const R l1 = kScatter ? X[6] : to_r<R>(Ls[1]);
    const R a0 = kScatter ? X[7] : to_r<R>(As[0]);
    const FirstFrame<R> ff = first_frame<R>(l0, l1, a0, args.p0, args.first_direction, args.initial_normal);
#pragma unroll
    for (int i = 0; i < 9; ++i) F[i] = ff.F[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) p2[i] = ff.p2[i];
    if constexpr (kScatter) __syncthreads();  // every thread has read l0, l1, a0 from atom slots 1, 2
    if (tid == 0) write_head_points<R>(X, ff.p0, ff.p1, ff.p2);
  }

  auto step = [&](int s, R& l, R& st, R& ct, R& sp, R& cp) {
    R th, ph;
    if constexpr (kScatter) {
      const R* slot = X + 3 * (s + 3);
      l = slot[0];
      th = slot[1];
      ph = slot[2];
    } else {
      l = to_r<R>(Ls[s + 2]);
      th = to_r<R>(As[s + 1]);
      ph = to_r<R>(Ds[s]);
    }
    sin_cos(th, st, ct);
    sin_cos(ph, sp, cp);
  };

  const StepRange range = step_range(tid, K, S);
  const Affine<R> total = sweep_local_prefix<R>(X, range, step);
  const Affine<R> carry = cta_exclusive_affine<R>(total, ex.warp_totals, nwarps);
  apply_carry<R>(X, carry, F, p2, range);
  store_xyz_row<T, R>(out, X, N, tid, nthr);
}

// Sweep 2 of the block backward.  `kGeneral` adds the first-frame term for a base frame that is not
// orthonormal (degenerate anchors or a collinear first angle); it is uniform over the CTA.
template <bool kGeneral, typename R, typename T, typename StepFn>
__device__ __forceinline__ R block_backward_sweep2(R* X, const T* Gs, const R* F, const Affine<R>& carry, R* Fs, R* Ms, const R* av,
                                                   const R* bv, StepRange r, StepFn step) {
  Affine<R> P = carry;
  R acc = R(0);
  R* slot = X + 3 * (r.first + 3);
  const T* g = Gs + 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, slot += 3, g += 3) {
    const R u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
    const R xp[3] = {P.v[0], P.v[1], P.v[2]};
    R l, st, ct, sp, cp;
    step(r.first + k, l, st, ct, sp, cp);
    advance(P, l, st, ct, sp, cp);
    R gt[3];
    base_grad<R, T>(g, F, gt);
    R tau[3];
    cross3(xp, Fs, tau);
#pragma unroll
    for (int i = 0; i < 3; ++i) tau[i] = Ms[i] - tau[i];
    const R d_phi = u0 * tau[0] + u1 * tau[1] + u2 * tau[2];
    const R d_theta = -(P.m[2] * tau[0] + P.m[5] * tau[1] + P.m[8] * tau[2]);
    const R d_len = P.m[0] * Fs[0] + P.m[3] * Fs[1] + P.m[6] * Fs[2];
    R mx[3];
    cross3(P.v, gt, mx);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] -= gt[i];
      Ms[i] -= mx[i];
    }
    if constexpr (kGeneral) {
      acc += (gt[0] * av[0] + gt[1] * av[1] + gt[2] * av[2]) * P.v[0] + (gt[0] * bv[0] + gt[1] * bv[1] + gt[2] * bv[2]) * P.v[1];
    }
    slot[0] = d_len;
    slot[1] = d_theta;
    slot[2] = d_phi;
  }
  return acc;
}

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp) block_backward_kernel(BlockArgs<T> args, const T* __restrict__ grad_xyz,
                                                                         T* __restrict__ grad_lengths, T* __restrict__ grad_angles,
                                                                         T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<R> ex;

  const int N = geo.points, S = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* Lr = args.lengths + chain * (N - 1);
  const T* Ar = args.angles + chain * (N - 2);
  const T* Dr = args.dihedrals + chain * (N - 3);
  const T* Gr = grad_xyz + chain * 3 * N;

  unsigned char* p = smem;
  R* X = reinterpret_cast<R*>(p);
  p += slot_bytes(N, sizeof(R));
  const T* Ls = nullptr;
  const T* As = nullptr;
  const T* Ds = nullptr;
  if constexpr (kScatter) {
    scatter_block_inputs<T>(reinterpret_cast<T*>(X), Lr, Ar, Dr, N, tid, nthr);
  } else {
    Ls = stage_row_async(p, Lr, N - 1, tid, nthr);
    p += staged_row_bytes(N - 1, sizeof(T));
    As = stage_row_async(p, Ar, N - 2, tid, nthr);
    p += staged_row_bytes(N - 2, sizeof(T));
    Ds = stage_row_async(p, Dr, N - 3, tid, nthr);
    p += staged_row_bytes(N - 3, sizeof(T));
  }
  T* Gs = stage_row_async(p, Gr, 3 * N, tid, nthr);
  cp_async_wait_all();
  __syncthreads();

  const R l0 = kScatter ? X[3] : to_r<R>(Ls[0]);
  const R l1 = kScatter ? X[6] : to_r<R>(Ls[1]);
  const R a0 = kScatter ? X[7] : to_r<R>(As[0]);
  R F[9];
  R av[3], bv[3];
  {
    const FirstFrame<R> ff = first_frame<R>(l0, l1, a0, args.p0, args.first_direction, args.initial_normal);
#pragma unroll
    for (int i = 0; i < 9; ++i) F[i] = ff.F[i];
    // projections of write_first_frame_param_grads (block.cu:224-227) in base coordinates
    R d_dir[3], d_side[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) d_dir[i] = ff.s0 * ff.dir0[i] + ff.c0 * ff.turn0[i];
    cross3(ff.normal, d_dir, d_side);
    to_base(F, d_dir[0], d_dir[1], d_dir[2], av);
    to_base(F, d_side[0], d_side[1], d_side[2], bv);
  }

  auto step = [&](int s, R& l, R& st, R& ct, R& sp, R& cp) {
    R th, ph;
    if constexpr (kScatter) {
      const R* slot = X + 3 * (s + 3);
      l = slot[0];
      th = slot[1];
      ph = slot[2];
    } else {
      l = to_r<R>(Ls[s + 2]);
      th = to_r<R>(As[s + 1]);
      ph = to_r<R>(Ds[s]);
    }
    sin_cos(th, st, ct);
    sin_cos(ph, sp, cp);
  };

  const StepRange range = step_range(tid, K, S);
  R gsum[3];
  R Q[9];
  const Affine<R> total = sweep_backward_totals<R, T>(Gs, F, range, step, gsum, Q);
  const Affine<R> carry = cta_exclusive_affine<R>(total, ex.warp_totals, nwarps);
  R Fs[3], Ms[3];
  suffix_base<R>(carry, gsum, Q, ex, nwarps, Fs, Ms);
  // thread 0's suffix base covers every atom >= 3 (S_0 of the reference)
  const R F3[3] = {Fs[0], Fs[1], Fs[2]};
  const R M3z = Ms[2];

  // For an orthonormal right-handed F, av = -sigma e_y and bv = sigma e_x (sigma = sign sin a0), so
  // sum_j (g~_j.av) x~_j[0] + (g~_j.bv) x~_j[1] = -bv[0] * M_z: no per-step term is needed.
  const R tol = static_cast<R>(1e-5);
  const bool general = !(abs_r(av[0]) + abs_r(av[2]) + abs_r(bv[1]) + abs_r(bv[2]) + abs_r(av[1] + bv[0]) <= tol &&
                         abs_r(bv[0]) >= static_cast<R>(0.5));
  R acc;
  if (general) {
    acc = block_backward_sweep2<true, R, T>(X, Gs, F, carry, Fs, Ms, av, bv, range, step);
  } else {
    acc = block_backward_sweep2<false, R, T>(X, Gs, F, carry, Fs, Ms, av, bv, range, step);
  }
  const R acc_total = general ? cta_sum_to_thread0<R>(acc, ex.warp_red, nwarps) : -bv[0] * M3z;
  if (tid == 0) {
    FirstFrame<R> ff = first_frame<R>(l0, l1, a0, args.p0, args.first_direction, args.initial_normal);
    R g1[3], g2[3], grad_p2[3], d_dir[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      g1[i] = to_r<R>(Gr[3 + i]);
      g2[i] = to_r<R>(Gr[6 + i]);
      d_dir[i] = ff.s0 * ff.dir0[i] + ff.c0 * ff.turn0[i];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) grad_p2[i] = g2[i] + F[3 * i + 0] * F3[0] + F[3 * i + 1] * F3[1] + F[3 * i + 2] * F3[2];
    X[3] = (g1[0] + grad_p2[0]) * ff.dir0[0] + (g1[1] + grad_p2[1]) * ff.dir0[1] + (g1[2] + grad_p2[2]) * ff.dir0[2];
    X[6] = dot3(grad_p2, ff.dir1);
    X[7] = l1 * dot3(grad_p2, d_dir) + acc_total;
  }
  __syncthreads();
  T* gl = grad_lengths + chain * (N - 1);
  T* ga = grad_angles + chain * (N - 2);
  T* gd = grad_dihedrals + chain * (N - 3);
#pragma unroll 2
  for (int i = tid; i < N - 1; i += nthr) {
    const R* slot = X + 3 * i;
    gl[i] = from_r<T>(slot[3]);
    if (i < N - 2) ga[i] = from_r<T>(slot[7]);
    if (i < N - 3) gd[i] = from_r<T>(slot[11]);
  }
}

// --------------------------------------------------------------------------------------------
// torsion-only path
// --------------------------------------------------------------------------------------------

// Fixed base frame of the torsion path (make_default_base_frame, torsion.cu:149-166).
template <typename R>
__device__ __forceinline__ void torsion_base(const TorsionConsts<R>& c, R* F, R* p1, R* p2) {
  const R s = c.sin_a[0], co = c.cos_a[0];
  // columns dir1 = (-c, s, 0), side = (-s, -c, 0), normal = (0, 0, 1)
  F[0] = -co;
  F[1] = -s;
  F[2] = R(0);
  F[3] = s;
  F[4] = -co;
  F[5] = R(0);
  F[6] = R(0);
  F[7] = R(0);
  F[8] = R(1);
  p1[0] = c.length[0];
  p1[1] = R(0);
  p1[2] = R(0);
  p2[0] = c.length[0] - c.length[1] * co;
  p2[1] = c.length[1] * s;
  p2[2] = R(0);
}

// (s, c) * rsqrt(max(s^2 + c^2, 1e-8f * 1e-8f)) (torsion.cu:119-141)
__device__ __forceinline__ float torsion_norm2(float s, float c) {
  const float n2 = s * s + c * c;
  constexpr float kEps2 = 1.0e-8f * 1.0e-8f;
  return n2 < kEps2 ? kEps2 : n2;
}
__device__ __forceinline__ double torsion_norm2(double s, double c) {
  const double n2 = s * s + c * c;
  constexpr double kEps2 = static_cast<double>(1.0e-8f * 1.0e-8f);
  return n2 < kEps2 ? kEps2 : n2;
}
__device__ __forceinline__ float torsion_rinv(float n2) { return rsqrtf(n2); }
__device__ __forceinline__ double torsion_rinv(double n2) { return 1.0 / sqrt(n2); }

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

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_forward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                           T* __restrict__ xyz, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<R> ex;

  const int N = geo.points, S = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* raw = raw_pairs + chain * raw_stride;
  T* out = xyz + chain * 3 * N;

  R* X;
  const T* Rs = nullptr;
  if constexpr (kScatter) {
    X = reinterpret_cast<R*>(smem + (reinterpret_cast<uintptr_t>(out) & 15u));
    scatter_pairs<T>(reinterpret_cast<T*>(X), raw, S, tid, nthr);
  } else {
    X = reinterpret_cast<R*>(smem);
    Rs = stage_row_async(smem + slot_bytes(N, sizeof(R)), raw, 2 * S, tid, nthr);
  }
  R F[9], p1[3], p2[3];
  torsion_base(consts, F, p1, p2);
  if (tid == 0) {
    const R zero[3] = {R(0), R(0), R(0)};
    write_head_points<R>(X, zero, p1, p2);  // atom slots 0..2 receive no input
  }
  cp_async_wait_all();
  __syncthreads();

  auto step = [&](int s, R& l, R& st, R& ct, R& sp, R& cp) {
    R rs, rc;
    if constexpr (kScatter) {
      rs = X[3 * (s + 3) + 1];
      rc = X[3 * (s + 3) + 2];
    } else {
      rs = to_r<R>(Rs[2 * s]);
      rc = to_r<R>(Rs[2 * s + 1]);
    }
    const R rinv = torsion_rinv(torsion_norm2(rs, rc));
    sp = rs * rinv;
    cp = rc * rinv;
    torsion_constants_for(consts, s, l, st, ct);
  };

  const StepRange range = step_range(tid, K, S);
  const Affine<R> total = sweep_local_prefix<R>(X, range, step);
  const Affine<R> carry = cta_exclusive_affine<R>(total, ex.warp_totals, nwarps);
  apply_carry<R>(X, carry, F, p2, range);
  store_xyz_row<T, R>(out, X, N, tid, nthr);
}

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_backward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                            const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride, ChainGeometry geo) {
  using R = typename ComputeOf<T>::type;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<R> ex;

  const int N = geo.points, S = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* raw = raw_pairs + chain * raw_stride;
  const T* Gr = grad_xyz + chain * 3 * N;

  unsigned char* p = smem;
  R* X = reinterpret_cast<R*>(p);
  p += slot_bytes(N, sizeof(R));
  const T* Rs = nullptr;
  if constexpr (kScatter) {
    scatter_pairs<T>(reinterpret_cast<T*>(X), raw, S, tid, nthr);
  } else {
    Rs = stage_row_async(p, raw, 2 * S, tid, nthr);
    p += staged_row_bytes(size_t(2) * S, sizeof(T));
  }
  T* Gs = stage_row_async(p, Gr, 3 * N, tid, nthr);
  cp_async_wait_all();
  __syncthreads();

  R F[9], p1[3], p2[3];
  torsion_base(consts, F, p1, p2);

  auto pair = [&](int s, R& rs, R& rc) {
    if constexpr (kScatter) {
      rs = X[3 * (s + 3) + 1];
      rc = X[3 * (s + 3) + 2];
    } else {
      rs = to_r<R>(Rs[2 * s]);
      rc = to_r<R>(Rs[2 * s + 1]);
    }
  };
  auto step = [&](int s, R& l, R& st, R& ct, R& sp, R& cp) {
    R rs, rc;
    pair(s, rs, rc);
    const R rinv = torsion_rinv(torsion_norm2(rs, rc));
    sp = rs * rinv;
    cp = rc * rinv;
    torsion_constants_for(consts, s, l, st, ct);
  };

  const StepRange range = step_range(tid, K, S);
  R gsum[3];
  R Q[9];
  const Affine<R> total = sweep_backward_totals<R, T>(Gs, F, range, step, gsum, Q);
  const Affine<R> carry = cta_exclusive_affine<R>(total, ex.warp_totals, nwarps);
  R Fs[3], Ms[3];
  suffix_base<R>(carry, gsum, Q, ex, nwarps, Fs, Ms);

  Affine<R> P = carry;
  R* slot = X + 3 * (range.first + 3);
  const T* g = Gs + 3 * (range.first + 3);
#pragma unroll 2
  for (int k = 0; k < range.count; ++k, slot += 3, g += 3) {
    const int s = range.first + k;
    const R u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
    const R xp[3] = {P.v[0], P.v[1], P.v[2]};
    R rs, rc;
    pair(s, rs, rc);
    const R n2 = torsion_norm2(rs, rc);
    const R rinv = torsion_rinv(n2);
    R l, st, ct;
    torsion_constants_for(consts, s, l, st, ct);
    advance(P, l, st, ct, rs * rinv, rc * rinv);
    R gt[3];
    base_grad<R, T>(g, F, gt);
    R tau[3];
    cross3(xp, Fs, tau);
#pragma unroll
    for (int i = 0; i < 3; ++i) tau[i] = Ms[i] - tau[i];
    const R d_phi = u0 * tau[0] + u1 * tau[1] + u2 * tau[2];
    R mx[3];
    cross3(P.v, gt, mx);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] -= gt[i];
      Ms[i] -= mx[i];
    }
    // raw-pair chain rule (torsion.cu:173-182): d raw = d phi * (c, -s) / n2
    const R scale = d_phi / n2;
    slot[1] = rc * scale;
    slot[2] = -rs * scale;
  }
  __syncthreads();
  T* gr = grad_raw + chain * grad_stride;
#pragma unroll 4
  for (int e = tid; e < 2 * S; e += nthr) gr[e] = from_r<T>(X[3 * ((e >> 1) + 3) + 1 + (e & 1)]);
}

}  // namespace cufkb
