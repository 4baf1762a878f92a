// sm_100a kernels for the cufk reconstruction path.
//
// block_forward_kernel          <- src/cufk/csrc/block.cu:157-204   (xyz from lengths/angles/dihedrals)
// block_backward_kernel         <- src/cufk/csrc/block.cu:206-313   (d lengths/angles/dihedrals)
// block_backward_xyz_kernel        the same gradients from the forward's xyz (no local transforms)
// torsion_forward_kernel        <- src/cufk/csrc/torsion.cu:254-295 (xyz from raw (sin, cos) pairs)
// torsion_backward_kernel       <- src/cufk/csrc/torsion.cu:297-381 (d raw pairs)
// torsion_backward_xyz_kernel      the same from the forward's xyz (as the reference's own does)
//
// One CTA reconstructs one chain with W = blockDim.x / 32 warps and K (odd) consecutive steps per
// thread.
//
// Forward: stage the chain's inputs into atom slots (LDGSTS), sweep each thread's K steps
// sequentially from the identity (the local prefix position written back into the slot), exclusive
// affine scan of the thread totals across the CTA, then x = p2 + F (C.v + C.m v) per slot in place
// and one bulk (TMA-engine) store of the (N, 3) row.
//
// Backward: the gradient of every parameter of step s follows from the force/moment suffix of the
// atoms it moves.  In world coordinates (P_s = (F, p2) L_0...L_s, x = P.v):
//   F_s = sum_{j >= s+3} g_j,  M_s = sum_{j >= s+3} x_j x g_j,  tau_s = M_s - x_{s+2} x F_s,
//   d dihedral[s]   =  P_{s-1}.col0 . tau_s   (rotation about the incoming bond)
//   d angle[s+1]    = -P_s.col2     . tau_s   (rotation about the frame normal)
//   d length[s+2]   =  P_s.col0     . F_s     (translation along the new bond)
// valid when the base frame F is orthonormal; otherwise the same formulas run in base-frame
// coordinates (x~ = P.v without (F, p2), g~ = F^T g), which is the derivative of the reference's
// forward for any F.  The first-frame terms (lengths[0..1], angles[0]) follow
// write_first_frame_param_grads (block.cu:206-228).
//   * Recompute form (block_backward_kernel, nothing saved): sweep 1 builds each thread's local
//     prefix, its sum of g and the 3x3 moment matrix Q = sum p (x) g (p = local position), so that
//     once the affine scan gives the thread's carry C its moment total is C.v x G + axial(C.m Q).
//   * xyz form (block_backward_xyz_kernel): the frame columns the formulas need are bond
//     directions and plane normals of the forward's xyz, so nothing is rebuilt from the inputs.
//   Either way an exclusive suffix scan of the thread sums gives each thread the sums of all later
//   threads, and sweep 2 recomputes the prefix from the carry, walks the running suffix down and
//   writes the gradients into the slots in place.
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

// The prefetches of a launch that overlaps the previous kernel ((B, N) batches, whose rows need no
// offsets from memory): the chain's three input rows (forward), or two (B, N, 3) rows (xyz backward:
// positions and grad).  Thread 0 of each chain, before it waits for the previous grid.
template <typename T>
__device__ __forceinline__ void prefetch_input_rows(const BlockArgs<T>& args, const ChainGeometry& g, int64_t chain) {
  if (chain >= g.batch) return;
  const ChainRows r = chain_rows(g, chain);
  prefetch_row_l2(args.lengths + r.lengths, sizeof(T) * (r.points - 1));
  prefetch_row_l2(args.angles + r.angles, sizeof(T) * (r.points - 2));
  prefetch_row_l2(args.dihedrals + r.dihedrals, sizeof(T) * (r.points - 3));
}

template <typename A, typename B>
__device__ __forceinline__ void prefetch_point_rows(const A* rows_a, const B* rows_b, const ChainGeometry& g, int64_t chain) {
  if (chain >= g.batch) return;
  const ChainRows r = chain_rows(g, chain);
  prefetch_row_l2(rows_a + r.xyz, sizeof(A) * 3 * r.points);
  prefetch_row_l2(rows_b + r.xyz, sizeof(B) * 3 * r.points);
}

template <typename R>
struct TorsionConsts {
  R length[3];  // bond lengths by phase, rounded to float first (torsion.cu:43-47)
  R sin_a[3];   // sin/cos of the bond angles by phase (torsion.cu:49-53)
  R cos_a[3];
};

// Shared memory of one CTA beyond the dynamic slots: scan exchange between warps.
template <typename V>
struct CtaExchange {
  Affine<V> warp_totals[kMaxWarps];
  V warp_sums[kMaxWarps * 6];  // suffix scan of (force, moment)
  V warp_red[kMaxWarps];       // first-frame reduction (separate: warps may still read warp_sums)
  V frame[12];                 // base frame F (row-major) and p2, built once by thread 0
};

// The chain's first frame from its anchors and (lengths[0], lengths[1], angles[0]), read from
// global memory (one thread per CTA builds it; the staged rows are still in flight).
template <typename T, typename V>
__device__ __forceinline__ ChainFrame<V> chain_frame_of(const BlockArgs<T>& args, const AnchorFrame<V>& af, const ChainRows& rows) {
  const V l0 = to_r<V>(args.lengths[rows.lengths]);
  const V l1 = to_r<V>(args.lengths[rows.lengths + 1]);
  const V a0 = to_r<V>(args.angles[rows.angles]);
  return chain_frame<V>(af, l0, l1, a0);
}

// --------------------------------------------------------------------------------------------
// shared-memory layout of one chain
// --------------------------------------------------------------------------------------------
// 4- and 8-byte types ("scatter"): [X slots, 3N elements of T, offset so that X has the residue of
//   the output row mod 16] [G staged grad row (backward)]; the xyz backward stages the forward's
//   xyz row where the slots would be
// 16-bit types: [X slots, 3N floats] [staged input rows (T)] [G staged grad row (backward)]
__host__ __device__ inline size_t slot_bytes(int points, size_t elem) { return staged_row_bytes(size_t(3) * points, elem); }

template <typename T>
__host__ __device__ inline size_t block_smem_bytes(int points, bool backward) {
  using R = typename ComputeOf<T>::type;
  size_t bytes = slot_bytes(points, sizeof(R));
  if (sizeof(T) < 4) {
    bytes += staged_row_bytes(points - 1, sizeof(T)) + staged_row_bytes(points - 2, sizeof(T)) + staged_row_bytes(points - 3, sizeof(T));
  }
  if (backward) bytes += staged_row_bytes(size_t(3) * points, sizeof(T));
  return bytes;
}

// The torsion xyz backward: the slots and the grad row of torsion_smem_bytes, and the raw row.
template <typename T>
__host__ __device__ inline size_t torsion_xyz_smem_bytes(int points) {
  return slot_bytes(points, sizeof(typename ComputeOf<T>::type)) + staged_row_bytes(size_t(3) * points, sizeof(T)) +
         staged_row_bytes(size_t(2) * (points - 3), sizeof(T));
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

// Shared-memory views of one chain.
template <typename T>
struct ChainViews {
  using R = typename ComputeOf<T>::type;
  R* X;               // atom slots
  const T* row[3];    // staged input rows of 16-bit types (lengths/angles/dihedrals or raw pairs)
  T* G;               // staged gradient row (backward)
  const T* Y;         // staged xyz row of the forward (xyz backward)

  __device__ __forceinline__ R slot(int off) const { return X[off]; }
  __device__ __forceinline__ void set_slot(int off, R v) const { X[off] = v; }
  __device__ __forceinline__ R staged(int which, int i) const { return to_r<R>(row[which][i]); }
  __device__ __forceinline__ R grad(int off) const { return to_r<R>(G[off]); }
  __device__ __forceinline__ void set_grad(int off, R v) const { G[off] = from_r<T>(v); }
  __device__ __forceinline__ R pos(int off) const { return to_r<R>(Y[off]); }
};

// Block path inputs of step s: (L[s+2], A[s+1], D[s]).
template <typename T>
__device__ __forceinline__ void block_step_inputs(const ChainViews<T>& cv, int s, typename ComputeOf<T>::type& l, typename ComputeOf<T>::type& th,
                                                  typename ComputeOf<T>::type& ph) {
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
  // the last two lengths and the last angle (indices N-3 and N-2 fall to two different threads)
  if (i < N - 1) cp_async<sizeof(T)>(X + 3 * i + 3, Lr + i);
  if (i < N - 2) cp_async<sizeof(T)>(X + 3 * i + 7, Ar + i);
}

// Stages a chain's inputs: scattered into the slots (4/8-byte types) or as rows (16-bit types, whose
// slots hold float results).  Returns the first free byte after the chain's input region.
template <typename T>
__device__ __forceinline__ unsigned char* stage_block_inputs(ChainViews<T>& cv, unsigned char* smem, const BlockArgs<T>& args, const ChainRows& rows,
                                                             uintptr_t slot_residue, int tid, int nthr) {
  using R = typename ComputeOf<T>::type;
  const int N = rows.points;
  const T* Lr = args.lengths + rows.lengths;
  const T* Ar = args.angles + rows.angles;
  const T* Dr = args.dihedrals + rows.dihedrals;
  cv.X = reinterpret_cast<R*>(smem + slot_residue);
  unsigned char* p = smem + slot_bytes(N, sizeof(R));
  if constexpr (sizeof(T) >= 4) {
    scatter_block_inputs<T>(reinterpret_cast<T*>(cv.X), Lr, Ar, Dr, N, tid, nthr);
  } else {
    cv.row[0] = stage_row_async(p, Lr, N - 1, tid, nthr);
    p += staged_row_bytes(N - 1, sizeof(T));
    cv.row[1] = stage_row_async(p, Ar, N - 2, tid, nthr);
    p += staged_row_bytes(N - 2, sizeof(T));
    cv.row[2] = stage_row_async(p, Dr, N - 3, tid, nthr);
    p += staged_row_bytes(N - 3, sizeof(T));
  }
  return p;
}

// World carry (F, p2) C: the frame in front of the thread's first step.
template <typename V>
__device__ __forceinline__ Affine<V> world_carry(const Affine<V>& carry, const V* F, const V* p2) {
  Affine<V> w;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      w.m[3 * i + j] = vfma(F[3 * i + 2], carry.m[6 + j], vfma(F[3 * i + 1], carry.m[3 + j], vmul(F[3 * i + 0], carry.m[0 + j])));
    }
    w.v[i] = vfma(F[3 * i + 2], carry.v[2], vfma(F[3 * i + 1], carry.v[1], vfma(F[3 * i + 0], carry.v[0], p2[i])));
  }
  return w;
}

// x = W.v + W.m v for every slot the thread owns (in place), W its world carry.
template <typename T, typename V>
__device__ __forceinline__ void apply_carry(const ChainViews<T>& cv, const Affine<V>& W, StepRange r) {
  int off = 3 * (r.first + 3);
#pragma unroll 4
  for (int k = 0; k < r.count; ++k, off += 3) {
    const V v0 = cv.slot(off), v1 = cv.slot(off + 1), v2 = cv.slot(off + 2);
    cv.set_slot(off + 0, vfma(W.m[2], v2, vfma(W.m[1], v1, vfma(W.m[0], v0, W.v[0]))));
    cv.set_slot(off + 1, vfma(W.m[5], v2, vfma(W.m[4], v1, vfma(W.m[3], v0, W.v[1]))));
    cv.set_slot(off + 2, vfma(W.m[8], v2, vfma(W.m[7], v1, vfma(W.m[6], v0, W.v[2]))));
  }
}

// Sweep 1 of the forward: local prefix positions into the slots; returns the thread total.
template <typename T, typename V, typename StepFn>
__device__ __forceinline__ Affine<V> sweep_local_prefix(const ChainViews<T>& cv, StepRange r, StepFn step) {
  Affine<V> P = affine_identity<V>();
  int off = 3 * (r.first + 3);
#pragma unroll 2  // 2, not 4: the inlined sine/cosine makes a 4-step body large enough to cost time
  for (int k = 0; k < r.count; ++k, off += 3) {
    advance(P, step(r.first + k));
    cv.set_slot(off, P.v[0]);
    cv.set_slot(off + 1, P.v[1]);
    cv.set_slot(off + 2, P.v[2]);
  }
  return P;
}

// Two floats rounded to a 16-bit type, packed low element first.
template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  uint32_t u;
  if constexpr (std::is_same_v<T, __half>) {
    const __half2 h = __floats2half2_rn(lo, hi);
    memcpy(&u, &h, sizeof u);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    memcpy(&u, &h, sizeof u);
  }
  return u;
}

// Residue mod 16 of the float slots of a 16-bit forward: the float32 output row's when there is
// one, else twice the 16-bit row's, so that the slots line up with the 16-bit row for
// store_half_row (and with a float32 row of the same shape, whose residue is that too).
__device__ __forceinline__ uintptr_t half_slot_residue(const void* out16, const float* out32) {
  return out32 != nullptr ? (reinterpret_cast<uintptr_t>(out32) & 15u) : ((2u * (reinterpret_cast<uintptr_t>(out16) & 15u)) & 15u);
}

// A 16-bit row from `count` floats in shared memory: where X + e and out + e line up (X at a
// 16-byte boundary where out is at an 8-byte one), four elements per thread and iteration (one
// 16-byte shared load, two packed roundings, one 8-byte global store; consecutive threads write
// consecutive 8 bytes); element by element at the ragged ends, and throughout when they do not.
template <typename T>
__device__ __forceinline__ void store_half_row(T* out, const float* X, int count, int tid, int nthr) {
  const uintptr_t o = reinterpret_cast<uintptr_t>(out);
  const int head = min(static_cast<int>(((8u - (o & 7u)) & 7u) / 2u), count);
  if ((reinterpret_cast<uintptr_t>(X + head) & 15u) != 0) {
#pragma unroll 4
    for (int e = tid; e < count; e += nthr) out[e] = from_r<T>(X[e]);
    return;
  }
  const int chunks = (count - head) / 4;
  const float4* src = reinterpret_cast<const float4*>(X + head);
  uint2* dst = reinterpret_cast<uint2*>(out + head);
#pragma unroll 4
  for (int c = tid; c < chunks; c += nthr) {
    const float4 v = src[c];
    dst[c] = make_uint2(pack_pair<T>(v.x, v.y), pack_pair<T>(v.z, v.w));
  }
  if (tid < head) out[tid] = from_r<T>(X[tid]);
  const int tail = head + 4 * chunks;
  if (tid < count - tail) out[tail + tid] = from_r<T>(X[tail + tid]);
}

// Writes the slot array (3N values in R) to the output row.  Scatter types hold final T values
// with the row's residue mod 16, so the row leaves in one bulk store; 16-bit types convert.
template <typename T, typename R>
__device__ __forceinline__ void store_xyz_row(T* out, const R* X, int N, int tid, int nthr) {
  if constexpr (sizeof(T) >= 4) {
    fence_proxy_async_smem();
    __syncthreads();
    store_row_bulk<T>(out, reinterpret_cast<const T*>(X), 3 * N, tid, nthr, 0);
    if (tid == 0) bulk_store_wait_read();
  } else {
    __syncthreads();
    store_half_row<T>(out, X, 3 * N, tid, nthr);
  }
}

// g~ = F^T g
template <typename V>
__device__ __forceinline__ void to_base(const V* F, V g0, V g1, V g2, V* out) {
  out[0] = vfma(F[6], g2, vfma(F[3], g1, vmul(F[0], g0)));
  out[1] = vfma(F[7], g2, vfma(F[4], g1, vmul(F[1], g0)));
  out[2] = vfma(F[8], g2, vfma(F[5], g1, vmul(F[2], g0)));
}

// Sweep 1 of the recompute backward: thread total of the local prefix, of g and of
// Q = sum p (x) g.  In base coordinates (kWorld false) g is g~ = F^T g, stored back in place for
// sweep 2 when the staged row is in the compute type.
template <bool kWorld, typename T, typename V, typename StepFn>
__device__ __forceinline__ Affine<V> sweep_backward_totals(const ChainViews<T>& cv, const V* F, StepRange r, StepFn step, V (&gsum)[3], V (&Q)[9]) {
  using R = typename ComputeOf<T>::type;
  Affine<V> P = affine_identity<V>();
#pragma unroll
  for (int i = 0; i < 3; ++i) gsum[i] = V(0);
#pragma unroll
  for (int i = 0; i < 9; ++i) Q[i] = V(0);
  int off = 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, off += 3) {
    advance(P, step(r.first + k));
    V g[3];
    if constexpr (kWorld) {
      g[0] = cv.grad(off);
      g[1] = cv.grad(off + 1);
      g[2] = cv.grad(off + 2);
    } else {
      to_base(F, cv.grad(off), cv.grad(off + 1), cv.grad(off + 2), g);
      if constexpr (std::is_same_v<T, R>) {
        cv.set_grad(off, g[0]);
        cv.set_grad(off + 1, g[1]);
        cv.set_grad(off + 2, g[2]);
      }
    }
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

// Suffix sums (force, moment) over all atoms from this thread's first step on, from the thread's own
// sums (gsum, msum).
template <typename V>
__device__ __forceinline__ void suffix_base(const V (&gsum)[3], const V* msum, CtaExchange<V>& ex, int nwarps, V* Fs, V* Ms) {
  V mine[6] = {gsum[0], gsum[1], gsum[2], msum[0], msum[1], msum[2]};
  V after[6];
  cta_exclusive_suffix<V, 6>(mine, after, ex.warp_sums, nwarps);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    Fs[i] = vadd(after[i], gsum[i]);
    Ms[i] = vadd(after[3 + i], msum[i]);
  }
}

// Sweep 2 of the block backward: prefix from the carry, gradients from the running suffix.
// kWorld: carry, positions and gradients in world coordinates.  Otherwise base-frame coordinates
// with g~ = F^T g, plus the per-step first-frame term `acc`
// (sum_j (g~_j.av) x~_j[0] + (g~_j.bv) x~_j[1]) that a non-orthonormal frame needs.
template <bool kWorld, typename T, typename V, typename StepFn>
__device__ __forceinline__ V block_backward_sweep2(const ChainViews<T>& cv, const V* F, const Affine<V>& carry, V* Fs, V* Ms, const V* av, const V* bv,
                                                   StepRange r, StepFn step) {
  using R = typename ComputeOf<T>::type;
  Affine<V> P = carry;
  V acc = V(0);
  int off = 3 * (r.first + 3);
#pragma unroll 2
  for (int k = 0; k < r.count; ++k, off += 3) {
    const V u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
    const V xp[3] = {P.v[0], P.v[1], P.v[2]};
    advance(P, step(r.first + k));
    V g[3];
    if constexpr (kWorld || std::is_same_v<T, R>) {
      g[0] = cv.grad(off);
      g[1] = cv.grad(off + 1);
      g[2] = cv.grad(off + 2);
    } else {
      to_base(F, cv.grad(off), cv.grad(off + 1), cv.grad(off + 2), g);
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

// First-frame quantities of the block backward shared by both forms.
template <typename V>
struct BackwardFrame {
  ChainFrame<V> ff;
  V av[3], bv[3];  // F^T d_dir and F^T (normal x d_dir) (block.cu:224-227)
  V l1;
  bool general;    // base frame not orthonormal: use base coordinates
};

template <typename V>
struct FirstFrame {
  AnchorFrame<V> af;
  BackwardFrame<V> bf;
};

template <typename V, typename S>
__device__ __forceinline__ BackwardFrame<V> backward_frame(const AnchorFrame<S>& af, V l0, V l1, V a0) {
  BackwardFrame<V> b;
  b.ff = chain_frame<V>(af, l0, l1, a0);
  b.l1 = l1;
  V d_dir[3], d_side[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) d_dir[i] = vfma(b.ff.c0, V(af.turn0[i]), vmul(b.ff.s0, V(af.dir0[i])));
  cross3(b.ff.normal, d_dir, d_side);
  to_base(b.ff.F, d_dir[0], d_dir[1], d_dir[2], b.av);
  to_base(b.ff.F, d_side[0], d_side[1], d_side[2], b.bv);
  // For an orthonormal right-handed F, av = -sigma e_y and bv = sigma e_x (sigma = sign sin a0).
  const V dev = fabs(b.av[0]) + fabs(b.av[2]) + fabs(b.bv[1]) + fabs(b.bv[2]) + fabs(b.av[1] + b.bv[0]);
  b.general = !(dev <= static_cast<V>(1e-5) && fabs(b.bv[0]) >= static_cast<V>(0.5));
  return b;
}

// Gradients of lengths[0], lengths[1] and angles[0] (write_first_frame_param_grads,
// block.cu:206-228) into atom slots 1 and 2, by thread 0.  F3 and M3 are the suffix sums over every
// atom >= 3 (world coordinates; kAboutP2: moments taken about p2) or F3 in base coordinates and
// `acc` the reduced first-frame term (base coordinates).
template <bool kWorld, typename T, typename V, bool kAboutP2 = false>
__device__ __forceinline__ void first_frame_grads(const ChainViews<T>& cv, const AnchorFrame<V>& af, const BackwardFrame<V>& bf, const T* grow, const V* F3,
                                                  const V* M3, V acc) {
  const ChainFrame<V>& ff = bf.ff;
  V g1[3], g2[3], grad_p2[3], d_dir[3], dir0[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    g1[i] = to_r<V>(grow[3 + i]);
    g2[i] = to_r<V>(grow[6 + i]);
    dir0[i] = af.dir0[i];
    d_dir[i] = vfma(ff.c0, V(af.turn0[i]), vmul(ff.s0, dir0[i]));
  }
  if constexpr (kWorld) {
    // the z moment about p2 in base coordinates is normal . (M3 - p2 x F3); for an orthonormal frame
    // the first-frame projection term is -bv[0] times it.  With kAboutP2, M3 is already about p2.
    V m_about_p2[3] = {M3[0], M3[1], M3[2]};
    if constexpr (!kAboutP2) {
      V pf[3];
      cross3(ff.p2, F3, pf);
#pragma unroll
      for (int i = 0; i < 3; ++i) m_about_p2[i] = vsub(M3[i], pf[i]);
    }
    acc = vneg(vmul(bf.bv[0], dot3(ff.normal, m_about_p2)));
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
  cv.set_slot(7, vfma(bf.l1, dot3(grad_p2, d_dir), acc));
}

// Recompute backward after staging, for one coordinate choice.
template <bool kWorld, typename T, typename V, typename StepFn>
__device__ __forceinline__ void block_backward_recompute(const ChainViews<T>& cv, CtaExchange<V>& ex, const AnchorFrame<V>& af, const BackwardFrame<V>& bf,
                                                      const T* grow, StepRange range, int nwarps, StepFn step) {
  V gsum[3];
  V Q[9];
  const Affine<V> total = sweep_backward_totals<kWorld, T, V>(cv, bf.ff.F, range, step, gsum, Q);
  Affine<V> carry = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  if constexpr (kWorld) carry = world_carry(carry, bf.ff.F, bf.ff.p2);
  V msum[3];
  moment_total<V>(carry, gsum, Q, msum);
  V Fs[3], Ms[3];
  suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);
  const V F3[3] = {Fs[0], Fs[1], Fs[2]};
  const V M3[3] = {Ms[0], Ms[1], Ms[2]};
  V acc = block_backward_sweep2<kWorld, T, V>(cv, bf.ff.F, carry, Fs, Ms, bf.av, bf.bv, range, step);
  if constexpr (!kWorld) acc = cta_sum_to_thread0<V>(acc, ex.warp_red, nwarps);
  if (threadIdx.x == 0) first_frame_grads<kWorld, T, V>(cv, af, bf, grow, F3, M3, acc);
}

// The base-coordinate form, for a base frame that is not orthonormal.
template <typename T, typename V, typename StepFn>
__device__ __forceinline__ void block_backward_general(const ChainViews<T>& cv, CtaExchange<V>& ex, const AnchorFrame<V>& af, const BackwardFrame<V>& bf,
                                                    const T* grow, StepRange range, int nwarps, StepFn step) {
  block_backward_recompute<false, T, V>(cv, ex, af, bf, grow, range, nwarps, step);
}

template <typename T>
__device__ __forceinline__ void write_block_grads(const ChainViews<T>& cv, T* grad_lengths, T* grad_angles, T* grad_dihedrals, const ChainRows& rows, int tid,
                                                  int nthr) {
  using R = typename ComputeOf<T>::type;
  const int N = rows.points;
  T* gl = grad_lengths + rows.lengths;
  T* ga = grad_angles + rows.angles;
  T* gd = grad_dihedrals + rows.dihedrals;
  const R* X = cv.X;
#pragma unroll 2
  for (int i = tid; i < N - 1; i += nthr) {
    const R* slot = X + 3 * i;
    gl[i] = from_r<T>(slot[3]);
    if (i < N - 2) ga[i] = from_r<T>(slot[7]);
    if (i < N - 3) gd[i] = from_r<T>(slot[11]);
  }
}

// --------------------------------------------------------------------------------------------
// block path
// --------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    block_forward_kernel(BlockArgs<T> args, T* __restrict__ xyz, ChainGeometry geo, float* __restrict__ xyz32) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, St = N - 3, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  T* out = xyz + rows.xyz;
  // 16-bit types: the float slots take half_slot_residue's residue (with xyz32, that row's, so that
  // they leave by bulk store too)
  float* out32 = (!kScatter && xyz32 != nullptr) ? xyz32 + rows.xyz : nullptr;
  ChainViews<T> cv;
  const uintptr_t residue = kScatter ? (reinterpret_cast<uintptr_t>(out) & 15u) : half_slot_residue(out, out32);
  stage_block_inputs<T>(cv, smem, args, rows, residue, tid, nthr);
  // thread 0 builds the first frame while the rows stage; the others read (F, p2) after the scan
  V first_points[9];
  if (tid == 0) {
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const ChainFrame<V> ff = chain_frame_of<T, V>(args, af, rows);
#pragma unroll
    for (int i = 0; i < 9; ++i) ex.frame[i] = ff.F[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      ex.frame[9 + i] = ff.p2[i];
      first_points[i] = af.p0[i];
      first_points[3 + i] = ff.p1[i];
      first_points[6 + i] = ff.p2[i];
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (tid == 0) {
    // atoms 0..2; their slots held lengths[0..1] and angles[0], which nothing else reads
#pragma unroll
    for (int i = 0; i < 9; ++i) cv.set_slot(i, first_points[i]);
  }

  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };

  const StepRange range = step_range(tid, K, St);
  const Affine<V> total = sweep_local_prefix<T, V>(cv, range, step);
  // ex.frame was written before the barrier that follows the staging
  const Affine<V> W = world_carry(cta_exclusive_affine<V>(total, ex.warp_totals, nwarps), ex.frame, ex.frame + 9);
  apply_carry<T, V>(cv, W, range);
  if constexpr (!kScatter) {
    if (out32 != nullptr) {
      // the float32 positions as well (the 16-bit xyz backward reads them)
      fence_proxy_async_smem();
      __syncthreads();
      store_row_bulk<float>(out32, reinterpret_cast<const float*>(cv.X), 3 * N, tid, nthr, 0);
      store_xyz_row<T, R>(out, cv.X, N, tid, nthr);
      if (tid == 0) bulk_store_wait_read();
      return;
    }
  }
  store_xyz_row<T, R>(out, cv.X, N, tid, nthr);
}

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp) block_backward_kernel(BlockArgs<T> args, const T* __restrict__ grad_xyz, T* __restrict__ grad_lengths,
                                                                         T* __restrict__ grad_angles, T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, St = N - 3, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const T* grow = grad_xyz + rows.xyz;
  ChainViews<T> cv;
  unsigned char* p = stage_block_inputs<T>(cv, smem, args, rows, 0, tid, nthr);
  cv.G = stage_row_async(p, grow, 3 * N, tid, nthr);
  // thread 0 builds the first frame from global memory while the rows stage; every thread reads it
  // from shared memory
  __shared__ FirstFrame<V> first;
  if (tid == 0) {
    const AnchorFrame<R> af0 = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const V l0 = to_r<V>(args.lengths[rows.lengths]);
    const V l1 = to_r<V>(args.lengths[rows.lengths + 1]);
    const V a0 = to_r<V>(args.angles[rows.angles]);
    first = FirstFrame<V>{af0, backward_frame<V>(af0, l0, l1, a0)};
  }
  cp_async_wait_all();
  __syncthreads();

  const AnchorFrame<V>& af = first.af;
  const BackwardFrame<V>& bf = first.bf;
  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };
  const StepRange range = step_range(tid, K, St);
  if (bf.general) {
    block_backward_general<T, V>(cv, ex, af, bf, grow, range, nwarps, step);
  } else {
    block_backward_recompute<true, T, V>(cv, ex, af, bf, grow, range, nwarps, step);
  }
  __syncthreads();
  write_block_grads<T>(cv, grad_lengths, grad_angles, grad_dihedrals, rows, tid, nthr);
}

// The xyz-form backward of one chain whose xyz (cv.Y) and grad row (cv.G) are staged in shared
// memory (slot_region and grad_region), with its first frame in `first`.  Leaves the three
// gradients in the slots cv.X points at: the grad row, or the slot region when the chain takes the
// recompute form.  restore_grad() puts the grad row back in shared memory for that form (the
// sweep may have written gradients over part of it before the chain was found degenerate): a
// restaging of the global row, or (fused consumer) a recomputation; the redo path waits for its
// copies and synchronises after it.
template <typename T, typename V, typename RestoreGrad>
__device__ __forceinline__ void backward_xyz_staged(ChainViews<T>& cv, CtaExchange<V>& ex, const FirstFrame<V>& first, const BlockArgs<T>& args,
                                                    const ChainRows& rows, unsigned char* slot_region, StepRange range, int nwarps,
                                                    RestoreGrad restore_grad) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const bool general = first.bf.general;  // uniform over the CTA
  bool redo = general;
  if (!redo) {
    // moments about o = p2 (the chain's own origin, atom 2 of the forward's xyz): the sums then lose
    // no precision to the chain's distance from the world origin
    const V o[3] = {cv.pos(6), cv.pos(7), cv.pos(8)};
    V gsum[3] = {V(0), V(0), V(0)};
    V msum[3] = {V(0), V(0), V(0)};
    V xmax2 = V(0);  // largest |x|^2 of the thread's atoms (world), for the short-bond test
    {
      const T* px = cv.Y + 3 * (range.first + 3);
      const T* pg = cv.G + 3 * (range.first + 3);
#pragma unroll 4
      for (int k = 0; k < range.count; ++k, px += 3, pg += 3) {
        const V g[3] = {to_r<V>(pg[0]), to_r<V>(pg[1]), to_r<V>(pg[2])};
        const V xw[3] = {to_r<V>(px[0]), to_r<V>(px[1]), to_r<V>(px[2])};
        xmax2 = fmax(xmax2, dot3(xw, xw));
        const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
        V mx[3];
        cross3(x, g, mx);
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          gsum[i] = vadd(gsum[i], g[i]);
          msum[i] = vadd(msum[i], mx[i]);
        }
      }
    }
    V Fs[3], Ms[3];
    suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);
    const V F3[3] = {Fs[0], Fs[1], Fs[2]};
    const V M3[3] = {Ms[0], Ms[1], Ms[2]};
    // sweep: x2 = x_{s+2} (world), up = u_{s+1}, tau = tau_s = sum_{j >= s+3} (x_j - x_{s+2}) x g_j,
    // carried from step to step as tau_{s+1} = tau_s - (x_{s+3} - x_{s+2}) x F_s.  Threads without
    // steps read nothing (their first step lies past the chain).
    V x2[3] = {V(0), V(0), V(0)};
    V up[3] = {V(0), V(0), V(0)};
    V tau[3] = {V(0), V(0), V(0)};
    V dmin2 = V(0);
    if (range.count > 0) {
      const int off = 3 * (range.first + 1);  // atoms first+1 and first+2 <= N-2
#pragma unroll
      for (int i = 0; i < 3; ++i) x2[i] = cv.pos(off + 3 + i);
      const V d[3] = {vsub(x2[0], cv.pos(off)), vsub(x2[1], cv.pos(off + 1)), vsub(x2[2], cv.pos(off + 2))};
      dmin2 = dot3(d, d);
      xmax2 = fmax(xmax2, dot3(x2, x2));
      const V inv = vrsqrt(dmin2);
#pragma unroll
      for (int i = 0; i < 3; ++i) up[i] = vmul(d[i], inv);
      const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
      V xf[3];
      cross3(xr, Fs, xf);
#pragma unroll
      for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
    }
    V wmin2 = V(1);
    {
      const T* px = cv.Y + 3 * (range.first + 3);
      T* pg = cv.G + 3 * (range.first + 3);
#pragma unroll 2
      for (int k = 0; k < range.count; ++k, px += 3, pg += 3) {
        const V x3[3] = {to_r<V>(px[0]), to_r<V>(px[1]), to_r<V>(px[2])};
        const V g[3] = {to_r<V>(pg[0]), to_r<V>(pg[1]), to_r<V>(pg[2])};
        const V d[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
        const V d2 = dot3(d, d);
        dmin2 = fmin(dmin2, d2);
        const V inv = vrsqrt(d2);
        const V uc[3] = {vmul(d[0], inv), vmul(d[1], inv), vmul(d[2], inv)};
        V w[3];
        cross3(up, uc, w);
        const V w2 = dot3(w, w);
        wmin2 = fmin(wmin2, w2);
        const V d_phi = dot3(up, tau);
        const V d_len = dot3(uc, Fs);
        const V d_theta = vneg(vmul(dot3(w, tau), vrsqrt(w2)));
        // tau -= d x Fs, then Fs -= g
        tau[0] = vfma(d[2], Fs[1], vfma(vneg(d[1]), Fs[2], tau[0]));
        tau[1] = vfma(d[0], Fs[2], vfma(vneg(d[2]), Fs[0], tau[1]));
        tau[2] = vfma(d[1], Fs[0], vfma(vneg(d[0]), Fs[1], tau[2]));
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          Fs[i] = vsub(Fs[i], g[i]);
          x2[i] = x3[i];
          up[i] = uc[i];
        }
        pg[0] = from_r<T>(d_len);
        pg[1] = from_r<T>(d_theta);
        pg[2] = from_r<T>(d_phi);
      }
    }
    // Positions are accurate to ~1 ulp of |x|, so a bond direction from them is good to
    // ~ulp(|x|) / |d|: bonds shorter than 1e-3 |x|max, a plane normal with sin^2 < 1e-2 (and any
    // non-finite value: the comparisons fail) send the chain to the recompute form.
    const bool bad = range.count > 0 && !(dmin2 >= static_cast<V>(1e-6) * xmax2 && wmin2 >= static_cast<V>(1e-2));
    redo = __syncthreads_or(bad) != 0;
    // g1, g2 from the staged grad row: slots 1 and 2 are not overwritten by the sweep
    if (!redo && tid == 0) first_frame_grads<true, T, V, true>(cv, first.af, first.bf, cv.G, F3, M3, V(0));
  }
  if (redo) {
    const AnchorFrame<V>& af = first.af;
    const BackwardFrame<V>& bf = first.bf;
    // recompute form, laid out as in block_backward_kernel: the grad row restored (the sweep may
    // have written gradients over part of it), then the inputs into the slots
    __syncthreads();
    restore_grad();
    stage_block_inputs<T>(cv, slot_region, args, rows, 0, tid, nthr);
    cp_async_wait_all();
    __syncthreads();
    auto step = [&](int s) {
      V l, th, ph, st, ct, sp, cp;
      block_step_inputs<T>(cv, s, l, th, ph);
      step_sincos(th, ph, st, ct, sp, cp);
      return step_rot(l, st, ct, sp, cp);
    };
    if (general) {
      block_backward_general<T, V>(cv, ex, af, bf, cv.G, range, nwarps, step);
    } else {
      block_backward_recompute<true, T, V>(cv, ex, af, bf, cv.G, range, nwarps, step);
    }
  }
}

// Backward from the forward's xyz (4- and 8-byte types, base frame orthonormal).  In world
// coordinates every gradient of step s needs only the positions around it and the suffix sums
// F_s = sum_{j >= s+3} g_j, M_s = sum_{j >= s+3} (x_j - o) x g_j (moments about the chain's own
// p2 = o, so that tau keeps its precision however far the chain is from the world origin):
//   u_b = (x_{b+1} - x_b) / |x_{b+1} - x_b|          (bond b; u_{s+1} = P_{s-1}.col0, u_{s+2} = P_s.col0)
//   P_s.col2 = (u_{s+1} x u_{s+2}) / sin(theta_s)    (the frame normal; |u_{s+1} x u_{s+2}| = sin theta_s)
// so no local transform is rebuilt: the chain's xyz and grad rows are staged (16-byte LDGSTS), each
// thread sums g and (x - o) x g over its atoms, an exclusive suffix scan gives the sums of all later
// threads, and one sweep up the thread's steps produces the three gradients, written over the
// grad row in place (step s only reads g_{s+3}, its own atom).  A chain is redone by the recompute
// form in the same CTA when its base frame is not orthonormal, when a bond is shorter than
// 1e-3 |x|max (its direction from rounded positions would be off by more than ~1e-4: a zero-length
// bond, or a chain far from the origin relative to its bond lengths), when a plane normal has
// sin^2 theta < 1e-2 (bond angle within ~6 degrees of 0 or pi), or when a value is not finite.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    block_backward_xyz_kernel(BlockArgs<T> args, const T* __restrict__ xyz, const T* __restrict__ grad_xyz, T* __restrict__ grad_lengths,
                              T* __restrict__ grad_angles, T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the xyz form serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, St = N - 3, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const T* grow = grad_xyz + rows.xyz;
  unsigned char* const slot_region = smem;
  unsigned char* const grad_region = smem + slot_bytes(N, sizeof(R));
  ChainViews<T> cv;
  cv.Y = stage_row_async(slot_region, xyz + rows.xyz, 3 * N, tid, nthr);
  cv.G = stage_row_async(grad_region, grow, 3 * N, tid, nthr);
  cv.X = cv.G;  // gradients go over the consumed grad row
  // thread 0 classifies the base frame while the rows stage; the first frame itself is only needed
  // again by thread 0 for the first-frame gradients (and by the recompute form)
  auto first_frame = [&]() {
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const R l0 = to_r<R>(args.lengths[rows.lengths]);
    const R l1 = to_r<R>(args.lengths[rows.lengths + 1]);
    const R a0 = to_r<R>(args.angles[rows.angles]);
    return FirstFrame<V>{af, backward_frame<V>(af, l0, l1, a0)};
  };
  // thread 0 builds the first frame while the rows stage and keeps it in shared memory for the
  // first-frame gradients at the end (no dependent global loads on the CTA's critical path there)
  __shared__ FirstFrame<V> first;
  if (tid == 0) first = first_frame();
  const StepRange range = step_range(tid, K, St);
  cp_async_wait_all();
  __syncthreads();

  auto restore_grad = [&]() { cv.G = stage_row_async(grad_region, grow, 3 * N, tid, nthr); };
  backward_xyz_staged<T, V>(cv, ex, first, args, rows, slot_region, range, nwarps, restore_grad);
  __syncthreads();
  write_block_grads<T>(cv, grad_lengths, grad_angles, grad_dihedrals, rows, tid, nthr);
}

// --------------------------------------------------------------------------------------------
// fused consumer: reconstruction, a coordinate loss and its backward in one CTA per chain
// --------------------------------------------------------------------------------------------
// loss[b] = (1/N) sum_j |x_j - t_j|^2 for the chain's xyz x (as block_forward_kernel builds it) and a
// target row t, and, when grad_lengths is not null, d loss[b] / d (lengths, angles, dihedrals) of
// the chain.  The chain never leaves shared memory: its inputs are staged into the slots and the
// target row into the grad region, the forward leaves x in the slots, one pass forms the loss and
// dL/dx = (2/N)(x - t) over the target row, and the xyz-form backward (backward_xyz_staged) turns
// that into the parameter gradients.  HBM traffic per atom (float32): 12 B of inputs + 12 B of
// target + 12 B of gradients, where the unfused chain (forward, a separate loss, backward) moves the
// xyz out and back in between.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    block_mse_kernel(BlockArgs<T> args, const T* __restrict__ target, T* __restrict__ loss, T* __restrict__ grad_lengths, T* __restrict__ grad_angles,
                     T* __restrict__ grad_dihedrals, ChainGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the fused consumer serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;
  __shared__ FirstFrame<V> first;

  const int64_t chain = blockIdx.x;
  const ChainRows rows = chain_rows(geo, chain);
  if (rows.points == 0) return;  // a packed chain outside [4, geo.points] (uniform over the CTA)
  const int N = rows.points, St = N - 3, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  unsigned char* const slot_region = smem;
  unsigned char* const grad_region = smem + slot_bytes(N, sizeof(R));
  const T* trow = target + rows.xyz;
  ChainViews<T> cv;
  stage_block_inputs<T>(cv, slot_region, args, rows, 0, tid, nthr);
  cv.G = stage_row_async(grad_region, trow, 3 * N, tid, nthr);
  if (tid == 0) {
    // the first frame from global memory while the rows stage (as the xyz backward builds it)
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const R l0 = to_r<R>(args.lengths[rows.lengths]);
    const R l1 = to_r<R>(args.lengths[rows.lengths + 1]);
    const R a0 = to_r<R>(args.angles[rows.angles]);
    first = FirstFrame<V>{af, backward_frame<V>(af, l0, l1, a0)};
  }
  cp_async_wait_all();
  __syncthreads();

  // forward: the operations of block_forward_kernel, xyz left in the slots
  const ChainFrame<V>& ff = first.bf.ff;
  if (tid == 0) {
    // atoms 0..2; their slots held lengths[0..1] and angles[0], which no step reads
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      cv.set_slot(i, first.af.p0[i]);
      cv.set_slot(3 + i, ff.p1[i]);
      cv.set_slot(6 + i, ff.p2[i]);
    }
  }
  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };
  const StepRange range = step_range(tid, K, St);
  const Affine<V> total = sweep_local_prefix<T, V>(cv, range, step);
  const Affine<V> W = world_carry(cta_exclusive_affine<V>(total, ex.warp_totals, nwarps), ff.F, ff.p2);
  apply_carry<T, V>(cv, W, range);
  __syncthreads();

  // loss and dL/dx = (2/N)(x - t) over the target row
  const V inv_n = V(1) / V(N);
  const V two_inv_n = V(2) * inv_n;
  auto make_grad = [&]() {
    V part = V(0);
    for (int e = tid; e < 3 * N; e += nthr) {
      const V d = vsub(cv.slot(e), to_r<V>(cv.G[e]));
      part = vfma(d, d, part);
      cv.G[e] = from_r<T>(vmul(two_inv_n, d));
    }
    return part;
  };
  const V sum = cta_sum_to_thread0<V>(make_grad(), ex.warp_red, nwarps);
  if (tid == 0) loss[chain] = from_r<T>(vmul(sum, inv_n));
  if (grad_lengths == nullptr) return;  // uniform over the CTA: the loss alone
  __syncthreads();

  // backward from x (in the slots) and dL/dx (over the target row)
  cv.Y = reinterpret_cast<const T*>(cv.X);
  cv.X = cv.G;
  auto restore_grad = [&]() {
    // the target again, and dL/dx from the positions, which are still in the slots
    stage_row_async(grad_region, trow, 3 * N, tid, nthr);
    cp_async_wait_all();
    __syncthreads();
    for (int e = tid; e < 3 * N; e += nthr) cv.G[e] = from_r<T>(vmul(two_inv_n, vsub(cv.pos(e), to_r<V>(cv.G[e]))));
    __syncthreads();
  };
  backward_xyz_staged<T, V>(cv, ex, first, args, rows, slot_region, range, nwarps, restore_grad);
  __syncthreads();
  write_block_grads<T>(cv, grad_lengths, grad_angles, grad_dihedrals, rows, tid, nthr);
}

// --------------------------------------------------------------------------------------------
// torsion-only path
// --------------------------------------------------------------------------------------------

// Fixed base frame of the torsion path (make_default_base_frame, torsion.cu:149-166).
template <typename V>
__device__ __forceinline__ void torsion_base(const TorsionConsts<V>& c, V* F, V* p1, V* p2) {
  const V s = c.sin_a[0], co = c.cos_a[0];
  // columns dir1 = (-c, s, 0), side = (-s, -c, 0), normal = (0, 0, 1)
  const V f[9] = {-co, -s, V(0), s, -co, V(0), V(0), V(0), V(1)};
#pragma unroll
  for (int i = 0; i < 9; ++i) F[i] = f[i];
  p1[0] = c.length[0];
  p1[1] = V(0);
  p1[2] = V(0);
  p2[0] = c.length[0] - c.length[1] * co;
  p2[1] = c.length[1] * s;
  p2[2] = V(0);
}

// |(s, c)|^2 clamped below at 1e-8f * 1e-8f (clamped_pair_norm2, torsion.cu:119-123)
template <typename V>
__device__ __forceinline__ V torsion_norm2(V s, V c) {
  const V n2 = vfma(s, s, vmul(c, c));
  const V eps2 = static_cast<V>(1.0e-8f * 1.0e-8f);
  return n2 < eps2 ? eps2 : n2;
}
// 1/sqrt(n2): rsqrtf in float (the reference builds this path with fast math), 1/sqrt in double
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
__device__ __forceinline__ void torsion_pair(const ChainViews<T>& cv, int s, typename ComputeOf<T>::type& rs, typename ComputeOf<T>::type& rc) {
  if constexpr (sizeof(T) >= 4) {
    rs = cv.slot(3 * (s + 3) + 1);
    rc = cv.slot(3 * (s + 3) + 2);
  } else {
    rs = cv.staged(0, 2 * s);
    rc = cv.staged(0, 2 * s + 1);
  }
}

// Sweep 1 of the torsion forward.  Step s takes its bond length and angle by phase (s % 3); the
// thread rotates the three constant triples once, to its first step's phase, and walks its steps
// three at a time, so that every step of an iteration uses fixed registers (no per-step modulo or
// selects).
// One step of the torsion forward sweep with its constants: local prefix advanced, its position
// written to the step's slot.
template <typename T, typename V, typename R>
__device__ __forceinline__ void torsion_sweep_step(const ChainViews<T>& cv, Affine<V>& P, int s, R l, R st, R ct) {
  V rs, rc;
  torsion_pair<T>(cv, s, rs, rc);
  const V rinv = torsion_rinv(torsion_norm2(rs, rc));
  advance(P, step_rot<V>(l, st, ct, vmul(rs, rinv), vmul(rc, rinv)));
  const int off = 3 * (s + 3);
  cv.set_slot(off, P.v[0]);
  cv.set_slot(off + 1, P.v[1]);
  cv.set_slot(off + 2, P.v[2]);
}

template <typename T, typename V, typename R>
__device__ __forceinline__ Affine<V> torsion_sweep(const ChainViews<T>& cv, StepRange r, const TorsionConsts<R>& consts) {
  R l0, l1, l2, s0, s1, s2, c0, c1, c2;
  torsion_constants_for(consts, r.first, l0, s0, c0);
  torsion_constants_for(consts, r.first + 1, l1, s1, c1);
  torsion_constants_for(consts, r.first + 2, l2, s2, c2);
  Affine<V> P = affine_identity<V>();
  int s = r.first;
  const int end = r.first + r.count;
#pragma unroll 1
  for (; s + 3 <= end; s += 3) {
    torsion_sweep_step<T, V, R>(cv, P, s, l0, s0, c0);
    torsion_sweep_step<T, V, R>(cv, P, s + 1, l1, s1, c1);
    torsion_sweep_step<T, V, R>(cv, P, s + 2, l2, s2, c2);
  }
  if (s < end) torsion_sweep_step<T, V, R>(cv, P, s, l0, s0, c0);
  if (s + 1 < end) torsion_sweep_step<T, V, R>(cv, P, s + 1, l1, s1, c1);
  return P;
}

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_forward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts, T* __restrict__ xyz,
                           ChainGeometry geo, float* __restrict__ xyz32) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* raw = raw_pairs + chain * raw_stride;
  T* out = xyz + chain * 3 * N;
  ChainViews<T> cv;
  if constexpr (kScatter) {
    cv.X = reinterpret_cast<R*>(smem + (reinterpret_cast<uintptr_t>(out) & 15u));
    scatter_pairs<T>(reinterpret_cast<T*>(cv.X), raw, St, tid, nthr);
  } else {
    // the float slots line up with out for store_half_row, and with xyz32's row when there is one
    cv.X = reinterpret_cast<R*>(smem + half_slot_residue(out, xyz32 != nullptr ? xyz32 + chain * 3 * N : nullptr));
    cv.row[0] = stage_row_async(smem + slot_bytes(N, sizeof(R)), raw, 2 * St, tid, nthr);
  }
  V F[9], p1[3], p2[3];
  torsion_base<V>(consts, F, p1, p2);
  if (tid == 0) {  // atom slots 0..2 receive no input
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      cv.set_slot(i, V(0));
      cv.set_slot(3 + i, p1[i]);
      cv.set_slot(6 + i, p2[i]);
    }
  }
  cp_async_wait_all();
  __syncthreads();

  const StepRange range = step_range(tid, K, St);
  const Affine<V> total = torsion_sweep<T, V, R>(cv, range, consts);
  const Affine<V> W = world_carry(cta_exclusive_affine<V>(total, ex.warp_totals, nwarps), F, p2);
  apply_carry<T, V>(cv, W, range);
  if constexpr (!kScatter) {
    if (xyz32 != nullptr) {
      // the float32 positions as well (the 16-bit xyz backward reads them)
      fence_proxy_async_smem();
      __syncthreads();
      store_row_bulk<float>(xyz32 + chain * 3 * N, reinterpret_cast<const float*>(cv.X), 3 * N, tid, nthr, 0);
      store_xyz_row<T, R>(out, cv.X, N, tid, nthr);
      if (tid == 0) bulk_store_wait_read();
      return;
    }
  }
  store_xyz_row<T, R>(out, cv.X, N, tid, nthr);
}

// One step of the torsion recompute form's sweep 1: local prefix advanced, the step's grad summed
// into the thread's totals of g and Q = sum p (x) g (world coordinates).
template <typename T, typename V, typename R>
__device__ __forceinline__ void torsion_totals_step(const ChainViews<T>& cv, Affine<V>& P, int s, R l, R st, R ct, V (&gsum)[3], V (&Q)[9]) {
  V rs, rc;
  torsion_pair<T>(cv, s, rs, rc);
  const V rinv = torsion_rinv(torsion_norm2(rs, rc));
  advance(P, step_rot<V>(l, st, ct, vmul(rs, rinv), vmul(rc, rinv)));
  const int off = 3 * (s + 3);
  const V g[3] = {cv.grad(off), cv.grad(off + 1), cv.grad(off + 2)};
#pragma unroll
  for (int c = 0; c < 3; ++c) gsum[c] = vadd(gsum[c], g[c]);
#pragma unroll
  for (int d = 0; d < 3; ++d) {
#pragma unroll
    for (int c = 0; c < 3; ++c) Q[3 * d + c] = vfma(P.v[d], g[c], Q[3 * d + c]);
  }
}

// One step of the torsion recompute form's sweep 2: prefix from the carry, d phi from the running
// force/moment suffix, the raw-pair chain rule d raw = d phi (c, -s) / n2 (torsion.cu:173-182)
// into the step's slot.
template <typename T, typename V, typename R>
__device__ __forceinline__ void torsion_grad_step(const ChainViews<T>& cv, Affine<V>& P, int s, R l, R st, R ct, V (&Fs)[3], V (&Ms)[3]) {
  const int off = 3 * (s + 3);
  const V u0 = P.m[0], u1 = P.m[3], u2 = P.m[6];
  const V xp[3] = {P.v[0], P.v[1], P.v[2]};
  V rs, rc;
  torsion_pair<T>(cv, s, rs, rc);
  const V rinv = torsion_rinv(torsion_norm2(rs, rc));
  advance(P, step_rot<V>(l, st, ct, vmul(rs, rinv), vmul(rc, rinv)));
  const V g[3] = {cv.grad(off), cv.grad(off + 1), cv.grad(off + 2)};
  V xf[3];
  cross3(xp, Fs, xf);
  const V tau[3] = {vsub(Ms[0], xf[0]), vsub(Ms[1], xf[1]), vsub(Ms[2], xf[2])};
  const V d_phi = vfma(u2, tau[2], vfma(u1, tau[1], vmul(u0, tau[0])));
  V mx[3];
  cross3(P.v, g, mx);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    Fs[i] = vsub(Fs[i], g[i]);
    Ms[i] = vsub(Ms[i], mx[i]);
  }
  const V scale = vmul(d_phi, vmul(rinv, rinv));
  cv.set_slot(off + 1, vmul(rc, scale));
  cv.set_slot(off + 2, vneg(vmul(rs, scale)));
}

// Recompute form of the torsion backward after staging (raw pairs in the slots or a staged row,
// grad row in cv.G): the same structure as the block recompute form; d raw goes into the slots.
// kRotate: both sweeps take their constants as torsion_sweep does (rotated once to the thread's
// first step's phase, three steps per iteration), at the cost of nine more live registers; the
// xyz form's fallback, which shares its kernel's register budget, picks them per step instead.
template <typename T, typename V, typename R, bool kRotate = true>
__device__ __forceinline__ void torsion_backward_recompute(const ChainViews<T>& cv, CtaExchange<V>& ex, const TorsionConsts<R>& consts, StepRange range,
                                                           int nwarps) {
  V F[9], p1[3], p2[3];
  torsion_base<V>(consts, F, p1, p2);
  if constexpr (!kRotate) {
    V gsum[3] = {V(0), V(0), V(0)};
    V Q[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) Q[i] = V(0);
    Affine<V> P = affine_identity<V>();
    const int end = range.first + range.count;
#pragma unroll 2
    for (int s = range.first; s < end; ++s) {
      R l, st, ct;
      torsion_constants_for(consts, s, l, st, ct);
      torsion_totals_step<T, V, R>(cv, P, s, l, st, ct, gsum, Q);
    }
    const Affine<V> carry = world_carry(cta_exclusive_affine<V>(P, ex.warp_totals, nwarps), F, p2);
    V msum[3];
    moment_total<V>(carry, gsum, Q, msum);
    V Fs[3], Ms[3];
    suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);
    P = carry;
#pragma unroll 2
    for (int s = range.first; s < end; ++s) {
      R l, st, ct;
      torsion_constants_for(consts, s, l, st, ct);
      torsion_grad_step<T, V, R>(cv, P, s, l, st, ct, Fs, Ms);
    }
  } else {
    R l0, l1, l2, s0, s1, s2, c0, c1, c2;
    torsion_constants_for(consts, range.first, l0, s0, c0);
    torsion_constants_for(consts, range.first + 1, l1, s1, c1);
    torsion_constants_for(consts, range.first + 2, l2, s2, c2);
    const int end = range.first + range.count;
    // the fixed torsion base frame is orthonormal: world coordinates throughout
    V gsum[3] = {V(0), V(0), V(0)};
    V Q[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) Q[i] = V(0);
    Affine<V> P = affine_identity<V>();
    int s = range.first;
#pragma unroll 1
    for (; s + 3 <= end; s += 3) {
      torsion_totals_step<T, V, R>(cv, P, s, l0, s0, c0, gsum, Q);
      torsion_totals_step<T, V, R>(cv, P, s + 1, l1, s1, c1, gsum, Q);
      torsion_totals_step<T, V, R>(cv, P, s + 2, l2, s2, c2, gsum, Q);
    }
    if (s < end) torsion_totals_step<T, V, R>(cv, P, s, l0, s0, c0, gsum, Q);
    if (s + 1 < end) torsion_totals_step<T, V, R>(cv, P, s + 1, l1, s1, c1, gsum, Q);
    const Affine<V> carry = world_carry(cta_exclusive_affine<V>(P, ex.warp_totals, nwarps), F, p2);
    V msum[3];
    moment_total<V>(carry, gsum, Q, msum);
    V Fs[3], Ms[3];
    suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);

    P = carry;
    s = range.first;
#pragma unroll 1
    for (; s + 3 <= end; s += 3) {
      torsion_grad_step<T, V, R>(cv, P, s, l0, s0, c0, Fs, Ms);
      torsion_grad_step<T, V, R>(cv, P, s + 1, l1, s1, c1, Fs, Ms);
      torsion_grad_step<T, V, R>(cv, P, s + 2, l2, s2, c2, Fs, Ms);
    }
    if (s < end) torsion_grad_step<T, V, R>(cv, P, s, l0, s0, c0, Fs, Ms);
    if (s + 1 < end) torsion_grad_step<T, V, R>(cv, P, s + 1, l1, s1, c1, Fs, Ms);
  }
}

// d raw from the slots (written by the recompute form) to the output row.
template <typename T, typename R>
__device__ __forceinline__ void write_pair_grads(const R* X, T* gr, int S, int tid, int nthr) {
#pragma unroll 4
  for (int e = tid; e < 2 * S; e += nthr) gr[e] = from_r<T>(X[3 * ((e >> 1) + 3) + 1 + (e & 1)]);
}

template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_backward_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                            const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride, ChainGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  constexpr bool kScatter = sizeof(T) >= 4;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* raw = raw_pairs + chain * raw_stride;
  ChainViews<T> cv;
  unsigned char* p = smem;
  cv.X = reinterpret_cast<R*>(p);
  p += slot_bytes(N, sizeof(R));
  if constexpr (kScatter) {
    scatter_pairs<T>(reinterpret_cast<T*>(cv.X), raw, St, tid, nthr);
  } else {
    cv.row[0] = stage_row_async(p, raw, 2 * St, tid, nthr);
    p += staged_row_bytes(size_t(2) * St, sizeof(T));
  }
  cv.G = stage_row_async(p, grad_xyz + chain * 3 * N, 3 * N, tid, nthr);
  cp_async_wait_all();
  __syncthreads();
  torsion_backward_recompute<T, V, R>(cv, ex, consts, step_range(tid, K, St), nwarps);
  __syncthreads();
  write_pair_grads<T, R>(cv.X, grad_raw + chain * grad_stride, St, tid, nthr);
}

// Torsion backward from the forward's xyz (4- and 8-byte types), as the reference's own torsion
// backward does (world_torsion_grad, torsion.cu:213-217 and :297-381): d phi_s = u_{s+1} . tau_s
// with u_{s+1} the direction of bond (x_{s+1}, x_{s+2}) and tau_s = M_s - (x_{s+2} - o) x F_s, the
// sums over atoms >= s+3 (moments about o = atom 2), carried from step to step.  The xyz, grad
// and raw rows are staged (16-byte LDGSTS); d phi goes over the grad row; the last loop applies the
// raw-pair chain rule d raw = d phi (c, -s) / n2 from the staged raw row.  A bond shorter than
// 1e-3 |x|max, a pair below the norm clamp (not a rotation), or a non-finite value sends the chain
// to the recompute form.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    torsion_backward_xyz_kernel(const T* __restrict__ raw_pairs, int64_t raw_stride, TorsionConsts<typename ComputeOf<T>::type> consts,
                                const T* __restrict__ xyz, const T* __restrict__ grad_xyz, T* __restrict__ grad_raw, int64_t grad_stride,
                                ChainGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the xyz form serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;

  const int N = geo.points, St = geo.steps, K = geo.items;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const int64_t chain = blockIdx.x;
  const T* raw = raw_pairs + chain * raw_stride;
  const T* grow = grad_xyz + chain * 3 * N;
  unsigned char* const slot_region = smem;
  unsigned char* const grad_region = smem + slot_bytes(N, sizeof(R));
  unsigned char* const raw_region = grad_region + staged_row_bytes(size_t(3) * N, sizeof(T));
  ChainViews<T> cv;
  cv.Y = stage_row_async(slot_region, xyz + chain * 3 * N, 3 * N, tid, nthr);
  cv.G = stage_row_async(grad_region, grow, 3 * N, tid, nthr);
  // the raw row, read once by the chain-rule loop at the end, stages with the others
  const T* raw_s = stage_row_async(raw_region, raw, 2 * St, tid, nthr);
  const StepRange range = step_range(tid, K, St);
  cp_async_wait_all();
  __syncthreads();

  const V o[3] = {cv.pos(6), cv.pos(7), cv.pos(8)};
  V gsum[3] = {V(0), V(0), V(0)};
  V msum[3] = {V(0), V(0), V(0)};
  V xmax2 = V(0);
  int off = 3 * (range.first + 3);
#pragma unroll 2
  for (int k = 0; k < range.count; ++k, off += 3) {
    const V g[3] = {cv.grad(off), cv.grad(off + 1), cv.grad(off + 2)};
    const V xw[3] = {cv.pos(off), cv.pos(off + 1), cv.pos(off + 2)};
    xmax2 = fmax(xmax2, dot3(xw, xw));
    const V x[3] = {vsub(xw[0], o[0]), vsub(xw[1], o[1]), vsub(xw[2], o[2])};
    V mx[3];
    cross3(x, g, mx);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      gsum[i] = vadd(gsum[i], g[i]);
      msum[i] = vadd(msum[i], mx[i]);
    }
  }
  V Fs[3], Ms[3];
  suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);
  // sweep: x1 = x_{s+1}, x2 = x_{s+2} and the torque about x_{s+2},
  // tau_s = sum_{j >= s+3} (x_j - x_{s+2}) x g_j, carried from step to step as
  // tau_{s+1} = tau_s - (x_{s+3} - x_{s+2}) x F_s (threads without steps read nothing)
  V x1[3] = {V(0), V(0), V(0)};
  V x2[3] = {V(0), V(0), V(0)};
  V tau[3] = {V(0), V(0), V(0)};
  if (range.count > 0) {
    off = 3 * (range.first + 1);  // atoms first+1 and first+2 <= N-2
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      x1[i] = cv.pos(off + i);
      x2[i] = cv.pos(off + 3 + i);
    }
    const V xr[3] = {vsub(x2[0], o[0]), vsub(x2[1], o[1]), vsub(x2[2], o[2])};
    V xf[3];
    cross3(xr, Fs, xf);
#pragma unroll
    for (int i = 0; i < 3; ++i) tau[i] = vsub(Ms[i], xf[i]);
  }
  V dmin2 = V(1e30);
  off = 3 * (range.first + 3);
#pragma unroll 2
  for (int k = 0; k < range.count; ++k, off += 3) {
    const V x3[3] = {cv.pos(off), cv.pos(off + 1), cv.pos(off + 2)};
    const V g[3] = {cv.grad(off), cv.grad(off + 1), cv.grad(off + 2)};
    const V d[3] = {vsub(x2[0], x1[0]), vsub(x2[1], x1[1]), vsub(x2[2], x1[2])};
    const V d2 = dot3(d, d);
    dmin2 = fmin(dmin2, d2);
    const V inv = vrsqrt(d2);
    const V d_phi = vmul(dot3(d, tau), inv);
    // tau -= (x3 - x2) x Fs, then Fs -= g
    const V e[3] = {vsub(x3[0], x2[0]), vsub(x3[1], x2[1]), vsub(x3[2], x2[2])};
    tau[0] = vfma(e[2], Fs[1], vfma(vneg(e[1]), Fs[2], tau[0]));
    tau[1] = vfma(e[0], Fs[2], vfma(vneg(e[2]), Fs[0], tau[1]));
    tau[2] = vfma(e[1], Fs[0], vfma(vneg(e[0]), Fs[1], tau[2]));
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      Fs[i] = vsub(Fs[i], g[i]);
      x1[i] = x2[i];
      x2[i] = x3[i];
    }
    cv.G[off] = d_phi;
  }
  // the last bond of the thread's range is x_{first+count+1} -> x_{first+count+2}: covered, every
  // bond a step uses is tested; non-finite values fail the comparison
  const bool bad = range.count > 0 && !(dmin2 >= static_cast<V>(1e-6) * xmax2);
  bool redo = __syncthreads_or(bad) != 0;
  T* gr = grad_raw + chain * grad_stride;
  if (!redo) {
    // chain rule from the staged raw row (each element and its partner, sin or cos, read from
    // shared memory).  A pair below the norm clamp is not normalised to a unit pair: that step is
    // not a rotation, the positions cannot give its gradient, and the chain is redone below.
    bool clamped = false;
#pragma unroll 4
    for (int e = tid; e < 2 * St; e += nthr) {
      const V v = to_r<V>(raw_s[e]);
      const V partner = to_r<V>(raw_s[e ^ 1]);
      const V rs = (e & 1) ? partner : v;
      const V rc = (e & 1) ? v : partner;
      const V n2raw = vfma(rs, rs, vmul(rc, rc));
      clamped |= !(n2raw >= static_cast<V>(1.0e-8f * 1.0e-8f));
      const V rinv = torsion_rinv(torsion_norm2(rs, rc));
      const V scale = vmul(cv.G[3 * ((e >> 1) + 3)], vmul(rinv, rinv));
      gr[e] = from_r<T>((e & 1) ? vneg(vmul(rs, scale)) : vmul(rc, scale));
    }
    redo = __syncthreads_or(clamped) != 0;
  }
  if (redo) {
    // recompute form, laid out as in torsion_backward_kernel
    __syncthreads();
    cv.X = reinterpret_cast<R*>(slot_region);
    scatter_pairs<T>(reinterpret_cast<T*>(cv.X), raw, St, tid, nthr);
    cv.G = stage_row_async(grad_region, grow, 3 * N, tid, nthr);
    cp_async_wait_all();
    __syncthreads();
    torsion_backward_recompute<T, V, R, false>(cv, ex, consts, range, nwarps);
    __syncthreads();
    write_pair_grads<T, R>(cv.X, gr, St, tid, nthr);
  }
}

}  // namespace cufkb
