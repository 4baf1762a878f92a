// Chains longer than one CTA's capacity (N - 3 > 2048 steps), float32 and float64.
//
// The reference stops at 2048 steps per chain (block.cu:88, reconstruct.py:5) and leaves longer
// chains to a separate scan it does not ship (README.md:52).  Here a chain is split into `segs`
// balanced segments of at most 2048 steps, one CTA each, and the segments meet through a small
// workspace in global memory (no CTA waits for another: every exchange is between two launches):
//
//   forward   long_totals_kernel    T_g = product of segment g's local transforms  -> totals[g]
//             long_scan_kernel      totals[g] <- T_0 ... T_{g-1} (one thread per chain, in place)
//             long_forward_kernel   world carry (F, p2) totals[g], then the one-CTA forward of the
//                                   segment from it
//   backward  long_totals_kernel    as above (the carries)
//             long_sums_kernel      G_g = sum g_j, M_g = sum x_j x g_j over segment g's atoms, from
//                                   the forward's xyz                              -> sums[g]
//             long_scan_kernel      totals as above, and sums[g] <- the sums of all later segments
//             long_backward_kernel  the one-CTA recompute backward of the segment (world
//                                   coordinates) from its carry and the sums of all later segments
//
// The scan between the launches keeps the work linear in the number of segments: every CTA reads
// one carry and one suffix instead of combining all the segments in front of (or behind) its own.
//
// Segment g covers steps [g L, min(S, (g + 1) L)), L = ceil(S / segs), and writes the atoms of its
// steps (s + 3); segment 0 also writes atoms 0..2 and the first-frame gradients.  Inside a
// segment the shared-memory layout and thread mapping are those of the one-CTA kernels, in the
// segment's local step numbering.  The backward needs an orthonormal base frame (world
// coordinates); a chain whose base frame is not (a collinear first angle, degenerate anchors)
// gets NaN gradients.
#pragma once

#include "nerf_kernels.cuh"

namespace cufkb {

struct LongGeometry {
  int batch;      // B
  int points;     // N
  int steps;      // S = N - 3
  int segs;       // segments per chain
  int seg_steps;  // L: steps per segment (the last one may have fewer)
  int items;      // K: steps per thread (odd)
};

constexpr int kTotalWords = 12;  // one affine total per (chain, segment)
constexpr int kSumWords = 6;     // one (sum g, sum x x g) per (chain, segment)

struct SegmentOf {
  int64_t chain;
  int g;      // segment index
  int first;  // first step
  int count;  // steps in the segment
};

__device__ __forceinline__ SegmentOf segment_of(const LongGeometry& geo) {
  const int64_t blk = blockIdx.x;
  SegmentOf s;
  s.chain = blk / geo.segs;
  s.g = static_cast<int>(blk - s.chain * geo.segs);
  s.first = s.g * geo.seg_steps;
  const int left = geo.steps - s.first;
  s.count = left < geo.seg_steps ? left : geo.seg_steps;
  return s;
}

// Scatters the inputs of a segment's steps into slots numbered from the segment's first step: local
// step i reads L[first+i+2], A[first+i+1], D[first+i] from slots 3(i+3) .. 3(i+3)+2.
template <typename T>
__device__ __forceinline__ void stage_segment_inputs(ChainViews<T>& cv, unsigned char* smem, const BlockArgs<T>& args, const SegmentOf& sg, int N,
                                                     uintptr_t slot_residue, int tid, int nthr) {
  cv.X = reinterpret_cast<typename ComputeOf<T>::type*>(smem + slot_residue);
  const T* Lr = args.lengths + sg.chain * (N - 1) + sg.first;
  const T* Ar = args.angles + sg.chain * (N - 2) + sg.first;
  const T* Dr = args.dihedrals + sg.chain * (N - 3) + sg.first;
  scatter_block_inputs<T>(reinterpret_cast<T*>(cv.X), Lr, Ar, Dr, sg.count + 3, tid, nthr);
}

template <typename V, typename R>
__device__ __forceinline__ void store_total(R* dst, const Affine<V>& a) {
#pragma unroll
  for (int i = 0; i < 9; ++i) dst[i] = a.m[i];
#pragma unroll
  for (int i = 0; i < 3; ++i) dst[9 + i] = a.v[i];
}

template <typename V, typename R>
__device__ __forceinline__ Affine<V> load_total(const R* src) {
  Affine<V> a;
#pragma unroll
  for (int i = 0; i < 9; ++i) a.m[i] = src[i];
#pragma unroll
  for (int i = 0; i < 3; ++i) a.v[i] = src[9 + i];
  return a;
}

// Exclusive prefix of every chain's segment totals, in place: totals[g] <- T_0 ... T_{g-1} (the
// identity for g = 0), composed left to right.  With sums non-null, also the exclusive suffix of the
// segment sums: sums[g] <- the sum over the segments after g.  One thread per chain.
template <typename R>
__global__ void long_scan_kernel(R* __restrict__ totals, R* __restrict__ sums, int batch, int segs) {
  enter_after_previous_grid();
  const int64_t chain = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (chain >= batch) return;
  R* t = totals + chain * segs * kTotalWords;
  Affine<R> C = affine_identity<R>();
  for (int g = 0; g < segs; ++g) {
    const Affine<R> T = load_total<R>(t + int64_t(g) * kTotalWords);
    store_total(t + int64_t(g) * kTotalWords, C);
    C = compose(C, T);
  }
  if (sums == nullptr) return;
  R* sm = sums + chain * segs * kSumWords;
  R acc[kSumWords] = {R(0), R(0), R(0), R(0), R(0), R(0)};
  for (int g = segs - 1; g >= 0; --g) {
#pragma unroll
    for (int i = 0; i < kSumWords; ++i) {
      const R v = sm[int64_t(g) * kSumWords + i];
      sm[int64_t(g) * kSumWords + i] = acc[i];
      acc[i] = acc[i] + v;
    }
  }
}

// T_g for every (chain, segment).
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp) long_totals_kernel(BlockArgs<T> args, typename ComputeOf<T>::type* __restrict__ totals, LongGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the long path serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const SegmentOf sg = segment_of(geo);
  ChainViews<T> cv;
  stage_segment_inputs<T>(cv, smem, args, sg, geo.points, 0, tid, nthr);
  cp_async_wait_all();
  __syncthreads();
  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };
  const Affine<V> total = sweep_local_prefix<T, V>(cv, step_range(tid, geo.items, sg.count), step);
  const Affine<V> excl = cta_exclusive_affine<V>(total, ex.warp_totals, nwarps);
  // threads past the segment's last step carry the identity: the last thread holds the product
  if (tid == nthr - 1) store_total(totals + (sg.chain * geo.segs + sg.g) * kTotalWords, compose(excl, total));
}

// xyz of every (chain, segment) from the totals.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    long_forward_kernel(BlockArgs<T> args, const typename ComputeOf<T>::type* __restrict__ totals, T* __restrict__ xyz, LongGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the long path serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;
  const int N = geo.points;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const SegmentOf sg = segment_of(geo);
  // segment 0 stores atoms 0 .. count+2 from slot 0; later segments atoms first+3 .. from slot 9
  const int first_slot = sg.g == 0 ? 0 : 9;
  T* dst = xyz + sg.chain * 3 * N + (sg.g == 0 ? 0 : 3 * int64_t(sg.first + 3));
  const uintptr_t residue = (reinterpret_cast<uintptr_t>(dst) - first_slot * sizeof(T)) & 15u;
  ChainViews<T> cv;
  stage_segment_inputs<T>(cv, smem, args, sg, N, residue, tid, nthr);
  V first_points[9];
  if (tid == 0) {
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const ChainFrame<V> ff = chain_frame_of<T, V>(args, af, rows_at(sg.chain, sg.chain * N, N));
    const Affine<V> W = world_carry(load_total<V>(totals + (sg.chain * geo.segs + sg.g) * kTotalWords), ff.F, ff.p2);
#pragma unroll
    for (int i = 0; i < 9; ++i) ex.frame[i] = W.m[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      ex.frame[9 + i] = W.v[i];
      first_points[i] = af.p0[i];
      first_points[3 + i] = ff.p1[i];
      first_points[6 + i] = ff.p2[i];
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (tid == 0 && sg.g == 0) {
#pragma unroll
    for (int i = 0; i < 9; ++i) cv.set_slot(i, first_points[i]);
  }
  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };
  const StepRange range = step_range(tid, geo.items, sg.count);
  const Affine<V> total = sweep_local_prefix<T, V>(cv, range, step);
  const Affine<V> W = world_carry(cta_exclusive_affine<V>(total, ex.warp_totals, nwarps), ex.frame, ex.frame + 9);
  apply_carry<T, V>(cv, W, range);
  fence_proxy_async_smem();
  __syncthreads();
  store_row_bulk<T>(dst, reinterpret_cast<const T*>(cv.X) + first_slot, 3 * (sg.count + 3) - first_slot, tid, nthr, 0);
  if (tid == 0) bulk_store_wait_read();
}

// (sum g, sum x x g) over each segment's atoms, from the forward's xyz.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    long_sums_kernel(const T* __restrict__ xyz, const T* __restrict__ grad_xyz, typename ComputeOf<T>::type* __restrict__ sums, LongGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  __shared__ V red[kMaxWarps * kSumWords];
  const int N = geo.points;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const SegmentOf sg = segment_of(geo);
  const T* x = xyz + sg.chain * 3 * N;
  const T* gr = grad_xyz + sg.chain * 3 * N;
  V acc[kSumWords] = {V(0), V(0), V(0), V(0), V(0), V(0)};
  for (int64_t a = sg.first + 3 + tid; a < int64_t(sg.first) + 3 + sg.count; a += nthr) {
    const V p[3] = {to_r<V>(x[3 * a]), to_r<V>(x[3 * a + 1]), to_r<V>(x[3 * a + 2])};
    const V g[3] = {to_r<V>(gr[3 * a]), to_r<V>(gr[3 * a + 1]), to_r<V>(gr[3 * a + 2])};
    V m[3];
    cross3(p, g, m);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      acc[i] = vadd(acc[i], g[i]);
      acc[3 + i] = vadd(acc[3 + i], m[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < kSumWords; ++i) {
#pragma unroll
    for (int off = kWarp / 2; off > 0; off >>= 1) acc[i] = vadd(acc[i], shfl_xor(acc[i], off));
  }
  const int lane = tid & (kWarp - 1), warp = tid / kWarp;
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < kSumWords; ++i) red[warp * kSumWords + i] = acc[i];
  }
  __syncthreads();
  if (tid < kSumWords) {
    V t = V(0);
    for (int w = 0; w < nwarps; ++w) t = vadd(t, red[w * kSumWords + tid]);
    sums[(sg.chain * geo.segs + sg.g) * kSumWords + tid] = t;
  }
}

// Gradients of every (chain, segment): the recompute backward of the segment in world coordinates,
// its carry from the totals, the force/moment of all later segments from the sums.
template <typename T>
__global__ void __launch_bounds__(kMaxWarps* kWarp)
    long_backward_kernel(BlockArgs<T> args, const typename ComputeOf<T>::type* __restrict__ totals, const typename ComputeOf<T>::type* __restrict__ sums,
                         const T* __restrict__ grad_xyz, T* __restrict__ grad_lengths, T* __restrict__ grad_angles, T* __restrict__ grad_dihedrals,
                         LongGeometry geo) {
  enter_after_previous_grid();
  using R = typename ComputeOf<T>::type;
  using V = R;
  static_assert(sizeof(T) >= 4, "the long path serves 32- and 64-bit types");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ CtaExchange<V> ex;
  __shared__ FirstFrame<V> first;
  __shared__ V later[kSumWords];
  const int N = geo.points;
  const int tid = threadIdx.x, nthr = blockDim.x, nwarps = nthr / kWarp;
  const SegmentOf sg = segment_of(geo);
  const T* grow = grad_xyz + sg.chain * 3 * N;
  ChainViews<T> cv;
  stage_segment_inputs<T>(cv, smem, args, sg, N, 0, tid, nthr);
  // the grad row of the segment's atoms first .. first+count+2, in the local numbering of the slots
  cv.G = stage_row_async(smem + slot_bytes(sg.count + 3, sizeof(R)), grow + 3 * int64_t(sg.first), 3 * (sg.count + 3), tid, nthr);
  if (tid == 0) {
    const AnchorFrame<R> af = anchor_frame<R>(args.p0, args.first_direction, args.initial_normal);
    const R l0 = args.lengths[sg.chain * (N - 1)];
    const R l1 = args.lengths[sg.chain * (N - 1) + 1];
    const R a0 = args.angles[sg.chain * (N - 2)];
    first = FirstFrame<V>{af, backward_frame<V>(af, l0, l1, a0)};
    const Affine<V> W = world_carry(load_total<V>(totals + (sg.chain * geo.segs + sg.g) * kTotalWords), first.bf.ff.F, first.bf.ff.p2);
#pragma unroll
    for (int i = 0; i < 9; ++i) ex.frame[i] = W.m[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) ex.frame[9 + i] = W.v[i];
    const R* cs = sums + (sg.chain * geo.segs + sg.g) * kSumWords;
#pragma unroll
    for (int i = 0; i < kSumWords; ++i) later[i] = cs[i];
  }
  cp_async_wait_all();
  __syncthreads();

  T* gl = grad_lengths + sg.chain * (N - 1);
  T* ga = grad_angles + sg.chain * (N - 2);
  T* gd = grad_dihedrals + sg.chain * (N - 3);
  // output entries of the segment: lengths[first+2 ..], angles[first+1 ..], dihedrals[first ..]
  // (segment 0 also lengths[0..1] and angles[0])
  const int l_lo = sg.g == 0 ? 0 : sg.first + 2, a_lo = sg.g == 0 ? 0 : sg.first + 1;
  const int l_hi = sg.first + sg.count + 2, a_hi = sg.first + sg.count + 1;
  if (first.bf.general) {
    const V nan = V(__int_as_float(0x7fc00000));
    for (int i = l_lo + tid; i < l_hi; i += nthr) gl[i] = from_r<T>(nan);
    for (int i = a_lo + tid; i < a_hi; i += nthr) ga[i] = from_r<T>(nan);
    for (int i = sg.first + tid; i < sg.first + sg.count; i += nthr) gd[i] = from_r<T>(nan);
    return;
  }
  auto step = [&](int s) {
    V l, th, ph, st, ct, sp, cp;
    block_step_inputs<T>(cv, s, l, th, ph);
    step_sincos(th, ph, st, ct, sp, cp);
    return step_rot(l, st, ct, sp, cp);
  };
  const StepRange range = step_range(tid, geo.items, sg.count);
  V gsum[3];
  V Q[9];
  const Affine<V> total = sweep_backward_totals<true, T, V>(cv, first.bf.ff.F, range, step, gsum, Q);
  const Affine<V> carry = world_carry(cta_exclusive_affine<V>(total, ex.warp_totals, nwarps), ex.frame, ex.frame + 9);
  V msum[3];
  moment_total<V>(carry, gsum, Q, msum);
  V Fs[3], Ms[3];
  suffix_base<V>(gsum, msum, ex, nwarps, Fs, Ms);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    Fs[i] = vadd(Fs[i], later[i]);
    Ms[i] = vadd(Ms[i], later[3 + i]);
  }
  const V F3[3] = {Fs[0], Fs[1], Fs[2]};
  const V M3[3] = {Ms[0], Ms[1], Ms[2]};
  block_backward_sweep2<true, T, V>(cv, first.bf.ff.F, carry, Fs, Ms, first.bf.av, first.bf.bv, range, step);
  if (sg.g == 0 && tid == 0) first_frame_grads<true, T, V>(cv, first.af, first.bf, cv.G, F3, M3, V(0));
  __syncthreads();
  // slot layout (local): lengths[first+i] in X[3+3i], angles[first+i] in X[7+3i], dihedrals[first+i]
  // in X[11+3i]
  const R* X = cv.X;
  for (int i = l_lo + tid; i < l_hi; i += nthr) gl[i] = from_r<T>(X[3 + 3 * (i - sg.first)]);
  for (int i = a_lo + tid; i < a_hi; i += nthr) ga[i] = from_r<T>(X[7 + 3 * (i - sg.first)]);
  for (int i = sg.first + tid; i < sg.first + sg.count; i += nthr) gd[i] = from_r<T>(X[11 + 3 * (i - sg.first)]);
}

// Bytes of dynamic shared memory of the long kernels for a segment of `seg_steps` steps.
template <typename T>
__host__ __device__ inline size_t long_smem_bytes(int seg_steps, bool backward) {
  return block_smem_bytes<T>(seg_steps + 3, backward);
}

}  // namespace cufkb
