/*
 * cufkb.h — C ABI of the B200 (sm_100a) NeRF chain-reconstruction library (libcufkb.so).
 *
 * Drop-in boundary for the reconstruction hot path of cufk (xsjk/cufk).  Each entry point takes
 * plain device pointers, sizes, a dtype code and a CUDA stream, launches asynchronously on that
 * stream and returns a status code; it never allocates, never synchronises and keeps no state
 * besides a per-device cache of the SM count and kernel attributes.  Inputs are read-only.
 *
 * Shapes (all row-major, contiguous rows):
 *   lengths (B, N-1), angles (B, N-2), dihedrals (B, N-3), xyz / grad_xyz (B, N, 3);
 *   raw_pairs (B, 2(N-3)) interleaved [sin_0, cos_0, sin_1, cos_1, ...] with any row stride;
 *   anchors p0 / first_direction / initial_normal: 3 elements each, or NULL for the reference's
 *   defaults (0,0,0), (1,0,0), (0,0,1).
 * Limits: 4 <= N <= CUFKB_MAX_POINT_COUNT (2051), 0 <= B <= INT32_MAX; B == 0 launches nothing.
 * Every pointer must be aligned to its element size.  All floating-point arithmetic of the 16-bit
 * types is done in float (rounded once on output); float64 computes in double.
 *
 * Reference interfaces replaced (paths relative to the cufk project root):
 *   cufkb_block_forward   <- forward_cuda_impl<T>   src/cufk/csrc/block.cu:319-329
 *                            (reached from _C.apply, block.cu:431-445 / _C.pyi:3-10)
 *   cufkb_block_backward  <- backward_cuda_impl<T>  src/cufk/csrc/block.cu:331-365
 *   cufkb_block_backward_from_xyz <- backward_cuda_impl<T> as well (same gradients, reads xyz)
 *   cufkb_torsion_forward <- forward_default_impl<T> src/cufk/csrc/torsion.cu:387-397
 *   cufkb_torsion_backward<- backward_xyz_impl<T>   src/cufk/csrc/torsion.cu:399-411
 *   cufkb_torsion_backward_from_xyz <- backward_xyz_impl<T> as well (reads the saved xyz, like it)
 *   validation codes      <- TORCH_CHECKs of src/cufk/csrc/extension_utils.cuh:57-143
 */
#ifndef CUFKB_H_
#define CUFKB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CUFKB_API __attribute__((visibility("default")))
#else
#define CUFKB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* cufkb_stream_t;

#define CUFKB_MAX_POINT_COUNT 2051
#define CUFKB_MAX_STEPS 2048

/* Storage dtype of every floating-point buffer of one call. */
enum cufkb_dtype {
  CUFKB_FLOAT32 = 0,
  CUFKB_FLOAT64 = 1,
  CUFKB_FLOAT16 = 2,
  CUFKB_BFLOAT16 = 3
};

enum cufkb_status {
  CUFKB_SUCCESS = 0,
  CUFKB_ERROR_INVALID_DTYPE = 1,  /* "must be float32, float64, float16, or bfloat16" */
  CUFKB_ERROR_NULL_POINTER = 2,   /* a required buffer is NULL while B > 0 */
  CUFKB_ERROR_POINT_COUNT = 3,    /* "point_count must be >= 4" */
  CUFKB_ERROR_TOO_MANY_STEPS = 4, /* "supports at most 2048 local transforms" */
  CUFKB_ERROR_SHAPE_LIMITS = 5,   /* "shape exceeds int32 kernel limits" (or B < 0) */
  CUFKB_ERROR_BAD_STRIDE = 6,     /* torsion row stride too small for the pairs */
  CUFKB_ERROR_MISALIGNED = 7,     /* a pointer not aligned to its element size */
  CUFKB_ERROR_INVALID_VALUE = 8,  /* NULL torsion constants */
  CUFKB_ERROR_CUDA = 9,           /* a CUDA runtime error; see cufkb_last_cuda_error() */
  CUFKB_ERROR_WORKSPACE = 10,     /* workspace smaller than cufkb_block_long_workspace_bytes */
  CUFKB_ERROR_UNSUPPORTED_DTYPE = 11, /* a dtype the entry point does not serve (long chains, fused loss: float32/float64; *_xyz32: 16-bit) */
  CUFKB_ERROR_SCRATCH_CAPACITY = 12   /* cufkb_block_forward_long_static: call too large for its scratch */
};

/* Backbone constants of compile_torsion(bond_lengths, bond_angles).  Bond i is used by every
 * step whose length phase is i; lengths are rounded to float32 inside the library, as the
 * reference compiles them (src/cufk/csrc/torsion.cu:43-47); the angle sine/cosine are given in
 * double, as src/cufk/torsion.py:81-86 computes them on the host. */
typedef struct cufkb_torsion_constants {
  double bond_lengths[3];
  double bond_angle_sin[3];
  double bond_angle_cos[3];
} cufkb_torsion_constants;

/* 2051 = BLOCK_SCAN_MAX_POINT_COUNT (src/cufk/reconstruct.py:5). */
CUFKB_API int cufkb_max_point_count(void);

/* xyz (B, N, 3) from lengths/angles/dihedrals and the three optional anchors. */
CUFKB_API int cufkb_block_forward(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                        const void* first_direction, const void* initial_normal, void* xyz, int64_t batch, int64_t points,
                        cufkb_stream_t stream);

/* Gradients of sum(grad_xyz * xyz) w.r.t. lengths, angles and dihedrals (no anchor gradients).
 * Recomputes the forward prefix; needs nothing saved from cufkb_block_forward. */
CUFKB_API int cufkb_block_backward(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                         const void* first_direction, const void* initial_normal, const void* grad_xyz, void* grad_lengths,
                         void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points, cufkb_stream_t stream);

/* The same gradients as cufkb_block_backward, from xyz = the output of cufkb_block_forward with
 * identical arguments: for an orthonormal base frame every gradient follows from the bond
 * directions and plane normals of xyz and the running sums of grad_xyz, so the chain is not
 * rebuilt.  Chains whose base frame is not orthonormal, or with a bond angle within ~6 degrees of 0
 * or pi, are recomputed as cufkb_block_backward does.  float16/bfloat16 ignore xyz (a 16-bit
 * position is too coarse for a bond direction) and recompute; cufkb_block_backward_from_xyz32
 * takes their float32 positions instead.  Replaces backward_cuda_impl<T> as
 * well; the reference's backward always recomputes the chain. */
CUFKB_API int cufkb_block_backward_from_xyz(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                  const void* first_direction, const void* initial_normal, const void* xyz, const void* grad_xyz,
                                  void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points,
                                  cufkb_stream_t stream);

/* float16/bfloat16 forward that also writes its float32 positions: xyz (B, N, 3) in the storage
 * dtype as cufkb_block_forward gives it, and xyz32 (B, N, 3) float32, the positions before rounding.
 * No counterpart in the reference.  With xyz32, cufkb_block_backward_from_xyz32 computes the
 * gradients from the positions (bond directions and plane normals) instead of walking the chain
 * again, as the float32 backward does from its xyz; a 16-bit xyz is too coarse for that.
 * float16/bfloat16 only (CUFKB_ERROR_UNSUPPORTED_DTYPE otherwise). */
CUFKB_API int cufkb_block_forward_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                              const void* first_direction, const void* initial_normal, void* xyz, float* xyz32, int64_t batch,
                              int64_t points, cufkb_stream_t stream);

/* Gradients of sum(grad_xyz * xyz) w.r.t. lengths, angles and dihedrals (float16/bfloat16) from
 * xyz32 = the float32 positions of cufkb_block_forward_xyz32 with identical arguments; grad_xyz and
 * the gradients in the storage dtype.  Replaces backward_cuda_impl<T> (src/cufk/csrc/block.cu:331-365)
 * for the 16-bit types; chains whose base frame is not orthonormal, or with a bond angle within ~6
 * degrees of 0 or pi, are recomputed as cufkb_block_backward does.  float16/bfloat16 only. */
CUFKB_API int cufkb_block_backward_from_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                    const void* first_direction, const void* initial_normal, const float* xyz32, const void* grad_xyz,
                                    void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points,
                                    cufkb_stream_t stream);

/* Fused consumer: loss[b] = (1/N) sum_j |xyz_j - target_j|^2 for each chain's reconstruction
 * (as cufkb_block_forward builds it, with the same arguments) and a target (B, N, 3), and, unless
 * grad_lengths, grad_angles and grad_dihedrals are all NULL, d loss[b] / d (lengths, angles,
 * dihedrals) of each chain.  One kernel: the chain's xyz stays in shared memory, so neither xyz nor
 * d loss / d xyz is written to device memory.  loss is (B,).  float32 and float64 only
 * (CUFKB_ERROR_UNSUPPORTED_DTYPE otherwise).  No counterpart in the reference, whose path ends at
 * xyz. */
CUFKB_API int cufkb_block_mse(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                    const void* first_direction, const void* initial_normal, const void* target, void* loss, void* grad_lengths,
                    void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points, cufkb_stream_t stream);

/* Packed (ragged) batches: chains of different lengths in one call.  No counterpart in the
 * reference, whose batches are (B, N) (src/cufk/csrc/block.cu:367-378).  chain_points is a device
 * array of B+1 nondecreasing int64 offsets with chain_points[0] = 0: chain b has the points
 * [chain_points[b], chain_points[b+1]) of the packed xyz (total_points, 3), and its rows sit packed
 * the same way in lengths (total_points - B), angles (total_points - 2B) and dihedrals
 * (total_points - 3B): chain b's lengths start at chain_points[b] - b, its angles at
 * chain_points[b] - 2b, its dihedrals at chain_points[b] - 3b.  total_points is the packed xyz's
 * point count (at least 4 B) and fixes the sizes of the four packed arrays.  max_points is the
 * largest chain (4 <= max_points <= 2051); the launch is planned for it.  A chain whose point
 * count lies outside [4, max_points], or any of whose four rows would reach outside its packed
 * array (negative or too large offsets), is skipped: its outputs are left as they were.  The
 * offsets stay on the device (nothing is read back), so these calls validate only what the host
 * knows; the kernels check every chain's rows against the packed sizes.  Anchors and dtypes as
 * for the (B, N) entry points; the backward reads the forward's xyz as
 * cufkb_block_backward_from_xyz does. */
CUFKB_API int cufkb_block_forward_packed(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                               const void* first_direction, const void* initial_normal, const int64_t* chain_points, void* xyz,
                               int64_t batch, int64_t total_points, int64_t max_points, cufkb_stream_t stream);

CUFKB_API int cufkb_block_backward_packed_from_xyz(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                         const void* first_direction, const void* initial_normal, const int64_t* chain_points,
                                         const void* xyz, const void* grad_xyz, void* grad_lengths, void* grad_angles,
                                         void* grad_dihedrals, int64_t batch, int64_t total_points, int64_t max_points,
                                         cufkb_stream_t stream);

/* Packed batches of float16/bfloat16 with the float32 positions: cufkb_block_forward_xyz32 and
 * cufkb_block_backward_from_xyz32 over the packed layout of cufkb_block_forward_packed (xyz and
 * xyz32 both (total_points, 3)).  No counterpart in the reference. */
CUFKB_API int cufkb_block_forward_packed_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                     const void* first_direction, const void* initial_normal, const int64_t* chain_points, void* xyz,
                                     float* xyz32, int64_t batch, int64_t total_points, int64_t max_points, cufkb_stream_t stream);

CUFKB_API int cufkb_block_backward_packed_from_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                           const void* first_direction, const void* initial_normal, const int64_t* chain_points,
                                           const float* xyz32, const void* grad_xyz, void* grad_lengths, void* grad_angles,
                                           void* grad_dihedrals, int64_t batch, int64_t total_points, int64_t max_points,
                                           cufkb_stream_t stream);

/* xyz (B, N, 3) from raw (sin, cos) pairs; raw row b starts at raw_pairs + b * raw_row_stride
 * elements (any stride >= 0, pairs within a row contiguous). */
CUFKB_API int cufkb_torsion_forward(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                          void* xyz, int64_t batch, int64_t points, cufkb_stream_t stream);

/* Gradient w.r.t. the raw pairs; grad row b starts at grad_raw_pairs + b * grad_row_stride
 * (stride >= 2(N-3) when B > 1).  Recomputes the forward; reads no saved xyz. */
CUFKB_API int cufkb_torsion_backward(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                           const void* grad_xyz, void* grad_raw_pairs, int64_t grad_row_stride, int64_t batch, int64_t points,
                           cufkb_stream_t stream);

/* The same gradient as cufkb_torsion_backward, from xyz = the output of cufkb_torsion_forward with
 * identical arguments, as the reference's own torsion backward reads its saved xyz
 * (src/cufk/csrc/torsion.cu:297-381): d dihedral = bond direction . torque, no chain rebuilt.
 * Chains with a bond shorter than 1e-3 of the largest coordinate are recomputed in the same
 * kernel.  float16/bfloat16 ignore xyz and recompute.  Replaces backward_xyz_impl<T>. */
CUFKB_API int cufkb_torsion_backward_from_xyz(int dtype, const void* raw_pairs, int64_t raw_row_stride,
                                    const cufkb_torsion_constants* constants, const void* xyz, const void* grad_xyz,
                                    void* grad_raw_pairs, int64_t grad_row_stride, int64_t batch, int64_t points,
                                    cufkb_stream_t stream);

/* float16/bfloat16 torsion forward that also writes its float32 positions (xyz32, (B, N, 3)), and
 * the raw-pair gradients from them: as cufkb_block_forward_xyz32 / cufkb_block_backward_from_xyz32
 * for the block path (a 16-bit position is too coarse for the bond directions the xyz form takes).
 * Replace forward_default_impl<T> / backward_xyz_impl<T> (src/cufk/csrc/torsion.cu:387-411) for the
 * 16-bit types; float16/bfloat16 only (CUFKB_ERROR_UNSUPPORTED_DTYPE otherwise). */
CUFKB_API int cufkb_torsion_forward_xyz32(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                                void* xyz, float* xyz32, int64_t batch, int64_t points, cufkb_stream_t stream);

CUFKB_API int cufkb_torsion_backward_from_xyz32(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                                      const float* xyz32, const void* grad_xyz, void* grad_raw_pairs, int64_t grad_row_stride,
                                      int64_t batch, int64_t points, cufkb_stream_t stream);

/* Chains of any length N >= 4 (no counterpart in the reference, which stops at
 * BLOCK_SCAN_MAX_POINT_COUNT = 2051 points and leaves longer chains to a scan it does not ship,
 * README.md:52).  A chain is split into balanced segments of at most 2048 steps, one CTA each;
 * segments exchange their affine totals (and, backward, their force/moment sums) through a
 * caller-provided device workspace of cufkb_block_long_workspace_bytes bytes (16-byte aligned,
 * nothing needs to be initialised; one workspace serves one call at a time).  float32 and float64.
 * Same arguments and results as cufkb_block_forward / cufkb_block_backward otherwise; the backward
 * reads the forward's xyz and needs an orthonormal base frame (a collinear first angle or
 * degenerate anchors give NaN gradients). */
CUFKB_API int cufkb_block_long_workspace_bytes(int dtype, int64_t batch, int64_t points, size_t* bytes);

CUFKB_API int cufkb_block_forward_long(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                             const void* first_direction, const void* initial_normal, void* xyz, int64_t batch, int64_t points,
                             void* workspace, size_t workspace_bytes, cufkb_stream_t stream);

/* cufkb_block_forward_long for callers that cannot provide a workspace.  No counterpart in the
 * reference.  It is meant for hosts that hold no device allocator of their own (a language binding
 * that only passes on the pointers it was given) and for code that must not allocate on its path
 * (a loop with a fixed device-memory budget).
 *
 * The call allocates nothing.  Its scratch is a file-scope static device array of 2 MiB inside
 * libcufkb.so; the library looks up its address with cudaGetSymbolAddress on the first call on a
 * device and keeps it for later calls there.  Make that first call outside any stream capture (a
 * plain warm-up call will do); a lookup that fails is returned as CUFKB_ERROR_CUDA and tried again
 * by the next call.  The cached address belongs to the device's current context: after
 * cudaDeviceReset on a device, this entry point must not be called again in that process.
 * Nothing in the scratch needs to start at zero: each call writes the segment totals before
 * reading them.
 *
 * Limits:
 * - batch x segments x 12 x sizeof(element) must fit in 2 MiB, where
 *   segments = ceil((points - 3) / 2048). For example, 4096 float32 chains of up to 20483 points.
 *   Larger calls return CUFKB_ERROR_SCRATCH_CAPACITY and launch nothing.
 * - The scratch is shared by every call on a device. Calls that overlap in time (on different
 *   streams, or from different threads) race on it and can return wrong coordinates. Keep calls of
 *   this entry point on one device in one stream, or use cufkb_block_forward_long with a workspace
 *   per stream. */
CUFKB_API int cufkb_block_forward_long_static(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                    const void* first_direction, const void* initial_normal, void* xyz, int64_t batch, int64_t points,
                                    cufkb_stream_t stream);

CUFKB_API int cufkb_block_backward_long(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                              const void* first_direction, const void* initial_normal, const void* xyz, const void* grad_xyz,
                              void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points,
                              void* workspace, size_t workspace_bytes, cufkb_stream_t stream);

/* Static text for a status code. */
CUFKB_API const char* cufkb_status_string(int status);

/* cudaError_t value of the last CUFKB_ERROR_CUDA returned on the calling thread (0 if none). */
CUFKB_API int cufkb_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* CUFKB_H_ */
