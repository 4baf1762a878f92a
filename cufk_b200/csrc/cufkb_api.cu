// C ABI of libcufkb.so: validation, launch planning and dispatch of the sm_100a chain kernels.
//
// Validation restates the reference's checks (src/cufk/csrc/extension_utils.cuh:119-143):
// N >= 4, steps = N - 3 <= 2048 (plan_capacity of the float plan, block.cu:88), int32 limits.
// Differences, by design: B == 0 is a successful no-op (the reference would launch an empty grid
// and raise), float64 backward is accepted up to 2048 steps (the reference caps it at 1024 by its
// register plan, block.cu:76-86), and anchors may be NULL for the defaults.
#include "cufkb.h"
#include "nerf_kernels.cuh"
#include "nerf_long.cuh"
#include "nerf_vec.cuh"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <initializer_list>
#include <mutex>
#include <type_traits>
#include <utility>

namespace {

using cufkb::ChainGeometry;

thread_local int g_last_cuda_error = 0;

constexpr int kMaxDevices = 64;
constexpr int kNumKernels = 156;  // kKindCount x 4 dtypes
constexpr int kTargetItems = 24;  // steps per thread a long chain is split down to
constexpr int kMinItems = 5;      // never split a chain below this many steps per thread
// Resident warps per SM the plan aims for, per kernel.  The xyz backward aims lower: its per-thread
// fixed work (staging, suffix scan, first frame) is large next to its per-step work, so fewer,
// longer threads per chain beat more resident warps (measured on B200: at N=768, 2 warps per chain
// and ~22 resident warps beat 3 warps per chain and 24).
#ifndef CUFKB_TARGET_WARPS_PER_SM
#define CUFKB_TARGET_WARPS_PER_SM 32
#endif
#ifndef CUFKB_XYZ_TARGET_WARPS_PER_SM
#define CUFKB_XYZ_TARGET_WARPS_PER_SM 20
#endif
// The torsion kernels aim lower too: with fewer warps per chain their scans cost less than the
// residency they give up (B200, config 3 fp32: forward 57.7 vs 67.7 us, xyz backward 108.4 vs
// 116.9 us at 16 against 32).
#ifndef CUFKB_TORSION_TARGET_WARPS_PER_SM
#define CUFKB_TORSION_TARGET_WARPS_PER_SM 16
#endif
// The 16-bit kernels aim lowest.  Their slots hold float results next to the staged 16-bit rows, so
// a chain needs more shared memory and the default target splits it over more warps (4 at N=1026),
// whose affine scan then costs more than the extra residency hides (B200, config 4: block forward
// 69.8 vs 83.4 us, recompute backward 136.0 vs 149.3 us; config 3 bf16: torsion backward 114.8 vs
// 121.5 us at 12 against 32).
#ifndef CUFKB_TARGET_WARPS_PER_SM_16BIT
#define CUFKB_TARGET_WARPS_PER_SM_16BIT 12
#endif
constexpr int kTargetWarpsPerSm = CUFKB_TARGET_WARPS_PER_SM;
constexpr int kXyzTargetWarpsPerSm = CUFKB_XYZ_TARGET_WARPS_PER_SM;
constexpr int kTorsionTargetWarpsPerSm = CUFKB_TORSION_TARGET_WARPS_PER_SM;
constexpr int kTargetWarpsPerSm16 = CUFKB_TARGET_WARPS_PER_SM_16BIT;

// The resident-warp target of a kernel for element type T whose 32/64-bit target is `wide`.
template <typename T>
constexpr int target_warps(int wide) {
  return sizeof(T) == 2 ? kTargetWarpsPerSm16 : wide;
}
// Warps per SM the block forward's grid must offer before a small batch stops splitting its chains
// over more warps.  Each extra warp adds scan work; on B200 at N=768 two warps per chain beat three
// to five at 1024 and 2048 chains, and four match them at 512 (per-launch times 12.3 vs 14.3 us and
// 17.0 vs 18.4 us).
constexpr int kForwardFillWarpsPerSm = 12;

struct DeviceCache {
  std::once_flag once;
  int sm_count = 0;
  int max_smem_optin = 0;     // per block, static + dynamic
  int smem_per_sm = 0;        // per SM, all blocks
  int reserved_per_block = 0; // runtime reservation per resident block
  int regs_per_sm = 0;
  int max_warps_per_sm = 0;
  int max_blocks_per_sm = 0;
  int error = 0;
};
DeviceCache g_devices[kMaxDevices];

// Per kernel: its register and static shared-memory footprint, and one bit per device saying that
// its dynamic shared-memory limit has been raised there.
struct KernelCache {
  std::once_flag once;
  int regs = 0;
  int static_smem = 0;
  int error = 0;
  std::atomic<uint64_t> attr_done{0};
};
KernelCache g_kernels[kNumKernels];

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (*dev < 0 || *dev >= kMaxDevices) return static_cast<int>(cudaErrorInvalidDevice);
  return 0;
}

const DeviceCache* device_cache(int dev) {
  DeviceCache& d = g_devices[dev];
  std::call_once(d.once, [&] {
    int warps_threads = 0;
    const struct {
      int* out;
      cudaDeviceAttr attr;
    } queries[] = {
        {&d.sm_count, cudaDevAttrMultiProcessorCount},
        {&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin},
        {&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor},
        {&d.reserved_per_block, cudaDevAttrReservedSharedMemoryPerBlock},
        {&d.regs_per_sm, cudaDevAttrMaxRegistersPerMultiprocessor},
        {&warps_threads, cudaDevAttrMaxThreadsPerMultiProcessor},
        {&d.max_blocks_per_sm, cudaDevAttrMaxBlocksPerMultiprocessor},
    };
    for (const auto& q : queries) {
      const cudaError_t e = cudaDeviceGetAttribute(q.out, q.attr, dev);
      if (e != cudaSuccess) {
        d.error = static_cast<int>(e);
        return;
      }
    }
    d.max_warps_per_sm = warps_threads / cufkb::kWarp;
  });
  return &d;
}

int fail_cuda(cudaError_t e) {
  g_last_cuda_error = static_cast<int>(e);
  return CUFKB_ERROR_CUDA;
}

template <typename Kernel>
const KernelCache* kernel_cache(Kernel kernel, int kernel_id) {
  KernelCache& k = g_kernels[kernel_id];
  std::call_once(k.once, [&] {
    cudaFuncAttributes attr;
    const cudaError_t e = cudaFuncGetAttributes(&attr, kernel);
    if (e != cudaSuccess) {
      k.error = static_cast<int>(e);
      return;
    }
    k.regs = attr.numRegs;
    k.static_smem = static_cast<int>(attr.sharedSizeBytes);
  });
  return &k;
}

template <typename Kernel>
cudaError_t ensure_smem_limit(Kernel kernel, KernelCache* k, int dev, int max_optin) {
  const uint64_t bit = uint64_t(1) << dev;
  if (k->attr_done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  // the opt-in maximum covers static + dynamic shared memory of a block
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_optin - k->static_smem);
  if (e == cudaSuccess) k->attr_done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Warps per chain (W) and steps per thread (K).  A chain needs W >= ceil(steps / (32 kTargetItems))
// so that a thread walks at most ~kTargetItems steps.  Beyond that, W grows while the SM would hold
// fewer than `target` resident warps (shared memory per chain and registers per thread bound the
// resident chains), and while the whole grid offers fewer than `fill` warps per SM (small
// batches), as long as a thread keeps >= kMinItems steps.  K is made odd so that the threads' slot
// strides (3K words) fall on 32 distinct shared-memory banks.
struct Plan {
  int threads;
  int items;
};

int resident_warps(const DeviceCache& d, const KernelCache& k, size_t dyn_smem, int warps) {
  const int chain_smem = static_cast<int>(dyn_smem) + k.static_smem + d.reserved_per_block;
  int chains = chain_smem > 0 ? d.smem_per_sm / chain_smem : d.max_blocks_per_sm;
  const int regs_per_warp = ((k.regs + 7) / 8) * 8 * cufkb::kWarp;
  const int by_regs = regs_per_warp > 0 ? d.regs_per_sm / (regs_per_warp * warps) : chains;
  if (by_regs < chains) chains = by_regs;
  if (d.max_blocks_per_sm < chains) chains = d.max_blocks_per_sm;
  if (d.max_warps_per_sm / warps < chains) chains = d.max_warps_per_sm / warps;
  return chains * warps;
}

Plan make_plan(int64_t batch, int points, const DeviceCache& d, const KernelCache& k, size_t dyn_smem, int target, int fill) {
  const int steps = points - 3;
  int warps = ceil_div(steps, cufkb::kWarp * kTargetItems);
  if (warps < 1) warps = 1;
  if (warps > cufkb::kMaxWarps) warps = cufkb::kMaxWarps;
  auto splittable = [&](int w) { return w < cufkb::kMaxWarps && ceil_div(steps, cufkb::kWarp * (w + 1)) >= kMinItems; };
  while (splittable(warps) && resident_warps(d, k, dyn_smem, warps) < target &&
         resident_warps(d, k, dyn_smem, warps + 1) > resident_warps(d, k, dyn_smem, warps)) {
    ++warps;
  }
  const int64_t grid_target = int64_t(d.sm_count) * fill;
  while (splittable(warps) && batch * warps < grid_target) ++warps;
  int items = ceil_div(steps, cufkb::kWarp * warps);
  if ((items & 1) == 0) ++items;
  return {cufkb::kWarp * warps, items};
}

size_t elem_size(int dtype) {
  switch (dtype) {
    case CUFKB_FLOAT32:
      return 4;
    case CUFKB_FLOAT64:
      return 8;
    case CUFKB_FLOAT16:
    case CUFKB_BFLOAT16:
      return 2;
    default:
      return 0;
  }
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shared validation of (dtype, batch, points); returns CUFKB_SUCCESS or an error code.
int check_shape(int dtype, int64_t batch, int64_t points) {
  if (elem_size(dtype) == 0) return CUFKB_ERROR_INVALID_DTYPE;
  if (batch < 0 || batch > INT32_MAX || points > INT32_MAX) return CUFKB_ERROR_SHAPE_LIMITS;
  if (points < 4) return CUFKB_ERROR_POINT_COUNT;
  if (points - 3 > CUFKB_MAX_STEPS) return CUFKB_ERROR_TOO_MANY_STEPS;
  return CUFKB_SUCCESS;
}

struct LaunchEnv {
  int dev;
  const DeviceCache* cache;
  Plan plan;
};

// Grids of at most this many CTAs per SM are launched with programmatic dependent launch.  Every
// kernel of this library lets the next kernel in the stream be scheduled as soon as all of its CTAs
// have started (enter_after_previous_grid); for a small grid that hides the launch latency between
// the two (B200, config-1 chains, forward + backward per step: 512 chains 12.5 -> 11.5 us, 1024
// chains 16.5 -> 15.5 us), but the next kernel's CTAs, resident early and waiting, slowed larger
// ones (2048 chains: 26.8 -> 29.1 us), which therefore launch plainly; the one exception is the
// (B, N) vector forward larger than one resident wave (forward_beyond_one_wave).
constexpr int kOverlapCtasPerSm = 8;

// Whether a grid of `ctas` CTAs is launched to overlap the previous kernel (kOverlapCtasPerSm).
bool overlap_launch(uint64_t ctas) {
  int dev = 0, sms = 148;
  if (current_device(&dev) == 0) {
    const DeviceCache* d = device_cache(dev);
    if (!d->error) sms = d->sm_count;
  }
  return ctas <= uint64_t(kOverlapCtasPerSm) * sms;
}

// Whether a chain launch takes the prefetching instantiation: an overlapping launch of a (B, N)
// batch, whose CTAs start while the previous kernel drains and each ask L2 for their chain's rows
// first (B200, config-1 chains, step of forward + backward: 512 chains 12.15 -> 11.68 us, 1024
// chains 17.03 -> 15.70 us).
bool prefetch_launch(int64_t batch, const cufkb::PackedLayout& packed) { return packed.offsets == nullptr && overlap_launch(uint64_t(batch)); }

// Launches `kernel` on `stream`, with programmatic dependent launch when `overlap`: the kernel may
// then be scheduled while the previous kernel in the stream finishes, and, like every kernel of this
// library, waits for that kernel's completion (enter_after_previous_grid) before touching global
// memory.  Returns the launch's own error.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_as(bool overlap, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = overlap ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with the small-grid rule (overlap_launch) for the overlap.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  const uint64_t ctas = uint64_t(grid.x) * grid.y * grid.z;
  return launch_kernel_as(overlap_launch(ctas), kernel, grid, block, smem, stream, std::forward<Args>(args)...);
}

// Device, kernel footprint, shared-memory opt-in and plan of one launch.
template <typename Kernel>
int launch_env(LaunchEnv* env, Kernel kernel, int kernel_id, int64_t batch, int points, size_t smem, int target = kTargetWarpsPerSm,
               int fill = 0) {
  const int e = current_device(&env->dev);
  if (e != 0) return fail_cuda(static_cast<cudaError_t>(e));
  env->cache = device_cache(env->dev);
  if (env->cache->error != 0) return fail_cuda(static_cast<cudaError_t>(env->cache->error));
  const KernelCache* k = kernel_cache(kernel, kernel_id);
  if (k->error != 0) return fail_cuda(static_cast<cudaError_t>(k->error));
  if (static_cast<int>(smem) + k->static_smem > env->cache->max_smem_optin) return fail_cuda(cudaErrorInvalidValue);
  if (cudaError_t err = ensure_smem_limit(kernel, &g_kernels[kernel_id], env->dev, env->cache->max_smem_optin)) return fail_cuda(err);
  env->plan = make_plan(batch, points, *env->cache, *k, smem, target, fill > 0 ? fill : target);
  return CUFKB_SUCCESS;
}

template <typename T>
constexpr int dtype_index() {
  if constexpr (std::is_same_v<T, float>) return 0;
  if constexpr (std::is_same_v<T, double>) return 1;
  if constexpr (std::is_same_v<T, __half>) return 2;
  return 3;
}

// Kernel ids for the caches: kind x dtype (4).
enum KernelKind {
  kBlockForward = 0,
  kBlockBackward = 1,
  kTorsionForward = 2,
  kTorsionBackward = 3,
  kBlockBackwardXyz = 4,
  kTorsionBackwardXyz = 5,
  kLongTotals = 6,
  kLongForward = 7,
  kLongSums = 8,
  kLongBackward = 9,
  kBlockMse = 10,
  // vector-slot kernels: kVecKindBase + family x warp count (vec_kind)
  kVecKindBase = 11,
  kKindCount = 39
};
constexpr int kernel_id(KernelKind kind, int dtype) { return kind * 4 + dtype; }

// ---------------------------------------------------------------------------------------------
// vector-slot kernels: plan and launch
// ---------------------------------------------------------------------------------------------
// Warps per chain of the vector kernels; 0 lets the plan choose (a count the kernels are built
// for, kVecWarpCounts).  A chain's K atoms per thread are a multiple of G = 16 / sizeof(slot
// element) and give an odd number of groups of G (three 16-byte shared accesses per group then fall
// on distinct banks across each quarter warp).
#ifndef CUFKB_VEC_FWD_WARPS
#define CUFKB_VEC_FWD_WARPS 0
#endif
#ifndef CUFKB_VEC_BWD_WARPS
#define CUFKB_VEC_BWD_WARPS 0
#endif
// Resident warps per SM the vector kernels' plans aim for (the forward is issue-bound and wants
// many warps; the xyz backward's per-thread fixed work favours fewer, longer threads).
#ifndef CUFKB_VEC_TARGET_WARPS
#define CUFKB_VEC_TARGET_WARPS 32
#endif
#ifndef CUFKB_VEC_BWD_TARGET_WARPS
#define CUFKB_VEC_BWD_TARGET_WARPS 20
#endif
#ifndef CUFKB_VEC_MAX_GROUPS
#define CUFKB_VEC_MAX_GROUPS 7
#endif

// Longest chain (points) the vector kernels take where a previous-generation kernel exists.
constexpr int kVecMaxPointsLong = 1024;

// The largest shift of a thread range in the batch: known exactly when every chain's output row has
// the residue mod 16 of the first one ((B, N) rows whose pitch is a multiple of 16 bytes).
template <typename T>
int vec_delta_max(const void* row0, int points, bool packed) {
  const bool uniform = !packed && (size_t(3) * points * sizeof(T)) % 16 == 0;
  return uniform ? cufkb::vec_delta<T>(reinterpret_cast<uintptr_t>(row0) & 15u) : cufkb::VecSlots<T>::kAtoms - 1;
}

// Items per thread for W warps: the fewest groups of G atoms that cover N + delta atoms with 32 W
// threads, made odd.
template <typename T>
int vec_items(int points, int delta, int warps) {
  constexpr int G = cufkb::VecSlots<T>::kAtoms;
  int groups = ceil_div(points + delta, int64_t(cufkb::kWarp) * warps * G);
  if ((groups & 1) == 0) ++groups;
  return groups * G;
}

// Resident CTAs per SM of a kernel instantiation with `smem` bytes of dynamic shared memory.
template <typename Kernel>
int resident_ctas(Kernel kernel, int kind, int dtype_idx, size_t smem, int warps_per_cta, int* error) {
  int dev = 0;
  if (int e = current_device(&dev)) {
    *error = e;
    return 0;
  }
  const DeviceCache* d = device_cache(dev);
  const KernelCache* k = kernel_cache(kernel, kernel_id(static_cast<KernelKind>(kind), dtype_idx));
  if (d->error || k->error) {
    *error = d->error ? d->error : k->error;
    return 0;
  }
  return resident_warps(*d, *k, smem, warps_per_cta) / warps_per_cta;
}

// Warp counts per chain the vector kernels are built for.  (Counts 3 and 6, which leave fewer
// threads without atoms at N = 1026 or 2051, measured slower on B200 than the nearest power of two:
// per-warp work, staging, scan and stores, outweighs the idle threads.)
constexpr int kVecWarpCounts[] = {1, 2, 4, 8};
constexpr int kNumVecWarpCounts = 4;
constexpr int vec_warp_slot(int w) { return w == 1 ? 0 : (w == 2 ? 1 : (w == 4 ? 2 : 3)); }

// Calls f(std::integral_constant<int, W>()) for the built warp count w.
template <typename F>
int with_vec_warps(int w, F&& f) {
  switch (w) {
    case 1:
      return f(std::integral_constant<int, 1>());
    case 2:
      return f(std::integral_constant<int, 2>());
    case 4:
      return f(std::integral_constant<int, 4>());
    default:
      return f(std::integral_constant<int, 8>());
  }
}

// The *Prefetch families are the instantiations for launches that overlap the previous kernel.
enum VecFamily {
  kVecForwardFamily = 0,
  kVecBackwardFamily = 1,
  kXyz32BackwardFamily = 2,
  kVecForwardPrefetchFamily = 3,
  kVecBackwardPrefetchFamily = 4,
  kTorsionBackwardFamily = 5,
  kTorsionXyz32Family = 6
};
constexpr KernelKind vec_kind(VecFamily f, int w) { return static_cast<KernelKind>(kVecKindBase + f * kNumVecWarpCounts + vec_warp_slot(w)); }
static_assert(kVecKindBase + 7 * kNumVecWarpCounts == kKindCount, "kind table");

// Warps per chain of a vector kernel whose slots hold `Elem`: the fewest with at most
// CUFKB_VEC_MAX_GROUPS groups of G atoms per thread, then twice as many while the SM would hold
// fewer than `target` resident warps and the doubled plan holds more (shared memory bounds the
// chains of one warp), or while the grid offers fewer than the target per SM (small batches), as
// long as the doubled plan keeps at least half of its threads on atoms.  resident(w, items) gives
// the resident warps per SM of the instantiation; `forced` (a build-time override) wins when set.
template <typename Elem, typename Resident>
int choose_vec_warps(int64_t batch, int points, int delta, int target, int forced, Resident resident) {
  constexpr int G = cufkb::VecSlots<Elem>::kAtoms;
  constexpr int kMax = kVecWarpCounts[kNumVecWarpCounts - 1];
  int w = 1;
  while (w < kMax && vec_items<Elem>(points, delta, w) / G > CUFKB_VEC_MAX_GROUPS) w *= 2;
  if (forced > 0) return forced > w ? forced : w;
  int dev = 0, sms = 148;
  if (current_device(&dev) == 0) {
    const DeviceCache* d = device_cache(dev);
    if (!d->error) sms = d->sm_count;
  }
  auto res = [&](int warps) { return resident(warps, vec_items<Elem>(points, delta, warps)); };
  auto busy = [&](int warps) { return 2 * ceil_div(points + delta, vec_items<Elem>(points, delta, warps)) > int64_t(cufkb::kWarp) * warps; };
  while (w < kMax && busy(2 * w)) {
    const bool low_residency = res(w) < target && res(2 * w) > res(w);
    const bool small_grid = batch * w < int64_t(sms) * target;
    if (!(low_residency || small_grid)) break;
    w *= 2;
  }
  return w;
}

// Resident warps per SM of family F's kernel with W warps for chains of `points` and `items`.
template <VecFamily F, typename T>
int vec_resident(int w, int points, int items);

template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kVecForwardFamily>) {
  return cufkb::block_forward_vec_kernel<T, W, 1>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kVecBackwardFamily>) {
  return cufkb::block_backward_xyz_vec_kernel<T, W>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kTorsionBackwardFamily>) {
  return cufkb::torsion_backward_xyz_vec_kernel<T, W>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kTorsionXyz32Family>) {
  return cufkb::torsion_backward_xyz32_kernel<T, W>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kVecForwardPrefetchFamily>) {
  return cufkb::block_forward_vec_kernel<T, W, 1, true>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kVecBackwardPrefetchFamily>) {
  return cufkb::block_backward_xyz_vec_kernel<T, W, true>;
}
template <typename T, int W>
auto vec_kernel(std::integral_constant<VecFamily, kXyz32BackwardFamily>) {
  return cufkb::block_backward_xyz32_kernel<T, W>;
}

// Dynamic shared memory of one chain of family F.
template <VecFamily F, typename T>
size_t vec_smem(int points, int items) {
  if constexpr (F == kVecForwardFamily || F == kVecForwardPrefetchFamily) return cufkb::vec_row_bytes(points, items, sizeof(T));
  if constexpr (F == kVecBackwardFamily || F == kVecBackwardPrefetchFamily) return 2 * cufkb::vec_row_bytes(points, items, sizeof(T));
  if constexpr (F == kTorsionXyz32Family) return cufkb::torsion_xyz32_bytes<T>(points, items);
  if constexpr (F == kTorsionBackwardFamily) {
    return 2 * cufkb::vec_row_bytes(points, items, sizeof(T)) + cufkb::staged_row_bytes(size_t(2) * (points - 3), sizeof(T));
  }
  return cufkb::xyz32_pos_region_bytes<T>(points, items) + cufkb::xyz32_grad_region_bytes<T>(points, items);
}

template <VecFamily F, typename T>
int vec_resident(int w, int points, int items) {
  return with_vec_warps(w, [&](auto wc) {
    constexpr int W = decltype(wc)::value;
    int err = 0;
    const int r = resident_ctas(vec_kernel<T, W>(std::integral_constant<VecFamily, F>()), vec_kind(F, W), dtype_index<T>(), vec_smem<F, T>(points, items), W, &err);
    return err ? 0 : r * W;
  });
}

// Plans family F for a batch: (warps per chain, items per thread).
template <VecFamily F, typename T>
std::pair<int, int> vec_plan(int64_t batch, int points, int delta) {
  using Elem = std::conditional_t<sizeof(T) == 2, float, T>;  // the slot element
  constexpr bool kForward = F == kVecForwardFamily || F == kVecForwardPrefetchFamily;
  const int target = kForward ? CUFKB_VEC_TARGET_WARPS : CUFKB_VEC_BWD_TARGET_WARPS;
  const int forced = kForward ? CUFKB_VEC_FWD_WARPS : CUFKB_VEC_BWD_WARPS;
  const int w = choose_vec_warps<Elem>(batch, points, delta, target, forced,
                                       [&](int ww, int items) { return vec_resident<F, T>(ww, points, items); });
  return {w, vec_items<Elem>(points, delta, w)};
}

// Whether a (B, N) vector forward of `batch` chains needs more than one resident wave.  Such a
// forward is launched overlapping the previous kernel, in the prefetching instantiation: it lets the
// next kernel in as soon as its last wave has started, and its own CTAs, let in early during the
// previous kernel's last wave, ask L2 for their input rows, which no earlier kernel writes, before
// they wait (B200, config 1: forward alone 21.7 -> 20.0 us, step 47.2 -> 45.7 us; config 2 fp32:
// forward 31.1 -> 27.7 us, step 78.2 -> 77.0 us).  The other families measured no faster or slower
// that way (the xyz backward after a forward that one wave holds, 3072 chains: step 37.4 -> 38.8 us;
// the torsion step at config 3: 150.5 -> 153.4 us), and packed forwards, which do not prefetch,
// keep the small-grid rule.
template <typename T, int W>
bool forward_beyond_one_wave(int64_t batch, int points, int items) {
  int dev = 0;
  if (current_device(&dev) != 0) return false;
  const DeviceCache* d = device_cache(dev);
  if (d->error) return false;
  const int per_sm = vec_resident<kVecForwardFamily, T>(W, points, items) / W;
  return per_sm > 0 && batch > int64_t(per_sm) * d->sm_count;
}

// Whether a launch of family F with W warps per chain overlaps the previous kernel: small grids
// (overlap_launch) in every family, and prefetching forwards beyond one resident wave.
template <VecFamily F, typename T, int W>
bool vec_overlap(int64_t batch, int points, int items) {
  if (overlap_launch(uint64_t(batch))) return true;
  if constexpr (F == kVecForwardPrefetchFamily) return forward_beyond_one_wave<T, W>(batch, points, items);
  return false;
}

// Launches family F's kernel with W warps per chain: one CTA per chain.
template <VecFamily F, typename T, int W, typename... Args>
int launch_vec(int64_t batch, int points, int items, cudaStream_t stream, Args... args) {
  auto kernel = vec_kernel<T, W>(std::integral_constant<VecFamily, F>());
  const size_t smem = vec_smem<F, T>(points, items);
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(vec_kind(F, W), dtype_index<T>()), batch, points, smem)) return st;
  const bool overlap = vec_overlap<F, T, W>(batch, points, items);
  if (cudaError_t e = launch_kernel_as(overlap, kernel, static_cast<unsigned>(batch), cufkb::kWarp * W, smem, stream, args...)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

template <typename T>
cufkb::BlockArgs<T> block_args(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn) {
  return {static_cast<const T*>(L),  static_cast<const T*>(A),  static_cast<const T*>(D),
          static_cast<const T*>(p0), static_cast<const T*>(fd), static_cast<const T*>(nn)};
}

template <typename T>
int block_forward_vec(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, void* xyz, int64_t batch, int points,
                      cudaStream_t stream, cufkb::PackedLayout packed) {
  const cufkb::BlockArgs<T> args = block_args<T>(L, A, D, p0, fd, nn);
  const int delta = vec_delta_max<T>(xyz, points, packed.offsets != nullptr);
  const std::pair<int, int> plan = vec_plan<kVecForwardFamily, T>(batch, points, delta);
  const int w = plan.first, items = plan.second;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, items, packed};
  return with_vec_warps(w, [&](auto wc) {
    constexpr int W = decltype(wc)::value;
    if (packed.offsets == nullptr && vec_overlap<kVecForwardPrefetchFamily, T, W>(batch, points, items)) return launch_vec<kVecForwardPrefetchFamily, T, W>(batch, points, items, stream, args, static_cast<T*>(xyz), geo);
    return launch_vec<kVecForwardFamily, T, W>(batch, points, items, stream, args, static_cast<T*>(xyz), geo);
  });
}

template <typename T>
int block_backward_xyz_vec(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, const void* xyz, const void* g,
                           void* gL, void* gA, void* gD, int64_t batch, int points, cudaStream_t stream, cufkb::PackedLayout packed) {
  const cufkb::BlockArgs<T> args = block_args<T>(L, A, D, p0, fd, nn);
  const int delta = vec_delta_max<T>(xyz, points, packed.offsets != nullptr);
  const std::pair<int, int> plan = vec_plan<kVecBackwardFamily, T>(batch, points, delta);
  const int w = plan.first, items = plan.second;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, items, packed};
  return with_vec_warps(w, [&](auto wc) {
    constexpr int W = decltype(wc)::value;
    const T* x = static_cast<const T*>(xyz);
    const T* gg = static_cast<const T*>(g);
    T *l = static_cast<T*>(gL), *a = static_cast<T*>(gA), *d = static_cast<T*>(gD);
    if (prefetch_launch(batch, packed)) return launch_vec<kVecBackwardPrefetchFamily, T, W>(batch, points, items, stream, args, x, gg, l, a, d, geo);
    return launch_vec<kVecBackwardFamily, T, W>(batch, points, items, stream, args, x, gg, l, a, d, geo);
  });
}

// The 16-bit backward from the forward's float32 positions.
template <typename T>
int block_backward_xyz32_impl(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, const float* xyz32,
                              const void* g, void* gL, void* gA, void* gD, int64_t batch, int points, cudaStream_t stream, cufkb::PackedLayout packed) {
  const cufkb::BlockArgs<T> args = block_args<T>(L, A, D, p0, fd, nn);
  const int delta = vec_delta_max<float>(xyz32, points, packed.offsets != nullptr);
  const std::pair<int, int> plan = vec_plan<kXyz32BackwardFamily, T>(batch, points, delta);
  const int w = plan.first, items = plan.second;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, items, packed};
  return with_vec_warps(w, [&](auto wc) {
    return launch_vec<kXyz32BackwardFamily, T, decltype(wc)::value>(batch, points, items, stream, args, xyz32, static_cast<const T*>(g),
                                                                     static_cast<T*>(gL), static_cast<T*>(gA), static_cast<T*>(gD), geo);
  });
}

template <typename T>
int block_forward_impl(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, void* xyz, int64_t batch, int points,
                       cudaStream_t stream, cufkb::PackedLayout packed_layout = {}, float* xyz32 = nullptr) {
  // the vector forward: float32 at every length, float64 up to kVecMaxPointsLong (beyond it the
  // one-slot-per-step kernel wins: measured on B200 at N = 2051, 71 against 80 us for 2048 chains).
  // The 16-bit types keep the one-slot-per-step kernel, which writes the float32 positions as
  // well when asked: a vector-slot form measured no faster at config 4 (65.9 / 67.0 / 84.3 us with
  // 2 / 3 / 4 warps per chain against 64.7)
  if constexpr (sizeof(T) == 4) return block_forward_vec<T>(L, A, D, p0, fd, nn, xyz, batch, points, stream, packed_layout);
  if constexpr (sizeof(T) == 8) {
    if (points <= kVecMaxPointsLong) return block_forward_vec<T>(L, A, D, p0, fd, nn, xyz, batch, points, stream, packed_layout);
  }
  const size_t smem = cufkb::block_smem_bytes<T>(points, false);
  auto kernel = cufkb::block_forward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kBlockForward, dtype_index<T>()), batch, points, smem, target_warps<T>(kTargetWarpsPerSm), kForwardFillWarpsPerSm)) {
    return st;
  }
  cufkb::BlockArgs<T> args{static_cast<const T*>(L),  static_cast<const T*>(A),  static_cast<const T*>(D),
                           static_cast<const T*>(p0), static_cast<const T*>(fd), static_cast<const T*>(nn)};
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items, packed_layout};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, args, static_cast<T*>(xyz), geo, xyz32)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

template <typename T>
int block_backward_impl(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, const void* g, void* gL, void* gA,
                        void* gD, int64_t batch, int points, cudaStream_t stream, cufkb::PackedLayout packed_layout = {}) {
  const size_t smem = cufkb::block_smem_bytes<T>(points, true);
  auto kernel = cufkb::block_backward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kBlockBackward, dtype_index<T>()), batch, points, smem, target_warps<T>(kTargetWarpsPerSm))) return st;
  cufkb::BlockArgs<T> args{static_cast<const T*>(L),  static_cast<const T*>(A),  static_cast<const T*>(D),
                           static_cast<const T*>(p0), static_cast<const T*>(fd), static_cast<const T*>(nn)};
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items, packed_layout};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, args, static_cast<const T*>(g), static_cast<T*>(gL), static_cast<T*>(gA),
                                                                          static_cast<T*>(gD), geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// Backward from the forward's xyz (32- and 64-bit types).
template <typename T>
int block_backward_xyz_impl(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, const void* xyz, const void* g,
                            void* gL, void* gA, void* gD, int64_t batch, int points, cudaStream_t stream, cufkb::PackedLayout packed_layout = {}) {
  // the vector kernel stages xyz and grad rows with one shift: their rows must share the residue mod
  // 16.  Up to kVecMaxPointsLong points: beyond, a chain's two staged rows leave room for only ~4
  // chains per SM and the one-slot-per-step kernel wins (B200, N = 2051 float32: 51 against 55 us
  // for 2048 chains)
  if (points <= kVecMaxPointsLong && (reinterpret_cast<uintptr_t>(xyz) - reinterpret_cast<uintptr_t>(g)) % 16 == 0) {
    return block_backward_xyz_vec<T>(L, A, D, p0, fd, nn, xyz, g, gL, gA, gD, batch, points, stream, packed_layout);
  }
  const size_t smem = cufkb::block_smem_bytes<T>(points, true);
  auto kernel = cufkb::block_backward_xyz_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kBlockBackwardXyz, dtype_index<T>()), batch, points, smem, kXyzTargetWarpsPerSm)) return st;
  cufkb::BlockArgs<T> args{static_cast<const T*>(L),  static_cast<const T*>(A),  static_cast<const T*>(D),
                           static_cast<const T*>(p0), static_cast<const T*>(fd), static_cast<const T*>(nn)};
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items, packed_layout};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, args, static_cast<const T*>(xyz), static_cast<const T*>(g), static_cast<T*>(gL),
                                                                          static_cast<T*>(gA), static_cast<T*>(gD), geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// Fused consumer: reconstruction, mean squared distance to a target, and (grads non-null) its
// gradient with respect to the parameters, in one kernel (32- and 64-bit types).
template <typename T>
int block_mse_impl(const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, const void* target, void* loss, void* gL,
                   void* gA, void* gD, int64_t batch, int points, cudaStream_t stream) {
  const size_t smem = cufkb::block_smem_bytes<T>(points, true);
  auto kernel = cufkb::block_mse_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kBlockMse, dtype_index<T>()), batch, points, smem, kXyzTargetWarpsPerSm)) return st;
  cufkb::BlockArgs<T> args{static_cast<const T*>(L),  static_cast<const T*>(A),  static_cast<const T*>(D),
                           static_cast<const T*>(p0), static_cast<const T*>(fd), static_cast<const T*>(nn)};
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, args, static_cast<const T*>(target), static_cast<T*>(loss), static_cast<T*>(gL),
                                                                          static_cast<T*>(gA), static_cast<T*>(gD), geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

template <typename R>
cufkb::TorsionConsts<R> torsion_consts(const cufkb_torsion_constants* c) {
  cufkb::TorsionConsts<R> out;
  for (int i = 0; i < 3; ++i) {
    out.length[i] = static_cast<R>(static_cast<float>(c->bond_lengths[i]));
    out.sin_a[i] = static_cast<R>(c->bond_angle_sin[i]);
    out.cos_a[i] = static_cast<R>(c->bond_angle_cos[i]);
  }
  return out;
}

template <typename T>
int torsion_forward_impl(const void* raw, int64_t raw_stride, const cufkb_torsion_constants* c, void* xyz, int64_t batch, int points, cudaStream_t stream,
                         float* xyz32 = nullptr) {
  using R = typename cufkb::ComputeOf<T>::type;
  const size_t smem = cufkb::torsion_smem_bytes<T>(points, false);
  auto kernel = cufkb::torsion_forward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kTorsionForward, dtype_index<T>()), batch, points, smem, target_warps<T>(kTorsionTargetWarpsPerSm))) return st;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, static_cast<const T*>(raw), raw_stride,
                                    torsion_consts<R>(c), static_cast<T*>(xyz), geo, xyz32)) {
    return fail_cuda(e);
  }
  return CUFKB_SUCCESS;
}

template <typename T>
int torsion_backward_impl(const void* raw, int64_t raw_stride, const cufkb_torsion_constants* c, const void* g, void* graw, int64_t grad_stride,
                          int64_t batch, int points, cudaStream_t stream) {
  using R = typename cufkb::ComputeOf<T>::type;
  const size_t smem = cufkb::torsion_smem_bytes<T>(points, true);
  auto kernel = cufkb::torsion_backward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kTorsionBackward, dtype_index<T>()), batch, points, smem, target_warps<T>(kTorsionTargetWarpsPerSm))) return st;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, static_cast<const T*>(raw), raw_stride, torsion_consts<R>(c),
                                                                          static_cast<const T*>(g), static_cast<T*>(graw), grad_stride, geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// Torsion backward from the forward's xyz (32- and 64-bit types).
template <typename T>
int torsion_backward_xyz_impl(const void* raw, int64_t raw_stride, const cufkb_torsion_constants* c, const void* xyz, const void* g, void* graw,
                              int64_t grad_stride, int64_t batch, int points, cudaStream_t stream) {
  using R = typename cufkb::ComputeOf<T>::type;
  // the vector form stages xyz and grad rows with one shift: their rows must share the residue mod 16
  if ((reinterpret_cast<uintptr_t>(xyz) - reinterpret_cast<uintptr_t>(g)) % 16 == 0) {
    const int delta = vec_delta_max<T>(xyz, points, false);
    const std::pair<int, int> plan = vec_plan<kTorsionBackwardFamily, T>(batch, points, delta);
    const int w = plan.first, items = plan.second;
    const ChainGeometry geo{static_cast<int>(batch), points, points - 3, items};
    return with_vec_warps(w, [&](auto wc) {
      return launch_vec<kTorsionBackwardFamily, T, decltype(wc)::value>(batch, points, items, stream, static_cast<const T*>(raw), raw_stride,
                                                                         torsion_consts<R>(c), static_cast<const T*>(xyz), static_cast<const T*>(g),
                                                                         static_cast<T*>(graw), grad_stride, geo);
    });
  }
  const size_t smem = cufkb::torsion_xyz_smem_bytes<T>(points);
  auto kernel = cufkb::torsion_backward_xyz_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kTorsionBackwardXyz, dtype_index<T>()), batch, points, smem, kTorsionTargetWarpsPerSm)) return st;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch), env.plan.threads, smem, stream, static_cast<const T*>(raw), raw_stride, torsion_consts<R>(c),
                                                                          static_cast<const T*>(xyz), static_cast<const T*>(g), static_cast<T*>(graw),
                                                                          grad_stride, geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// The 16-bit torsion backward from the torsion forward's float32 positions.
template <typename T>
int torsion_backward_xyz32_impl(const void* raw, int64_t raw_stride, const cufkb_torsion_constants* c, const float* xyz32, const void* g, void* graw,
                                int64_t grad_stride, int64_t batch, int points, cudaStream_t stream) {
  const int delta = vec_delta_max<float>(xyz32, points, false);
  const std::pair<int, int> plan = vec_plan<kTorsionXyz32Family, T>(batch, points, delta);
  const int w = plan.first, items = plan.second;
  const ChainGeometry geo{static_cast<int>(batch), points, points - 3, items};
  return with_vec_warps(w, [&](auto wc) {
    return launch_vec<kTorsionXyz32Family, T, decltype(wc)::value>(batch, points, items, stream, static_cast<const T*>(raw), raw_stride,
                                                                   torsion_consts<float>(c), xyz32, static_cast<const T*>(g), static_cast<T*>(graw),
                                                                   grad_stride, geo);
  });
}

// ---- chains longer than one CTA: segments of at most CUFKB_MAX_STEPS steps ----
struct LongPlan {
  int segs;
  int seg_steps;
};

LongPlan long_plan(int64_t points) {
  const int64_t steps = points - 3;
  const int64_t segs = (steps + CUFKB_MAX_STEPS - 1) / CUFKB_MAX_STEPS;
  return {static_cast<int>(segs), static_cast<int>((steps + segs - 1) / segs)};
}

// workspace words: the totals (12 per segment) then the sums (6 per segment)
size_t long_workspace_words(int64_t batch, const LongPlan& lp) {
  return static_cast<size_t>(batch) * lp.segs * (cufkb::kTotalWords + cufkb::kSumWords);
}

template <typename T>
int long_totals_launch(const cufkb::BlockArgs<T>& args, typename cufkb::ComputeOf<T>::type* totals, int64_t batch, int64_t points, const LongPlan& lp,
                       cudaStream_t stream) {
  const size_t smem = cufkb::long_smem_bytes<T>(lp.seg_steps, false);
  auto kernel = cufkb::long_totals_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kLongTotals, dtype_index<T>()), batch * lp.segs, lp.seg_steps + 3, smem)) return st;
  const cufkb::LongGeometry geo{static_cast<int>(batch), static_cast<int>(points), static_cast<int>(points - 3), lp.segs, lp.seg_steps, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch * lp.segs), env.plan.threads, smem, stream, args, totals, geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// Turns the segment totals (and sums) into carries (and suffixes): one thread per chain.
template <typename R>
int long_scan_launch(R* totals, R* sums, int64_t batch, const LongPlan& lp, cudaStream_t stream) {
  constexpr int kThreads = 128;
  if (cudaError_t e = launch_kernel(cufkb::long_scan_kernel<R>, static_cast<unsigned>(ceil_div(batch, kThreads)), kThreads, 0, stream, totals, sums, static_cast<int>(batch), lp.segs)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

template <typename T>
int block_forward_long_impl(const cufkb::BlockArgs<T>& args, void* xyz, int64_t batch, int64_t points, void* workspace, cudaStream_t stream) {
  using R = typename cufkb::ComputeOf<T>::type;
  const LongPlan lp = long_plan(points);
  R* totals = static_cast<R*>(workspace);
  if (int st = long_totals_launch<T>(args, totals, batch, points, lp, stream)) return st;
  if (int st = long_scan_launch<R>(totals, nullptr, batch, lp, stream)) return st;
  const size_t smem = cufkb::long_smem_bytes<T>(lp.seg_steps, false);
  auto kernel = cufkb::long_forward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kLongForward, dtype_index<T>()), batch * lp.segs, lp.seg_steps + 3, smem)) return st;
  const cufkb::LongGeometry geo{static_cast<int>(batch), static_cast<int>(points), static_cast<int>(points - 3), lp.segs, lp.seg_steps, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch * lp.segs), env.plan.threads, smem, stream, args, totals, static_cast<T*>(xyz), geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

template <typename T>
int block_backward_long_impl(const cufkb::BlockArgs<T>& args, const void* xyz, const void* g, void* gL, void* gA, void* gD, int64_t batch,
                             int64_t points, void* workspace, cudaStream_t stream) {
  using R = typename cufkb::ComputeOf<T>::type;
  const LongPlan lp = long_plan(points);
  R* totals = static_cast<R*>(workspace);
  R* sums = totals + static_cast<size_t>(batch) * lp.segs * cufkb::kTotalWords;
  if (int st = long_totals_launch<T>(args, totals, batch, points, lp, stream)) return st;
  {
    auto kernel = cufkb::long_sums_kernel<T>;
    LaunchEnv env;
    if (int st = launch_env(&env, kernel, kernel_id(kLongSums, dtype_index<T>()), batch * lp.segs, lp.seg_steps + 3, 0)) return st;
    const cufkb::LongGeometry geo{static_cast<int>(batch), static_cast<int>(points), static_cast<int>(points - 3), lp.segs, lp.seg_steps, env.plan.items};
    if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch * lp.segs), env.plan.threads, 0, stream, static_cast<const T*>(xyz), static_cast<const T*>(g), sums, geo)) return fail_cuda(e);
  }
  if (int st = long_scan_launch<R>(totals, sums, batch, lp, stream)) return st;
  const size_t smem = cufkb::long_smem_bytes<T>(lp.seg_steps, true);
  auto kernel = cufkb::long_backward_kernel<T>;
  LaunchEnv env;
  if (int st = launch_env(&env, kernel, kernel_id(kLongBackward, dtype_index<T>()), batch * lp.segs, lp.seg_steps + 3, smem)) return st;
  const cufkb::LongGeometry geo{static_cast<int>(batch), static_cast<int>(points), static_cast<int>(points - 3), lp.segs, lp.seg_steps, env.plan.items};
  if (cudaError_t e = launch_kernel(kernel, static_cast<unsigned>(batch * lp.segs), env.plan.threads, smem, stream, args, totals, sums, static_cast<const T*>(g), static_cast<T*>(gL),
                                                                                    static_cast<T*>(gA), static_cast<T*>(gD), geo)) return fail_cuda(e);
  return CUFKB_SUCCESS;
}

// Validation shared by the long entry points (dtype float32/float64, 4 <= N <= INT32_MAX,
// B * segments within one grid).
int check_long(int dtype, int64_t batch, int64_t points) {
  if (elem_size(dtype) == 0) return CUFKB_ERROR_INVALID_DTYPE;
  if (dtype != CUFKB_FLOAT32 && dtype != CUFKB_FLOAT64) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch < 0 || batch > INT32_MAX || points > INT32_MAX) return CUFKB_ERROR_SHAPE_LIMITS;
  if (points < 4) return CUFKB_ERROR_POINT_COUNT;
  if (batch * long_plan(points).segs > INT32_MAX) return CUFKB_ERROR_SHAPE_LIMITS;
  return CUFKB_SUCCESS;
}

// Scratch of cufkb_block_forward_long_static: a fixed device array, so that the call allocates
// nothing.  It holds the segment totals only, written by the first kernel of a call before the
// second reads them: nothing in it needs to start at zero or survive between calls.
constexpr size_t kStaticScratchBytes = size_t(2) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct ScratchAddress {
  std::mutex lock;
  std::atomic<void*> ptr{nullptr};
};
ScratchAddress g_scratch_address[kMaxDevices];

// The array's address on device `dev` (the current device), looked up on the first call that
// succeeds there and cached from then on; a failed lookup is returned and retried by the next call.
void* static_scratch(int dev, int* error) {
  ScratchAddress& a = g_scratch_address[dev];
  *error = 0;
  if (void* p = a.ptr.load(std::memory_order_acquire)) return p;
  std::lock_guard<std::mutex> guard(a.lock);
  if (void* p = a.ptr.load(std::memory_order_relaxed)) return p;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) {
    *error = static_cast<int>(e);
    return nullptr;
  }
  a.ptr.store(p, std::memory_order_release);
  return p;
}

}  // namespace

namespace {

int check_block_pointers(int dtype, std::initializer_list<const void*> required, std::initializer_list<const void*> all) {
  for (const void* p : required) {
    if (!p) return CUFKB_ERROR_NULL_POINTER;
  }
  const size_t es = elem_size(dtype);
  for (const void* p : all) {
    if (!aligned(p, es)) return CUFKB_ERROR_MISALIGNED;
  }
  return CUFKB_SUCCESS;
}

// The packed total (points of all chains) must be >= 4 B; offsets outside it only skip chains.
int check_packed_total(int64_t batch, int64_t total_points) {
  return (total_points < 0 || (batch > 0 && total_points < 4 * batch)) ? CUFKB_ERROR_SHAPE_LIMITS : CUFKB_SUCCESS;
}

// Packed batches: the offsets array (B+1 int64) must be given, 8-byte aligned.
int check_offsets(const int64_t* offsets, bool packed) {
  if (!packed) return CUFKB_SUCCESS;
  if (!offsets) return CUFKB_ERROR_NULL_POINTER;
  return aligned(offsets, alignof(int64_t)) ? CUFKB_SUCCESS : CUFKB_ERROR_MISALIGNED;
}

int block_forward_dispatch(int dtype, const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, void* xyz, int64_t batch,
                           int64_t points, cufkb_stream_t stream, bool packed = false, cufkb::PackedLayout packed_layout = {}) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {L, A, D, xyz}, {L, A, D, p0, fd, nn, xyz})) return st;
  if (int st = check_offsets(packed_layout.offsets, packed)) return st;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CUFKB_FLOAT32:
      return block_forward_impl<float>(L, A, D, p0, fd, nn, xyz, batch, n, s, packed_layout);
    case CUFKB_FLOAT64:
      return block_forward_impl<double>(L, A, D, p0, fd, nn, xyz, batch, n, s, packed_layout);
    case CUFKB_FLOAT16:
      return block_forward_impl<__half>(L, A, D, p0, fd, nn, xyz, batch, n, s, packed_layout);
    default:
      return block_forward_impl<__nv_bfloat16>(L, A, D, p0, fd, nn, xyz, batch, n, s, packed_layout);
  }
}

int block_backward_dispatch(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                            const void* initial_normal, const void* grad_xyz, void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch,
                            int64_t points, cufkb_stream_t stream, bool packed = false, cufkb::PackedLayout packed_layout = {}) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, grad_xyz, grad_lengths, grad_angles, grad_dihedrals},
                                    {lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                     grad_dihedrals})) {
    return st;
  }
  if (int st = check_offsets(packed_layout.offsets, packed)) return st;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CUFKB_FLOAT32:
      return block_backward_impl<float>(lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                        grad_dihedrals, batch, n, s, packed_layout);
    case CUFKB_FLOAT64:
      return block_backward_impl<double>(lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                         grad_dihedrals, batch, n, s, packed_layout);
    case CUFKB_FLOAT16:
      return block_backward_impl<__half>(lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                         grad_dihedrals, batch, n, s, packed_layout);
    default:
      return block_backward_impl<__nv_bfloat16>(lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                                grad_dihedrals, batch, n, s, packed_layout);
  }
}

int block_backward_from_xyz_dispatch(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                                     const void* initial_normal, const void* xyz, const void* grad_xyz, void* grad_lengths, void* grad_angles,
                                     void* grad_dihedrals, int64_t batch, int64_t points, cufkb_stream_t stream, bool packed = false,
                                     cufkb::PackedLayout packed_layout = {}) {
  if (dtype != CUFKB_FLOAT32 && dtype != CUFKB_FLOAT64) {
    if (int st = check_shape(dtype, batch, points)) return st;
    if (batch > 0 && !xyz) return CUFKB_ERROR_NULL_POINTER;
    return block_backward_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                   grad_dihedrals, batch, points, stream, packed, packed_layout);
  }
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, xyz, grad_xyz, grad_lengths, grad_angles, grad_dihedrals},
                                    {lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths, grad_angles,
                                     grad_dihedrals})) {
    return st;
  }
  if (int st = check_offsets(packed_layout.offsets, packed)) return st;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT32) {
    return block_backward_xyz_impl<float>(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths, grad_angles,
                                          grad_dihedrals, batch, n, s, packed_layout);
  }
  return block_backward_xyz_impl<double>(lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths, grad_angles,
                                         grad_dihedrals, batch, n, s, packed_layout);
}

}  // namespace

extern "C" {

int cufkb_max_point_count(void) { return CUFKB_MAX_POINT_COUNT; }

int cufkb_block_forward(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                        const void* initial_normal, void* xyz, int64_t batch, int64_t points, cufkb_stream_t stream) {
  return block_forward_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, batch, points, stream);
}

int cufkb_block_backward(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                         const void* initial_normal, const void* grad_xyz, void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch,
                         int64_t points, cufkb_stream_t stream) {
  return block_backward_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, grad_xyz, grad_lengths, grad_angles,
                                 grad_dihedrals, batch, points, stream);
}

int cufkb_block_backward_from_xyz(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                                  const void* initial_normal, const void* xyz, const void* grad_xyz, void* grad_lengths, void* grad_angles,
                                  void* grad_dihedrals, int64_t batch, int64_t points, cufkb_stream_t stream) {
  return block_backward_from_xyz_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths,
                                          grad_angles, grad_dihedrals, batch, points, stream);
}

}  // extern "C" (the float32-position dispatchers below are internal)

namespace {
int block_forward_xyz32_dispatch(int dtype, const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn, void* xyz,
                                 float* xyz32, int64_t batch, int64_t points, cufkb_stream_t stream, bool packed, cufkb::PackedLayout layout) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (dtype != CUFKB_FLOAT16 && dtype != CUFKB_BFLOAT16) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {L, A, D, xyz, xyz32}, {L, A, D, p0, fd, nn, xyz})) return st;
  if (!aligned(xyz32, sizeof(float))) return CUFKB_ERROR_MISALIGNED;
  if (int st = check_offsets(layout.offsets, packed)) return st;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT16) return block_forward_impl<__half>(L, A, D, p0, fd, nn, xyz, batch, n, s, layout, xyz32);
  return block_forward_impl<__nv_bfloat16>(L, A, D, p0, fd, nn, xyz, batch, n, s, layout, xyz32);
}

int block_backward_xyz32_dispatch(int dtype, const void* L, const void* A, const void* D, const void* p0, const void* fd, const void* nn,
                                  const float* xyz32, const void* g, void* gL, void* gA, void* gD, int64_t batch, int64_t points, cufkb_stream_t stream,
                                  bool packed, cufkb::PackedLayout layout) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (dtype != CUFKB_FLOAT16 && dtype != CUFKB_BFLOAT16) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {L, A, D, xyz32, g, gL, gA, gD}, {L, A, D, p0, fd, nn, g, gL, gA, gD})) return st;
  if (!aligned(xyz32, sizeof(float))) return CUFKB_ERROR_MISALIGNED;
  if (int st = check_offsets(layout.offsets, packed)) return st;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT16) return block_backward_xyz32_impl<__half>(L, A, D, p0, fd, nn, xyz32, g, gL, gA, gD, batch, n, s, layout);
  return block_backward_xyz32_impl<__nv_bfloat16>(L, A, D, p0, fd, nn, xyz32, g, gL, gA, gD, batch, n, s, layout);
}
}  // namespace

extern "C" {

int cufkb_block_forward_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                              const void* initial_normal, void* xyz, float* xyz32, int64_t batch, int64_t points, cufkb_stream_t stream) {
  return block_forward_xyz32_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, xyz32, batch, points, stream, false, {});
}

int cufkb_block_backward_from_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                    const void* first_direction, const void* initial_normal, const float* xyz32, const void* grad_xyz,
                                    void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch, int64_t points,
                                    cufkb_stream_t stream) {
  return block_backward_xyz32_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz32, grad_xyz, grad_lengths,
                                       grad_angles, grad_dihedrals, batch, points, stream, false, {});
}

int cufkb_block_forward_packed_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                     const void* first_direction, const void* initial_normal, const int64_t* chain_points, void* xyz, float* xyz32,
                                     int64_t batch, int64_t total_points, int64_t max_points, cufkb_stream_t stream) {
  if (int st = check_packed_total(batch, total_points)) return st;
  return block_forward_xyz32_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, xyz32, batch, max_points, stream, true,
                                      cufkb::PackedLayout{chain_points, total_points});
}

int cufkb_block_backward_packed_from_xyz32(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                           const void* first_direction, const void* initial_normal, const int64_t* chain_points, const float* xyz32,
                                           const void* grad_xyz, void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch,
                                           int64_t total_points, int64_t max_points, cufkb_stream_t stream) {
  if (int st = check_packed_total(batch, total_points)) return st;
  return block_backward_xyz32_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz32, grad_xyz, grad_lengths,
                                       grad_angles, grad_dihedrals, batch, max_points, stream, true, cufkb::PackedLayout{chain_points, total_points});
}

int cufkb_block_mse(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                    const void* initial_normal, const void* target, void* loss, void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch,
                    int64_t points, cufkb_stream_t stream) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (dtype != CUFKB_FLOAT32 && dtype != CUFKB_FLOAT64) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch == 0) return CUFKB_SUCCESS;
  const bool grads = grad_lengths || grad_angles || grad_dihedrals;
  if (grads && !(grad_lengths && grad_angles && grad_dihedrals)) return CUFKB_ERROR_NULL_POINTER;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, target, loss},
                                    {lengths, angles, dihedrals, p0, first_direction, initial_normal, target, loss, grad_lengths, grad_angles,
                                     grad_dihedrals})) {
    return st;
  }
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT32) {
    return block_mse_impl<float>(lengths, angles, dihedrals, p0, first_direction, initial_normal, target, loss, grad_lengths, grad_angles, grad_dihedrals,
                                 batch, n, s);
  }
  return block_mse_impl<double>(lengths, angles, dihedrals, p0, first_direction, initial_normal, target, loss, grad_lengths, grad_angles, grad_dihedrals,
                                batch, n, s);
}

int cufkb_block_forward_packed(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                               const void* initial_normal, const int64_t* chain_points, void* xyz, int64_t batch, int64_t total_points,
                               int64_t max_points, cufkb_stream_t stream) {
  if (int st = check_packed_total(batch, total_points)) return st;
  return block_forward_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, batch, max_points, stream, true,
                                cufkb::PackedLayout{chain_points, total_points});
}

int cufkb_block_backward_packed_from_xyz(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                         const void* first_direction, const void* initial_normal, const int64_t* chain_points, const void* xyz,
                                         const void* grad_xyz, void* grad_lengths, void* grad_angles, void* grad_dihedrals, int64_t batch,
                                         int64_t total_points, int64_t max_points, cufkb_stream_t stream) {
  if (int st = check_packed_total(batch, total_points)) return st;
  return block_backward_from_xyz_dispatch(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths,
                                          grad_angles, grad_dihedrals, batch, max_points, stream, true,
                                          cufkb::PackedLayout{chain_points, total_points});
}

int cufkb_torsion_forward(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                          void* xyz, int64_t batch, int64_t points, cufkb_stream_t stream) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (!raw_pairs || !xyz) return CUFKB_ERROR_NULL_POINTER;
  if (!constants) return CUFKB_ERROR_INVALID_VALUE;
  if (raw_row_stride < 0) return CUFKB_ERROR_BAD_STRIDE;
  const size_t es = elem_size(dtype);
  if (!aligned(raw_pairs, es) || !aligned(xyz, es)) return CUFKB_ERROR_MISALIGNED;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CUFKB_FLOAT32:
      return torsion_forward_impl<float>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s);
    case CUFKB_FLOAT64:
      return torsion_forward_impl<double>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s);
    case CUFKB_FLOAT16:
      return torsion_forward_impl<__half>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s);
    default:
      return torsion_forward_impl<__nv_bfloat16>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s);
  }
}

int cufkb_torsion_backward(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                           const void* grad_xyz, void* grad_raw_pairs, int64_t grad_row_stride, int64_t batch, int64_t points,
                           cufkb_stream_t stream) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (!raw_pairs || !grad_xyz || !grad_raw_pairs) return CUFKB_ERROR_NULL_POINTER;
  if (!constants) return CUFKB_ERROR_INVALID_VALUE;
  if (raw_row_stride < 0 || grad_row_stride < 0 || (batch > 1 && grad_row_stride < 2 * (points - 3))) return CUFKB_ERROR_BAD_STRIDE;
  const size_t es = elem_size(dtype);
  if (!aligned(raw_pairs, es) || !aligned(grad_xyz, es) || !aligned(grad_raw_pairs, es)) return CUFKB_ERROR_MISALIGNED;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CUFKB_FLOAT32:
      return torsion_backward_impl<float>(raw_pairs, raw_row_stride, constants, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
    case CUFKB_FLOAT64:
      return torsion_backward_impl<double>(raw_pairs, raw_row_stride, constants, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
    case CUFKB_FLOAT16:
      return torsion_backward_impl<__half>(raw_pairs, raw_row_stride, constants, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
    default:
      return torsion_backward_impl<__nv_bfloat16>(raw_pairs, raw_row_stride, constants, grad_xyz, grad_raw_pairs, grad_row_stride, batch,
                                                  n, s);
  }
}

int cufkb_torsion_backward_from_xyz(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                                    const void* xyz, const void* grad_xyz, void* grad_raw_pairs, int64_t grad_row_stride, int64_t batch,
                                    int64_t points, cufkb_stream_t stream) {
  if (dtype != CUFKB_FLOAT32 && dtype != CUFKB_FLOAT64) {
    if (int st = check_shape(dtype, batch, points)) return st;
    if (batch > 0 && !xyz) return CUFKB_ERROR_NULL_POINTER;
    return cufkb_torsion_backward(dtype, raw_pairs, raw_row_stride, constants, grad_xyz, grad_raw_pairs, grad_row_stride, batch, points, stream);
  }
  if (int st = check_shape(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (!raw_pairs || !xyz || !grad_xyz || !grad_raw_pairs) return CUFKB_ERROR_NULL_POINTER;
  if (!constants) return CUFKB_ERROR_INVALID_VALUE;
  if (raw_row_stride < 0 || grad_row_stride < 0 || (batch > 1 && grad_row_stride < 2 * (points - 3))) return CUFKB_ERROR_BAD_STRIDE;
  const size_t es = elem_size(dtype);
  if (!aligned(raw_pairs, es) || !aligned(xyz, es) || !aligned(grad_xyz, es) || !aligned(grad_raw_pairs, es)) return CUFKB_ERROR_MISALIGNED;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT32) {
    return torsion_backward_xyz_impl<float>(raw_pairs, raw_row_stride, constants, xyz, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
  }
  return torsion_backward_xyz_impl<double>(raw_pairs, raw_row_stride, constants, xyz, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
}

int cufkb_torsion_forward_xyz32(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants, void* xyz,
                                float* xyz32, int64_t batch, int64_t points, cufkb_stream_t stream) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (dtype != CUFKB_FLOAT16 && dtype != CUFKB_BFLOAT16) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch == 0) return CUFKB_SUCCESS;
  if (!raw_pairs || !xyz || !xyz32) return CUFKB_ERROR_NULL_POINTER;
  if (!constants) return CUFKB_ERROR_INVALID_VALUE;
  if (raw_row_stride < 0) return CUFKB_ERROR_BAD_STRIDE;
  if (!aligned(raw_pairs, 2) || !aligned(xyz, 2) || !aligned(xyz32, sizeof(float))) return CUFKB_ERROR_MISALIGNED;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT16) return torsion_forward_impl<__half>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s, xyz32);
  return torsion_forward_impl<__nv_bfloat16>(raw_pairs, raw_row_stride, constants, xyz, batch, n, s, xyz32);
}

int cufkb_torsion_backward_from_xyz32(int dtype, const void* raw_pairs, int64_t raw_row_stride, const cufkb_torsion_constants* constants,
                                      const float* xyz32, const void* grad_xyz, void* grad_raw_pairs, int64_t grad_row_stride, int64_t batch,
                                      int64_t points, cufkb_stream_t stream) {
  if (int st = check_shape(dtype, batch, points)) return st;
  if (dtype != CUFKB_FLOAT16 && dtype != CUFKB_BFLOAT16) return CUFKB_ERROR_UNSUPPORTED_DTYPE;
  if (batch == 0) return CUFKB_SUCCESS;
  if (!raw_pairs || !xyz32 || !grad_xyz || !grad_raw_pairs) return CUFKB_ERROR_NULL_POINTER;
  if (!constants) return CUFKB_ERROR_INVALID_VALUE;
  if (raw_row_stride < 0 || grad_row_stride < 0 || (batch > 1 && grad_row_stride < 2 * (points - 3))) return CUFKB_ERROR_BAD_STRIDE;
  if (!aligned(raw_pairs, 2) || !aligned(xyz32, sizeof(float)) || !aligned(grad_xyz, 2) || !aligned(grad_raw_pairs, 2)) return CUFKB_ERROR_MISALIGNED;
  const int n = static_cast<int>(points);
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT16) {
    return torsion_backward_xyz32_impl<__half>(raw_pairs, raw_row_stride, constants, xyz32, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
  }
  return torsion_backward_xyz32_impl<__nv_bfloat16>(raw_pairs, raw_row_stride, constants, xyz32, grad_xyz, grad_raw_pairs, grad_row_stride, batch, n, s);
}

int cufkb_block_long_workspace_bytes(int dtype, int64_t batch, int64_t points, size_t* bytes) {
  if (!bytes) return CUFKB_ERROR_NULL_POINTER;
  *bytes = 0;
  if (int st = check_long(dtype, batch, points)) return st;
  *bytes = long_workspace_words(batch, long_plan(points)) * elem_size(dtype);
  return CUFKB_SUCCESS;
}

int cufkb_block_forward_long(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                             const void* initial_normal, void* xyz, int64_t batch, int64_t points, void* workspace, size_t workspace_bytes,
                             cufkb_stream_t stream) {
  if (int st = check_long(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, xyz, workspace}, {lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz})) {
    return st;
  }
  if (!aligned(workspace, 16)) return CUFKB_ERROR_MISALIGNED;
  const LongPlan lp = long_plan(points);
  if (workspace_bytes < static_cast<size_t>(batch) * lp.segs * cufkb::kTotalWords * elem_size(dtype)) return CUFKB_ERROR_WORKSPACE;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT32) {
    const cufkb::BlockArgs<float> a{static_cast<const float*>(lengths), static_cast<const float*>(angles), static_cast<const float*>(dihedrals),
                                    static_cast<const float*>(p0), static_cast<const float*>(first_direction), static_cast<const float*>(initial_normal)};
    return block_forward_long_impl<float>(a, xyz, batch, points, workspace, s);
  }
  const cufkb::BlockArgs<double> a{static_cast<const double*>(lengths), static_cast<const double*>(angles), static_cast<const double*>(dihedrals),
                                   static_cast<const double*>(p0), static_cast<const double*>(first_direction), static_cast<const double*>(initial_normal)};
  return block_forward_long_impl<double>(a, xyz, batch, points, workspace, s);
}

int cufkb_block_forward_long_static(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0,
                                    const void* first_direction, const void* initial_normal, void* xyz, int64_t batch, int64_t points,
                                    cufkb_stream_t stream) {
  if (int st = check_long(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, xyz}, {lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz})) {
    return st;
  }
  if (static_cast<size_t>(batch) * long_plan(points).segs * cufkb::kTotalWords * elem_size(dtype) > kStaticScratchBytes) {
    return CUFKB_ERROR_SCRATCH_CAPACITY;
  }
  int dev = 0;
  if (int e = current_device(&dev)) return fail_cuda(static_cast<cudaError_t>(e));
  int err = 0;
  void* scratch = static_scratch(dev, &err);
  if (err != 0) return fail_cuda(static_cast<cudaError_t>(err));
  return cufkb_block_forward_long(dtype, lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, batch, points, scratch,
                                  kStaticScratchBytes, stream);
}

int cufkb_block_backward_long(int dtype, const void* lengths, const void* angles, const void* dihedrals, const void* p0, const void* first_direction,
                              const void* initial_normal, const void* xyz, const void* grad_xyz, void* grad_lengths, void* grad_angles,
                              void* grad_dihedrals, int64_t batch, int64_t points, void* workspace, size_t workspace_bytes, cufkb_stream_t stream) {
  if (int st = check_long(dtype, batch, points)) return st;
  if (batch == 0) return CUFKB_SUCCESS;
  if (int st = check_block_pointers(dtype, {lengths, angles, dihedrals, xyz, grad_xyz, grad_lengths, grad_angles, grad_dihedrals, workspace},
                                    {lengths, angles, dihedrals, p0, first_direction, initial_normal, xyz, grad_xyz, grad_lengths, grad_angles,
                                     grad_dihedrals})) {
    return st;
  }
  if (!aligned(workspace, 16)) return CUFKB_ERROR_MISALIGNED;
  const LongPlan lp = long_plan(points);
  if (workspace_bytes < long_workspace_words(batch, lp) * elem_size(dtype)) return CUFKB_ERROR_WORKSPACE;
  auto s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CUFKB_FLOAT32) {
    const cufkb::BlockArgs<float> a{static_cast<const float*>(lengths), static_cast<const float*>(angles), static_cast<const float*>(dihedrals),
                                    static_cast<const float*>(p0), static_cast<const float*>(first_direction), static_cast<const float*>(initial_normal)};
    return block_backward_long_impl<float>(a, xyz, grad_xyz, grad_lengths, grad_angles, grad_dihedrals, batch, points, workspace, s);
  }
  const cufkb::BlockArgs<double> a{static_cast<const double*>(lengths), static_cast<const double*>(angles), static_cast<const double*>(dihedrals),
                                   static_cast<const double*>(p0), static_cast<const double*>(first_direction), static_cast<const double*>(initial_normal)};
  return block_backward_long_impl<double>(a, xyz, grad_xyz, grad_lengths, grad_angles, grad_dihedrals, batch, points, workspace, s);
}

const char* cufkb_status_string(int status) {
  switch (status) {
    case CUFKB_SUCCESS:
      return "success";
    case CUFKB_ERROR_INVALID_DTYPE:
      return "dtype must be float32, float64, float16, or bfloat16";
    case CUFKB_ERROR_NULL_POINTER:
      return "a required buffer is NULL";
    case CUFKB_ERROR_POINT_COUNT:
      return "point_count must be >= 4";
    case CUFKB_ERROR_TOO_MANY_STEPS:
      return "supports at most 2048 local transforms";
    case CUFKB_ERROR_SHAPE_LIMITS:
      return "shape exceeds int32 kernel limits";
    case CUFKB_ERROR_BAD_STRIDE:
      return "row stride too small for the pairs of one chain";
    case CUFKB_ERROR_MISALIGNED:
      return "pointer not aligned to its element size";
    case CUFKB_ERROR_INVALID_VALUE:
      return "torsion constants must not be NULL";
    case CUFKB_ERROR_CUDA:
      return "CUDA runtime error";
    case CUFKB_ERROR_WORKSPACE:
      return "workspace is smaller than cufkb_block_long_workspace_bytes";
    case CUFKB_ERROR_UNSUPPORTED_DTYPE:
      return "dtype not served here: chains longer than 2051 points and the fused loss take float32 and float64 only, the float32-position (xyz32) entries float16 and bfloat16 only";
    case CUFKB_ERROR_SCRATCH_CAPACITY:
      return "batch x segments exceeds the 2 MiB static scratch of cufkb_block_forward_long_static";
    default:
      return "unknown status";
  }
}

int cufkb_last_cuda_error(void) { return g_last_cuda_error; }

}  // extern "C"
