// PyTorch boundary of cufk_b200: the C++ autograd `apply` wrappers around the C ABI (cufkb.h).
//
// Mirrors the reference's extension (src/cufk/csrc/block.cu:367-445, torsion.cu:413-447) and its
// checks (src/cufk/csrc/extension_utils.cuh:57-143): same argument meaning, same error texts, outputs
// allocated through the caching allocator on the input's device, launches on the current stream
// under a device guard, no host synchronisation.  Anchors may be None (the kernel then uses the
// defaults without any host-to-device copy).  This file holds host code only; every kernel lives in
// libcufkb.so.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/autograd.h>
#include <torch/extension.h>

#include <optional>
#include <vector>

#include "cufkb.h"

namespace {

using torch::Tensor;
using torch::autograd::AutogradContext;
using torch::autograd::tensor_list;

constexpr int kMaxSteps = CUFKB_MAX_STEPS;

bool supported_dtype(torch::ScalarType t) {
  return t == torch::kFloat32 || t == torch::kFloat64 || t == torch::kFloat16 || t == torch::kBFloat16;
}

int dtype_code(torch::ScalarType t) {
  switch (t) {
    case torch::kFloat32:
      return CUFKB_FLOAT32;
    case torch::kFloat64:
      return CUFKB_FLOAT64;
    case torch::kFloat16:
      return CUFKB_FLOAT16;
    case torch::kBFloat16:
      return CUFKB_BFLOAT16;
    default:
      TORCH_CHECK(false, "unsupported dtype");
  }
}

// extension_utils.cuh:57-61
void check_cuda_float(const Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(supported_dtype(x.scalar_type()), name, " must be float32, float64, float16, or bfloat16");
  TORCH_CHECK(x.is_contiguous(), name, " must be contiguous");
}

// extension_utils.cuh:63-68
void check_cuda_float_row_contiguous(const Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(supported_dtype(x.scalar_type()), name, " must be float32, float64, float16, or bfloat16");
  TORCH_CHECK(x.dim() == 2, name, " must have shape (B, K)");
  TORCH_CHECK(x.stride(1) == 1, name, " must have stride(1) == 1");
}

// extension_utils.cuh:70-74
void check_like(const Tensor& x, const Tensor& ref, const char* name) {
  check_cuda_float(x, name);
  TORCH_CHECK(x.scalar_type() == ref.scalar_type(), name, " must have the same dtype as reference");
  TORCH_CHECK(x.device() == ref.device(), name, " must be on the same device as reference");
}

// extension_utils.cuh:76-82; an undefined tensor means "use the default anchor"
Tensor checked_anchor(const Tensor& x, const Tensor& ref, const char* name) {
  if (!x.defined()) return x;
  TORCH_CHECK(x.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(x.scalar_type() == ref.scalar_type(), name, " must have the same dtype as reference");
  TORCH_CHECK(x.device() == ref.device(), name, " must be on the same device as reference");
  TORCH_CHECK(x.sizes() == torch::IntArrayRef({3}), name, " must have shape (3,)");
  TORCH_CHECK(!x.requires_grad(), name, " gradients are not supported");
  return x.contiguous();
}

struct Shape {
  int64_t batch;
  int64_t points;
};

// extension_utils.cuh:119-126
Shape chain_shape_from_steps(const Tensor& ref, int64_t steps) {
  TORCH_CHECK(ref.size(0) <= INT32_MAX && steps + 3 <= INT32_MAX, "shape exceeds int32 kernel limits");
  TORCH_CHECK(steps >= 1, "point_count must be >= 4");
  return {ref.size(0), steps + 3};
}

// the step cap of ChainLaunch (extension_utils.cuh:128-143), checked after the anchors
void check_max_local_transforms(const Shape& shape, const char* op_name) {
  TORCH_CHECK(shape.points - 3 <= kMaxSteps, op_name, " supports at most ", kMaxSteps, " local transforms");
}

// block.cu:367-378
Shape check_geom(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals) {
  check_cuda_float(lengths, "lengths");
  check_like(angles, lengths, "angles");
  check_like(dihedrals, lengths, "dihedrals");
  TORCH_CHECK(lengths.dim() == 2, "lengths must have shape (B, N-1)");
  TORCH_CHECK(angles.dim() == 2, "angles must have shape (B, N-2)");
  TORCH_CHECK(dihedrals.dim() == 2, "dihedrals must have shape (B, N-3)");
  const Shape shape = chain_shape_from_steps(lengths, lengths.size(1) - 2);
  TORCH_CHECK(angles.sizes() == torch::IntArrayRef({shape.batch, shape.points - 2}), "bad angles shape");
  TORCH_CHECK(dihedrals.sizes() == torch::IntArrayRef({shape.batch, shape.points - 3}), "bad dihedrals shape");
  return shape;
}

// torsion.cu:413-417
Shape check_pairs(const Tensor& raw) {
  check_cuda_float_row_contiguous(raw, "raw_pairs");
  TORCH_CHECK(raw.size(1) % 2 == 0, "raw_pairs second dimension must be even");
  const Shape shape = chain_shape_from_steps(raw, raw.size(1) / 2);
  check_max_local_transforms(shape, "torsion_pairs");
  return shape;
}

void check_status(int status, const char* op) {
  if (status == CUFKB_SUCCESS) return;
  if (status == CUFKB_ERROR_CUDA) {
    const auto err = static_cast<cudaError_t>(cufkb_last_cuda_error());
    TORCH_CHECK(false, op, ": CUDA error: ", cudaGetErrorString(err));
  }
  TORCH_CHECK(false, op, ": ", cufkb_status_string(status));
}

const void* ptr_or_null(const Tensor& t) { return t.defined() ? t.data_ptr() : nullptr; }
void* out_ptr_or_null(const Tensor& t) { return t.defined() ? t.data_ptr() : nullptr; }

cufkb_stream_t current_stream() { return reinterpret_cast<cufkb_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

struct Anchors {
  Tensor p0, first_direction, initial_normal;
};

Anchors checked_anchors(const Tensor& p0, const Tensor& fd, const Tensor& nn, const Tensor& ref, const Shape& shape, bool step_cap = true) {
  Anchors a{checked_anchor(p0, ref, "p0"), checked_anchor(fd, ref, "first_direction"), checked_anchor(nn, ref, "initial_normal")};
  if (step_cap) check_max_local_transforms(shape, "reconstruct");
  return a;
}

Tensor block_forward_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a, const Shape& shape,
                          Tensor* xyz32 = nullptr) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor xyz = torch::empty({shape.batch, shape.points, 3}, lengths.options());
  if (xyz32 != nullptr) {
    // float16/bfloat16: the float32 positions as well, for the backward
    *xyz32 = torch::empty({shape.batch, shape.points, 3}, lengths.options().dtype(torch::kFloat32));
    check_status(cufkb_block_forward_xyz32(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                           ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), xyz.data_ptr(),
                                           xyz32->data_ptr<float>(), shape.batch, shape.points, current_stream()),
                 "reconstruct");
    return xyz;
  }
  check_status(cufkb_block_forward(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                   ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), xyz.data_ptr(),
                                   shape.batch, shape.points, current_stream()),
               "reconstruct");
  return xyz;
}

bool is_16bit(const Tensor& t) { return t.scalar_type() == torch::kHalf || t.scalar_type() == torch::kBFloat16; }

// Backward from the forward's output xyz (float32/float64; 16-bit types recompute).
std::vector<Tensor> block_backward_xyz_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a, const Tensor& xyz,
                                            const Tensor& grad_points, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor gl = torch::empty_like(lengths);
  Tensor ga = torch::empty_like(angles);
  Tensor gd = torch::empty_like(dihedrals);
  if (is_16bit(lengths) && xyz.scalar_type() == torch::kFloat32) {
    // float16/bfloat16 with the forward's float32 positions
    check_status(cufkb_block_backward_from_xyz32(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                                 ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                                 xyz.data_ptr<float>(), grad_points.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(),
                                                 shape.batch, shape.points, current_stream()),
                 "reconstruct backward");
    return {gl, ga, gd};
  }
  check_status(cufkb_block_backward_from_xyz(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                             ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), xyz.data_ptr(),
                                             grad_points.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(), shape.batch, shape.points,
                                             current_stream()),
               "reconstruct backward");
  return {gl, ga, gd};
}

std::vector<Tensor> block_backward_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a,
                                        const Tensor& grad_points, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor gl = torch::empty_like(lengths);
  Tensor ga = torch::empty_like(angles);
  Tensor gd = torch::empty_like(dihedrals);
  check_status(cufkb_block_backward(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                    ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                    grad_points.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(), shape.batch, shape.points,
                                    current_stream()),
               "reconstruct backward");
  return {gl, ga, gd};
}

Tensor opt(const std::optional<Tensor>& t) { return t.has_value() ? *t : Tensor(); }

// block.cu:393-429
class ReconstructAutograd : public torch::autograd::Function<ReconstructAutograd> {
 public:
  // Anchors are optional non-variable arguments: torch's autograd Function records every Tensor
  // argument as a differentiable input and cannot take an undefined one.
  static Tensor forward(AutogradContext* ctx, Tensor lengths, Tensor angles, Tensor dihedrals, std::optional<Tensor> p0,
                        std::optional<Tensor> first_direction, std::optional<Tensor> initial_normal) {
    const Shape shape = check_geom(lengths, angles, dihedrals);
    const Anchors a = checked_anchors(opt(p0), opt(first_direction), opt(initial_normal), lengths, shape);
    // the backward reads the output instead of walking the chain again; the version counter of the
    // saved output catches in-place edits of xyz
    // float16/bfloat16 save the float32 positions instead (a 16-bit position is too coarse for the
    // bond directions the backward takes from it); they are not visible to the caller
    Tensor xyz32;
    Tensor xyz = block_forward_impl(lengths, angles, dihedrals, a, shape, is_16bit(lengths) ? &xyz32 : nullptr);
    ctx->save_for_backward({lengths, angles, dihedrals, xyz32.defined() ? xyz32 : xyz});
    ctx->saved_data["p0"] = a.p0.defined() ? c10::IValue(a.p0) : c10::IValue();
    ctx->saved_data["first_direction"] = a.first_direction.defined() ? c10::IValue(a.first_direction) : c10::IValue();
    ctx->saved_data["initial_normal"] = a.initial_normal.defined() ? c10::IValue(a.initial_normal) : c10::IValue();
    return xyz;
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
    const auto saved = ctx->get_saved_variables();
    const Tensor& lengths = saved[0];
    const Tensor& angles = saved[1];
    const Tensor& dihedrals = saved[2];
    Tensor grad_points = grad_outputs[0].is_contiguous() ? grad_outputs[0] : grad_outputs[0].contiguous();
    check_like(grad_points, lengths, "grad_points");
    const Shape shape = check_geom(lengths, angles, dihedrals);
    auto anchor = [&](const char* key) {
      const c10::IValue& v = ctx->saved_data[key];
      return v.isTensor() ? v.toTensor() : Tensor();
    };
    const Anchors a{anchor("p0"), anchor("first_direction"), anchor("initial_normal")};
    auto grads = block_backward_xyz_impl(lengths, angles, dihedrals, a, saved[3], grad_points, shape);
    return {grads[0], grads[1], grads[2], Tensor(), Tensor(), Tensor()};
  }
};

// ---- chains of any length (segments of at most 2048 steps; no counterpart in the reference) ----
Tensor long_workspace(const Tensor& like, const Shape& shape) {
  size_t bytes = 0;
  check_status(cufkb_block_long_workspace_bytes(dtype_code(like.scalar_type()), shape.batch, shape.points, &bytes), "reconstruct_long");
  return torch::empty({static_cast<int64_t>(bytes)}, like.options().dtype(torch::kUInt8));
}

Tensor block_forward_long_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor xyz = torch::empty({shape.batch, shape.points, 3}, lengths.options());
  Tensor ws = long_workspace(lengths, shape);
  check_status(cufkb_block_forward_long(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                        ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), xyz.data_ptr(),
                                        shape.batch, shape.points, ws.data_ptr(), static_cast<size_t>(ws.numel()), current_stream()),
               "reconstruct_long");
  return xyz;
}

std::vector<Tensor> block_backward_long_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a, const Tensor& xyz,
                                             const Tensor& grad_points, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor gl = torch::empty_like(lengths);
  Tensor ga = torch::empty_like(angles);
  Tensor gd = torch::empty_like(dihedrals);
  Tensor ws = long_workspace(lengths, shape);
  check_status(cufkb_block_backward_long(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                         ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), xyz.data_ptr(),
                                         grad_points.data_ptr(), gl.data_ptr(), ga.data_ptr(), gd.data_ptr(), shape.batch, shape.points,
                                         ws.data_ptr(), static_cast<size_t>(ws.numel()), current_stream()),
               "reconstruct_long backward");
  return {gl, ga, gd};
}

class LongAutograd : public torch::autograd::Function<LongAutograd> {
 public:
  static Tensor forward(AutogradContext* ctx, Tensor lengths, Tensor angles, Tensor dihedrals, std::optional<Tensor> p0,
                        std::optional<Tensor> first_direction, std::optional<Tensor> initial_normal) {
    const Shape shape = check_geom(lengths, angles, dihedrals);
    const Anchors a = checked_anchors(opt(p0), opt(first_direction), opt(initial_normal), lengths, shape, /*step_cap=*/false);
    Tensor xyz = block_forward_long_impl(lengths, angles, dihedrals, a, shape);
    ctx->save_for_backward({lengths, angles, dihedrals, xyz});
    ctx->saved_data["p0"] = a.p0.defined() ? c10::IValue(a.p0) : c10::IValue();
    ctx->saved_data["first_direction"] = a.first_direction.defined() ? c10::IValue(a.first_direction) : c10::IValue();
    ctx->saved_data["initial_normal"] = a.initial_normal.defined() ? c10::IValue(a.initial_normal) : c10::IValue();
    return xyz;
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
    const auto saved = ctx->get_saved_variables();
    Tensor grad_points = grad_outputs[0].is_contiguous() ? grad_outputs[0] : grad_outputs[0].contiguous();
    check_like(grad_points, saved[0], "grad_points");
    const Shape shape = check_geom(saved[0], saved[1], saved[2]);
    auto anchor = [&](const char* key) {
      const c10::IValue& v = ctx->saved_data[key];
      return v.isTensor() ? v.toTensor() : Tensor();
    };
    const Anchors a{anchor("p0"), anchor("first_direction"), anchor("initial_normal")};
    auto grads = block_backward_long_impl(saved[0], saved[1], saved[2], a, saved[3], grad_points, shape);
    return {grads[0], grads[1], grads[2], Tensor(), Tensor(), Tensor()};
  }
};

Tensor apply_long(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                  const std::optional<Tensor>& first_direction, const std::optional<Tensor>& initial_normal) {
  return LongAutograd::apply(lengths, angles, dihedrals, p0, first_direction, initial_normal);
}

Tensor apply_autograd(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                      const std::optional<Tensor>& first_direction, const std::optional<Tensor>& initial_normal) {
  return ReconstructAutograd::apply(lengths, angles, dihedrals, p0, first_direction, initial_normal);
}

// ---- packed (ragged) batches: chains of different lengths in one call (no counterpart in the
// reference).  lengths/angles/dihedrals are 1-D packed rows, chain_points the (B+1,) int64 point
// offsets on the device; the point total follows from the sizes (lengths has total - B entries), so
// nothing is read back from the device.
struct PackedShape {
  int64_t batch;
  int64_t total;  // points of all chains
  int64_t max_points;
};

PackedShape check_packed(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Tensor& chain_points, int64_t max_points) {
  check_cuda_float(lengths, "lengths");
  check_like(angles, lengths, "angles");
  check_like(dihedrals, lengths, "dihedrals");
  TORCH_CHECK(lengths.dim() == 1 && angles.dim() == 1 && dihedrals.dim() == 1, "packed lengths, angles and dihedrals must be 1-D");
  TORCH_CHECK(chain_points.is_cuda() && chain_points.device() == lengths.device(), "chain_points must be CUDA, on the device of lengths");
  TORCH_CHECK(chain_points.scalar_type() == torch::kInt64 && chain_points.dim() == 1 && chain_points.is_contiguous(),
              "chain_points must be a contiguous 1-D int64 tensor of B+1 offsets");
  const int64_t batch = chain_points.size(0) - 1;
  TORCH_CHECK(batch >= 0, "chain_points must hold B+1 offsets");
  const int64_t total = lengths.size(0) + batch;
  TORCH_CHECK(angles.size(0) == total - 2 * batch, "bad angles shape");
  TORCH_CHECK(dihedrals.size(0) == total - 3 * batch, "bad dihedrals shape");
  TORCH_CHECK(batch <= INT32_MAX, "shape exceeds int32 kernel limits");
  TORCH_CHECK(total >= 4 * batch, "packed chains must hold at least 4 points each on average");
  TORCH_CHECK(batch == 0 || max_points >= 4, "point_count must be >= 4");
  TORCH_CHECK(max_points - 3 <= kMaxSteps, "reconstruct supports at most ", kMaxSteps, " local transforms");
  return {batch, total, max_points};
}

Tensor packed_forward_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a, const Tensor& chain_points,
                           const PackedShape& shape, Tensor* xyz32 = nullptr) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor xyz = torch::empty({shape.total, 3}, lengths.options());
  if (xyz32 != nullptr) {
    // float16/bfloat16: the float32 positions as well, for the backward
    *xyz32 = torch::empty({shape.total, 3}, lengths.options().dtype(torch::kFloat32));
    check_status(cufkb_block_forward_packed_xyz32(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                                  ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                                  chain_points.data_ptr<int64_t>(), xyz.data_ptr(), xyz32->data_ptr<float>(), shape.batch, shape.total,
                                                  shape.max_points, current_stream()),
                 "reconstruct_packed");
    return xyz;
  }
  check_status(cufkb_block_forward_packed(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                          ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                          chain_points.data_ptr<int64_t>(), xyz.data_ptr(), shape.batch, shape.total, shape.max_points, current_stream()),
               "reconstruct_packed");
  return xyz;
}

std::vector<Tensor> packed_backward_impl(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Anchors& a,
                                         const Tensor& chain_points, const Tensor& xyz, const Tensor& grad_points, const PackedShape& shape) {
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor gl = torch::empty_like(lengths);
  Tensor ga = torch::empty_like(angles);
  Tensor gd = torch::empty_like(dihedrals);
  if (is_16bit(lengths) && xyz.scalar_type() == torch::kFloat32) {
    check_status(cufkb_block_backward_packed_from_xyz32(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                                        ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                                        chain_points.data_ptr<int64_t>(), xyz.data_ptr<float>(), grad_points.data_ptr(), gl.data_ptr(),
                                                        ga.data_ptr(), gd.data_ptr(), shape.batch, shape.total, shape.max_points, current_stream()),
                 "reconstruct_packed backward");
    return {gl, ga, gd};
  }
  check_status(cufkb_block_backward_packed_from_xyz(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(),
                                                    ptr_or_null(a.p0), ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal),
                                                    chain_points.data_ptr<int64_t>(), xyz.data_ptr(), grad_points.data_ptr(), gl.data_ptr(),
                                                    ga.data_ptr(), gd.data_ptr(), shape.batch, shape.total, shape.max_points, current_stream()),
               "reconstruct_packed backward");
  return {gl, ga, gd};
}

class PackedAutograd : public torch::autograd::Function<PackedAutograd> {
 public:
  static Tensor forward(AutogradContext* ctx, Tensor lengths, Tensor angles, Tensor dihedrals, Tensor chain_points, int64_t max_points,
                       std::optional<Tensor> p0, std::optional<Tensor> first_direction, std::optional<Tensor> initial_normal) {
    const PackedShape shape = check_packed(lengths, angles, dihedrals, chain_points, max_points);
    const Anchors a{checked_anchor(opt(p0), lengths, "p0"), checked_anchor(opt(first_direction), lengths, "first_direction"),
                    checked_anchor(opt(initial_normal), lengths, "initial_normal")};
    Tensor xyz32;  // float16/bfloat16 save the float32 positions instead, as the (B, N) wrapper does
    Tensor xyz = packed_forward_impl(lengths, angles, dihedrals, a, chain_points, shape, is_16bit(lengths) ? &xyz32 : nullptr);
    ctx->save_for_backward({lengths, angles, dihedrals, chain_points, xyz32.defined() ? xyz32 : xyz});
    ctx->saved_data["max_points"] = max_points;
    ctx->saved_data["p0"] = a.p0.defined() ? c10::IValue(a.p0) : c10::IValue();
    ctx->saved_data["first_direction"] = a.first_direction.defined() ? c10::IValue(a.first_direction) : c10::IValue();
    ctx->saved_data["initial_normal"] = a.initial_normal.defined() ? c10::IValue(a.initial_normal) : c10::IValue();
    return xyz;
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
    const auto saved = ctx->get_saved_variables();
    Tensor grad_points = grad_outputs[0].is_contiguous() ? grad_outputs[0] : grad_outputs[0].contiguous();
    check_like(grad_points, saved[0], "grad_points");
    const PackedShape shape = check_packed(saved[0], saved[1], saved[2], saved[3], ctx->saved_data["max_points"].toInt());
    auto anchor = [&](const char* key) {
      const c10::IValue& v = ctx->saved_data[key];
      return v.isTensor() ? v.toTensor() : Tensor();
    };
    const Anchors a{anchor("p0"), anchor("first_direction"), anchor("initial_normal")};
    auto grads = packed_backward_impl(saved[0], saved[1], saved[2], a, saved[3], saved[4], grad_points, shape);
    return {grads[0], grads[1], grads[2], Tensor(), Tensor(), Tensor(), Tensor(), Tensor()};
  }
};

Tensor apply_packed(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const Tensor& chain_points, int64_t max_points,
                    const std::optional<Tensor>& p0, const std::optional<Tensor>& first_direction, const std::optional<Tensor>& initial_normal) {
  return PackedAutograd::apply(lengths, angles, dihedrals, chain_points, max_points, p0, first_direction, initial_normal);
}

// ---------------------------------------------------------------------------------------------
// torsion path: constants are a run-time argument (9 doubles), not a JIT build
// ---------------------------------------------------------------------------------------------
cufkb_torsion_constants torsion_constants(const std::vector<double>& c) {
  TORCH_CHECK(c.size() == 9, "torsion constants must be 3 bond lengths, 3 angle sines and 3 angle cosines");
  cufkb_torsion_constants out;
  for (int i = 0; i < 3; ++i) {
    out.bond_lengths[i] = c[i];
    out.bond_angle_sin[i] = c[3 + i];
    out.bond_angle_cos[i] = c[6 + i];
  }
  return out;
}

Tensor torsion_forward_impl(const Tensor& raw, const std::vector<double>& consts, const Shape& shape, Tensor* xyz32 = nullptr) {
  const c10::cuda::CUDAGuard guard(raw.device());
  const cufkb_torsion_constants c = torsion_constants(consts);
  Tensor xyz = torch::empty({shape.batch, shape.points, 3}, raw.options());
  if (xyz32 != nullptr) {
    // float16/bfloat16: the float32 positions as well, for the backward
    *xyz32 = torch::empty({shape.batch, shape.points, 3}, raw.options().dtype(torch::kFloat32));
    check_status(cufkb_torsion_forward_xyz32(dtype_code(raw.scalar_type()), raw.data_ptr(), raw.stride(0), &c, xyz.data_ptr(), xyz32->data_ptr<float>(),
                                             shape.batch, shape.points, current_stream()),
                 "torsion_pairs");
    return xyz;
  }
  check_status(cufkb_torsion_forward(dtype_code(raw.scalar_type()), raw.data_ptr(), raw.stride(0), &c, xyz.data_ptr(), shape.batch,
                                     shape.points, current_stream()),
               "torsion_pairs");
  return xyz;
}

// gradient tensor with raw's strides (empty_strided_like, extension_utils.cuh:162-164); rows that
// would overlap (a broadcast row stride) get a contiguous gradient instead
Tensor pair_grad_like(const Tensor& raw, const Shape& shape) {
  return (shape.batch <= 1 || raw.stride(0) >= raw.size(1)) ? torch::empty_strided(raw.sizes(), raw.strides(), raw.options())
                                                            : torch::empty(raw.sizes(), raw.options());
}

Tensor torsion_backward_xyz_impl(const Tensor& raw, const std::vector<double>& consts, const Tensor& xyz, const Tensor& grad_points, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(raw.device());
  const cufkb_torsion_constants c = torsion_constants(consts);
  Tensor grad = pair_grad_like(raw, shape);
  if (is_16bit(raw) && xyz.scalar_type() == torch::kFloat32) {
    // float16/bfloat16 with the forward's float32 positions
    check_status(cufkb_torsion_backward_from_xyz32(dtype_code(raw.scalar_type()), raw.data_ptr(), raw.stride(0), &c, xyz.data_ptr<float>(),
                                                   grad_points.data_ptr(), grad.data_ptr(), grad.stride(0), shape.batch, shape.points,
                                                   current_stream()),
                 "torsion_pairs backward");
    return grad;
  }
  check_status(cufkb_torsion_backward_from_xyz(dtype_code(raw.scalar_type()), raw.data_ptr(), raw.stride(0), &c, xyz.data_ptr(),
                                               grad_points.data_ptr(), grad.data_ptr(), grad.stride(0), shape.batch, shape.points,
                                               current_stream()),
               "torsion_pairs backward");
  return grad;
}

Tensor torsion_backward_impl(const Tensor& raw, const std::vector<double>& consts, const Tensor& grad_points, const Shape& shape) {
  const c10::cuda::CUDAGuard guard(raw.device());
  const cufkb_torsion_constants c = torsion_constants(consts);
  Tensor grad = pair_grad_like(raw, shape);
  check_status(cufkb_torsion_backward(dtype_code(raw.scalar_type()), raw.data_ptr(), raw.stride(0), &c, grad_points.data_ptr(),
                                      grad.data_ptr(), grad.stride(0), shape.batch, shape.points, current_stream()),
               "torsion_pairs backward");
  return grad;
}

// torsion.cu:419-437: the forward saves raw_pairs and its output, which the backward reads
class TorsionAutograd : public torch::autograd::Function<TorsionAutograd> {
 public:
  static Tensor forward(AutogradContext* ctx, Tensor raw_pairs, std::vector<double> consts) {
    const Shape shape = check_pairs(raw_pairs);
    // float16/bfloat16 save the float32 positions instead, as the block wrapper does
    Tensor xyz32;
    Tensor xyz = torsion_forward_impl(raw_pairs, consts, shape, is_16bit(raw_pairs) ? &xyz32 : nullptr);
    ctx->save_for_backward({raw_pairs, xyz32.defined() ? xyz32 : xyz});
    ctx->saved_data["consts"] = c10::IValue(consts);
    return xyz;
  }

  static tensor_list backward(AutogradContext* ctx, tensor_list grad_outputs) {
    const auto saved = ctx->get_saved_variables();
    const Tensor& raw = saved[0];
    const std::vector<double> consts = ctx->saved_data["consts"].toDoubleVector();
    Tensor grad_points = grad_outputs[0].is_contiguous() ? grad_outputs[0] : grad_outputs[0].contiguous();
    check_like(grad_points, raw, "grad_points");
    const Shape shape = check_pairs(raw);
    return {torsion_backward_xyz_impl(raw, consts, saved[1], grad_points, shape), Tensor()};
  }
};

Tensor torsion_apply(const Tensor& raw_pairs, const std::vector<double>& consts) { return TorsionAutograd::apply(raw_pairs, consts); }

// ---------------------------------------------------------------------------------------------
// autograd-free entry points (benchmarks, CUDA-graph capture); same checks and kernels
// ---------------------------------------------------------------------------------------------
Tensor block_forward(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                     const std::optional<Tensor>& fd, const std::optional<Tensor>& nn) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  return block_forward_impl(lengths, angles, dihedrals, a, shape);
}

std::vector<Tensor> block_backward(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                                   const std::optional<Tensor>& fd, const std::optional<Tensor>& nn, const Tensor& grad_points) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  check_like(grad_points, lengths, "grad_points");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  return block_backward_impl(lengths, angles, dihedrals, a, grad_points, shape);
}

std::vector<Tensor> block_backward_from_xyz(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                                            const std::optional<Tensor>& fd, const std::optional<Tensor>& nn, const Tensor& xyz,
                                            const Tensor& grad_points) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  check_like(grad_points, lengths, "grad_points");
  check_like(xyz, lengths, "xyz");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  TORCH_CHECK(xyz.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "xyz must have shape (B, N, 3)");
  return block_backward_xyz_impl(lengths, angles, dihedrals, a, xyz, grad_points, shape);
}

// float16/bfloat16: the forward with its float32 positions, and the backward that reads them
// (cufkb_block_forward_xyz32, cufkb_block_backward_from_xyz32)
std::vector<Tensor> block_forward_xyz32(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                                        const std::optional<Tensor>& fd, const std::optional<Tensor>& nn) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  TORCH_CHECK(is_16bit(lengths), "block_forward_xyz32 supports float16 and bfloat16");
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  Tensor xyz32;
  Tensor xyz = block_forward_impl(lengths, angles, dihedrals, a, shape, &xyz32);
  return {xyz, xyz32};
}

std::vector<Tensor> block_backward_from_xyz32(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                                              const std::optional<Tensor>& fd, const std::optional<Tensor>& nn, const Tensor& xyz32,
                                              const Tensor& grad_points) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  TORCH_CHECK(is_16bit(lengths), "block_backward_from_xyz32 supports float16 and bfloat16");
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  check_like(grad_points, lengths, "grad_points");
  check_cuda_float(xyz32, "xyz32");
  TORCH_CHECK(xyz32.scalar_type() == torch::kFloat32, "xyz32 must be float32");
  TORCH_CHECK(xyz32.device() == lengths.device(), "xyz32 must be on the same device as reference");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  TORCH_CHECK(xyz32.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "xyz32 must have shape (B, N, 3)");
  return block_backward_xyz_impl(lengths, angles, dihedrals, a, xyz32, grad_points, shape);
}

// Fused consumer (cufkb_block_mse): per-chain mean squared distance of the reconstruction to a
// target and, with_grads, its gradient with respect to lengths, angles and dihedrals.
std::vector<Tensor> block_mse(const Tensor& lengths, const Tensor& angles, const Tensor& dihedrals, const std::optional<Tensor>& p0,
                              const std::optional<Tensor>& fd, const std::optional<Tensor>& nn, const Tensor& target, bool with_grads) {
  const Shape shape = check_geom(lengths, angles, dihedrals);
  const Anchors a = checked_anchors(opt(p0), opt(fd), opt(nn), lengths, shape);
  TORCH_CHECK(lengths.scalar_type() == torch::kFloat32 || lengths.scalar_type() == torch::kFloat64, "reconstruct_mse supports float32 and float64");
  check_like(target, lengths, "target");
  TORCH_CHECK(target.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "target must have shape (B, N, 3)");
  const c10::cuda::CUDAGuard guard(lengths.device());
  Tensor loss = torch::empty({shape.batch}, lengths.options());
  Tensor gl, ga, gd;
  if (with_grads) {
    gl = torch::empty_like(lengths);
    ga = torch::empty_like(angles);
    gd = torch::empty_like(dihedrals);
  }
  check_status(cufkb_block_mse(dtype_code(lengths.scalar_type()), lengths.data_ptr(), angles.data_ptr(), dihedrals.data_ptr(), ptr_or_null(a.p0),
                               ptr_or_null(a.first_direction), ptr_or_null(a.initial_normal), target.data_ptr(), loss.data_ptr(), out_ptr_or_null(gl),
                               out_ptr_or_null(ga), out_ptr_or_null(gd), shape.batch, shape.points, current_stream()),
               "reconstruct_mse");
  return {loss, gl, ga, gd};
}

Tensor torsion_forward(const Tensor& raw, const std::vector<double>& consts) { return torsion_forward_impl(raw, consts, check_pairs(raw)); }

Tensor torsion_backward(const Tensor& raw, const std::vector<double>& consts, const Tensor& grad_points) {
  const Shape shape = check_pairs(raw);
  check_like(grad_points, raw, "grad_points");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  return torsion_backward_impl(raw, consts, grad_points, shape);
}

// float16/bfloat16: the torsion forward with its float32 positions, and the backward reading them
std::vector<Tensor> torsion_forward_xyz32(const Tensor& raw, const std::vector<double>& consts) {
  const Shape shape = check_pairs(raw);
  TORCH_CHECK(is_16bit(raw), "torsion_forward_xyz32 supports float16 and bfloat16");
  Tensor xyz32;
  Tensor xyz = torsion_forward_impl(raw, consts, shape, &xyz32);
  return {xyz, xyz32};
}

Tensor torsion_backward_from_xyz32(const Tensor& raw, const std::vector<double>& consts, const Tensor& xyz32, const Tensor& grad_points) {
  const Shape shape = check_pairs(raw);
  TORCH_CHECK(is_16bit(raw), "torsion_backward_from_xyz32 supports float16 and bfloat16");
  check_like(grad_points, raw, "grad_points");
  check_cuda_float(xyz32, "xyz32");
  TORCH_CHECK(xyz32.scalar_type() == torch::kFloat32, "xyz32 must be float32");
  TORCH_CHECK(xyz32.device() == raw.device(), "xyz32 must be on the same device as reference");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  TORCH_CHECK(xyz32.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "xyz32 must have shape (B, N, 3)");
  return torsion_backward_xyz_impl(raw, consts, xyz32, grad_points, shape);
}

Tensor torsion_backward_from_xyz(const Tensor& raw, const std::vector<double>& consts, const Tensor& xyz, const Tensor& grad_points) {
  const Shape shape = check_pairs(raw);
  check_like(grad_points, raw, "grad_points");
  check_like(xyz, raw, "xyz");
  TORCH_CHECK(grad_points.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}), "grad_points must have shape (B, N, 3)");
  TORCH_CHECK(xyz.sizes() == torch::IntArrayRef({shape.batch, shape.points, 3}) && xyz.is_contiguous(), "xyz must be the (B, N, 3) output of the forward");
  return torsion_backward_xyz_impl(raw, consts, xyz, grad_points, shape);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("apply", &apply_autograd, "reconstruct autograd apply", pybind11::arg("lengths"), pybind11::arg("angles"),
        pybind11::arg("dihedrals"), pybind11::arg("p0") = pybind11::none(), pybind11::arg("first_direction") = pybind11::none(),
        pybind11::arg("initial_normal") = pybind11::none());
  m.def("apply_long", &apply_long, "reconstruct autograd apply for chains of any length", pybind11::arg("lengths"), pybind11::arg("angles"),
        pybind11::arg("dihedrals"), pybind11::arg("p0") = pybind11::none(), pybind11::arg("first_direction") = pybind11::none(),
        pybind11::arg("initial_normal") = pybind11::none());
  m.def("apply_packed", &apply_packed, "reconstruct autograd apply for a packed (ragged) batch", pybind11::arg("lengths"), pybind11::arg("angles"),
        pybind11::arg("dihedrals"), pybind11::arg("chain_points"), pybind11::arg("max_points"), pybind11::arg("p0") = pybind11::none(),
        pybind11::arg("first_direction") = pybind11::none(), pybind11::arg("initial_normal") = pybind11::none());
  m.def("torsion_apply", &torsion_apply, "torsion-only autograd apply", pybind11::arg("raw_pairs"), pybind11::arg("constants"));
  m.def("block_forward", &block_forward, "forward kernel only", pybind11::arg("lengths"), pybind11::arg("angles"),
        pybind11::arg("dihedrals"), pybind11::arg("p0") = pybind11::none(), pybind11::arg("first_direction") = pybind11::none(),
        pybind11::arg("initial_normal") = pybind11::none());
  m.def("block_backward", &block_backward, "backward kernel only", pybind11::arg("lengths"), pybind11::arg("angles"),
        pybind11::arg("dihedrals"), pybind11::arg("p0"), pybind11::arg("first_direction"), pybind11::arg("initial_normal"),
        pybind11::arg("grad_points"));
  m.def("block_backward_from_xyz", &block_backward_from_xyz, "backward kernel reading the forward's xyz", pybind11::arg("lengths"),
        pybind11::arg("angles"), pybind11::arg("dihedrals"), pybind11::arg("p0"), pybind11::arg("first_direction"), pybind11::arg("initial_normal"),
        pybind11::arg("xyz"), pybind11::arg("grad_points"));
  m.def("block_forward_xyz32", &block_forward_xyz32, "16-bit forward kernel writing float32 positions as well", pybind11::arg("lengths"),
        pybind11::arg("angles"), pybind11::arg("dihedrals"), pybind11::arg("p0") = pybind11::none(),
        pybind11::arg("first_direction") = pybind11::none(), pybind11::arg("initial_normal") = pybind11::none());
  m.def("block_backward_from_xyz32", &block_backward_from_xyz32, "16-bit backward kernel reading the forward's float32 positions",
        pybind11::arg("lengths"), pybind11::arg("angles"), pybind11::arg("dihedrals"), pybind11::arg("p0"), pybind11::arg("first_direction"),
        pybind11::arg("initial_normal"), pybind11::arg("xyz32"), pybind11::arg("grad_points"));
  m.def("block_mse", &block_mse, "fused reconstruction + mean squared distance to a target (+ gradients)", pybind11::arg("lengths"),
        pybind11::arg("angles"), pybind11::arg("dihedrals"), pybind11::arg("p0"), pybind11::arg("first_direction"), pybind11::arg("initial_normal"),
        pybind11::arg("target"), pybind11::arg("with_grads"));
  m.def("torsion_forward", &torsion_forward, "torsion forward kernel only");
  m.def("torsion_backward", &torsion_backward, "torsion backward kernel only");
  m.def("torsion_backward_from_xyz", &torsion_backward_from_xyz, "torsion backward kernel reading the forward's xyz");
  m.def("torsion_forward_xyz32", &torsion_forward_xyz32, "16-bit torsion forward kernel writing float32 positions as well");
  m.def("torsion_backward_from_xyz32", &torsion_backward_from_xyz32, "16-bit torsion backward kernel reading the forward's float32 positions");
  m.def("max_point_count", &cufkb_max_point_count);
}
