// torch custom ops over the C ABI: torch.ops.pla_b200.*
//
// The reference reaches its kernels through a torch extension op
// (data/stencil_direct_cuda_v7/stencil_cuda.cpp:10-41,
// data/stencil_cuda_v2/stencil_cuda.cpp:7-37): TORCH_CHECK argument errors,
// a CUDAGuard on the input's device, the output allocated by the op
// (contiguous, shaped like the input) and the launch on the current stream.
// These ops keep that behaviour on top of include/pla_b200.h, and add what
// the torch.compile / CUDA-graph world needs:
//   * a Meta kernel per op (shapes, dtypes and memory formats only), so fake
//     tensors trace through them;
//   * an Autograd kernel that lets the forward run on tensors that require
//     grad and raises if a backward is ever asked of it (the reference ops
//     are forward only);
//   * every filter is read from device memory by the kernel at run time, so
//     a graph replay after an in-place weight update uses the new weights.
// A non-zero status from the C ABI becomes a RuntimeError naming the entry
// point and the status text; no CPU path exists (a CPU tensor is an error).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/autograd_not_implemented_fallback.h>
#include <torch/library.h>

#include <optional>
#include <string>

#include "../../include/pla_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kHalf: return PLA_F16;
    case at::kFloat: return PLA_F32;
    case at::kDouble: return PLA_F64;
    case at::kBFloat16: return PLA_BF16;
    default: TORCH_CHECK(false, "pla_b200: unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_status(int st, const char* what) {
  if (st == PLA_OK) return;
  std::string detail = st == PLA_ERR_CUDA || st == PLA_ERR_TOO_LARGE ? pla_last_cuda_error() : "";
  TORCH_CHECK(false, what, ": ", pla_status_string(st), detail.empty() ? "" : " (" + detail + ")");
}

pla_stream_t current_stream(const at::Tensor& x) {
  return reinterpret_cast<pla_stream_t>(c10::cuda::getCurrentCUDAStream(x.device().index()).stream());
}

void check_param(const at::Tensor& x, const at::Tensor& p, const char* name, int64_t numel) {
  TORCH_CHECK(p.is_cuda() && p.device() == x.device(), name, " must be a CUDA tensor on the input's device");
  TORCH_CHECK(p.scalar_type() == x.scalar_type(), name, " dtype ", p.scalar_type(), " does not match x's ",
              x.scalar_type());
  TORCH_CHECK(p.numel() == numel, name, " must have ", numel, " elements, got ", p.numel());
}

const void* opt_ptr(const std::optional<at::Tensor>& t) { return t ? t->data_ptr() : nullptr; }

std::optional<at::Tensor> opt_contig(const std::optional<at::Tensor>& t) {
  if (!t) return std::nullopt;
  return t->contiguous();
}

// ---- single-step stencil: data/stencil_7x7.py:10-12 ----------------------
void check_stencil_input(const at::Tensor& x) {
  TORCH_CHECK(x.is_cuda(), "stencil7x7: x must be a CUDA tensor");
  TORCH_CHECK((x.dim() == 4 && x.size(1) == 1) || (x.dim() == 3 && x.size(0) == 1),
              "stencil7x7: expected [N,1,H,W] or [1,H,W] input, got ", x.sizes());
}

at::Tensor stencil7x7_cuda(const at::Tensor& x, const at::Tensor& weight, const std::optional<at::Tensor>& bias) {
  check_stencil_input(x);
  check_param(x, weight, "weight", 49);
  if (bias) check_param(x, *bias, "bias", 1);
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = at::empty(x.sizes(), x.options());
  if (y.numel() == 0) return y;
  const at::Tensor w = weight.contiguous();
  const auto b = opt_contig(bias);
  const int64_t n = x.dim() == 4 ? x.size(0) : 1;
  const int64_t h = x.size(-2), wd = x.size(-1);
  const int64_t sn = x.dim() == 4 ? x.stride(0) : h * wd;
  TORCH_CHECK(n <= INT32_MAX && h <= INT32_MAX && wd <= INT32_MAX, "stencil7x7: size exceeds int32");
  check_status(pla_stencil7x7_forward(x.data_ptr(), w.data_ptr(), opt_ptr(b), y.data_ptr(), static_cast<int>(n),
                                      static_cast<int>(h), static_cast<int>(wd), sn, x.stride(-2), x.stride(-1),
                                      dtype_code(x), current_stream(x)),
               "pla_stencil7x7_forward");
  return y;
}

// Meta kernels use the symbolic-size API, so dynamic shapes stay symbolic
// under torch.compile / torch.export.
at::Tensor stencil7x7_meta(const at::Tensor& x, const at::Tensor& weight, const std::optional<at::Tensor>& bias) {
  return at::empty_symint(x.sym_sizes(), x.options());
}

// ---- depthwise k x k: data/depthwise_conv_7x7.py:15-29 --------------------
// Layout from the input's memory format, as torch's own convolution does.
at::MemoryFormat depthwise_format(const at::Tensor& x) {
  if (x.is_contiguous()) return at::MemoryFormat::Contiguous;
  if (x.is_contiguous(at::MemoryFormat::ChannelsLast)) return at::MemoryFormat::ChannelsLast;
  return at::MemoryFormat::Contiguous;
}

int64_t filter_side(const at::Tensor& x, const at::Tensor& weight) {
  const int64_t k = weight.dim() == 4 ? weight.size(-1) : 7;
  TORCH_CHECK(k == 3 || k == 5 || k == 7, "depthwise: only 3x3, 5x5 and 7x7 filters are supported");
  TORCH_CHECK(weight.dim() != 4 || (weight.size(0) == x.size(1) && weight.size(1) == 1 && weight.size(2) == k),
              "depthwise: weight must have shape [C,1,", k, ",", k, "], got ", weight.sizes());
  return k;
}

at::Tensor depthwise_impl(const at::Tensor& x_in, const at::Tensor& weight, const std::optional<at::Tensor>& bias,
                          int64_t k) {
  TORCH_CHECK(x_in.is_cuda(), "depthwise: x must be a CUDA tensor");
  TORCH_CHECK(x_in.dim() == 4, "depthwise: input must have shape [N,C,H,W], got ", x_in.sizes());
  const int64_t C = x_in.size(1);
  check_param(x_in, weight, "weight", C * k * k);
  if (bias) check_param(x_in, *bias, "bias", C);
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::MemoryFormat fmt = depthwise_format(x_in);
  const at::Tensor x = x_in.contiguous(fmt);
  at::Tensor y = at::empty(x.sizes(), x.options().memory_format(fmt));
  if (y.numel() == 0) return y;
  TORCH_CHECK(x.size(0) <= INT32_MAX && C <= INT32_MAX && x.size(2) <= INT32_MAX && x.size(3) <= INT32_MAX,
              "depthwise: size exceeds int32");
  const at::Tensor w = weight.contiguous();
  const auto b = opt_contig(bias);
  const int layout = fmt == at::MemoryFormat::ChannelsLast ? PLA_NHWC : PLA_NCHW;
  check_status(pla_depthwise_forward(x.data_ptr(), w.data_ptr(), opt_ptr(b), y.data_ptr(),
                                     static_cast<int>(x.size(0)), static_cast<int>(C), static_cast<int>(x.size(2)),
                                     static_cast<int>(x.size(3)), static_cast<int>(k), dtype_code(x), layout,
                                     current_stream(x)),
               "pla_depthwise_forward");
  return y;
}

at::Tensor depthwise_meta_impl(const at::Tensor& x) {
  return at::empty_symint(x.sym_sizes(), x.options().memory_format(depthwise_format(x)));
}

at::Tensor depthwise7x7_cuda(const at::Tensor& x, const at::Tensor& weight, const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.dim() == 4, "depthwise7x7: input must have shape [N,C,H,W], got ", x.sizes());
  TORCH_CHECK(weight.dim() != 4 || weight.size(-1) == 7, "depthwise7x7: weight must have shape [C,1,7,7]");
  return depthwise_impl(x, weight, bias, 7);
}

at::Tensor depthwise_cuda(const at::Tensor& x, const at::Tensor& weight, const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.dim() == 4, "depthwise: input must have shape [N,C,H,W], got ", x.sizes());
  return depthwise_impl(x, weight, bias, filter_side(x, weight));
}

at::Tensor depthwise_meta(const at::Tensor& x, const at::Tensor& weight, const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.dim() == 4, "depthwise: input must have shape [N,C,H,W], got ", x.sym_sizes());
  return depthwise_meta_impl(x);
}

// ---- depthwise 7x7 + LayerNorm over C (NHWC), fused ----------------------
at::Tensor depthwise7x7_layernorm_cuda(const at::Tensor& x, const at::Tensor& weight,
                                       const std::optional<at::Tensor>& bias,
                                       const std::optional<at::Tensor>& norm_weight,
                                       const std::optional<at::Tensor>& norm_bias, double eps) {
  TORCH_CHECK(x.is_cuda(), "depthwise7x7_layernorm: x must be a CUDA tensor");
  TORCH_CHECK(x.dim() == 4 && x.is_contiguous(at::MemoryFormat::ChannelsLast),
              "depthwise7x7_layernorm normalises NHWC pixels: pass a channels_last [N,C,H,W] input");
  const int64_t C = x.size(1);
  check_param(x, weight, "weight", C * 49);
  for (const auto* t : {&bias, &norm_weight, &norm_bias})
    if (*t) check_param(x, **t, "bias / norm_weight / norm_bias", C);
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::ChannelsLast));
  if (y.numel() == 0) return y;
  TORCH_CHECK(x.size(0) <= INT32_MAX && C <= INT32_MAX && x.size(2) <= INT32_MAX && x.size(3) <= INT32_MAX,
              "depthwise7x7_layernorm: size exceeds int32");
  const at::Tensor w = weight.contiguous();
  const auto b = opt_contig(bias), g = opt_contig(norm_weight), be = opt_contig(norm_bias);
  check_status(pla_depthwise7x7_layernorm_nhwc(x.data_ptr(), w.data_ptr(), opt_ptr(b), opt_ptr(g), opt_ptr(be),
                                               static_cast<float>(eps), y.data_ptr(), static_cast<int>(x.size(0)),
                                               static_cast<int>(C), static_cast<int>(x.size(2)),
                                               static_cast<int>(x.size(3)), dtype_code(x), current_stream(x)),
               "pla_depthwise7x7_layernorm_nhwc");
  return y;
}

at::Tensor depthwise7x7_layernorm_meta(const at::Tensor& x, const at::Tensor& weight,
                                       const std::optional<at::Tensor>& bias,
                                       const std::optional<at::Tensor>& norm_weight,
                                       const std::optional<at::Tensor>& norm_bias, double eps) {
  return at::empty_symint(x.sym_sizes(), x.options().memory_format(at::MemoryFormat::ChannelsLast));
}

// ---- iterated stencil on one device (zero Dirichlet boundary) ------------
at::Tensor stencil7x7_iterate_cuda(const at::Tensor& x_in, const at::Tensor& weight, int64_t steps,
                                   const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x_in.is_cuda(), "stencil7x7_iterate: x must be a CUDA tensor");
  TORCH_CHECK(x_in.dim() == 2, "stencil7x7_iterate: expected a [H, W] grid, got ", x_in.sizes());
  TORCH_CHECK(steps >= 0 && steps <= INT32_MAX, "stencil7x7_iterate: steps must be in [0, 2^31)");
  check_param(x_in, weight, "weight", 49);
  if (bias) check_param(x_in, *bias, "bias", 1);
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.contiguous();
  at::Tensor y = at::empty_like(x);
  if (y.numel() == 0) return y;
  TORCH_CHECK(x.size(0) <= INT32_MAX && x.size(1) <= INT32_MAX, "stencil7x7_iterate: size exceeds int32");
  at::Tensor scratch = steps > 0 ? at::empty_like(x) : y;
  const at::Tensor w = weight.contiguous();
  const auto b = opt_contig(bias);
  check_status(pla_stencil7x7_iterate(x.data_ptr(), w.data_ptr(), opt_ptr(b), y.data_ptr(),
                                      steps > 0 ? scratch.data_ptr() : nullptr, static_cast<int>(x.size(0)),
                                      static_cast<int>(x.size(1)), static_cast<int>(steps), dtype_code(x),
                                      current_stream(x)),
               "pla_stencil7x7_iterate");
  return y;
}

at::Tensor stencil7x7_iterate_meta(const at::Tensor& x, const at::Tensor& weight, int64_t steps,
                                   const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.dim() == 2, "stencil7x7_iterate: expected a [H, W] grid, got ", x.sym_sizes());
  return at::empty_symint(x.sym_sizes(), x.options());
}

}  // namespace

TORCH_LIBRARY(pla_b200, m) {
  m.def("stencil7x7(Tensor x, Tensor weight, Tensor? bias=None) -> Tensor");
  m.def("depthwise7x7(Tensor x, Tensor weight, Tensor? bias=None) -> Tensor");
  m.def("depthwise(Tensor x, Tensor weight, Tensor? bias=None) -> Tensor");
  m.def(
      "depthwise7x7_layernorm(Tensor x, Tensor weight, Tensor? bias=None, Tensor? norm_weight=None, "
      "Tensor? norm_bias=None, float eps=1e-6) -> Tensor");
  m.def("stencil7x7_iterate(Tensor x, Tensor weight, int steps, Tensor? bias=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(pla_b200, CUDA, m) {
  m.impl("stencil7x7", &stencil7x7_cuda);
  m.impl("depthwise7x7", &depthwise7x7_cuda);
  m.impl("depthwise", &depthwise_cuda);
  m.impl("depthwise7x7_layernorm", &depthwise7x7_layernorm_cuda);
  m.impl("stencil7x7_iterate", &stencil7x7_iterate_cuda);
}

TORCH_LIBRARY_IMPL(pla_b200, Meta, m) {
  m.impl("stencil7x7", &stencil7x7_meta);
  m.impl("depthwise7x7", &depthwise_meta);
  m.impl("depthwise", &depthwise_meta);
  m.impl("depthwise7x7_layernorm", &depthwise7x7_layernorm_meta);
  m.impl("stencil7x7_iterate", &stencil7x7_iterate_meta);
}

TORCH_LIBRARY_IMPL(pla_b200, Autograd, m) {
  for (const char* op : {"stencil7x7", "depthwise7x7", "depthwise", "depthwise7x7_layernorm", "stencil7x7_iterate"})
    m.impl(op, torch::autograd::autogradNotImplementedFallback());
}
