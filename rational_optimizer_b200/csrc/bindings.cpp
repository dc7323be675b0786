// PyTorch bindings for the sm_100a kernels.  This file owns validation
// (device, dtype, contiguity, shape), output allocation and stream selection;
// the .cu files only see raw pointers.  Mirrors the checks of the reference's
// activation/csrc/rational_ext.cpp:10-14, 197-198 (CUDA, contiguous,
// group width <= 256, <= 4 basis atoms) but accepts bf16 as well as fp32.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cuda_runtime.h>
#include <vector>

#include "ext_api.h"

namespace {

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

int dtype_code(const torch::Tensor& t, const char* name) {
  if (t.scalar_type() == torch::kFloat32) return 0;
  if (t.scalar_type() == torch::kBFloat16) return 1;
  TORCH_CHECK(false, name, " must be float32 or bfloat16");
  return -1;
}

torch::ScalarType code_dtype(int code) { return code == 0 ? torch::kFloat32 : torch::kBFloat16; }

void check_f32(const torch::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kFloat32, name, " must be float32");
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed with code ", rc,
              rc > 0 ? cudaGetErrorString(static_cast<cudaError_t>(rc)) : "");
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

void check_grain_coeffs(const torch::Tensor& num, const torch::Tensor& den,
                        const torch::Tensor& logits, const torch::Tensor& centers,
                        const torch::Tensor& beta, int64_t groups) {
  check_f32(num, "numerator");
  check_f32(den, "denominator");
  check_f32(logits, "coeff_logits");
  check_f32(centers, "centers");
  check_f32(beta, "beta");
  TORCH_CHECK(num.dim() == 2 && num.size(0) == groups && num.size(1) == 6, "numerator must be [groups, 6]");
  TORCH_CHECK(den.dim() == 2 && den.size(0) == groups && den.size(1) == 4, "denominator must be [groups, 4]");
  TORCH_CHECK(centers.dim() == 2 && centers.size(0) == groups, "centers must be [groups, basis]");
  const int64_t nb = centers.size(1);
  TORCH_CHECK(nb <= 4, "GRAIN supports at most 4 local basis atoms");
  TORCH_CHECK(beta.sizes() == centers.sizes(), "beta must match centers");
  TORCH_CHECK(logits.dim() == 3 && logits.size(0) == groups && logits.size(1) == nb && logits.size(2) == 2,
              "coeff_logits must be [groups, basis, 2]");
}

std::vector<torch::Tensor> grain_forward(torch::Tensor x, torch::Tensor num, torch::Tensor den,
                                         torch::Tensor logits, torch::Tensor centers,
                                         torch::Tensor beta, double coeff_limit, double eps,
                                         int64_t hidden, int64_t groups, int64_t out_code,
                                         bool want_rho) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  check_grain_coeffs(num, den, logits, centers, beta, groups);
  TORCH_CHECK(x.size(-1) == hidden, "x last dimension must equal hidden_dim");
  TORCH_CHECK(hidden % groups == 0 && hidden / groups <= 256, "GRAIN supports group width <= 256");
  const int xc = dtype_code(x, "x");
  const int oc = out_code < 0 ? xc : static_cast<int>(out_code);
  auto y = torch::empty(x.sizes(), x.options().dtype(code_dtype(oc)));
  const int64_t rows = x.numel() / hidden;
  torch::Tensor rho;
  if (want_rho) rho = torch::empty({rows, groups}, x.options().dtype(torch::kFloat32));
  const int rc = ro::grain_forward(x.data_ptr(), xc, num.data_ptr<float>(), den.data_ptr<float>(),
                                   logits.data_ptr<float>(), centers.data_ptr<float>(),
                                   beta.data_ptr<float>(), y.data_ptr(), oc,
                                   want_rho ? rho.data_ptr<float>() : nullptr, rows,
                                   static_cast<int>(hidden), static_cast<int>(groups),
                                   static_cast<int>(centers.size(1)),
                                   static_cast<float>(coeff_limit), static_cast<float>(eps), stream());
  check_rc(rc, "grain_forward");
  if (want_rho) return {y, rho};
  return {y};
}

std::vector<torch::Tensor> grain_backward(torch::Tensor gy, torch::Tensor x, torch::Tensor num,
                                          torch::Tensor den, torch::Tensor logits,
                                          torch::Tensor centers, torch::Tensor beta,
                                          double coeff_limit, double eps, int64_t hidden,
                                          int64_t groups, c10::optional<torch::Tensor> alpha,
                                          c10::optional<torch::Tensor> abeta) {
  check_cuda(gy, "grad_output");
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  check_grain_coeffs(num, den, logits, centers, beta, groups);
  TORCH_CHECK(gy.sizes() == x.sizes(), "grad_output must match x");
  TORCH_CHECK(hidden % groups == 0 && hidden / groups <= 256, "GRAIN supports group width <= 256");
  const bool restricted = alpha.has_value();
  TORCH_CHECK(restricted == abeta.has_value(), "affine alpha and beta come together");
  if (restricted) {
    check_f32(*alpha, "affine_alpha");
    check_f32(*abeta, "affine_beta");
    TORCH_CHECK(alpha->numel() == groups && abeta->numel() == groups, "affine terms must be [groups]");
  }
  const int xc = dtype_code(x, "x");
  const int gc = dtype_code(gy, "grad_output");
  auto gx = torch::empty(x.sizes(), x.options());
  auto gnum = torch::zeros_like(num);
  auto gden = torch::zeros_like(den);
  auto gcoeff = torch::zeros_like(logits);
  const int64_t rows = x.numel() / hidden;
  const int nb = static_cast<int>(centers.size(1));
  auto partial = torch::empty({std::max<int64_t>(1, ro::grain_backward_partial_size(rows, groups, nb))},
                              x.options().dtype(torch::kFloat32));
  torch::Tensor nonlinear;
  if (restricted) nonlinear = torch::empty(x.sizes(), x.options().dtype(torch::kFloat32));
  const int rc = ro::grain_backward(
      gy.data_ptr(), gc, x.data_ptr(), xc, num.data_ptr<float>(), den.data_ptr<float>(),
      logits.data_ptr<float>(), centers.data_ptr<float>(), beta.data_ptr<float>(),
      restricted ? alpha->data_ptr<float>() : nullptr, restricted ? abeta->data_ptr<float>() : nullptr,
      restricted ? nonlinear.data_ptr<float>() : nullptr, gx.data_ptr(), xc, gnum.data_ptr<float>(),
      gden.data_ptr<float>(), gcoeff.data_ptr<float>(), partial.data_ptr<float>(), rows,
      static_cast<int>(hidden), static_cast<int>(groups), nb, static_cast<float>(coeff_limit),
      static_cast<float>(eps), stream());
  check_rc(rc, "grain_backward");
  if (restricted) return {nonlinear, gx, gnum, gden, gcoeff};
  return {gx, gnum, gden, gcoeff};
}

std::vector<torch::Tensor> grain_affine_statistics(torch::Tensor x, torch::Tensor feature,
                                                   double eps, int64_t hidden, int64_t groups) {
  check_cuda(x, "x");
  check_cuda(feature, "feature");
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.sizes() == feature.sizes() && x.scalar_type() == feature.scalar_type(),
              "feature must match x");
  TORCH_CHECK(hidden % groups == 0 && hidden / groups <= 256, "GRAIN supports group width <= 256");
  const int64_t rows = x.numel() / hidden;
  auto rho = torch::empty({rows, groups, 1}, x.options().dtype(torch::kFloat32));
  auto stats = torch::empty({groups, 5}, x.options().dtype(torch::kFloat64));
  auto partial = torch::empty({std::max<int64_t>(1, ro::grain_affine_partial_size(rows, groups))},
                              x.options().dtype(torch::kFloat64));
  const int rc = ro::grain_affine_statistics(x.data_ptr(), feature.data_ptr(), dtype_code(x, "x"),
                                             rho.data_ptr<float>(), stats.data_ptr<double>(),
                                             partial.data_ptr<double>(), rows,
                                             static_cast<int>(hidden), static_cast<int>(groups),
                                             static_cast<float>(eps), stream());
  check_rc(rc, "grain_affine_statistics");
  return {stats, rho};
}

torch::Tensor legacy_forward(torch::Tensor x, torch::Tensor a, torch::Tensor b, bool signed_den) {
  check_f32(x, "x");
  check_f32(a, "numerator");
  check_f32(b, "denominator");
  TORCH_CHECK(a.numel() == 6 && b.numel() == 4, "legacy rational has 6+4 coefficients");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  check_rc(ro::legacy_rational_forward(x.data_ptr<float>(), a.data_ptr<float>(), b.data_ptr<float>(),
                                       y.data_ptr<float>(), x.numel(), signed_den, stream()),
           "legacy_forward");
  return y;
}

std::vector<torch::Tensor> legacy_backward(torch::Tensor gy, torch::Tensor x, torch::Tensor a,
                                           torch::Tensor b, bool signed_den) {
  check_f32(gy, "grad_output");
  check_f32(x, "x");
  check_f32(a, "numerator");
  check_f32(b, "denominator");
  TORCH_CHECK(gy.sizes() == x.sizes(), "grad_output must match x");
  const c10::cuda::CUDAGuard guard(x.device());
  auto gx = torch::empty_like(x);
  auto ga = torch::empty_like(a);
  auto gb = torch::empty_like(b);
  auto partial = torch::empty({ro::legacy_rational_blocks(x.numel()) * 10}, x.options());
  check_rc(ro::legacy_rational_backward(gy.data_ptr<float>(), x.data_ptr<float>(), a.data_ptr<float>(),
                                        b.data_ptr<float>(), gx.data_ptr<float>(), ga.data_ptr<float>(),
                                        gb.data_ptr<float>(), partial.data_ptr<float>(), x.numel(),
                                        signed_den, stream()),
           "legacy_backward");
  return {gx, ga, gb};
}

std::vector<torch::Tensor> rmsnorm_forward(torch::Tensor x, torch::Tensor w, double eps,
                                           int64_t out_code) {
  check_cuda(x, "x");
  check_f32(w, "weight");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t d = x.size(-1);
  TORCH_CHECK(w.numel() == d, "weight must match the last dimension");
  const int64_t rows = x.numel() / d;
  const int xc = dtype_code(x, "x");
  const int oc = out_code < 0 ? xc : static_cast<int>(out_code);
  auto y = torch::empty(x.sizes(), x.options().dtype(code_dtype(oc)));
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  check_rc(ro::rmsnorm_forward(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(),
                               rows, static_cast<int>(d), static_cast<float>(eps), xc, oc, stream()),
           "rmsnorm_forward");
  return {y, rstd};
}

std::vector<torch::Tensor> rmsnorm_backward(torch::Tensor dy, torch::Tensor x, torch::Tensor w,
                                            torch::Tensor rstd) {
  check_cuda(dy, "dy");
  check_cuda(x, "x");
  check_f32(w, "weight");
  check_f32(rstd, "rstd");
  TORCH_CHECK(dy.sizes() == x.sizes(), "dy must match x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  auto dx = torch::empty_like(x);
  auto dw = torch::empty_like(w);
  auto partial = torch::empty({std::max<int64_t>(1, ro::rmsnorm_backward_partial_size(rows, static_cast<int>(d)))},
                              x.options().dtype(torch::kFloat32));
  check_rc(ro::rmsnorm_backward(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(),
                                dx.data_ptr(), dw.data_ptr<float>(), partial.data_ptr<float>(), rows,
                                static_cast<int>(d), dtype_code(x, "x"), dtype_code(dy, "dy"), 0, stream()),
           "rmsnorm_backward");
  return {dx, dw};
}

std::vector<torch::Tensor> rope_qkv_forward(torch::Tensor qkv, torch::Tensor cos_t,
                                            torch::Tensor sin_t, int64_t B, int64_t S, int64_t H,
                                            int64_t hd) {
  check_cuda(qkv, "qkv");
  check_f32(cos_t, "cos");
  check_f32(sin_t, "sin");
  TORCH_CHECK(qkv.numel() == B * S * 3 * H * hd, "qkv has the wrong size");
  TORCH_CHECK(cos_t.size(0) >= S && cos_t.size(1) == hd / 2, "rope tables too small");
  TORCH_CHECK(hd % 8 == 0, "head_dim must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto opts = qkv.options();
  auto q = torch::empty({B, H, S, hd}, opts);
  auto k = torch::empty({B, H, S, hd}, opts);
  auto v = torch::empty({B, H, S, hd}, opts);
  check_rc(ro::rope_qkv_forward(qkv.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                q.data_ptr(), k.data_ptr(), v.data_ptr(), static_cast<int>(B),
                                static_cast<int>(S), static_cast<int>(H), static_cast<int>(hd),
                                dtype_code(qkv, "qkv"), stream()),
           "rope_qkv_forward");
  return {q, k, v};
}

torch::Tensor rope_qkv_backward(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv,
                                torch::Tensor cos_t, torch::Tensor sin_t) {
  check_cuda(dq, "dq");
  check_cuda(dk, "dk");
  check_cuda(dv, "dv");
  check_f32(cos_t, "cos");
  check_f32(sin_t, "sin");
  TORCH_CHECK(dq.dim() == 4 && dq.sizes() == dk.sizes() && dq.sizes() == dv.sizes(), "dq/dk/dv shapes");
  const c10::cuda::CUDAGuard guard(dq.device());
  const int64_t B = dq.size(0), H = dq.size(1), S = dq.size(2), hd = dq.size(3);
  auto dqkv = torch::empty({B * S, 3 * H * hd}, dq.options());
  check_rc(ro::rope_qkv_backward(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), cos_t.data_ptr<float>(),
                                 sin_t.data_ptr<float>(), dqkv.data_ptr(), static_cast<int>(B),
                                 static_cast<int>(S), static_cast<int>(H), static_cast<int>(hd),
                                 dtype_code(dq, "dq"), stream()),
           "rope_qkv_backward");
  return dqkv;
}

torch::Tensor cross_entropy_fwd_bwd(torch::Tensor logits, torch::Tensor target, double grad_scale,
                                    int64_t ignore_index) {
  check_cuda(logits, "logits");
  check_cuda(target, "target");
  TORCH_CHECK(logits.dim() == 2, "logits must be [rows, vocab]");
  TORCH_CHECK(target.scalar_type() == torch::kInt64 && target.numel() == logits.size(0),
              "target must be int64 [rows]");
  const c10::cuda::CUDAGuard guard(logits.device());
  auto loss = torch::empty({logits.size(0)}, logits.options().dtype(torch::kFloat32));
  check_rc(ro::cross_entropy_fwd_bwd(logits.data_ptr(), target.data_ptr<int64_t>(), loss.data_ptr<float>(),
                                     logits.size(0), static_cast<int>(logits.size(1)),
                                     static_cast<float>(grad_scale), ignore_index,
                                     dtype_code(logits, "logits"), stream()),
           "cross_entropy_fwd_bwd");
  return loss;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels for rational_optimizer_b200";
  m.def("grain_forward", &grain_forward);
  m.def("grain_backward", &grain_backward);
  m.def("grain_affine_statistics", &grain_affine_statistics);
  m.def("legacy_forward", &legacy_forward);
  m.def("legacy_backward", &legacy_backward);
  m.def("rmsnorm_forward", &rmsnorm_forward);
  m.def("rmsnorm_backward", &rmsnorm_backward);
  m.def("rope_qkv_forward", &rope_qkv_forward);
  m.def("rope_qkv_backward", &rope_qkv_backward);
  m.def("cross_entropy_fwd_bwd", &cross_entropy_fwd_bwd);
}
