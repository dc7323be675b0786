// PyTorch bindings for the sm_100a kernels.  This file owns validation
// (device, dtype, contiguity, shape), output allocation and stream selection;
// the .cu files only see raw pointers.  Mirrors the checks of the reference's
// activation/csrc/rational_ext.cpp:10-14, 197-198 (CUDA, contiguous,
// group width <= 256, <= 4 basis atoms) but accepts bf16 as well as fp32.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
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

// Fused residual add + RMSNorm.  x fp32 [rows, d]; delta bf16 or None.
// Returns (x_new fp32, y bf16, rstd).  With delta None, x_new is x itself.
std::vector<torch::Tensor> add_rmsnorm_forward(torch::Tensor x, c10::optional<torch::Tensor> delta,
                                               torch::Tensor w, double eps) {
  check_f32(x, "x");
  check_f32(w, "weight");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  torch::Tensor x_new = x;
  const void* dptr = nullptr;
  if (delta.has_value()) {
    check_cuda(*delta, "delta");
    TORCH_CHECK(delta->scalar_type() == torch::kBFloat16 && delta->numel() == x.numel(), "delta must be bf16 like x");
    dptr = delta->data_ptr();
    x_new = torch::empty_like(x);
  }
  auto y = torch::empty(x.sizes(), x.options().dtype(torch::kBFloat16));
  auto rstd = torch::empty({rows}, x.options());
  check_rc(ro::add_rmsnorm_forward(x.data_ptr<float>(), dptr, w.data_ptr<float>(), x_new.data_ptr<float>(),
                                   y.data_ptr(), rstd.data_ptr<float>(), rows, static_cast<int>(d),
                                   static_cast<float>(eps), at::cuda::getCurrentCUDAStream()),
           "add_rmsnorm_forward");
  return {x_new, y, rstd};
}

// Returns (dx fp32, ddelta bf16 or undefined, dw).
// dw_into: the weight's fp32 gradient buffer; when given, dw is added into it
// (in the reduction kernel) and the returned dw is undefined.
std::vector<torch::Tensor> add_rmsnorm_backward(torch::Tensor dy, c10::optional<torch::Tensor> dres,
                                                torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                                                bool want_ddelta, c10::optional<torch::Tensor> dw_into) {
  check_cuda(dy, "dy");
  check_f32(x, "x");
  check_f32(w, "weight");
  check_f32(rstd, "rstd");
  TORCH_CHECK(dy.scalar_type() == torch::kBFloat16 && dy.numel() == x.numel(), "dy must be bf16 like x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t d = x.size(-1);
  const int64_t rows = x.numel() / d;
  const float* rp = nullptr;
  if (dres.has_value()) {
    check_f32(*dres, "dres");
    rp = dres->data_ptr<float>();
  }
  auto dx = torch::empty_like(x);
  torch::Tensor dd;
  if (want_ddelta) dd = torch::empty(x.sizes(), x.options().dtype(torch::kBFloat16));
  torch::Tensor dw;
  if (dw_into.has_value()) {
    check_f32(*dw_into, "dw_into");
    TORCH_CHECK(dw_into->numel() == d, "dw_into size");
  } else {
    dw = torch::empty_like(w);
  }
  float* dwp = dw_into.has_value() ? dw_into->data_ptr<float>() : dw.data_ptr<float>();
  auto partial = torch::empty({std::max<int64_t>(1, ro::rmsnorm_backward_partial_size(rows, static_cast<int>(d)))},
                              x.options());
  check_rc(ro::add_rmsnorm_backward(dy.data_ptr(), rp, x.data_ptr<float>(), w.data_ptr<float>(),
                                    rstd.data_ptr<float>(), dx.data_ptr<float>(),
                                    want_ddelta ? dd.data_ptr() : nullptr, dwp, dw_into.has_value(),
                                    partial.data_ptr<float>(), rows, static_cast<int>(d),
                                    at::cuda::getCurrentCUDAStream()),
           "add_rmsnorm_backward");
  return {dx, dd, dw};
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
  // [B, S, H, hd] storage (token-major, the layout the attention kernels
  // read and write without transposes), returned as [B, H, S, hd] views.
  auto q = torch::empty({B, S, H, hd}, opts);
  auto k = torch::empty({B, S, H, hd}, opts);
  auto v = torch::empty({B, S, H, hd}, opts);
  check_rc(ro::rope_qkv_forward(qkv.data_ptr(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
                                q.data_ptr(), k.data_ptr(), v.data_ptr(), static_cast<int>(B),
                                static_cast<int>(S), static_cast<int>(H), static_cast<int>(hd),
                                dtype_code(qkv, "qkv"), stream()),
           "rope_qkv_forward");
  return {q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)};
}

torch::Tensor rope_qkv_backward(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv,
                                torch::Tensor cos_t, torch::Tensor sin_t) {
  TORCH_CHECK(dq.dim() == 4 && dq.sizes() == dk.sizes() && dq.sizes() == dv.sizes(), "dq/dk/dv shapes");
  const c10::cuda::CUDAGuard guard(dq.device());
  const int64_t B = dq.size(0), H = dq.size(1), S = dq.size(2), hd = dq.size(3);
  // gradients of the [B, H, S, hd] views: token-major storage (a copy only
  // when the producer chose another layout)
  dq = dq.transpose(1, 2).contiguous();
  dk = dk.transpose(1, 2).contiguous();
  dv = dv.transpose(1, 2).contiguous();
  check_cuda(dq, "dq");
  check_cuda(dk, "dk");
  check_cuda(dv, "dv");
  check_f32(cos_t, "cos");
  check_f32(sin_t, "sin");
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

// ---------------------------------------------------------------------------
// tcgen05 GEMM.  a_km: a is [.., K, M] (else [.., M, K]); b_nk: b is [.., N, K]
// (else [.., K, N]).  Returns None when the layout is unsupported so the
// caller can use another path.

torch::Tensor& gemm_error_flag(const torch::Device& dev) {
  static std::vector<torch::Tensor> flags(64);
  auto& f = flags.at(dev.index());
  if (!f.defined()) f = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  return f;
}

c10::optional<torch::Tensor> gemm_bf16_impl(torch::Tensor a, torch::Tensor b, bool a_km, bool b_nk,
                                            bool out_f32, c10::optional<torch::Tensor> d, double alpha,
                                            double beta) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "gemm operands must be CUDA tensors");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "gemm operands must be bfloat16");
  TORCH_CHECK(a.dim() == b.dim() && (a.dim() == 2 || a.dim() == 3), "gemm operands must be 2-D or 3-D");
  const c10::cuda::CUDAGuard guard(a.device());
  const bool batched = a.dim() == 3;
  const int64_t batch = batched ? a.size(0) : 1;
  if (batched) TORCH_CHECK(b.size(0) == batch, "batch mismatch");
  if (a.stride(-1) != 1 || b.stride(-1) != 1) return c10::nullopt;
  const int64_t M = a_km ? a.size(-1) : a.size(-2);
  const int64_t K = a_km ? a.size(-2) : a.size(-1);
  const int64_t N = b_nk ? b.size(-2) : b.size(-1);
  const int64_t Kb = b_nk ? b.size(-1) : b.size(-2);
  TORCH_CHECK(K == Kb, "gemm inner dimensions differ");
  auto opts = a.options().dtype(out_f32 ? torch::kFloat32 : torch::kBFloat16);
  torch::Tensor c = batched ? torch::empty({batch, M, N}, opts) : torch::empty({M, N}, opts);
  const void* dptr = nullptr;
  int64_t ldd = 0, sd = 0;
  if (d.has_value()) {
    TORCH_CHECK(d->scalar_type() == torch::kBFloat16 && d->stride(-1) == 1, "gemm D must be bf16 row-major");
    TORCH_CHECK(d->size(-2) == M && d->size(-1) == N, "gemm D shape");
    dptr = d->data_ptr();
    ldd = d->stride(-2);
    sd = batched ? d->stride(0) : 0;
  }
  auto& flag = gemm_error_flag(a.device());
  const int rc = ro::gemm_bf16_tn(a.data_ptr(), a.stride(-2), batched ? a.stride(0) : 0, a_km, b.data_ptr(),
                                  b.stride(-2), batched ? b.stride(0) : 0, !b_nk, c.data_ptr(), N,
                                  batched ? M * N : 0, out_f32, dptr, ldd, sd, static_cast<float>(alpha),
                                  static_cast<float>(beta), static_cast<int>(M), static_cast<int>(N),
                                  static_cast<int>(K), static_cast<int>(batch), flag.data_ptr<int>(),
                                  at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "gemm_bf16");
  return c;
}

c10::optional<torch::Tensor> gemm_bf16(torch::Tensor a, torch::Tensor b, bool a_km, bool b_nk, bool out_f32) {
  return gemm_bf16_impl(a, b, a_km, b_nk, out_f32, c10::nullopt, 1.0, 0.0);
}

c10::optional<torch::Tensor> gemm_bf16_ex(torch::Tensor a, torch::Tensor b, bool a_km, bool b_nk,
                                          bool out_f32, c10::optional<torch::Tensor> d, double alpha,
                                          double beta) {
  return gemm_bf16_impl(a, b, a_km, b_nk, out_f32, d, alpha, beta);
}

torch::Tensor gemm_error(torch::Tensor like) { return gemm_error_flag(like.device()); }

// fp32 c = a . b (layouts as gemm_bf16, 2-D) written to a raw device address
// with row stride ldc - which may be a peer GPU's memory mapped through CUDA
// IPC: every epilogue tile then travels over NVLink as plain 16-byte stores
// while later tiles are still being multiplied.  False when the layout is
// unsupported (nothing is written).
bool gemm_bf16_to(torch::Tensor a, torch::Tensor b, bool a_km, bool b_nk, int64_t c_addr, int64_t ldc) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dim() == 2 && b.dim() == 2, "gemm_bf16_to expects 2-D CUDA tensors");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "gemm_bf16_to expects bfloat16 operands");
  if (a.stride(-1) != 1 || b.stride(-1) != 1 || (c_addr & 15) != 0 || ldc % 4 != 0) return false;
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t M = a_km ? a.size(1) : a.size(0);
  const int64_t K = a_km ? a.size(0) : a.size(1);
  const int64_t N = b_nk ? b.size(0) : b.size(1);
  TORCH_CHECK(K == (b_nk ? b.size(1) : b.size(0)), "gemm_bf16_to inner dimensions differ");
  TORCH_CHECK(ldc >= N, "gemm_bf16_to: ldc < N");
  auto& flag = gemm_error_flag(a.device());
  const int rc = ro::gemm_bf16_tn(a.data_ptr(), a.stride(0), 0, a_km, b.data_ptr(), b.stride(0), 0, !b_nk,
                                  reinterpret_cast<void*>(c_addr), ldc, 0, true, nullptr, 0, 0, 1.0f, 0.0f,
                                  static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), 1,
                                  flag.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
  if (rc < 0) return false;
  check_rc(rc, "gemm_bf16_to");
  return true;
}

// 2-SM tcgen05 GEMM: c[M, N] = a[M, K] . b[N, K]^T (bf16, both K-major).
// None when the shape or alignment is unsupported (callers fall back).
c10::optional<torch::Tensor> gemm2_bf16(torch::Tensor a, torch::Tensor b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.dim() == 2 && b.dim() == 2, "gemm2 expects 2-D CUDA tensors");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16, "gemm2 expects bf16");
  TORCH_CHECK(a.size(1) == b.size(1), "gemm2 inner dimensions differ");
  if (a.stride(1) != 1 || b.stride(1) != 1) return c10::nullopt;
  const c10::cuda::CUDAGuard guard(a.device());
  auto c = torch::empty({a.size(0), b.size(0)}, a.options());
  const int rc = ro::gemm2_bf16_nt(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), c.data_ptr(), c.stride(0),
                                   static_cast<int>(a.size(0)), static_cast<int>(b.size(0)),
                                   static_cast<int>(a.size(1)), gemm_error_flag(a.device()).data_ptr<int>(),
                                   at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "gemm2_bf16");
  return c;
}

// Out-projection input gradient with the GRAIN backward fused into the GEMM
// epilogue: returns (gx = dGRAIN(h, bf16(dO W_out)), grad_numerator,
// grad_denominator); w_out_t is W_out^T in bf16 ([N, K], K-major).  None when
// unsupported.
c10::optional<std::vector<torch::Tensor>> grain_out_proj_backward(torch::Tensor dO, torch::Tensor w_out_t,
                                                                  torch::Tensor h, torch::Tensor num,
                                                                  torch::Tensor den, double eps,
                                                                  c10::optional<torch::Tensor> gnum_into,
                                                                  c10::optional<torch::Tensor> gden_into) {
  TORCH_CHECK(dO.is_cuda() && w_out_t.is_cuda() && h.is_cuda() && dO.dim() == 2 && w_out_t.dim() == 2 &&
                  h.dim() == 2, "expects 2-D CUDA tensors");
  TORCH_CHECK(dO.scalar_type() == torch::kBFloat16 && w_out_t.scalar_type() == torch::kBFloat16 &&
                  h.scalar_type() == torch::kBFloat16, "expects bf16");
  TORCH_CHECK(dO.size(1) == w_out_t.size(1) && h.size(0) == dO.size(0) && h.size(1) == w_out_t.size(0),
              "shape mismatch");
  check_f32(num, "numerator");
  check_f32(den, "denominator");
  const int64_t M = dO.size(0), N = w_out_t.size(0), K = dO.size(1);
  if (dO.stride(1) != 1 || w_out_t.stride(1) != 1 || h.stride(1) != 1 || N % 256 != 0 ||
      num.numel() != (N / 256) * 6 || den.numel() != (N / 256) * 4)
    return c10::nullopt;
  const c10::cuda::CUDAGuard guard(dO.device());
  const int groups = static_cast<int>(N / 256);
  const int chunks = ro::gemm2_grain_partial_rows(static_cast<int>(M));
  auto gx = torch::empty({M, N}, dO.options());
  auto partial = torch::empty({static_cast<int64_t>(chunks) * groups * 10}, num.options());
  // gnum_into / gden_into: the coefficients' fp32 gradient buffers; when given
  // the gradients are added into them and the returned tensors are undefined
  const bool into = gnum_into.has_value() && gden_into.has_value();
  if (into) {
    check_f32(*gnum_into, "gnum_into");
    check_f32(*gden_into, "gden_into");
    TORCH_CHECK(gnum_into->numel() == groups * 6 && gden_into->numel() == groups * 4, "gradient buffer sizes");
  }
  torch::Tensor gnum, gden;
  if (!into) {
    gnum = torch::empty({groups, 6}, num.options());
    gden = torch::empty({groups, 4}, num.options());
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  static const bool trace = std::getenv("RO_TRACE_LAUNCH") != nullptr;
  if (trace) std::fprintf(stderr, "grain_out_proj_backward: M=%lld N=%lld K=%lld launch\n", (long long)M, (long long)N, (long long)K);
  const int rc = ro::gemm2_grain_backward(dO.data_ptr(), dO.stride(0), w_out_t.data_ptr(), w_out_t.stride(0),
                                          h.data_ptr(), h.stride(0), gx.data_ptr(), partial.data_ptr<float>(),
                                          static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                          num.data_ptr<float>(), den.data_ptr<float>(), static_cast<float>(eps),
                                          gemm_error_flag(dO.device()).data_ptr<int>(), stream);
  if (trace) std::fprintf(stderr, "grain_out_proj_backward: rc=%d\n", rc);
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "grain_out_proj_backward");
  check_rc(ro::grain_reduce_coefficients(partial.data_ptr<float>(), chunks, groups,
                                         into ? gnum_into->data_ptr<float>() : gnum.data_ptr<float>(),
                                         into ? gden_into->data_ptr<float>() : gden.data_ptr<float>(), into, stream),
           "grain_reduce_coefficients");
  return std::vector<torch::Tensor>{gx, gnum, gden};
}

// q/k/v projection with RoPE in the GEMM epilogue: x [M, K] . w [3d, K]^T,
// rotated q and k, returned as one [3, M, d] tensor of token-major planes.
// None when unsupported.
c10::optional<torch::Tensor> qkv_rope_forward(torch::Tensor x, torch::Tensor w, torch::Tensor cos_t,
                                              torch::Tensor sin_t, int64_t seq, int64_t hd) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 2 && w.dim() == 2, "expects 2-D CUDA tensors");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "expects bf16");
  TORCH_CHECK(x.size(1) == w.size(1), "inner dimensions differ");
  check_f32(cos_t, "cos");
  check_f32(sin_t, "sin");
  const int64_t N = w.size(0);
  if (x.stride(1) != 1 || w.stride(1) != 1 || N % 3 || !cos_t.is_contiguous() || !sin_t.is_contiguous() ||
      cos_t.size(0) < seq || cos_t.size(-1) != hd / 2)
    return c10::nullopt;
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty({3, x.size(0), N / 3}, x.options());
  const int rc = ro::gemm2_qkv_rope(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), out.data_ptr(),
                                    static_cast<int>(x.size(0)), static_cast<int>(N), static_cast<int>(x.size(1)),
                                    cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), static_cast<int>(seq),
                                    static_cast<int>(hd), gemm_error_flag(x.device()).data_ptr<int>(),
                                    at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "qkv_rope_forward");
  return out;
}

// In-projection with the GRAIN activation fused into the GEMM epilogue:
// returns (h = bf16(x w^T), y = GRAIN(h)) for groups of 256 columns; None
// when unsupported.
c10::optional<std::vector<torch::Tensor>> grain_in_proj_forward(torch::Tensor x, torch::Tensor w,
                                                                torch::Tensor num, torch::Tensor den,
                                                                double eps) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 2 && w.dim() == 2, "expects 2-D CUDA tensors");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "expects bf16");
  TORCH_CHECK(x.size(1) == w.size(1), "inner dimensions differ");
  check_f32(num, "numerator");
  check_f32(den, "denominator");
  const int64_t N = w.size(0);
  if (x.stride(1) != 1 || w.stride(1) != 1 || N % 256 != 0 || num.numel() != (N / 256) * 6 ||
      den.numel() != (N / 256) * 4)
    return c10::nullopt;
  const c10::cuda::CUDAGuard guard(x.device());
  auto h = torch::empty({x.size(0), N}, x.options());
  auto y = torch::empty({x.size(0), N}, x.options());
  const int rc = ro::gemm2_grain_forward(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), h.data_ptr(),
                                         y.data_ptr(), static_cast<int>(x.size(0)), static_cast<int>(N),
                                         static_cast<int>(x.size(1)), num.data_ptr<float>(), den.data_ptr<float>(),
                                         static_cast<float>(eps), gemm_error_flag(x.device()).data_ptr<int>(),
                                         at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "grain_in_proj_forward");
  return std::vector<torch::Tensor>{h, y};
}

// Flash attention forward over token-major planes: q, k, v [B, S, ld] bf16
// (head h at columns h*hd), returns (o [B, S, H*hd] bf16, lse2 [B, H, S] fp32);
// None for unsupported shapes or strides.
c10::optional<std::vector<torch::Tensor>> attention_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                                            int64_t heads, int64_t hd, double scale,
                                                            bool causal) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "attention_forward expects CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16, "attention_forward expects bf16");
  TORCH_CHECK(q.dim() == 3 && k.sizes() == q.sizes() && v.sizes() == q.sizes(), "q, k, v must be [B, S, ld]");
  const int64_t B = q.size(0), S = q.size(1), ld = q.stride(1);
  for (const auto& t : {q, k, v})
    if (t.stride(2) != 1 || t.stride(1) != ld || t.stride(0) != ld * S) return c10::nullopt;
  if (q.size(2) < heads * hd) return c10::nullopt;
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({B, S, heads * hd}, q.options());
  auto lse2 = torch::empty({B, heads, S}, q.options().dtype(torch::kFloat32));
  const int rc = ro::attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                       lse2.data_ptr<float>(), static_cast<int>(B), static_cast<int>(S),
                                       static_cast<int>(heads), static_cast<int>(hd), ld, heads * hd,
                                       static_cast<float>(scale), causal,
                                       gemm_error_flag(q.device()).data_ptr<int>(),
                                       at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "attention_forward");
  return std::vector<torch::Tensor>{o, lse2};
}

// Backward of attention_forward: (dq, dk, dv) as [B, S, H*hd] bf16 planes, or
// None for unsupported arguments.  o, dout: [B, S, H*hd] (made contiguous).
c10::optional<std::vector<torch::Tensor>> attention_backward(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                                             torch::Tensor o, torch::Tensor dout,
                                                             torch::Tensor lse2, int64_t heads, int64_t hd,
                                                             double scale, bool causal) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && k.sizes() == q.sizes() && v.sizes() == q.sizes(),
              "q, k, v must be CUDA [B, S, ld]");
  const int64_t B = q.size(0), S = q.size(1), ld = q.stride(1), cols = heads * hd;
  for (const auto& t : {q, k, v})
    if (t.stride(2) != 1 || t.stride(1) != ld || t.stride(0) != ld * S || t.scalar_type() != torch::kBFloat16)
      return c10::nullopt;
  o = o.contiguous();
  dout = dout.contiguous();
  TORCH_CHECK(o.sizes() == dout.sizes() && o.size(0) == B && o.size(1) == S && o.size(2) == cols,
              "o and dout must be [B, S, H*hd]");
  TORCH_CHECK(lse2.is_contiguous() && lse2.scalar_type() == torch::kFloat32 && lse2.numel() == B * heads * S,
              "lse2 must be fp32 [B, H, S]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = torch::empty_like(o), dk = torch::empty_like(o), dv = torch::empty_like(o);
  auto delta = torch::empty({B, heads, S}, lse2.options());
  const int rc = ro::attention_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), ld, o.data_ptr(), dout.data_ptr(),
                                        lse2.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), cols,
                                        delta.data_ptr<float>(), static_cast<int>(B), static_cast<int>(S),
                                        static_cast<int>(heads), static_cast<int>(hd), static_cast<float>(scale),
                                        causal, gemm_error_flag(q.device()).data_ptr<int>(),
                                        at::cuda::getCurrentCUDAStream());
  if (rc < 0) return c10::nullopt;
  check_rc(rc, "attention_backward");
  return std::vector<torch::Tensor>{dq, dk, dv};
}

// Reduce-to-owner (csrc/owner_comm.cu).  `dst` and `counter` are addresses in
// the owner's memory (CUDA IPC mappings); the kernels run on the current stream.
// mode: 0 fp32, 1 bf16, 2 int8 (per-256 fp32 scales); see owner_slot_bytes.
int64_t owner_slot_bytes(int64_t n, int64_t mode) { return ro::owner_slot_bytes(n, static_cast<int>(mode)); }

// counter 0: no arrival (a later owner_signal accounts for the data).
void owner_signal(int64_t counter, int64_t count) {
  check_rc(ro::owner_signal(reinterpret_cast<unsigned int*>(counter), static_cast<unsigned int>(count),
                            at::cuda::getCurrentCUDAStream()),
           "owner_signal");
}

// fp32 payload copied into the owner's slot by a copy engine (no arrival).
void owner_copy(torch::Tensor src, int64_t dst) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kFloat32 && src.is_contiguous(),
              "owner_copy expects a contiguous fp32 CUDA tensor");
  const c10::cuda::CUDAGuard guard(src.device());
  check_rc(ro::owner_copy(src.data_ptr<float>(), reinterpret_cast<void*>(dst), src.numel(),
                          at::cuda::getCurrentCUDAStream()),
           "owner_copy");
}

void owner_send(torch::Tensor src, int64_t dst, int64_t mode, int64_t counter, int64_t ctas) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kFloat32 && src.is_contiguous(),
              "owner_send expects a contiguous fp32 CUDA tensor");
  const c10::cuda::CUDAGuard guard(src.device());
  check_rc(ro::owner_send(src.data_ptr<float>(), reinterpret_cast<void*>(dst), src.numel(), static_cast<int>(mode),
                          reinterpret_cast<unsigned int*>(counter), static_cast<int>(ctas),
                          at::cuda::getCurrentCUDAStream()),
           "owner_send");
}

void owner_reduce(torch::Tensor grad, int64_t recv, torch::Tensor counters, torch::Tensor offsets,
                  torch::Tensor sizes, torch::Tensor recv_offsets, torch::Tensor sumsq, int64_t rank,
                  int64_t world, int64_t expected, double scale, int64_t mode, torch::Tensor err,
                  int64_t timeout_ns) {
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == torch::kFloat32, "owner_reduce: fp32 gradient buffer");
  TORCH_CHECK(offsets.scalar_type() == torch::kInt64 && sizes.scalar_type() == torch::kInt64 &&
                  recv_offsets.scalar_type() == torch::kInt64 && offsets.is_cuda(),
              "owner_reduce: int64 CUDA layout tensors");
  TORCH_CHECK(sumsq.scalar_type() == torch::kFloat32 && err.scalar_type() == torch::kInt32, "owner_reduce dtypes");
  const c10::cuda::CUDAGuard guard(grad.device());
  check_rc(ro::owner_reduce(grad.data_ptr<float>(), reinterpret_cast<const void*>(recv),
                            reinterpret_cast<unsigned int*>(counters.data_ptr()), offsets.data_ptr<int64_t>(),
                            sizes.data_ptr<int64_t>(), recv_offsets.data_ptr<int64_t>(), sumsq.data_ptr<float>(),
                            static_cast<int>(sumsq.numel()), static_cast<int>(offsets.numel()),
                            static_cast<int>(rank), static_cast<int>(world), static_cast<unsigned int>(expected),
                            static_cast<float>(scale), static_cast<int>(mode), err.data_ptr<int>(),
                            static_cast<uint64_t>(timeout_ns), at::cuda::getCurrentCUDAStream()),
           "owner_reduce");
}

// Owner weight all-gather (csrc/owner_comm.cu): publish bumps this rank's
// counter; pull copies `dst.numel()` fp32 values from a peer address into
// `dst` once the peer's counter (address `published`) has reached this rank's
// own counter `mine`.
void owner_publish(torch::Tensor published) {
  const c10::cuda::CUDAGuard guard(published.device());
  check_rc(ro::owner_publish(reinterpret_cast<unsigned int*>(published.data_ptr()),
                             at::cuda::getCurrentCUDAStream()),
           "owner_publish");
}

void owner_pull(int64_t src, torch::Tensor dst, int64_t published, torch::Tensor mine, torch::Tensor err,
                int64_t timeout_ns, int64_t ctas) {
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == torch::kFloat32 && dst.is_contiguous(),
              "owner_pull: contiguous fp32 destination");
  const c10::cuda::CUDAGuard guard(dst.device());
  check_rc(ro::owner_pull(reinterpret_cast<const float*>(src), dst.data_ptr<float>(), nullptr, dst.numel(),
                          reinterpret_cast<const unsigned int*>(published),
                          reinterpret_cast<const unsigned int*>(mine.data_ptr()), err.data_ptr<int>(),
                          static_cast<uint64_t>(timeout_ns), static_cast<int>(ctas),
                          at::cuda::getCurrentCUDAStream()),
           "owner_pull");
}

void adamw_multi_tensor(std::vector<torch::Tensor> p, std::vector<torch::Tensor> g,
                        std::vector<torch::Tensor> m, std::vector<torch::Tensor> v, double lr,
                        double beta1, double beta2, double eps, double wd, double step) {
  const size_t n = p.size();
  TORCH_CHECK(g.size() == n && m.size() == n && v.size() == n, "adamw list lengths differ");
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(p[0].device());
  std::vector<float*> pp(n), mp(n), vp(n);
  std::vector<const float*> gp(n);
  std::vector<int64_t> sizes(n);
  for (size_t i = 0; i < n; ++i) {
    for (auto* t : {&p[i], &g[i], &m[i], &v[i]}) {
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous(),
                  "adamw tensors must be contiguous fp32 CUDA tensors");
    }
    TORCH_CHECK(g[i].numel() == p[i].numel() && m[i].numel() == p[i].numel() && v[i].numel() == p[i].numel(),
                "adamw tensor sizes differ");
    pp[i] = p[i].data_ptr<float>();
    gp[i] = g[i].data_ptr<float>();
    mp[i] = m[i].data_ptr<float>();
    vp[i] = v[i].data_ptr<float>();
    sizes[i] = p[i].numel();
  }
  check_rc(ro::adamw_multi_tensor(pp.data(), gp.data(), mp.data(), vp.data(), sizes.data(), static_cast<int>(n),
                                  static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
                                  static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(step),
                                  at::cuda::getCurrentCUDAStream()),
           "adamw_multi_tensor");
}

// Sum over tensors of <a_t, b_t> times scale, as a 0-dim fp32 tensor.
torch::Tensor multi_tensor_dot(std::vector<torch::Tensor> a, std::vector<torch::Tensor> b, double scale) {
  const size_t n = a.size();
  TORCH_CHECK(n > 0 && b.size() == n, "multi_tensor_dot list lengths");
  const c10::cuda::CUDAGuard guard(a[0].device());
  std::vector<const float*> ap(n), bp(n);
  std::vector<int64_t> sizes(n);
  for (size_t i = 0; i < n; ++i) {
    for (auto* t : {&a[i], &b[i]}) {
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous(),
                  "multi_tensor_dot tensors must be contiguous fp32 CUDA tensors");
    }
    TORCH_CHECK(a[i].numel() == b[i].numel(), "multi_tensor_dot sizes differ");
    ap[i] = a[i].data_ptr<float>();
    bp[i] = b[i].data_ptr<float>();
    sizes[i] = a[i].numel();
  }
  auto opts = a[0].options();
  auto part = torch::empty({std::max<int64_t>(1, ro::multi_tensor_dot_partials(sizes.data(), static_cast<int>(n)))}, opts);
  auto out = torch::empty({}, opts);
  check_rc(ro::multi_tensor_dot(ap.data(), bp.data(), sizes.data(), static_cast<int>(n), static_cast<float>(scale),
                                part.data_ptr<float>(), out.data_ptr<float>(), at::cuda::getCurrentCUDAStream()),
           "multi_tensor_dot");
  return out;
}

// x *= min(max_norm / (sqrt(sumsq) + 1e-6), 1) with sumsq a 1-element device tensor.
void clip_scale_(torch::Tensor x, torch::Tensor sumsq, double max_norm) {
  check_f32(x, "x");
  check_f32(sumsq, "sumsq");
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(ro::clip_scale(x.data_ptr<float>(), x.numel(), sumsq.data_ptr<float>(), static_cast<float>(max_norm),
                          at::cuda::getCurrentCUDAStream()),
           "clip_scale_");
}

// ---------------------------------------------------------------------------
// TILLER direction kernels.

std::vector<float*> ptrs_of(std::vector<torch::Tensor>& ts, int64_t numel, const char* what) {
  std::vector<float*> out;
  for (auto& t : ts) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous() && t.numel() == numel,
                what, " must be contiguous fp32 CUDA tensors of equal size");
    out.push_back(t.data_ptr<float>());
  }
  return out;
}

std::vector<torch::Tensor> tiller_nesterov(std::vector<torch::Tensor> grads, std::vector<torch::Tensor> bufs,
                                           bool transpose, double mu) {
  TORCH_CHECK(!grads.empty() && grads.size() == bufs.size(), "tiller_nesterov lists");
  const c10::cuda::CUDAGuard guard(grads[0].device());
  TORCH_CHECK(grads[0].dim() == 2, "tiller_nesterov expects matrices");
  const int64_t P = grads[0].size(0), Q = grads[0].size(1);
  auto gp = ptrs_of(grads, P * Q, "grads");
  auto bp = ptrs_of(bufs, P * Q, "momentum buffers");
  const int64_t L = grads.size();
  auto opts = grads[0].options();
  std::vector<int64_t> shape = transpose ? std::vector<int64_t>{L, Q, P} : std::vector<int64_t>{L, P, Q};
  auto m = torch::empty(shape, opts);
  auto g = torch::empty(shape, opts);
  auto m16 = torch::empty(shape, opts.dtype(torch::kBFloat16));
  check_rc(ro::tiller_nesterov(gp.data(), bp.data(), m.data_ptr<float>(), g.data_ptr<float>(),
                               reinterpret_cast<__nv_bfloat16*>(m16.data_ptr()), static_cast<int>(L),
                               static_cast<int>(P), static_cast<int>(Q), transpose, static_cast<float>(mu),
                               at::cuda::getCurrentCUDAStream()),
           "tiller_nesterov");
  return {m, g, m16};
}

torch::Tensor tiller_transpose_bf16(torch::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous() && x.dim() == 3,
              "transpose expects contiguous bf16 [L, P, Q]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty({x.size(0), x.size(2), x.size(1)}, x.options());
  check_rc(ro::tiller_transpose_bf16(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                     reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), static_cast<int>(x.size(0)),
                                     static_cast<int>(x.size(1)), static_cast<int>(x.size(2)),
                                     at::cuda::getCurrentCUDAStream()),
           "tiller_transpose_bf16");
  return y;
}

std::vector<torch::Tensor> tiller_chord(torch::Tensor polar, torch::Tensor m, torch::Tensor g,
                                        torch::Tensor row_m, torch::Tensor col_m, torch::Tensor participation,
                                        torch::Tensor congruence, int64_t nblocks, int64_t R, int64_t C,
                                        double scale, int64_t step, double adj) {
  const c10::cuda::CUDAGuard guard(m.device());
  TORCH_CHECK(polar.scalar_type() == torch::kBFloat16 && polar.is_contiguous() && polar.numel() == nblocks * R * C,
              "polar must be bf16 [nblocks*R*C]");
  check_f32(m, "m");
  check_f32(g, "g");
  check_f32(row_m, "row moment");
  check_f32(col_m, "column moment");
  check_f32(participation, "participation");
  check_f32(congruence, "congruence");
  TORCH_CHECK(m.numel() == nblocks * R * C && g.numel() == m.numel(), "m/g size");
  TORCH_CHECK(row_m.numel() == nblocks * R && col_m.numel() == nblocks * C, "moment sizes");
  TORCH_CHECK(participation.numel() == nblocks && congruence.numel() == nblocks, "route sizes");
  const int chunks = ro::tiller_chunks(static_cast<int>(R));
  auto opts = m.options();
  auto colpart = torch::empty({nblocks * chunks * C}, opts);
  auto dotpart = torch::empty({nblocks * chunks * 8}, opts);
  auto row_total = torch::empty({nblocks}, opts);
  auto out = torch::empty({nblocks, 16}, opts);
  check_rc(ro::tiller_chord(reinterpret_cast<const __nv_bfloat16*>(polar.data_ptr()), m.data_ptr<float>(),
                            g.data_ptr<float>(), row_m.data_ptr<float>(), col_m.data_ptr<float>(),
                            colpart.data_ptr<float>(), dotpart.data_ptr<float>(), row_total.data_ptr<float>(),
                            participation.data_ptr<float>(), congruence.data_ptr<float>(), out.data_ptr<float>(),
                            static_cast<int>(nblocks), static_cast<int>(R), static_cast<int>(C),
                            static_cast<float>(scale), static_cast<int>(step), static_cast<float>(adj),
                            at::cuda::getCurrentCUDAStream()),
           "tiller_chord");
  return {out, row_total};
}

c10::optional<torch::Tensor> tiller_apply(std::vector<torch::Tensor> params, torch::Tensor polar, torch::Tensor m,
                                          torch::Tensor row_m, torch::Tensor col_m, torch::Tensor row_total,
                                          torch::Tensor chord, torch::Tensor coef, bool want_selected,
                                          bool update_param, int64_t blocks_per_layer, int64_t R, int64_t C,
                                          bool transpose, double scale, int64_t step, double decay,
                                          double alpha, double adj) {
  TORCH_CHECK(!params.empty(), "tiller_apply params");
  const c10::cuda::CUDAGuard guard(m.device());
  const int64_t L = params.size();
  auto pp = ptrs_of(params, blocks_per_layer * R * C, "params");
  check_f32(m, "m");
  check_f32(coef, "coef");
  check_f32(chord, "chord");
  TORCH_CHECK(coef.numel() == L * blocks_per_layer, "coef size");
  torch::Tensor sel;
  if (want_selected) sel = torch::empty_like(m);
  check_rc(ro::tiller_apply(pp.data(), reinterpret_cast<const __nv_bfloat16*>(polar.data_ptr()), m.data_ptr<float>(),
                            row_m.data_ptr<float>(), col_m.data_ptr<float>(), row_total.data_ptr<float>(),
                            chord.data_ptr<float>(), coef.data_ptr<float>(),
                            want_selected ? sel.data_ptr<float>() : nullptr, static_cast<int>(L),
                            static_cast<int>(blocks_per_layer), static_cast<int>(R), static_cast<int>(C),
                            transpose, static_cast<float>(scale), static_cast<int>(step),
                            static_cast<float>(decay), static_cast<float>(alpha), static_cast<float>(adj),
                            update_param, at::cuda::getCurrentCUDAStream()),
           "tiller_apply");
  if (want_selected) return sel;
  return c10::nullopt;
}

torch::Tensor ns_normalize(torch::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous() && x.dim() == 3,
              "ns_normalize expects contiguous bf16 [B, r, c]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  const int64_t n = x.size(1) * x.size(2);
  auto part = torch::empty({x.size(0) * ro::ns_normalize_chunks(n)}, x.options().dtype(torch::kFloat32));
  check_rc(ro::ns_normalize(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                            reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), part.data_ptr<float>(),
                            static_cast<int>(x.size(0)), n, at::cuda::getCurrentCUDAStream()),
           "ns_normalize");
  return y;
}

// ---------------------------------------------------------------------------
// NVLink peer-memory collectives.

torch::Tensor comm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  const cudaError_t e = cudaMalloc(&ptr, static_cast<size_t>(nbytes));
  TORCH_CHECK(e == cudaSuccess, "comm_alloc: ", cudaGetErrorString(e));
  TORCH_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)) == cudaSuccess, "comm_alloc memset");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(ptr, {nbytes}, [device](void* p) {
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
    cudaFree(p);
  }, opts);
}

py::bytes comm_handle(torch::Tensor base) {
  char h[64];
  check_rc(ro::comm_ipc_handle(base.data_ptr(), h), "cudaIpcGetMemHandle");
  return py::bytes(h, 64);
}

int64_t comm_open(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "IPC handle must be 64 bytes");
  void* ptr = nullptr;
  check_rc(ro::comm_ipc_open(s.data(), &ptr), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(ptr);
}

void comm_close(int64_t ptr) { ro::comm_ipc_close(reinterpret_cast<void*>(ptr)); }

std::vector<void*> as_ptrs(const std::vector<int64_t>& v) {
  std::vector<void*> out;
  for (auto x : v) out.push_back(reinterpret_cast<void*>(x));
  return out;
}

std::vector<unsigned int*> as_flag_ptrs(const std::vector<int64_t>& v) {
  std::vector<unsigned int*> out;
  for (auto x : v) out.push_back(reinterpret_cast<unsigned int*>(x));
  return out;
}

void comm_allreduce_f32(std::vector<int64_t> data, std::vector<int64_t> flags, int64_t rank, int64_t n,
                        double scale, int64_t epoch, torch::Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(data.size() == flags.size(), "data/flag lists differ");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32, "err must be a CUDA int32 tensor");
  const c10::cuda::CUDAGuard guard(err.device());
  auto d = as_ptrs(data);
  auto f = as_flag_ptrs(flags);
  check_rc(ro::comm_allreduce_f32(d.data(), f.data(), static_cast<int>(rank), static_cast<int>(data.size()), n,
                                  static_cast<float>(scale), static_cast<unsigned int>(epoch), err.data_ptr<int>(),
                                  static_cast<uint64_t>(timeout_ns), at::cuda::getCurrentCUDAStream()),
           "comm_allreduce_f32");
}

void comm_allreduce_i8(torch::Tensor src, torch::Tensor out, std::vector<int64_t> data, std::vector<int64_t> flags,
                       int64_t rank, double scale, int64_t epoch, torch::Tensor err, int64_t timeout_ns) {
  check_f32(src, "src");
  check_f32(out, "out");
  TORCH_CHECK(src.numel() == out.numel(), "src/out sizes");
  const c10::cuda::CUDAGuard guard(src.device());
  auto d = as_ptrs(data);
  auto f = as_flag_ptrs(flags);
  check_rc(ro::comm_allreduce_i8(src.data_ptr<float>(), out.data_ptr<float>(), d.data(), f.data(),
                                 static_cast<int>(rank), static_cast<int>(data.size()), src.numel(),
                                 static_cast<float>(scale), static_cast<unsigned int>(epoch), err.data_ptr<int>(),
                                 static_cast<uint64_t>(timeout_ns), at::cuda::getCurrentCUDAStream()),
           "comm_allreduce_i8");
}

int64_t comm_i8_bytes(int64_t n) { return ro::comm_i8_bytes(n); }

void comm_wait_only(std::vector<int64_t> data, std::vector<int64_t> flags, int64_t rank, int64_t epoch,
                    torch::Tensor err, int64_t timeout_ns) {
  const c10::cuda::CUDAGuard guard(err.device());
  auto d = as_ptrs(data);
  auto f = as_flag_ptrs(flags);
  check_rc(ro::comm_wait_only(d.data(), f.data(), static_cast<int>(rank), static_cast<int>(data.size()),
                              static_cast<unsigned int>(epoch), err.data_ptr<int>(),
                              static_cast<uint64_t>(timeout_ns), at::cuda::getCurrentCUDAStream()),
           "comm_wait_only");
}

// ---------------------------------------------------------------------------
// TILLER ledger + transaction (single CTA, fp64).
// state: dict-like tensors; scal: fp32 [8] = [tail, discarded_fraction, shrinkage, ref_row_norm, ...]

std::vector<torch::Tensor> tiller_ledger_transaction(
    c10::optional<torch::Tensor> cur_scores, c10::optional<torch::Tensor> cur_decay, torch::Tensor exact,
    torch::Tensor momentum, torch::Tensor weights, torch::Tensor layer_ids,
    c10::optional<torch::Tensor> decay_derivative, torch::Tensor pers_scores, torch::Tensor pers_total_diag,
    torch::Tensor pers_decay_cross, torch::Tensor scal, torch::Tensor ws, int64_t prev_rows,
    int64_t total_layers, double eta, c10::optional<torch::Tensor> timing) {
  const c10::cuda::CUDAGuard guard(exact.device());
  check_f32(exact, "exact");
  check_f32(momentum, "momentum");
  check_f32(weights, "weights");
  check_f32(pers_scores, "persistent scores");
  check_f32(pers_total_diag, "persistent diagonal");
  check_f32(pers_decay_cross, "persistent decay cross");
  check_f32(scal, "ledger scalars");
  TORCH_CHECK(layer_ids.is_cuda() && layer_ids.scalar_type() == torch::kInt64, "layer ids must be int64 CUDA");
  const int64_t C = weights.numel();
  TORCH_CHECK(exact.numel() == 2 * C && momentum.numel() == 2 * C && layer_ids.numel() == C, "transaction sizes");
  TORCH_CHECK(pers_scores.numel() >= 64 * C && pers_total_diag.numel() == C && pers_decay_cross.numel() == C,
              "ledger buffer sizes");
  TORCH_CHECK(scal.numel() >= 8, "ledger scalars");
  TORCH_CHECK(ws.scalar_type() == torch::kFloat64 && ws.numel() >= ro::ledger_workspace_doubles(static_cast<int>(C)),
              "workspace too small");
  const bool functional = cur_scores.has_value();
  if (functional) {
    check_f32(*cur_scores, "current scores");
    check_f32(*cur_decay, "current decay");
    TORCH_CHECK(cur_scores->numel() == 32 * C && cur_decay->numel() == 32, "current rows");
  } else {
    TORCH_CHECK(decay_derivative.has_value(), "surrogate mode needs the decay derivative");
    check_f32(*decay_derivative, "decay derivative");
  }
  unsigned long long* timing_ptr = nullptr;
  if (timing.has_value()) {
    TORCH_CHECK(timing->is_cuda() && timing->scalar_type() == torch::kInt64 && timing->numel() >= 16,
                "timing buffer must be int64 CUDA with 16 entries");
    timing_ptr = reinterpret_cast<unsigned long long*>(timing->data_ptr<int64_t>());
  }
  auto coef = torch::empty({C}, weights.options());
  auto cand = torch::empty({C}, weights.options());
  auto result = torch::zeros({16}, weights.options());
  float* sp = scal.data_ptr<float>();
  check_rc(ro::ledger_transaction(functional ? cur_scores->data_ptr<float>() : nullptr,
                                  functional ? cur_decay->data_ptr<float>() : nullptr, exact.data_ptr<float>(),
                                  momentum.data_ptr<float>(), weights.data_ptr<float>(),
                                  layer_ids.data_ptr<int64_t>(),
                                  functional ? nullptr : decay_derivative->data_ptr<float>(),
                                  pers_scores.data_ptr<float>(), pers_total_diag.data_ptr<float>(),
                                  pers_decay_cross.data_ptr<float>(), sp + 0, sp + 1, sp + 2, sp + 3,
                                  coef.data_ptr<float>(), cand.data_ptr<float>(), result.data_ptr<float>(),
                                  ws.data_ptr<double>(), static_cast<int>(C), static_cast<int>(prev_rows),
                                  static_cast<int>(total_layers), functional, eta, timing_ptr,
                                  at::cuda::getCurrentCUDAStream()),
           "tiller_ledger_transaction");
  return {coef, cand, result};
}

int64_t tiller_ledger_workspace(int64_t C) { return ro::ledger_workspace_doubles(static_cast<int>(C)); }

// Failed RO_CHECKs per kernel file since the last call (0 = none; always 0
// unless the module was built with -DRO_BOUNDS_CHECK).  Synchronises.
std::map<std::string, uint64_t> bounds_faults() {
  check_rc(static_cast<int>(cudaDeviceSynchronize()), "bounds_faults");
  return {{"grain", ro::grain_bounds_word()}, {"nn_ops", ro::nn_ops_bounds_word()},
          {"optim", ro::optim_bounds_word()}};
}

void bounds_selftest(torch::Tensor buf, int64_t index) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == torch::kFloat32 && buf.is_contiguous(),
              "bounds_selftest: contiguous fp32 CUDA tensor expected");
  const int rc = ro::bounds_selftest(buf.data_ptr<float>(), buf.numel(), index, stream());
  TORCH_CHECK(rc != -1, "bounds_selftest needs a -DRO_BOUNDS_CHECK build");
  check_rc(rc, "bounds_selftest");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels for rational_optimizer_b200";
#ifdef RO_BOUNDS_CHECK
  m.attr("bounds_checked") = true;
#else
  m.attr("bounds_checked") = false;
#endif
  m.def("bounds_faults", &bounds_faults);
  m.def("bounds_selftest", &bounds_selftest);
  m.def("grain_forward", &grain_forward);
  m.def("grain_backward", &grain_backward);
  m.def("grain_affine_statistics", &grain_affine_statistics);
  m.def("legacy_forward", &legacy_forward);
  m.def("legacy_backward", &legacy_backward);
  m.def("rmsnorm_forward", &rmsnorm_forward);
  m.def("rmsnorm_backward", &rmsnorm_backward);
  m.def("add_rmsnorm_forward", &add_rmsnorm_forward);
  m.def("add_rmsnorm_backward", &add_rmsnorm_backward, py::arg("dy"), py::arg("dres"), py::arg("x"), py::arg("w"),
        py::arg("rstd"), py::arg("want_ddelta"), py::arg("dw_into") = py::none());
  m.def("rope_qkv_forward", &rope_qkv_forward);
  m.def("rope_qkv_backward", &rope_qkv_backward);
  m.def("cross_entropy_fwd_bwd", &cross_entropy_fwd_bwd);
  m.def("gemm_bf16", &gemm_bf16);
  m.def("gemm_bf16_ex", &gemm_bf16_ex);
  m.def("gemm_bf16_to", &gemm_bf16_to);
  m.def("gemm_error", &gemm_error);
  m.def("adamw_multi_tensor", &adamw_multi_tensor);
  m.def("multi_tensor_dot", &multi_tensor_dot);
  m.def("clip_scale_", &clip_scale_);
  m.def("gemm2_bf16", &gemm2_bf16);
  m.def("grain_in_proj_forward", &grain_in_proj_forward);
  m.def("qkv_rope_forward", &qkv_rope_forward);
  m.def("owner_slot_bytes", &owner_slot_bytes);
  m.def("owner_send", &owner_send);
  m.def("owner_signal", &owner_signal);
  m.def("owner_copy", &owner_copy);
  m.def("owner_reduce", &owner_reduce);
  m.def("owner_publish", &owner_publish);
  m.def("owner_pull", &owner_pull);
  m.def("attention_forward", &attention_forward);
  m.def("attention_backward", &attention_backward);
  m.def("grain_out_proj_backward", &grain_out_proj_backward, py::arg("dO"), py::arg("w_out_t"), py::arg("h"),
        py::arg("num"), py::arg("den"), py::arg("eps"), py::arg("gnum_into") = py::none(),
        py::arg("gden_into") = py::none());
  m.def("tiller_nesterov", &tiller_nesterov);
  m.def("tiller_transpose_bf16", &tiller_transpose_bf16);
  m.def("tiller_chord", &tiller_chord);
  m.def("tiller_apply", &tiller_apply);
  m.def("ns_normalize", &ns_normalize);
  m.def("comm_alloc", &comm_alloc);
  m.def("comm_handle", &comm_handle);
  m.def("comm_open", &comm_open);
  m.def("comm_close", &comm_close);
  m.def("comm_allreduce_f32", &comm_allreduce_f32);
  m.def("comm_allreduce_i8", &comm_allreduce_i8);
  m.def("comm_i8_bytes", &comm_i8_bytes);
  m.def("comm_wait_only", &comm_wait_only);
  m.def("tiller_ledger_transaction", &tiller_ledger_transaction, py::arg("cur_scores"), py::arg("cur_decay"),
        py::arg("exact"), py::arg("momentum"), py::arg("weights"), py::arg("layer_ids"),
        py::arg("decay_derivative"), py::arg("pers_scores"), py::arg("pers_total_diag"),
        py::arg("pers_decay_cross"), py::arg("scal"), py::arg("ws"), py::arg("prev_rows"),
        py::arg("total_layers"), py::arg("eta"), py::arg("timing") = py::none());
  m.def("tiller_ledger_workspace", &tiller_ledger_workspace);
}
