// Host-side launch API of the .cu kernel files (raw pointers + stream).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace ro {

// grain.cu
int grain_forward(const void* x, int x_dtype, const float* num, const float* den,
                  const float* logits, const float* centers, const float* beta, void* y,
                  int y_dtype, float* rho_out, int64_t rows, int hidden, int groups, int nb,
                  float coeff_limit, float eps, cudaStream_t stream);
int grain_backward_partial_size(int64_t rows, int groups, int nb);
int grain_backward(const void* gy, int gy_dtype, const void* x, int x_dtype, const float* num,
                   const float* den, const float* logits, const float* centers,
                   const float* beta, const float* affine_alpha, const float* affine_beta,
                   float* nonlinear_y, void* gx, int gx_dtype, float* gnum, float* gden,
                   float* gcoeff, float* partial, int64_t rows, int hidden, int groups, int nb,
                   float coeff_limit, float eps, cudaStream_t stream);
int grain_affine_partial_size(int64_t rows, int groups);
int grain_affine_statistics(const void* x, const void* feature, int dtype, float* rho_out,
                            double* stats, double* partial, int64_t rows, int hidden,
                            int groups, float eps, cudaStream_t stream);
int legacy_rational_blocks(int64_t n);
int legacy_rational_forward(const float* x, const float* a, const float* b, float* y, int64_t n,
                            bool signed_den, cudaStream_t stream);
int legacy_rational_backward(const float* gy, const float* x, const float* a, const float* b,
                             float* gx, float* ga, float* gb, float* partial, int64_t n,
                             bool signed_den, cudaStream_t stream);

// nn_ops.cu
int rmsnorm_forward(const void* x, const float* w, void* y, float* rstd, int64_t rows, int d,
                    float eps, int dtype, int out_dtype, cudaStream_t stream);
int rmsnorm_backward_partial_size(int64_t rows, int d);
int rmsnorm_backward(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                     float* dw, float* partial, int64_t rows, int d, int dtype, int out_dtype,
                     int accumulate_dw, cudaStream_t stream);
int rope_qkv_forward(const void* qkv, const float* cos_t, const float* sin_t, void* q, void* k,
                     void* v, int B, int S, int H, int hd, int dtype, cudaStream_t stream);
int rope_qkv_backward(const void* dq, const void* dk, const void* dv, const float* cos_t,
                      const float* sin_t, void* dqkv, int B, int S, int H, int hd, int dtype,
                      cudaStream_t stream);
int cross_entropy_fwd_bwd(void* logits, const int64_t* target, float* loss_row, int64_t rows,
                          int V, float grad_scale, int64_t ignore_index, int dtype,
                          cudaStream_t stream);

}  // namespace ro
