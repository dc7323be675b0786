// Host-side launch API of the .cu kernel files (raw pointers + stream).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cuda_bf16.h>

namespace ro {

// First failed RO_CHECK of each kernel file in a -DRO_BOUNDS_CHECK build,
// (site << 32) | line, cleared by the read; always 0 in normal builds.
unsigned long long grain_bounds_word();
unsigned long long nn_ops_bounds_word();
unsigned long long optim_bounds_word();
// Checked builds only: a kernel that guards buf[index] (n elements) with
// RO_CHECK and writes 1 there when the check passes; returns the launch status.
int bounds_selftest(float* buf, int64_t n, int64_t index, cudaStream_t stream);

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
int add_rmsnorm_forward(const float* x, const void* delta, const float* w, float* x_new, void* y,
                        float* rstd, int64_t rows, int d, float eps, cudaStream_t stream);
int add_rmsnorm_backward(const void* dy, const float* dres, const float* x, const float* w,
                         const float* rstd, float* dx, void* ddelta, float* dw, bool accumulate_dw, float* partial,
                         int64_t rows, int d, cudaStream_t stream);
int rope_qkv_forward(const void* qkv, const float* cos_t, const float* sin_t, void* q, void* k,
                     void* v, int B, int S, int H, int hd, int dtype, cudaStream_t stream);
int rope_qkv_backward(const void* dq, const void* dk, const void* dv, const float* cos_t,
                      const float* sin_t, void* dqkv, int B, int S, int H, int hd, int dtype,
                      cudaStream_t stream);
int cross_entropy_fwd_bwd(void* logits, const int64_t* target, float* loss_row, int64_t rows,
                          int V, float grad_scale, int64_t ignore_index, int dtype,
                          cudaStream_t stream);


// gemm_sm100.cu
int gemm2_bf16_nt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int M, int N,
                  int K, int* err, cudaStream_t stream);
int gemm2_grain_forward(const void* X, int64_t ldx, const void* W, int64_t ldw, void* H, void* Y, int M, int N,
                        int K, const float* num, const float* den, float eps, int* err, cudaStream_t stream);
int gemm2_qkv_rope(const void* X, int64_t ldx, const void* W, int64_t ldw, void* QKV, int M, int N, int K,
                   const float* cos_t, const float* sin_t, int seq, int hd, int* err, cudaStream_t stream);
int gemm2_grain_partial_rows(int M);
// Reduce-to-owner transport formats: mode 0 fp32, 1 bf16, 2 int8 with one
// fp32 scale per 256 elements.  recv_offsets are byte offsets.
int64_t owner_slot_bytes(int64_t n, int mode);
int owner_signal(unsigned int* counter, unsigned int count, cudaStream_t stream);
int owner_copy(const float* src, void* dst, int64_t n, cudaStream_t stream);
int owner_send(const float* src, void* dst, int64_t n, int mode, unsigned int* counter, int ctas,
               cudaStream_t stream);
int owner_reduce(float* grad, const void* recv, unsigned int* counters, const int64_t* offsets,
                 const int64_t* sizes, const int64_t* recv_offsets, float* sumsq, int ctas, int layers,
                 int rank, int world, unsigned int expected, float scale, int mode, int* err,
                 uint64_t timeout_ns, cudaStream_t stream);
int owner_publish(unsigned int* published, cudaStream_t stream);
int owner_pull(const float* src, float* dst, __nv_bfloat16* dst16, int64_t n, const unsigned int* published,
               const unsigned int* mine, int* err, uint64_t timeout_ns, int ctas, cudaStream_t stream);
int attention_backward(const void* q, const void* k, const void* v, int64_t ld, const void* o, const void* dout,
                       const float* lse2, void* dq, void* dk, void* dv, int64_t ld2, float* delta, int B, int S,
                       int H, int hd, float scale, bool causal, int* err, cudaStream_t stream);
int attention_forward(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int S, int H,
                      int hd, int64_t ld, int64_t ldo, float scale, bool causal, int* err, cudaStream_t stream);
int gemm2_grain_backward(const void* dO, int64_t ldo, const void* wt, int64_t ldw, const void* h, int64_t ldh,
                         void* GX, float* partial, int M, int N, int K, const float* num, const float* den,
                         float eps, int* err, cudaStream_t stream);
int grain_reduce_coefficients(const float* partial, int chunks, int groups, float* gnum, float* gden,
                              bool accumulate, cudaStream_t stream);
int gemm_bf16_tn(const void* A, int64_t lda, int64_t strideA, bool a_mn, const void* B, int64_t ldb,
                 int64_t strideB, bool b_mn, void* C, int64_t ldc, int64_t strideC, bool out_f32,
                 const void* D, int64_t ldd, int64_t strideD, float alpha, float beta, int M, int N,
                 int K, int batch, int* err, cudaStream_t stream);


// optim.cu
int adamw_multi_tensor(float* const* p, const float* const* g, float* const* m, float* const* v,
                       const int64_t* sizes, int count, float lr, float beta1, float beta2, float eps,
                       float wd, float step, cudaStream_t stream);
int64_t multi_tensor_dot_partials(const int64_t* sizes, int count);
int clip_scale(float* x, int64_t n, const float* sumsq, float max_norm, cudaStream_t stream);
int multi_tensor_dot(const float* const* a, const float* const* b, const int64_t* sizes, int count,
                     float scale, float* part, float* out, cudaStream_t stream);


// tiller.cu
int tiller_nesterov(float* const* grads, float* const* bufs, float* m_out, float* g_out,
                    __nv_bfloat16* m16_out, int L, int P, int Q, bool transpose, float mu,
                    cudaStream_t stream);
int tiller_transpose_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, int L, int P, int Q,
                          cudaStream_t stream);
int tiller_chunks(int R);
int tiller_chord(const __nv_bfloat16* polar, const float* m, const float* g, float* row_m, float* col_m,
                 float* colpart, float* dotpart, float* row_total, const float* participation,
                 const float* congruence, float* chord_out, int nblocks, int R, int C, float scale,
                 int step, float adj, cudaStream_t stream);
int tiller_apply(float* const* params, const __nv_bfloat16* polar, const float* m, const float* row_m,
                 const float* col_m, const float* row_total, const float* chord, const float* coef,
                 float* sel_out, int L, int blocks_per_layer, int R, int C, bool transpose, float scale,
                 int step, float decay, float alpha, float adj, bool update_param, cudaStream_t stream);
int64_t ns_normalize_chunks(int64_t n);
int ns_normalize(const __nv_bfloat16* x, __nv_bfloat16* y, float* part, int batch, int64_t n,
                 cudaStream_t stream);


// comm.cu
int comm_ipc_handle(const void* base, void* handle_out);
int comm_ipc_open(const void* handle, void** ptr);
int comm_ipc_close(void* ptr);
int comm_allreduce_f32(void* const* data, unsigned int* const* flags, int rank, int world, int64_t n,
                       float scale, unsigned int epoch, int* err, uint64_t timeout_ns,
                       cudaStream_t stream);
int64_t comm_i8_scale_offset(int64_t n);
int64_t comm_i8_bytes(int64_t n);
int comm_allreduce_i8(const float* src, float* out, void* const* data, unsigned int* const* flags, int rank,
                      int world, int64_t n, float scale, unsigned int epoch, int* err,
                      uint64_t timeout_ns, cudaStream_t stream);
int comm_wait_only(void* const* data, unsigned int* const* flags, int rank, int world, unsigned int epoch,
                   int* err, uint64_t timeout_ns, cudaStream_t stream);


// ledger.cu
int64_t ledger_workspace_doubles(int C);
int ledger_transaction(const float* cur_scores, const float* cur_decay, const float* exact,
                       const float* momentum, const float* weights, const int64_t* layer_ids,
                       const float* decay_derivative, float* pers_scores, float* pers_total_diag,
                       float* pers_decay_cross, float* pers_tail, float* discarded_fraction,
                       float* shrinkage, float* ref_row_norm, float* coefficients, float* candidate,
                       float* result, double* ws, int C, int prev_rows, int total_layers,
                       bool functional, double eta, unsigned long long* timing,
                       cudaStream_t stream);

}  // namespace ro
