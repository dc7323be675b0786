// Optimizer kernels for sm_100a.
//
// adamw_multi_tensor: every tensor of a parameter group in one launch.
// Tensor metadata (pointers, sizes, chunk prefix offsets) travels in the
// kernel parameter block (no per-step host->device copy); each CTA owns one
// 4096-element chunk and locates its tensor by one binary search.
// multi_tensor_dot: sum over tensors of <a_t, b_t> in one launch plus a
// fixed-order final reduction.  The arithmetic is the
// decoupled-weight-decay AdamW of torch.optim.AdamW (single-tensor path):
//   p *= 1 - lr*wd;  m = lerp(m, g, 1-b1);  v = b2 v + (1-b2) g^2;
//   p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps).
#include "common.cuh"

namespace ro {
namespace optim {

constexpr int kMaxTensors = 192;
constexpr int kChunk = 4096;  // elements per CTA
constexpr int kV = 8;

struct TensorList {
  float* p[kMaxTensors];
  const float* g[kMaxTensors];
  float* m[kMaxTensors];
  float* v[kMaxTensors];
  int64_t n[kMaxTensors];
  int64_t cstart[kMaxTensors + 1];  // prefix of per-tensor chunk counts
  int count;
};

__device__ __forceinline__ float lerp_torch(float self, float end, float w) {
  return (fabsf(w) < 0.5f) ? fmaf(w, end - self, self) : end - (end - self) * (1.0f - w);
}

// The CTA's tensor: the largest index whose first chunk is <= blockIdx.x
// (empty tensors are never selected: they share their first chunk with the
// next tensor).
__device__ __forceinline__ int chunk_owner(const int64_t* cstart, int count, int64_t c) {
  int lo = 0, hi = count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cstart[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct AdamScalars {
  float lr, beta1, beta2, eps, wd, step_size, bc2_sqrt;
};

__device__ __forceinline__ void adamw_element(float& p, float g, float& m, float& v, const AdamScalars& a) {
  p *= 1.0f - a.lr * a.wd;
  m = lerp_torch(m, g, 1.0f - a.beta1);
  v = fmaf(1.0f - a.beta2, g * g, v * a.beta2);
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p = fmaf(-a.step_size, m / denom, p);
}

// One CTA per 4096-element chunk of one tensor; 8-wide vector accesses when
// the tensor's four arrays are 16-byte aligned, element accesses otherwise.
__global__ void __launch_bounds__(256)
adamw_kernel(const __grid_constant__ TensorList tl, AdamScalars a) {
  const int t = chunk_owner(tl.cstart, tl.count, blockIdx.x);
  const int64_t start = (static_cast<int64_t>(blockIdx.x) - tl.cstart[t]) * kChunk;
  const int64_t end = start + kChunk < tl.n[t] ? start + kChunk : tl.n[t];
  if (!RO_CHECK(t >= 0 && t < tl.count && start >= 0 && end <= tl.n[t], 1)) return;
  float* __restrict__ P = tl.p[t];
  const float* __restrict__ G = tl.g[t];
  float* __restrict__ M = tl.m[t];
  float* __restrict__ Vv = tl.v[t];
  int64_t tail = start;
  if (aligned16(P) && aligned16(G) && aligned16(M) && aligned16(Vv)) {
    const int64_t vec_end = start + ((end - start) / kV) * kV;
    for (int64_t i = start + threadIdx.x * kV; i < vec_end; i += 256 * kV) {
      float p[kV], g[kV], m[kV], v[kV];
      load_vec<float, kV>(P + i, p);
      load_vec<float, kV>(G + i, g);
      load_vec<float, kV>(M + i, m);
      load_vec<float, kV>(Vv + i, v);
#pragma unroll
      for (int k = 0; k < kV; ++k) adamw_element(p[k], g[k], m[k], v[k], a);
      store_vec<float, kV>(P + i, p);
      store_vec<float, kV>(M + i, m);
      store_vec<float, kV>(Vv + i, v);
    }
    tail = vec_end;
  }
  for (int64_t i = tail + threadIdx.x; i < end; i += 256) {
    float p = P[i], m = M[i], v = Vv[i];
    adamw_element(p, G[i], m, v, a);
    P[i] = p;
    M[i] = m;
    Vv[i] = v;
  }
}

// Sum over tensors of <a_t, b_t>: per-chunk fp32 partials, then one CTA adds
// the partials in a fixed order in fp64 (bitwise reproducible).
struct DotList {
  const float* a[kMaxTensors];
  const float* b[kMaxTensors];
  int64_t n[kMaxTensors];
  int64_t cstart[kMaxTensors + 1];
  int count;
  int64_t part_offset;
};

__global__ void __launch_bounds__(256)
dot_chunks_kernel(const __grid_constant__ DotList dl, float* __restrict__ part) {
  __shared__ float red[8];
  const int t = chunk_owner(dl.cstart, dl.count, blockIdx.x);
  const int64_t start = (static_cast<int64_t>(blockIdx.x) - dl.cstart[t]) * kChunk;
  const int64_t end = start + kChunk < dl.n[t] ? start + kChunk : dl.n[t];
  // uniform per CTA, so the __syncthreads below is reached by all or none
  if (!RO_CHECK(t >= 0 && t < dl.count && start >= 0 && end <= dl.n[t], 2)) return;
  const float* __restrict__ A = dl.a[t];
  const float* __restrict__ B = dl.b[t];
  float s = 0.f;
  int64_t tail = start;
  if (aligned16(A) && aligned16(B)) {
    const int64_t vec_end = start + ((end - start) / kV) * kV;
    for (int64_t i = start + threadIdx.x * kV; i < vec_end; i += 256 * kV) {
      float x[kV], y[kV];
      load_vec<float, kV>(A + i, x);
      load_vec<float, kV>(B + i, y);
#pragma unroll
      for (int k = 0; k < kV; ++k) s = fmaf(x[k], y[k], s);
    }
    tail = vec_end;
  }
  for (int64_t i = tail + threadIdx.x; i < end; i += 256) s = fmaf(A[i], B[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float u = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) u += red[w];
    part[dl.part_offset + blockIdx.x] = u;
  }
}

__global__ void __launch_bounds__(1024)
sum_partials_kernel(const float* __restrict__ part, int64_t n, float scale, float* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += static_cast<double>(part[i]);
  s = warp_sum_d(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    out[0] = static_cast<float>(t * static_cast<double>(scale));
  }
}

// In-place gradient clipping: x *= min(max_norm / (sqrt(sumsq) + 1e-6), 1),
// the coefficient of torch.nn.utils.clip_grad_norm_, read from the device.
__global__ void __launch_bounds__(256)
clip_scale_kernel(float* __restrict__ x, int64_t n, const float* __restrict__ sumsq, float max_norm) {
  const float coef = fminf(max_norm / (sqrtf(sumsq[0]) + 1e-6f), 1.0f);
  const int64_t nvec = n / kV;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    float w[kV];
    load_vec<float, kV>(x + v * kV, w);
#pragma unroll
    for (int k = 0; k < kV; ++k) w[k] *= coef;
    store_vec<float, kV>(x + v * kV, w);
  }
  for (int64_t i = nvec * kV + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] *= coef;
}

}  // namespace optim

int adamw_multi_tensor(float* const* p, const float* const* g, float* const* m, float* const* v,
                       const int64_t* sizes, int count, float lr, float beta1, float beta2, float eps,
                       float wd, float step, cudaStream_t stream) {
  using namespace optim;
  const double bc1 = 1.0 - pow(static_cast<double>(beta1), static_cast<double>(step));
  const double bc2 = 1.0 - pow(static_cast<double>(beta2), static_cast<double>(step));
  AdamScalars a{lr, beta1, beta2, eps, wd, static_cast<float>(lr / bc1), static_cast<float>(sqrt(bc2))};
  int i = 0;
  while (i < count) {
    TensorList tl;
    int n = 0;
    tl.cstart[0] = 0;
    for (; i < count && n < kMaxTensors; ++i) {
      if (sizes[i] <= 0) continue;
      tl.p[n] = p[i];
      tl.g[n] = g[i];
      tl.m[n] = m[i];
      tl.v[n] = v[i];
      tl.n[n] = sizes[i];
      tl.cstart[n + 1] = tl.cstart[n] + (sizes[i] + kChunk - 1) / kChunk;
      ++n;
    }
    tl.count = n;
    if (n == 0) continue;
    adamw_kernel<<<static_cast<unsigned>(tl.cstart[n]), 256, 0, stream>>>(tl, a);
  }
  return static_cast<int>(cudaGetLastError());
}

int clip_scale(float* x, int64_t n, const float* sumsq, float max_norm, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (!aligned16(x)) return -1;
  int64_t blocks = (n / optim::kV + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  optim::clip_scale_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, n, sumsq, max_norm);
  return static_cast<int>(cudaGetLastError());
}

int64_t multi_tensor_dot_partials(const int64_t* sizes, int count) {
  int64_t c = 0;
  for (int i = 0; i < count; ++i) c += (sizes[i] + optim::kChunk - 1) / optim::kChunk;
  return c;
}

// out[0] = scale * sum_t <a_t, b_t>; part: multi_tensor_dot_partials floats.
int multi_tensor_dot(const float* const* a, const float* const* b, const int64_t* sizes, int count,
                     float scale, float* part, float* out, cudaStream_t stream) {
  using namespace optim;
  int i = 0;
  int64_t offset = 0;
  while (i < count) {
    DotList dl;
    int n = 0;
    dl.cstart[0] = 0;
    for (; i < count && n < kMaxTensors; ++i) {
      if (sizes[i] <= 0) continue;
      dl.a[n] = a[i];
      dl.b[n] = b[i];
      dl.n[n] = sizes[i];
      dl.cstart[n + 1] = dl.cstart[n] + (sizes[i] + kChunk - 1) / kChunk;
      ++n;
    }
    dl.count = n;
    dl.part_offset = offset;
    if (n == 0) continue;
    dot_chunks_kernel<<<static_cast<unsigned>(dl.cstart[n]), 256, 0, stream>>>(dl, part);
    offset += dl.cstart[n];
  }
  sum_partials_kernel<<<1, 1024, 0, stream>>>(part, offset, scale, out);
  return static_cast<int>(cudaGetLastError());
}

RO_BOUNDS_QUERY(optim_bounds_word)

}  // namespace ro
