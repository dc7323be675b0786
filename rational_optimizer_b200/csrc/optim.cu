// Optimizer kernels for sm_100a.
//
// adamw_multi_tensor: every tensor of a parameter group in one launch.
// Tensor metadata (pointers, sizes, prefix offsets) travels in the kernel
// parameter block (no per-step host->device copy); each CTA locates its
// tensor by binary search over the prefix offsets.  The arithmetic is the
// decoupled-weight-decay AdamW of torch.optim.AdamW (single-tensor path):
//   p *= 1 - lr*wd;  m = lerp(m, g, 1-b1);  v = b2 v + (1-b2) g^2;
//   p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps).
#include "common.cuh"

namespace ro {
namespace optim {

constexpr int kMaxTensors = 192;

struct TensorList {
  float* p[kMaxTensors];
  const float* g[kMaxTensors];
  float* m[kMaxTensors];
  float* v[kMaxTensors];
  int64_t start[kMaxTensors + 1];  // prefix offsets in elements
  int count;
};

__device__ __forceinline__ float lerp_torch(float self, float end, float w) {
  return (fabsf(w) < 0.5f) ? fmaf(w, end - self, self) : end - (end - self) * (1.0f - w);
}

__global__ void __launch_bounds__(256)
adamw_kernel(const __grid_constant__ TensorList tl, float lr, float beta1, float beta2, float eps,
             float wd, float step_size, float bc2_sqrt) {
  const int64_t total = tl.start[tl.count];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    int lo = 0, hi = tl.count - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tl.start[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int64_t j = i - tl.start[lo];
    float p = tl.p[lo][j];
    const float g = tl.g[lo][j];
    float m = tl.m[lo][j];
    float v = tl.v[lo][j];
    p *= 1.0f - lr * wd;
    m = lerp_torch(m, g, 1.0f - beta1);
    v = fmaf(1.0f - beta2, g * g, v * beta2);
    const float denom = sqrtf(v) / bc2_sqrt + eps;
    p = fmaf(-step_size, m / denom, p);
    tl.p[lo][j] = p;
    tl.m[lo][j] = m;
    tl.v[lo][j] = v;
  }
}

}  // namespace optim

int adamw_multi_tensor(float* const* p, const float* const* g, float* const* m, float* const* v,
                       const int64_t* sizes, int count, float lr, float beta1, float beta2, float eps,
                       float wd, float step, cudaStream_t stream) {
  using namespace optim;
  const double bc1 = 1.0 - pow(static_cast<double>(beta1), static_cast<double>(step));
  const double bc2 = 1.0 - pow(static_cast<double>(beta2), static_cast<double>(step));
  const float step_size = static_cast<float>(lr / bc1);
  const float bc2_sqrt = static_cast<float>(sqrt(bc2));
  for (int base = 0; base < count; base += kMaxTensors) {
    TensorList tl;
    const int n = count - base < kMaxTensors ? count - base : kMaxTensors;
    tl.count = n;
    tl.start[0] = 0;
    for (int i = 0; i < n; ++i) {
      tl.p[i] = p[base + i];
      tl.g[i] = g[base + i];
      tl.m[i] = m[base + i];
      tl.v[i] = v[base + i];
      tl.start[i + 1] = tl.start[i] + sizes[base + i];
    }
    const int64_t total = tl.start[n];
    if (total == 0) continue;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    adamw_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(tl, lr, beta1, beta2, eps, wd,
                                                                 step_size, bc2_sqrt);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro
