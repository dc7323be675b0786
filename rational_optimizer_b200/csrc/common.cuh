// Shared device helpers for the sm_100a kernels of this package.
//
// Every kernel file includes only CUDA headers; the PyTorch binding layer
// (bindings.cpp) owns tensor validation and passes raw pointers plus the
// current stream.  Keeping ATen out of the .cu files keeps nvcc builds short.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace ro {

enum class DType : int { kFloat32 = 0, kBFloat16 = 1 };

__host__ __device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float sign0(float x) {
  return (x > 0.0f) ? 1.0f : ((x < 0.0f) ? -1.0f : 0.0f);
}

// Scalar conversions.
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Load/store N contiguous elements as float.  N*sizeof(T) of 4, 8, 16 or 32
// bytes uses vector accesses (the address must be aligned to min(16, size));
// other sizes fall back to element accesses.  Callers guarantee alignment.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  if constexpr (sizeof(T) * N == 32) {
    // two 16-byte loads (32 bytes, 16-byte aligned)
    const uint4 raw0 = reinterpret_cast<const uint4*>(p)[0];
    const uint4 raw1 = reinterpret_cast<const uint4*>(p)[1];
    const T* e0 = reinterpret_cast<const T*>(&raw0);
    const T* e1 = reinterpret_cast<const T*>(&raw1);
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      out[i] = to_f<T>(e0[i]);
      out[N / 2 + i] = to_f<T>(e1[i]);
    }
  } else if constexpr (sizeof(T) * N == 16) {
    uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else if constexpr (sizeof(T) * N == 8) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else if constexpr (sizeof(T) * N == 4) {
    uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f<T>(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&in)[N]) {
  if constexpr (sizeof(T) * N == 32) {
    uint4 raw0, raw1;
    T* e0 = reinterpret_cast<T*>(&raw0);
    T* e1 = reinterpret_cast<T*>(&raw1);
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      e0[i] = from_f<T>(in[i]);
      e1[i] = from_f<T>(in[N / 2 + i]);
    }
    reinterpret_cast<uint4*>(p)[0] = raw0;
    reinterpret_cast<uint4*>(p)[1] = raw1;
  } else if constexpr (sizeof(T) * N == 16) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint4*>(p) = raw;
  } else if constexpr (sizeof(T) * N == 8) {
    uint2 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint2*>(p) = raw;
  } else if constexpr (sizeof(T) * N == 4) {
    uint32_t raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < N; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint32_t*>(p) = raw;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f<T>(in[i]);
  }
}

inline int ceil_div_i(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// ---------------------------------------------------------------------------
// Bounds-checked builds.  Compiled with -DRO_BOUNDS_CHECK, RO_CHECK(cond, site)
// evaluates `cond`; when it is false the first such failure of this source
// file is recorded in a device word as (site << 32) | source line and the
// macro yields false, so the caller skips the access it guards instead of
// touching memory it does not own (no trap, the context stays usable).  In
// normal builds RO_CHECK is the constant true and costs nothing.  Every .cu
// file that uses it defines a host query with RO_BOUNDS_QUERY(name), which
// returns the word and clears it (0 = no failure).
#ifdef RO_BOUNDS_CHECK
static __device__ unsigned long long g_bounds_word = 0ull;

static __device__ __noinline__ void bounds_record(unsigned site, unsigned line) {
  atomicCAS(&g_bounds_word, 0ull, (static_cast<unsigned long long>(site) << 32) | line);
}

#define RO_CHECK(cond, site) \
  (__builtin_expect(!!(cond), 1) ? true : (::ro::bounds_record((site), __LINE__), false))

#define RO_BOUNDS_QUERY(name)                                                          \
  unsigned long long name() {                                                          \
    unsigned long long word = 0ull;                                                    \
    const unsigned long long zero = 0ull;                                              \
    if (cudaMemcpyFromSymbol(&word, ::ro::g_bounds_word, sizeof(word)) != cudaSuccess) \
      return ~0ull;                                                                    \
    cudaMemcpyToSymbol(::ro::g_bounds_word, &zero, sizeof(zero));                      \
    return word;                                                                       \
  }
#else
#define RO_CHECK(cond, site) true
#define RO_BOUNDS_QUERY(name) \
  unsigned long long name() { return 0ull; }
#endif

// Row r, columns [c0, c1) of a [rows, cols] row-major plane.
__device__ __forceinline__ bool span_ok(int64_t r, int64_t c0, int64_t c1, int64_t rows, int64_t cols,
                                        unsigned site) {
  return RO_CHECK(r >= 0 && r < rows && c0 >= 0 && c0 <= c1 && c1 <= cols, site);
}

}  // namespace ro
