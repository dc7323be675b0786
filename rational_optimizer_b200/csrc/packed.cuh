// Packed fp32x2 arithmetic (sm_100 FFMA2/FMUL2/FADD2: two fp32 lanes per
// instruction) and register-pair loads/stores for elementwise kernels.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace ro {

__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 abs2(float2 a) { return make_float2(fabsf(a.x), fabsf(a.y)); }
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }
__device__ __forceinline__ float2 sign02(float2 a) { return make_float2(sign0(a.x), sign0(a.y)); }
// Fast reciprocal of each lane (the __fdividef(1, x) intrinsic); callers use
// it only where x >= 1.
__device__ __forceinline__ float2 rcp2(float2 a) {
  return make_float2(__fdividef(1.0f, a.x), __fdividef(1.0f, a.y));
}

// 2^x by the hardware approximation (ex2.approx.ftz.f32: about 2 ulp,
// subnormal results flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// P = E / 2 consecutive pairs from E contiguous elements (16-byte aligned for
// the vector paths: E * sizeof(T) in {8, 16, 32}).
template <typename T, int E>
__device__ __forceinline__ void load_pairs(const T* __restrict__ p, float2 (&out)[E / 2]);

template <int E>
__device__ __forceinline__ void load_pairs_bf16(const __nv_bfloat16* __restrict__ p, float2 (&out)[E / 2]) {
  static_assert(E == 2 || E == 4 || E == 8, "bf16 pair loads cover 4, 8 or 16 bytes");
  if constexpr (E == 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    out[0] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    out[1] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    out[2] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.z));
    out[3] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.w));
  } else if constexpr (E == 4) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    out[0] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    out[1] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  } else {
    const uint32_t raw = *reinterpret_cast<const uint32_t*>(p);
    out[0] = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw));
  }
}

template <int E>
__device__ __forceinline__ void load_pairs_f32(const float* __restrict__ p, float2 (&out)[E / 2]) {
  static_assert(E % 2 == 0 && E <= 8, "fp32 pair loads cover 8 to 32 bytes");
  if constexpr (E >= 4) {
#pragma unroll
    for (int i = 0; i < E / 4; ++i) {
      const float4 v = reinterpret_cast<const float4*>(p)[i];
      out[2 * i] = make_float2(v.x, v.y);
      out[2 * i + 1] = make_float2(v.z, v.w);
    }
  } else {
    out[0] = *reinterpret_cast<const float2*>(p);
  }
}

template <> __device__ __forceinline__ void load_pairs<__nv_bfloat16, 8>(const __nv_bfloat16* p, float2 (&o)[4]) { load_pairs_bf16<8>(p, o); }
template <> __device__ __forceinline__ void load_pairs<__nv_bfloat16, 4>(const __nv_bfloat16* p, float2 (&o)[2]) { load_pairs_bf16<4>(p, o); }
template <> __device__ __forceinline__ void load_pairs<__nv_bfloat16, 2>(const __nv_bfloat16* p, float2 (&o)[1]) { load_pairs_bf16<2>(p, o); }
template <> __device__ __forceinline__ void load_pairs<float, 8>(const float* p, float2 (&o)[4]) { load_pairs_f32<8>(p, o); }
template <> __device__ __forceinline__ void load_pairs<float, 4>(const float* p, float2 (&o)[2]) { load_pairs_f32<4>(p, o); }
template <> __device__ __forceinline__ void load_pairs<float, 2>(const float* p, float2 (&o)[1]) { load_pairs_f32<2>(p, o); }

template <typename T, int E>
__device__ __forceinline__ void store_pairs(T* __restrict__ p, const float2 (&in)[E / 2]) {
  if constexpr (sizeof(T) == 2) {
    uint32_t w[E / 2];
#pragma unroll
    for (int i = 0; i < E / 2; ++i) {
      const __nv_bfloat162 h = __float22bfloat162_rn(in[i]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if constexpr (E == 8) *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    else if constexpr (E == 4) *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
    else *reinterpret_cast<uint32_t*>(p) = w[0];
  } else {
    if constexpr (E >= 4) {
#pragma unroll
      for (int i = 0; i < E / 4; ++i)
        reinterpret_cast<float4*>(p)[i] = make_float4(in[2 * i].x, in[2 * i].y, in[2 * i + 1].x, in[2 * i + 1].y);
    } else {
      *reinterpret_cast<float2*>(p) = in[0];
    }
  }
}

}  // namespace ro
