// Memory-bound transformer ops for sm_100a: RMSNorm (fwd/bwd with a
// deterministic weight-gradient reduction), fused QKV split + interleaved-pair
// RoPE (fwd/bwd), and a one-pass softmax cross-entropy that writes the logit
// gradient in place.  Semantics follow training/train.py:24-45 (RMSNorm,
// precompute_rope/apply_rope) and the F.cross_entropy mean loss of
// training/train.py:2868-2870.
#include <cstdlib>

#include "common.cuh"
#include "packed.cuh"

namespace ro {
namespace nn {

// ---------------------------------------------------------------------------
// RMSNorm: y = w * x * rsqrt(mean(x^2) + eps).  One warp per row.  The fast
// path keeps the row in registers (d = 256 * NCH, lane owns 8 contiguous
// elements of each 256-wide chunk); the generic path re-reads the row.
constexpr int kNormWarps = 8;

template <typename T, typename TO, int NCH>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_fwd_fast(const T* __restrict__ x, const float* __restrict__ w, TO* __restrict__ y,
                 float* __restrict__ rstd_out, int64_t rows, float eps) {
  constexpr int d = NCH * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows || !span_ok(row, lane * 8, (NCH - 1) * 256 + lane * 8 + 8, rows, d, 1)) return;
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    load_vec<T, 8>(x + row * d + c * 256 + lane * 8, v[c]);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(d) + eps);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float wv[8];
    load_vec<float, 8>(w + c * 256 + lane * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[c][j] = wv[j] * (v[c][j] * r);
    store_vec<TO, 8>(y + row * d + c * 256 + lane * 8, v[c]);
  }
  if (lane == 0) rstd_out[row] = r;
}

template <typename T, typename TO>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_fwd_generic(const T* __restrict__ x, const float* __restrict__ w, TO* __restrict__ y,
                    float* __restrict__ rstd_out, int64_t rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * d;
  float ss = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float v = to_f<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(d) + eps);
  for (int i = lane; i < d; i += 32) y[row * d + i] = from_f<TO>(w[i] * (to_f<T>(xr[i]) * r));
  if (lane == 0) rstd_out[row] = r;
}

// Backward: dx = r * (w dy - xhat * mean(w dy xhat)), xhat = x r.
// Weight gradient partial per CTA: partial[blockIdx.x][d] = sum_rows dy*xhat.
template <typename T, typename TO, int NCH>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_bwd_fast(const TO* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                 const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ partial,
                 int64_t rows, int rows_per_block) {
  constexpr int d = NCH * 256;
  __shared__ float red[kNormWarps][256];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[c][j] = 0.f;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  int64_t r1 = r0 + rows_per_block;
  if (r1 > rows) r1 = rows;
  for (int64_t row = r0 + warp; row < r1; row += kNormWarps) {
    const float r = rstd[row];
    float xv[NCH][8], gv[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      load_vec<T, 8>(x + row * d + c * 256 + lane * 8, xv[c]);
      load_vec<TO, 8>(dy + row * d + c * 256 + lane * 8, gv[c]);
      float wv[8];
      load_vec<float, 8>(w + c * 256 + lane * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xv[c][j] * r;
        acc[c][j] = fmaf(gv[c][j], xh, acc[c][j]);
        const float wg = wv[j] * gv[c][j];
        dot = fmaf(wg, xh, dot);
        xv[c][j] = xh;
        gv[c][j] = wg;
      }
    }
    dot = warp_sum(dot) / static_cast<float>(d);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (gv[c][j] - xv[c][j] * dot);
      store_vec<T, 8>(dx + row * d + c * 256 + lane * 8, o);
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = acc[c][j];
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < kNormWarps; ++wi) s += red[wi][threadIdx.x];
    partial[static_cast<int64_t>(blockIdx.x) * d + c * 256 + threadIdx.x] = s;
    __syncthreads();
  }
}

template <typename T, typename TO>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_bwd_generic(const TO* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                    const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ partial,
                    int64_t rows, int d, int rows_per_block) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  int64_t r1 = r0 + rows_per_block;
  if (r1 > rows) r1 = rows;
  for (int64_t row = r0 + warp; row < r1; row += kNormWarps) {
    const float r = rstd[row];
    float dot = 0.f;
    for (int i = lane; i < d; i += 32)
      dot = fmaf(w[i] * to_f<TO>(dy[row * d + i]), to_f<T>(x[row * d + i]) * r, dot);
    dot = warp_sum(dot) / static_cast<float>(d);
    for (int i = lane; i < d; i += 32) {
      const float xh = to_f<T>(x[row * d + i]) * r;
      dx[row * d + i] = from_f<T>(r * (w[i] * to_f<TO>(dy[row * d + i]) - xh * dot));
    }
  }
  // Column partials: thread-per-column loop over the CTA's rows (fixed order).
  for (int col = threadIdx.x; col < d; col += blockDim.x) {
    float s = 0.f;
    for (int64_t row = r0; row < r1; ++row)
      s = fmaf(to_f<TO>(dy[row * d + col]), to_f<T>(x[row * d + col]) * rstd[row], s);
    partial[static_cast<int64_t>(blockIdx.x) * d + col] = s;
  }
}

// Column sums of partial [blocks, d]: CTA x covers 32 columns with 8 warps;
// warp w adds rows w, w+8, ... for its lane's column (coalesced 128-byte rows),
// then the 8 warp sums are added in warp order (fixed order: deterministic).
__global__ void __launch_bounds__(256)
column_reduce_kernel(const float* __restrict__ partial, int blocks, int d, float* __restrict__ out,
                     int accumulate) {
  __shared__ float red[8][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (col < d)
    for (int b = warp; b < blocks; b += 8) s += partial[static_cast<int64_t>(b) * d + col];
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && col < d) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    out[col] = accumulate ? out[col] + t : t;
  }
}


// Fused residual add + RMSNorm:  x_new = x + delta (fp32), y = w * x_new * rsqrt(mean(x_new^2)+eps).
// delta may be null (plain norm with x_new written as a copy only if x_new != x).
template <int NCH>
__global__ void __launch_bounds__(kNormWarps * 32)
add_rmsnorm_fwd_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                       const float* __restrict__ w, float* __restrict__ x_new,
                       __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int64_t rows,
                       float eps) {
  constexpr int d = NCH * 256;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows || !span_ok(row, lane * 8, (NCH - 1) * 256 + lane * 8 + 8, rows, d, 1)) return;
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t off = row * d + c * 256 + lane * 8;
    load_vec<float, 8>(x + off, v[c]);
    if (delta != nullptr) {
      float dv[8];
      load_vec<__nv_bfloat16, 8>(delta + off, dv);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c][j] += dv[j];
      store_vec<float, 8>(x_new + off, v[c]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(d) + eps);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float wv[8], o[8];
    load_vec<float, 8>(w + c * 256 + lane * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = wv[j] * (v[c][j] * r);
    store_vec<__nv_bfloat16, 8>(y + row * d + c * 256 + lane * 8, o);
  }
  if (lane == 0) rstd_out[row] = r;
}

// Backward of the fused op: dx = dres + r * (w dy - xhat * mean(w dy xhat)) (fp32); optionally
// also written as bf16 (the gradient of the bf16 delta branch).  dres may be null.
template <int NCH>
__global__ void __launch_bounds__(kNormWarps * 32)
add_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const float* __restrict__ dres,
                       const float* __restrict__ x, const float* __restrict__ w,
                       const float* __restrict__ rstd, float* __restrict__ dx,
                       __nv_bfloat16* __restrict__ ddelta, float* __restrict__ partial, int64_t rows,
                       int rows_per_block) {
  constexpr int d = NCH * 256;
  __shared__ float red[kNormWarps][256];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float acc[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[c][j] = 0.f;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  int64_t r1 = r0 + rows_per_block;
  if (r1 > rows) r1 = rows;
  for (int64_t row = r0 + warp; row < r1; row += kNormWarps) {
    const float r = rstd[row];
    float xv[NCH][8], gv[NCH][8], ov[NCH][8];
    float dot = 0.f;
    // the residual gradient is loaded with x and dy, so a row costs one
    // round trip to memory instead of two
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t off = row * d + c * 256 + lane * 8;
      if (dres != nullptr) {
        load_vec<float, 8>(dres + off, ov[c]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) ov[c][j] = 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t off = row * d + c * 256 + lane * 8;
      load_vec<float, 8>(x + off, xv[c]);
      load_vec<__nv_bfloat16, 8>(dy + off, gv[c]);
      float wv[8];
      load_vec<float, 8>(w + c * 256 + lane * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xv[c][j] * r;
        acc[c][j] = fmaf(gv[c][j], xh, acc[c][j]);
        const float wg = wv[j] * gv[c][j];
        dot = fmaf(wg, xh, dot);
        xv[c][j] = xh;
        gv[c][j] = wg;
      }
    }
    dot = warp_sum(dot) / static_cast<float>(d);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t off = row * d + c * 256 + lane * 8;
      float (&o)[8] = ov[c];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] += r * (gv[c][j] - xv[c][j] * dot);
      store_vec<float, 8>(dx + off, o);
      if (ddelta != nullptr) store_vec<__nv_bfloat16, 8>(ddelta + off, o);
    }
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = acc[c][j];
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < kNormWarps; ++wi) s += red[wi][threadIdx.x];
    partial[static_cast<int64_t>(blockIdx.x) * d + c * 256 + threadIdx.x] = s;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// QKV split + RoPE.  qkv: [B*S, 3*H*hd] (row = token); outputs q, k, v as
// [B, H, S, hd] contiguous.  Interleaved pairs (2j, 2j+1) rotate by
// angle = pos * theta^(-2j/hd) using fp32 cos/sin tables [S, hd/2].
// One CTA per token row (blockIdx.x = b * S + s); thread t owns 8 contiguous
// head-dim elements of (which, h) = (t / (H * hd/8), (t / (hd/8)) % H).  The
// qkv row is read contiguously; each (which, h) segment of hd elements is
// written contiguously.
__device__ __forceinline__ void rope_rotate(float (&val)[8], const float* __restrict__ cs,
                                            const float* __restrict__ sn, bool inverse) {
  const float4 c4 = *reinterpret_cast<const float4*>(cs);
  const float4 s4 = *reinterpret_cast<const float4*>(sn);
  const float c[4] = {c4.x, c4.y, c4.z, c4.w}, si[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float e = val[2 * p], o = val[2 * p + 1];
    if (!inverse) {
      val[2 * p] = e * c[p] - o * si[p];
      val[2 * p + 1] = e * si[p] + o * c[p];
    } else {
      val[2 * p] = e * c[p] + o * si[p];
      val[2 * p + 1] = -e * si[p] + o * c[p];
    }
  }
}

template <typename T>
__global__ void rope_qkv_fwd_kernel(const T* __restrict__ qkv, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, T* __restrict__ q,
                                    T* __restrict__ k, T* __restrict__ v, int B, int S, int H,
                                    int hd) {
  const int vec = hd / 8;
  const int t = blockIdx.y * blockDim.x + threadIdx.x;
  if (t >= 3 * H * vec) return;
  const int token = blockIdx.x;
  const int b = token / S, s = token - b * S;
  const int which = t / (H * vec);
  const int rem = t - which * H * vec;
  const int h = rem / vec, jv = rem - h * vec;
  const int d = H * hd;
  const int64_t tokens = static_cast<int64_t>(B) * S;
  if (!(span_ok(static_cast<int64_t>(token) * 3 + which, h * hd + jv * 8, h * hd + jv * 8 + 8, tokens * 3, d, 2) &&
        span_ok(static_cast<int64_t>(token) * H + h, jv * 8, jv * 8 + 8, tokens * H, hd, 2) &&
        span_ok(s, jv * 4, jv * 4 + 4, S, hd / 2, 2)))
    return;
  float val[8];
  load_vec<T, 8>(qkv + (static_cast<int64_t>(token) * 3 + which) * d + h * hd + jv * 8, val);
  if (which < 2) {
    const int half = hd / 2;
    rope_rotate(val, cos_t + s * half + jv * 4, sin_t + s * half + jv * 4, false);
  }
  T* out = which == 0 ? q : (which == 1 ? k : v);
  store_vec<T, 8>(out + (static_cast<int64_t>(token) * H + h) * hd + jv * 8, val);
}

template <typename T>
__global__ void rope_qkv_bwd_kernel(const T* __restrict__ dq, const T* __restrict__ dk,
                                    const T* __restrict__ dv, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, T* __restrict__ dqkv, int B,
                                    int S, int H, int hd) {
  const int vec = hd / 8;
  const int t = blockIdx.y * blockDim.x + threadIdx.x;
  if (t >= 3 * H * vec) return;
  const int token = blockIdx.x;
  const int b = token / S, s = token - b * S;
  const int which = t / (H * vec);
  const int rem = t - which * H * vec;
  const int h = rem / vec, jv = rem - h * vec;
  const int d = H * hd;
  const int64_t tokens = static_cast<int64_t>(B) * S;
  if (!(span_ok(static_cast<int64_t>(token) * 3 + which, h * hd + jv * 8, h * hd + jv * 8 + 8, tokens * 3, d, 3) &&
        span_ok(static_cast<int64_t>(token) * H + h, jv * 8, jv * 8 + 8, tokens * H, hd, 3) &&
        span_ok(s, jv * 4, jv * 4 + 4, S, hd / 2, 3)))
    return;
  const T* in = which == 0 ? dq : (which == 1 ? dk : dv);
  float val[8];
  load_vec<T, 8>(in + (static_cast<int64_t>(token) * H + h) * hd + jv * 8, val);
  if (which < 2) {
    const int half = hd / 2;
    rope_rotate(val, cos_t + s * half + jv * 4, sin_t + s * half + jv * 4, true);
  }
  store_vec<T, 8>(dqkv + (static_cast<int64_t>(token) * 3 + which) * d + h * hd + jv * 8, val);
}

// ---------------------------------------------------------------------------
// Cross-entropy with in-place gradient.  One CTA per row: one online pass for
// max and sum of exp, then the gradient pass re-reads the row (an L2 hit: the
// rows of all resident CTAs are a few tens of MB) or, with use_smem, reads it
// from a shared-memory copy made by the first pass (rows of up to 200 KB).
// Either way logits come from HBM once and the gradient is written once.
// loss_row[r] = lse - x[target]; logits are overwritten by
// (softmax - onehot) * grad_scale.  Rows whose target equals ignore_index get
// loss 0 and gradient 0.
constexpr int kCeThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kCeThreads)
ce_fwd_bwd_kernel(T* __restrict__ logits, const int64_t* __restrict__ target,
                  float* __restrict__ loss_row, int64_t rows, int V, float grad_scale,
                  int64_t ignore_index, int use_smem) {
  // With use_smem the row is staged in shared memory in its own dtype (bf16:
  // 100 KB for a 50k vocabulary, two CTAs per SM); max and sum of exp are
  // taken in one online pass, then the gradient is written over the logits.
  extern __shared__ __align__(16) unsigned char ce_smem[];
  T* srow = reinterpret_cast<T*>(ce_smem);
  __shared__ float red_m[kCeThreads / 32], red_s[kCeThreads / 32];
  __shared__ float bcast;
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  T* lr = logits + row * V;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tgt = target[row];
  const bool vec_ok = (V % 8 == 0) && (reinterpret_cast<uintptr_t>(lr) % 16 == 0);
  // The vector path works in base-2 units of the logits (u = v log2 e):
  // m is the running max of v, s the sum of 2^(u - m log2 e), so each element
  // costs one packed FMA and one ex2 per pass.
  constexpr float kLog2e = 1.4426950408889634f;
  const float2 l2e = splat2(kLog2e);
  float m = -INFINITY, s = 0.f;
  auto absorb = [&](const float (&v)[8], int count) {
    float mx = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j)
      if (j < count) mx = fmaxf(mx, v[j]);
    if (mx > m) {
      s *= __expf(m - mx);
      m = mx;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < count) s += __expf(v[j] - m);
  };
  if (vec_ok) {
    float2 s2 = splat2(0.f);
    for (int i = tid * 8; i < V; i += kCeThreads * 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(lr + i);
      if (use_smem) *reinterpret_cast<uint4*>(srow + i) = raw;
      float v8[8];
      load_vec<T, 8>(reinterpret_cast<const T*>(&raw), v8);
      const float mx = fmaxf(fmaxf(fmaxf(v8[0], v8[1]), fmaxf(v8[2], v8[3])),
                             fmaxf(fmaxf(v8[4], v8[5]), fmaxf(v8[6], v8[7])));
      if (mx > m) {
        const float r = exp2f((m - mx) * kLog2e);  // 0 while m = -inf
        s2 = mul2(s2, splat2(r));
        m = mx;
      }
      const float2 nm = splat2(-m * kLog2e);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 u = fma2(make_float2(v8[j], v8[j + 1]), l2e, nm);
        s2 = add2(s2, make_float2(ex2_approx(u.x), ex2_approx(u.y)));
      }
    }
    s = s2.x + s2.y;
  } else {
    for (int i = tid; i < V; i += kCeThreads) {
      const T raw = lr[i];
      if (use_smem) srow[i] = raw;
      float v8[8] = {to_f<T>(raw), 0, 0, 0, 0, 0, 0, 0};
      absorb(v8, 1);
    }
  }
  // combine (m, s) pairs: warp, then block
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    float wm = lane < kCeThreads / 32 ? red_m[lane] : -INFINITY;
    float ws = lane < kCeThreads / 32 ? red_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, wm, o);
      const float os = __shfl_xor_sync(0xffffffffu, ws, o);
      const float nm = fmaxf(wm, om);
      ws = (wm == -INFINITY ? 0.f : ws * __expf(wm - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      wm = nm;
    }
    if (lane == 0) bcast = wm + __logf(ws);
  }
  // The target logit is read before the barrier: after it, every thread
  // overwrites its elements of the row with the gradient.
  const bool ignored = (tgt == ignore_index) || tgt < 0 || tgt >= V;
  float xt = 0.f;
  if (tid == 0 && !ignored && RO_CHECK(tgt >= 0 && tgt < V, 4)) xt = to_f<T>(use_smem ? srow[tgt] : lr[tgt]);
  __syncthreads();
  const float lse = bcast;
  if (tid == 0) loss_row[row] = ignored ? 0.f : (lse - xt);
  const float scale = ignored ? 0.f : grad_scale;
  if (vec_ok) {
    const float2 nl = splat2(-lse * kLog2e), sc = splat2(scale);
    for (int i = tid * 8; i < V; i += kCeThreads * 8) {
      float v8[8];
      load_vec<T, 8>(use_smem ? srow + i : lr + i, v8);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 u = fma2(make_float2(v8[j], v8[j + 1]), l2e, nl);
        v8[j] = ex2_approx(u.x);
        v8[j + 1] = ex2_approx(u.y);
      }
      // the target's probability loses 1 (one vector of the row holds it)
      if (static_cast<uint64_t>(tgt - i) < 8u) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i + j == tgt) v8[j] -= 1.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 g = mul2(make_float2(v8[j], v8[j + 1]), sc);
        v8[j] = g.x;
        v8[j + 1] = g.y;
      }
      store_vec<T, 8>(lr + i, v8);
    }
  } else {
    for (int i = tid; i < V; i += kCeThreads) {
      const float v = to_f<T>(use_smem ? srow[i] : lr[i]);
      float p = __expf(v - lse);
      if (i == tgt) p -= 1.0f;
      lr[i] = from_f<T>(p * scale);
    }
  }
}

}  // namespace nn

// ---------------------------------------------------------------------------
// Host launchers.

int rmsnorm_forward(const void* x, const float* w, void* y, float* rstd, int64_t rows, int d,
                    float eps, int dtype, int out_dtype, cudaStream_t stream) {
  using namespace nn;
  if (rows <= 0) return 0;
  const int blocks = ceil_div_i(rows, kNormWarps);
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  auto go = [&](auto tv, auto tov) {
    using T = decltype(tv);
    using TO = decltype(tov);
    const T* xp = static_cast<const T*>(x);
    TO* yp = static_cast<TO*>(y);
    if (aligned && d % 256 == 0 && d / 256 <= 8) {
      switch (d / 256) {
        case 1: rmsnorm_fwd_fast<T, TO, 1><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        case 2: rmsnorm_fwd_fast<T, TO, 2><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        case 3: rmsnorm_fwd_fast<T, TO, 3><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        case 4: rmsnorm_fwd_fast<T, TO, 4><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        case 6: rmsnorm_fwd_fast<T, TO, 6><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        case 8: rmsnorm_fwd_fast<T, TO, 8><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, eps); return;
        default: break;
      }
    }
    rmsnorm_fwd_generic<T, TO><<<blocks, kNormWarps * 32, 0, stream>>>(xp, w, yp, rstd, rows, d, eps);
  };
  if (dtype == 0 && out_dtype == 0) go(float{}, float{});
  else if (dtype == 1 && out_dtype == 1) go(__nv_bfloat16{}, __nv_bfloat16{});
  else if (dtype == 0 && out_dtype == 1) go(float{}, __nv_bfloat16{});
  else return -2;
  return static_cast<int>(cudaGetLastError());
}

void rmsnorm_backward_plan(int64_t rows, int& blocks, int& rows_per_block) {
  int64_t b = 148 * 4;
  const int64_t maxb = (rows + nn::kNormWarps - 1) / nn::kNormWarps;
  if (b > maxb) b = maxb;
  if (b < 1) b = 1;
  rows_per_block = static_cast<int>((rows + b - 1) / b);
  blocks = static_cast<int>((rows + rows_per_block - 1) / rows_per_block);
}

int rmsnorm_backward_partial_size(int64_t rows, int d) {
  int blocks, rpb;
  rmsnorm_backward_plan(rows, blocks, rpb);
  return blocks * d;
}

int rmsnorm_backward(const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                     float* dw, float* partial, int64_t rows, int d, int dtype, int out_dtype,
                     int accumulate_dw, cudaStream_t stream) {
  using namespace nn;
  int blocks = 0, rpb = 1;
  if (rows > 0) {
    rmsnorm_backward_plan(rows, blocks, rpb);
    const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(dy) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(dx) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(w) % 16 == 0);
    auto go = [&](auto tv, auto tov) {
      using T = decltype(tv);
      using TO = decltype(tov);
      const TO* dyp = static_cast<const TO*>(dy);
      const T* xp = static_cast<const T*>(x);
      T* dxp = static_cast<T*>(dx);
      if (aligned && d % 256 == 0 && d / 256 <= 4) {
        switch (d / 256) {
          case 1: rmsnorm_bwd_fast<T, TO, 1><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, xp, w, rstd, dxp, partial, rows, rpb); return;
          case 2: rmsnorm_bwd_fast<T, TO, 2><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, xp, w, rstd, dxp, partial, rows, rpb); return;
          case 3: rmsnorm_bwd_fast<T, TO, 3><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, xp, w, rstd, dxp, partial, rows, rpb); return;
          case 4: rmsnorm_bwd_fast<T, TO, 4><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, xp, w, rstd, dxp, partial, rows, rpb); return;
          default: break;
        }
      }
      rmsnorm_bwd_generic<T, TO><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, xp, w, rstd, dxp, partial, rows, d, rpb);
    };
    if (dtype == 0 && out_dtype == 0) go(float{}, float{});
    else if (dtype == 1 && out_dtype == 1) go(__nv_bfloat16{}, __nv_bfloat16{});
    else if (dtype == 0 && out_dtype == 1) go(float{}, __nv_bfloat16{});
    else return -2;
  }
  column_reduce_kernel<<<ceil_div_i(d, 32), 256, 0, stream>>>(partial, blocks, d, dw, accumulate_dw);
  return static_cast<int>(cudaGetLastError());
}

int add_rmsnorm_forward(const float* x, const void* delta, const float* w, float* x_new, void* y,
                        float* rstd, int64_t rows, int d, float eps, cudaStream_t stream) {
  using namespace nn;
  if (rows <= 0) return 0;
  if (d % 256 || d / 256 > 8) return -1;
  const int blocks = ceil_div_i(rows, kNormWarps);
  const auto* dp = static_cast<const __nv_bfloat16*>(delta);
  auto* yp = static_cast<__nv_bfloat16*>(y);
  switch (d / 256) {
    case 1: add_rmsnorm_fwd_kernel<1><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    case 2: add_rmsnorm_fwd_kernel<2><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    case 3: add_rmsnorm_fwd_kernel<3><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    case 4: add_rmsnorm_fwd_kernel<4><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    case 6: add_rmsnorm_fwd_kernel<6><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    case 8: add_rmsnorm_fwd_kernel<8><<<blocks, kNormWarps * 32, 0, stream>>>(x, dp, w, x_new, yp, rstd, rows, eps); break;
    default: return -1;
  }
  return static_cast<int>(cudaGetLastError());
}

int add_rmsnorm_backward(const void* dy, const float* dres, const float* x, const float* w,
                         const float* rstd, float* dx, void* ddelta, float* dw, bool accumulate_dw,
                         float* partial, int64_t rows, int d, cudaStream_t stream) {
  using namespace nn;
  if (d % 256 || d / 256 > 4) return -1;
  int blocks = 0, rpb = 1;
  if (rows > 0) {
    rmsnorm_backward_plan(rows, blocks, rpb);
    const auto* dyp = static_cast<const __nv_bfloat16*>(dy);
    auto* ddp = static_cast<__nv_bfloat16*>(ddelta);
#define RO_NORM_BWD(N) \
  add_rmsnorm_bwd_kernel<N><<<blocks, kNormWarps * 32, 0, stream>>>(dyp, dres, x, w, rstd, dx, ddp, partial, rows, rpb)
    switch (d / 256) {
      case 1: RO_NORM_BWD(1); break;
      case 2: RO_NORM_BWD(2); break;
      case 3: RO_NORM_BWD(3); break;
      case 4: RO_NORM_BWD(4); break;
      default: return -1;
    }
#undef RO_NORM_BWD
  }
  column_reduce_kernel<<<ceil_div_i(d, 32), 256, 0, stream>>>(partial, blocks, d, dw, accumulate_dw ? 1 : 0);
  return static_cast<int>(cudaGetLastError());
}

int rope_qkv_forward(const void* qkv, const float* cos_t, const float* sin_t, void* q, void* k,
                     void* v, int B, int S, int H, int hd, int dtype, cudaStream_t stream) {
  if (hd % 8) return -1;
  if (static_cast<int64_t>(B) * S * H == 0) return 0;
  const int per_token = 3 * H * (hd / 8);
  const int threads = per_token < 512 ? ((per_token + 31) / 32) * 32 : 512;
  const dim3 blocks(static_cast<unsigned>(B * S), static_cast<unsigned>((per_token + threads - 1) / threads));
  if (dtype == 0)
    nn::rope_qkv_fwd_kernel<float><<<blocks, threads, 0, stream>>>(
        static_cast<const float*>(qkv), cos_t, sin_t, static_cast<float*>(q), static_cast<float*>(k),
        static_cast<float*>(v), B, S, H, hd);
  else if (dtype == 1)
    nn::rope_qkv_fwd_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(qkv), cos_t, sin_t, static_cast<__nv_bfloat16*>(q),
        static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v), B, S, H, hd);
  else return -2;
  return static_cast<int>(cudaGetLastError());
}

int rope_qkv_backward(const void* dq, const void* dk, const void* dv, const float* cos_t,
                      const float* sin_t, void* dqkv, int B, int S, int H, int hd, int dtype,
                      cudaStream_t stream) {
  if (hd % 8) return -1;
  if (static_cast<int64_t>(B) * S * H == 0) return 0;
  const int per_token = 3 * H * (hd / 8);
  const int threads = per_token < 512 ? ((per_token + 31) / 32) * 32 : 512;
  const dim3 blocks(static_cast<unsigned>(B * S), static_cast<unsigned>((per_token + threads - 1) / threads));
  if (dtype == 0)
    nn::rope_qkv_bwd_kernel<float><<<blocks, threads, 0, stream>>>(
        static_cast<const float*>(dq), static_cast<const float*>(dk), static_cast<const float*>(dv),
        cos_t, sin_t, static_cast<float*>(dqkv), B, S, H, hd);
  else if (dtype == 1)
    nn::rope_qkv_bwd_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(dq), static_cast<const __nv_bfloat16*>(dk),
        static_cast<const __nv_bfloat16*>(dv), cos_t, sin_t, static_cast<__nv_bfloat16*>(dqkv), B, S,
        H, hd);
  else return -2;
  return static_cast<int>(cudaGetLastError());
}

constexpr size_t kCeMaxSmemBytes = 200 * 1024;

int cross_entropy_fwd_bwd(void* logits, const int64_t* target, float* loss_row, int64_t rows,
                          int V, float grad_scale, int64_t ignore_index, int dtype,
                          cudaStream_t stream) {
  if (rows <= 0) return 0;
  const size_t elem = dtype == 1 ? 2 : 4;
  // The gradient pass re-reads the row (from L2: the rows of the resident
  // CTAs fit easily) instead of staging it in shared memory, which would
  // limit residency to two CTAs per SM: 0.360 against 0.442 ms for 32768 x
  // 50304 bf16 logits on one B200.  RO_CE_SMEM=1 restores the staging.
  static const bool smem_ok = [] {
    const char* v = std::getenv("RO_CE_SMEM");
    return v != nullptr && v[0] == '1';
  }();
  const int use_smem = smem_ok && static_cast<size_t>(V) * elem <= kCeMaxSmemBytes ? 1 : 0;
  const size_t smem = use_smem ? (static_cast<size_t>(V) * elem + 15) / 16 * 16 : 0;
  auto go = [&](auto tv) {
    using T = decltype(tv);
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(nn::ce_fwd_bwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
    nn::ce_fwd_bwd_kernel<T><<<static_cast<unsigned>(rows), nn::kCeThreads, smem, stream>>>(
        static_cast<T*>(logits), target, loss_row, rows, V, grad_scale, ignore_index, use_smem);
  };
  if (dtype == 0) go(float{});
  else if (dtype == 1) go(__nv_bfloat16{});
  else return -2;
  return static_cast<int>(cudaGetLastError());
}

RO_BOUNDS_QUERY(nn_ops_bounds_word)

#ifdef RO_BOUNDS_CHECK
namespace nn {
// Writes buf[index] = 1 only when 0 <= index < n; otherwise records site 99.
__global__ void bounds_selftest_kernel(float* buf, int64_t n, int64_t index) {
  if (RO_CHECK(index >= 0 && index < n, 99)) buf[index] = 1.0f;
}
}  // namespace nn

int bounds_selftest(float* buf, int64_t n, int64_t index, cudaStream_t stream) {
  nn::bounds_selftest_kernel<<<1, 1, 0, stream>>>(buf, n, index);
  return static_cast<int>(cudaGetLastError());
}
#else
// Without the checks the guarded store would not be skipped: refuse.
int bounds_selftest(float*, int64_t, int64_t, cudaStream_t) { return -1; }
#endif

}  // namespace ro
