// GRAIN: grouped, RMS-normalised P5/Q4 rational activation (sm_100a).
//
// Operator (per row r and group g of width w, "Version A" denominator):
//   rho = sqrt(mean(z^2) + eps),  t = z / rho,
//   f(t) = P(t) / Q(t) + sum_k [c_odd_k * odd_k(t) + c_bump_k * bump_k(t)],
//   P(t) = sum_{j<6} a_j t^j,  Q(t) = 1 + |b0||t| + |b1|t^2 + |b2||t|^3 + |b3|t^4,
//   y = rho * f(t).
// Semantics follow activation/rational_opt/rational.py:40-107 (torch oracle)
// and the fused kernels of activation/csrc/rational_cuda_kernel.cu:355-687
// (K6-K10 of the reference), including the optional <=4 local-basis atoms,
// the affine-statistics reduction and the restricted-morphology backward.
//
// Layout and scheduling are this package's own: one warp owns one
// (row, group) segment and keeps it in registers (w <= 256 -> <= 8 values per
// lane, 16-byte vector loads for bf16/fp32), a CTA of 8 warps owns one group
// and a contiguous chunk of rows so the group's coefficients live in
// registers, and coefficient gradients are reduced deterministically in two
// stages (per-CTA partials, then a fixed-order reduction) instead of fp32
// atomics, so data-parallel replicas stay bitwise identical.
#include <mutex>

#include "common.cuh"
#include "packed.cuh"

namespace ro {
namespace grain {

constexpr int kNum = 6;
constexpr int kDen = 4;
constexpr int kBase = kNum + kDen;
constexpr int kMaxBasis = 4;
constexpr int kMaxGrad = kBase + 2 * kMaxBasis;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct Coeffs {
  float a[kNum];
  float b[kDen];   // |b_raw|
  float bs[kDen];  // sign(b_raw), 0 at 0 (matches the reference's sign0)
  int nb;
  float center[kMaxBasis];
  float beta[kMaxBasis];
  float codd[kMaxBasis];
  float cbump[kMaxBasis];
  float dodd[kMaxBasis];   // coeff_limit * (1 - tanh^2) for the odd logit
  float dbump[kMaxBasis];  // same for the bump logit
  float zero_level[kMaxBasis];
};

__device__ __forceinline__ void load_coeffs(Coeffs& c, int g, const float* __restrict__ num,
                                            const float* __restrict__ den,
                                            const float* __restrict__ logits,
                                            const float* __restrict__ centers,
                                            const float* __restrict__ beta, int nb,
                                            float coeff_limit) {
#pragma unroll
  for (int j = 0; j < kNum; ++j) c.a[j] = num[g * kNum + j];
#pragma unroll
  for (int j = 0; j < kDen; ++j) {
    const float r = den[g * kDen + j];
    c.b[j] = fabsf(r);
    c.bs[j] = sign0(r);
  }
  c.nb = nb;
#pragma unroll
  for (int k = 0; k < kMaxBasis; ++k) {
    if (k < nb) {
      c.center[k] = centers[g * nb + k];
      c.beta[k] = beta[g * nb + k];
      const float to = tanhf(logits[(g * nb + k) * 2 + 0]);
      const float tb = tanhf(logits[(g * nb + k) * 2 + 1]);
      c.codd[k] = coeff_limit * to;
      c.cbump[k] = coeff_limit * tb;
      c.dodd[k] = coeff_limit * (1.0f - to * to);
      c.dbump[k] = coeff_limit * (1.0f - tb * tb);
      c.zero_level[k] = 1.0f / (1.0f + c.beta[k] * c.center[k] * c.center[k]);
    } else {
      c.center[k] = c.beta[k] = c.codd[k] = c.cbump[k] = 0.f;
      c.dodd[k] = c.dbump[k] = 0.f;
      c.zero_level[k] = 0.f;
    }
  }
}

// f(t) only.
__device__ __forceinline__ float eval_f(const Coeffs& c, float t) {
  const float at = fabsf(t);
  const float t2 = t * t;
  const float p = fmaf(fmaf(fmaf(fmaf(fmaf(c.a[5], t, c.a[4]), t, c.a[3]), t, c.a[2]), t, c.a[1]), t, c.a[0]);
  const float q = 1.0f + c.b[0] * at + c.b[1] * t2 + c.b[2] * at * t2 + c.b[3] * t2 * t2;
  float f = __fdividef(p, q);
  for (int k = 0; k < c.nb; ++k) {
    const float u = t - c.center[k];
    const float inv = __fdividef(1.0f, 1.0f + c.beta[k] * u * u);
    f += c.codd[k] * u * inv + c.cbump[k] * (inv - c.zero_level[k]);
  }
  return f;
}

// f, f' and the coefficient partials d f / d theta (without the rho factor).
template <int NGRAD>
__device__ __forceinline__ void eval_full(const Coeffs& c, float t, float& f, float& df,
                                          float (&part)[NGRAD]) {
  const float at = fabsf(t);
  const float t2 = t * t;
  const float t3 = t2 * t;
  const float t4 = t2 * t2;
  const float at3 = at * t2;
  const float p = fmaf(fmaf(fmaf(fmaf(fmaf(c.a[5], t, c.a[4]), t, c.a[3]), t, c.a[2]), t, c.a[1]), t, c.a[0]);
  const float dp = fmaf(fmaf(fmaf(fmaf(5.0f * c.a[5], t, 4.0f * c.a[4]), t, 3.0f * c.a[3]), t, 2.0f * c.a[2]), t, c.a[1]);
  const float q = 1.0f + c.b[0] * at + c.b[1] * t2 + c.b[2] * at3 + c.b[3] * t4;
  const float dq = c.b[0] * sign0(t) + 2.0f * c.b[1] * t + 3.0f * c.b[2] * t * at + 4.0f * c.b[3] * t3;
  const float iq = __fdividef(1.0f, q);  // q >= 1: fast reciprocal is well conditioned
  const float iq2 = iq * iq;
  f = p * iq;
  df = (dp * q - p * dq) * iq2;
  if constexpr (NGRAD >= kBase) {
    part[0] = iq;
    part[1] = t * iq;
    part[2] = t2 * iq;
    part[3] = t3 * iq;
    part[4] = t4 * iq;
    part[5] = t4 * t * iq;
    const float bsc = -p * iq2;
    part[6] = bsc * c.bs[0] * at;
    part[7] = bsc * c.bs[1] * t2;
    part[8] = bsc * c.bs[2] * at3;
    part[9] = bsc * c.bs[3] * t4;
  }
#pragma unroll
  for (int k = 0; k < kMaxBasis; ++k) {
    if (k < c.nb) {
      const float u = t - c.center[k];
      const float u2 = u * u;
      const float inv = __fdividef(1.0f, 1.0f + c.beta[k] * u2);
      const float inv2 = inv * inv;
      const float odd = u * inv;
      const float odd_dt = (1.0f - c.beta[k] * u2) * inv2;
      const float bump = inv - c.zero_level[k];
      const float bump_dt = -2.0f * c.beta[k] * u * inv2;
      f += c.codd[k] * odd + c.cbump[k] * bump;
      df += c.codd[k] * odd_dt + c.cbump[k] * bump_dt;
      if constexpr (NGRAD > kBase) {
        part[kBase + 2 * k] = c.dodd[k] * odd;
        part[kBase + 2 * k + 1] = c.dbump[k] * bump;
      }
    }
  }
}

// Per-lane element mapping: CONTIG lanes own [lane*E, lane*E+E); otherwise
// lane owns {lane + 32*j}.  E*32 >= w always.
template <typename T, int E, bool CONTIG>
__device__ __forceinline__ void load_seg(const T* __restrict__ base, int w, int lane,
                                         float (&v)[E]) {
  if constexpr (CONTIG) {
    load_vec<T, E>(base + lane * E, v);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int i = lane + 32 * j;
      v[j] = (i < w) ? to_f<T>(base[i]) : 0.0f;
    }
  }
}

template <typename T, int E, bool CONTIG>
__device__ __forceinline__ void store_seg(T* __restrict__ base, int w, int lane,
                                          const float (&v)[E]) {
  if constexpr (CONTIG) {
    store_vec<T, E>(base + lane * E, v);
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int i = lane + 32 * j;
      if (i < w) base[i] = from_f<T>(v[j]);
    }
  }
}

template <int E, bool CONTIG>
__device__ __forceinline__ bool valid_elem(int w, int lane, int j) {
  if constexpr (CONTIG) return true;
  return lane + 32 * j < w;
}

template <typename TI, typename TO, int E, bool CONTIG>
__global__ void __launch_bounds__(kThreads)
forward_kernel(const TI* __restrict__ x, const float* __restrict__ num,
               const float* __restrict__ den, const float* __restrict__ logits,
               const float* __restrict__ centers, const float* __restrict__ beta,
               TO* __restrict__ y, float* __restrict__ rho_out, int64_t rows, int hidden,
               int groups, int nb, float coeff_limit, float eps, int rows_per_chunk) {
  const int g = blockIdx.y;
  const int w = hidden / groups;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  Coeffs c;
  load_coeffs(c, g, num, den, logits, centers, beta, nb, coeff_limit);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_chunk;
  int64_t r1 = r0 + rows_per_chunk;
  if (r1 > rows) r1 = rows;
  const float inv_w = 1.0f / static_cast<float>(w);
  constexpr int U = 4;  // rows in flight per warp (memory-level parallelism)
  for (int64_t rb = r0 + warp; rb < r1; rb += kWarps * U) {
    float v[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r < r1 && span_ok(r, static_cast<int64_t>(g) * w, static_cast<int64_t>(g + 1) * w, rows, hidden, 1))
        load_seg<TI, E, CONTIG>(x + r * hidden + static_cast<int64_t>(g) * w, w, lane, v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r >= r1) break;
      if (!span_ok(r, static_cast<int64_t>(g) * w, static_cast<int64_t>(g + 1) * w, rows, hidden, 1)) continue;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss = fmaf(v[u][j], v[u][j], ss);
      ss = warp_sum(ss);
      const float rho = sqrtf(ss * inv_w + eps);
      const float irho = __fdividef(1.0f, rho);
#pragma unroll
      for (int j = 0; j < E; ++j) v[u][j] = rho * eval_f(c, v[u][j] * irho);
      store_seg<TO, E, CONTIG>(y + r * hidden + static_cast<int64_t>(g) * w, w, lane, v[u]);
      if (rho_out != nullptr && lane == 0) rho_out[r * groups + g] = rho;
    }
  }
}

// Backward.  Writes grad_x and per-CTA coefficient partials
// partial[(chunk * groups + g) * ngrad + k].  RESTRICT adds the affine
// projection removal of the reference's restricted-morphology branch
// (rational_cuda_kernel.cu:663-673): nonlinear_y = rho f - z alpha - rho beta,
// grad_x -= gy alpha + (t / w) beta sum(gy).
template <typename TG, typename TI, typename TO, int E, bool CONTIG, int NGRAD, bool RESTRICT>
__global__ void __launch_bounds__(kThreads, 3)
backward_kernel(const TG* __restrict__ gy_ptr, const TI* __restrict__ x,
                const float* __restrict__ num, const float* __restrict__ den,
                const float* __restrict__ logits, const float* __restrict__ centers,
                const float* __restrict__ beta, const float* __restrict__ affine_alpha,
                const float* __restrict__ affine_beta, float* __restrict__ nonlinear_y,
                TO* __restrict__ gx, float* __restrict__ partial, int64_t rows, int hidden,
                int groups, int nb, float coeff_limit, float eps, int rows_per_chunk) {
  __shared__ float red[kWarps][kMaxGrad];
  const int g = blockIdx.y;
  const int w = hidden / groups;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ngrad = kBase + 2 * nb;
  Coeffs c;
  load_coeffs(c, g, num, den, logits, centers, beta, nb, coeff_limit);
  float alpha_g = 0.f, beta_g = 0.f;
  if constexpr (RESTRICT) {
    alpha_g = affine_alpha[g];
    beta_g = affine_beta[g];
  }
  float acc[NGRAD];
#pragma unroll
  for (int k = 0; k < NGRAD; ++k) acc[k] = 0.f;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_chunk;
  int64_t r1 = r0 + rows_per_chunk;
  if (r1 > rows) r1 = rows;
  const float inv_w = 1.0f / static_cast<float>(w);
  constexpr int U = 2;  // rows in flight per warp
  for (int64_t rb = r0 + warp; rb < r1; rb += kWarps * U) {
    float z[U][E], gy[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r < r1 && span_ok(r, static_cast<int64_t>(g) * w, static_cast<int64_t>(g + 1) * w, rows, hidden, 2)) {
        const int64_t off = r * hidden + static_cast<int64_t>(g) * w;
        load_seg<TI, E, CONTIG>(x + off, w, lane, z[u]);
        load_seg<TG, E, CONTIG>(gy_ptr + off, w, lane, gy[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r >= r1) break;
      if (!span_ok(r, static_cast<int64_t>(g) * w, static_cast<int64_t>(g + 1) * w, rows, hidden, 2)) continue;
      const int64_t off = r * hidden + static_cast<int64_t>(g) * w;
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss = fmaf(z[u][j], z[u][j], ss);
      ss = warp_sum(ss);
      const float rho = sqrtf(ss * inv_w + eps);
      const float irho = __fdividef(1.0f, rho);
      float t[E], df[E];
      float s = 0.f, sg = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        t[j] = z[u][j] * irho;
        float f;
        if constexpr (NGRAD == kBase) {
          // Base coefficients only: accumulate in factored form,
          // d/da_k -> t^k / q, d/d|b_j| -> -p/q^2 * {|t|, t^2, |t|^3, t^4}
          // (the sign of b_j is applied once per CTA at the end).
          const float tv = t[j];
          const float at = fabsf(tv);
          const float t2 = tv * tv;
          const float p = fmaf(fmaf(fmaf(fmaf(fmaf(c.a[5], tv, c.a[4]), tv, c.a[3]), tv, c.a[2]), tv, c.a[1]), tv, c.a[0]);
          const float dp = fmaf(fmaf(fmaf(fmaf(5.0f * c.a[5], tv, 4.0f * c.a[4]), tv, 3.0f * c.a[3]), tv, 2.0f * c.a[2]), tv, c.a[1]);
          const float at3 = at * t2;
          const float t4 = t2 * t2;
          const float q = fmaf(c.b[3], t4, fmaf(c.b[2], at3, fmaf(c.b[1], t2, fmaf(c.b[0], at, 1.0f))));
          const float dq = fmaf(4.0f * c.b[3], t2 * tv, fmaf(3.0f * c.b[2], tv * at, fmaf(2.0f * c.b[1], tv, c.b[0] * sign0(tv))));
          const float iq = __fdividef(1.0f, q);
          f = p * iq;
          df[j] = (dp - f * dq) * iq;
          if (valid_elem<E, CONTIG>(w, lane, j)) {
            const float gr = gy[u][j] * rho;
            float ua = gr * iq;
            acc[0] += ua;
            ua *= tv; acc[1] += ua;
            ua *= tv; acc[2] += ua;
            ua *= tv; acc[3] += ua;
            ua *= tv; acc[4] += ua;
            ua *= tv; acc[5] += ua;
            const float vb = -gr * f * iq;
            acc[6] = fmaf(vb, at, acc[6]);
            acc[7] = fmaf(vb, t2, acc[7]);
            acc[8] = fmaf(vb, at3, acc[8]);
            acc[9] = fmaf(vb, t4, acc[9]);
          }
        } else {
          float part[NGRAD];
          eval_full<NGRAD>(c, t[j], f, df[j], part);
          if (valid_elem<E, CONTIG>(w, lane, j)) {
            const float gr = gy[u][j] * rho;
#pragma unroll
            for (int k = 0; k < NGRAD; ++k) acc[k] = fmaf(gr, part[k], acc[k]);
          }
        }
        if (valid_elem<E, CONTIG>(w, lane, j)) {
          s = fmaf(gy[u][j], f - df[j] * t[j], s);
          sg += gy[u][j];
        } else {
          gy[u][j] = 0.f;
        }
        if constexpr (RESTRICT) z[u][j] = rho * f - z[u][j] * alpha_g - rho * beta_g;
      }
      s = warp_sum(s);
      if constexpr (RESTRICT) sg = warp_sum(sg);
      float out[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        float gr = gy[u][j] * df[j] + t[j] * inv_w * s;
        if constexpr (RESTRICT) {
          gr -= gy[u][j] * alpha_g;
          gr -= t[j] * inv_w * beta_g * sg;
        }
        out[j] = gr;
      }
      store_seg<TO, E, CONTIG>(gx + off, w, lane, out);
      if constexpr (RESTRICT) store_seg<float, E, CONTIG>(nonlinear_y + off, w, lane, z[u]);
    }
  }
  if constexpr (NGRAD == kBase) {
#pragma unroll
    for (int k = 0; k < kDen; ++k) acc[kNum + k] *= c.bs[k];
  }
#pragma unroll
  for (int k = 0; k < NGRAD; ++k) {
    const float v = warp_sum(acc[k]);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < ngrad && RO_CHECK(ngrad <= kMaxGrad && g < groups, 2)) {
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < kWarps; ++wi) v += red[wi][threadIdx.x];
    partial[(static_cast<int64_t>(blockIdx.x) * groups + g) * ngrad + threadIdx.x] = v;
  }
}

// ---------------------------------------------------------------------------
// Packed fast path (no local-basis atoms, no affine restriction, lanes own
// E = w / 32 contiguous elements, E even).  Every elementwise step runs on
// fp32 pairs with FFMA2/FMUL2, which halves the FP32 issue slots of the
// scalar kernels above; the denominator is evaluated by Horner's rule in |t|
// (Q = 1 + |t|(|b0| + |t|(|b1| + |t|(|b2| + |t||b3|)))), the same polynomial.

struct PairCoeffs {
  float2 a[kNum];   // numerator
  float2 b[kDen];   // |denominator|
};

__device__ __forceinline__ void load_pair_coeffs(PairCoeffs& c, int g, const float* __restrict__ num,
                                                 const float* __restrict__ den) {
#pragma unroll
  for (int j = 0; j < kNum; ++j) c.a[j] = splat2(num[g * kNum + j]);
#pragma unroll
  for (int j = 0; j < kDen; ++j) c.b[j] = splat2(fabsf(den[g * kDen + j]));
}

template <typename TI, typename TO, int E>
__global__ void __launch_bounds__(kThreads, 4)
forward_packed_kernel(const TI* __restrict__ x, const float* __restrict__ num,
                      const float* __restrict__ den, TO* __restrict__ y, float* __restrict__ rho_out,
                      int64_t rows, int hidden, int groups, float eps, int rows_per_chunk) {
  constexpr int P = E / 2;
  const int g = blockIdx.y;
  const int w = hidden / groups;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  PairCoeffs c;
  load_pair_coeffs(c, g, num, den);
  const float2 one = splat2(1.0f);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  const float inv_w = 1.0f / static_cast<float>(w);
  constexpr int U = E == 2 ? 4 : 2;  // rows in flight per warp (register budget)
  const int64_t col = static_cast<int64_t>(g) * w + lane * E;
  for (int64_t rb = r0 + warp; rb < r1; rb += kWarps * U) {
    float2 v[U][P];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r < r1 && span_ok(r, col, col + E, rows, hidden, 3)) load_pairs<TI, E>(x + r * hidden + col, v[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r >= r1) break;
      // the whole warp takes the same branch: a failure anywhere skips the row
      if (!__all_sync(0xffffffffu, span_ok(r, col, col + E, rows, hidden, 3))) continue;
      float2 s2 = splat2(0.0f);
#pragma unroll
      for (int i = 0; i < P; ++i) s2 = fma2(v[u][i], v[u][i], s2);
      const float ss = warp_sum(s2.x + s2.y);
      const float rho = sqrtf(ss * inv_w + eps);
      const float2 ir = splat2(__fdividef(1.0f, rho)), rh = splat2(rho);
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const float2 t = mul2(v[u][i], ir);
        const float2 at = abs2(t);
        float2 p = fma2(c.a[5], t, c.a[4]);
        p = fma2(p, t, c.a[3]);
        p = fma2(p, t, c.a[2]);
        p = fma2(p, t, c.a[1]);
        p = fma2(p, t, c.a[0]);
        float2 q = fma2(c.b[3], at, c.b[2]);
        q = fma2(q, at, c.b[1]);
        q = fma2(q, at, c.b[0]);
        q = fma2(q, at, one);
        v[u][i] = mul2(mul2(p, rh), rcp2(q));
      }
      store_pairs<TO, E>(y + r * hidden + col, v[u]);
      if (rho_out != nullptr && lane == 0) rho_out[r * groups + g] = rho;
    }
  }
}

// Backward of the packed path.  Coefficient partials are accumulated in the
// factored form of the scalar kernel: d/da_k -> gy rho t^k / Q and
// d/d|b_j| -> -gy rho f / Q {|t|, t^2, |t|^3, t^4}; the signs of b_j are
// applied once per CTA.
template <typename TG, typename TI, typename TO, int E>
__global__ void __launch_bounds__(kThreads, 3)
backward_packed_kernel(const TG* __restrict__ gy_ptr, const TI* __restrict__ x,
                       const float* __restrict__ num, const float* __restrict__ den,
                       TO* __restrict__ gx, float* __restrict__ partial, int64_t rows, int hidden,
                       int groups, float eps, int rows_per_chunk) {
  constexpr int P = E / 2;
  __shared__ float red[kWarps][kBase];
  const int g = blockIdx.y;
  const int w = hidden / groups;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  PairCoeffs c;
  load_pair_coeffs(c, g, num, den);
  // derivative coefficients: P' = a1 + 2a2 t + 3a3 t^2 + 4a4 t^3 + 5a5 t^4,
  // dQ/dt = sign0(t)|b0| + t (2|b1| + |t| (3|b2| + 4|b3||t|))
  const float2 da5 = mul2(splat2(5.0f), c.a[5]), da4 = mul2(splat2(4.0f), c.a[4]);
  const float2 da3 = mul2(splat2(3.0f), c.a[3]), da2 = mul2(splat2(2.0f), c.a[2]);
  const float2 db3 = mul2(splat2(4.0f), c.b[3]), db2 = mul2(splat2(3.0f), c.b[2]);
  const float2 db1 = mul2(splat2(2.0f), c.b[1]);
  const float2 one = splat2(1.0f);
  float2 acc[kBase];
#pragma unroll
  for (int k = 0; k < kBase; ++k) acc[k] = splat2(0.0f);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  const float inv_w = 1.0f / static_cast<float>(w);
  const int64_t col = static_cast<int64_t>(g) * w + lane * E;
  constexpr int U = E == 8 ? 1 : 2;  // rows in flight per warp (register budget)
  for (int64_t rb = r0 + warp; rb < r1; rb += kWarps * U) {
    float2 z[U][P], gy[U][P];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r < r1 && span_ok(r, col, col + E, rows, hidden, 4)) {
        load_pairs<TI, E>(x + r * hidden + col, z[u]);
        load_pairs<TG, E>(gy_ptr + r * hidden + col, gy[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + static_cast<int64_t>(u) * kWarps;
      if (r >= r1) break;
      if (!__all_sync(0xffffffffu, span_ok(r, col, col + E, rows, hidden, 4))) continue;
      float2 s2 = splat2(0.0f);
#pragma unroll
      for (int i = 0; i < P; ++i) s2 = fma2(z[u][i], z[u][i], s2);
      const float ss = warp_sum(s2.x + s2.y);
      const float rho = sqrtf(ss * inv_w + eps);
      const float2 ir = splat2(__fdividef(1.0f, rho)), rh = splat2(rho);
      float2 sacc = splat2(0.0f);
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const float2 t = mul2(z[u][i], ir);
        const float2 at = abs2(t);
        const float2 t2 = mul2(t, t);
        float2 p = fma2(c.a[5], t, c.a[4]);
        p = fma2(p, t, c.a[3]);
        p = fma2(p, t, c.a[2]);
        p = fma2(p, t, c.a[1]);
        p = fma2(p, t, c.a[0]);
        float2 dp = fma2(da5, t, da4);
        dp = fma2(dp, t, da3);
        dp = fma2(dp, t, da2);
        dp = fma2(dp, t, c.a[1]);
        float2 q = fma2(c.b[3], at, c.b[2]);
        q = fma2(q, at, c.b[1]);
        q = fma2(q, at, c.b[0]);
        q = fma2(q, at, one);
        float2 h = fma2(db3, at, db2);
        h = fma2(h, at, db1);
        const float2 dq = fma2(t, h, mul2(c.b[0], sign02(t)));
        const float2 iq = rcp2(q);
        const float2 f = mul2(p, iq);
        const float2 df = mul2(fma2(neg2(f), dq, dp), iq);
        const float2 g2 = gy[u][i];
        // sum over the group of gy (f - t f')
        sacc = fma2(g2, fma2(neg2(t), df, f), sacc);
        // coefficient partials
        const float2 s1 = mul2(mul2(g2, rh), iq);
        const float2 t3 = mul2(t2, t), t4 = mul2(t2, t2);
        acc[0] = add2(acc[0], s1);
        acc[1] = fma2(s1, t, acc[1]);
        acc[2] = fma2(s1, t2, acc[2]);
        acc[3] = fma2(s1, t3, acc[3]);
        acc[4] = fma2(s1, t4, acc[4]);
        acc[5] = fma2(s1, mul2(t4, t), acc[5]);
        const float2 vb = mul2(s1, f);
        acc[6] = fma2(vb, at, acc[6]);
        acc[7] = fma2(vb, t2, acc[7]);
        acc[8] = fma2(vb, mul2(at, t2), acc[8]);
        acc[9] = fma2(vb, t4, acc[9]);
        // keep t and gy f' for grad_x
        z[u][i] = t;
        gy[u][i] = mul2(g2, df);
      }
      const float2 sw = splat2(warp_sum(sacc.x + sacc.y) * inv_w);
#pragma unroll
      for (int i = 0; i < P; ++i) z[u][i] = fma2(z[u][i], sw, gy[u][i]);
      store_pairs<TO, E>(gx + r * hidden + col, z[u]);
    }
  }
  float sgn[kDen];
#pragma unroll
  for (int k = 0; k < kDen; ++k) sgn[k] = -sign0(den[g * kDen + k]);
#pragma unroll
  for (int k = 0; k < kBase; ++k) {
    float v = acc[k].x + acc[k].y;
    if (k >= kNum) v *= sgn[k - kNum];
    v = warp_sum(v);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < kBase && RO_CHECK(g < groups, 4)) {
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < kWarps; ++wi) v += red[wi][threadIdx.x];
    partial[(static_cast<int64_t>(blockIdx.x) * groups + g) * kBase + threadIdx.x] = v;
  }
}

// Fixed-order reduction of the per-chunk partials into the three gradient
// tensors (fp64 accumulation; output fp32).
__global__ void reduce_coeff_kernel(const float* __restrict__ partial, int chunks, int groups,
                                    int nb, float* __restrict__ gnum, float* __restrict__ gden,
                                    float* __restrict__ gcoeff, int accumulate = 0) {
  const int ngrad = kBase + 2 * nb;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= groups * ngrad || !RO_CHECK(nb >= 0 && nb <= kMaxBasis && chunks >= 0, 5)) return;
  const int g = idx / ngrad;
  const int k = idx % ngrad;
  double s = 0.0;
  for (int ch = 0; ch < chunks; ++ch) s += partial[(static_cast<int64_t>(ch) * groups + g) * ngrad + k];
  const float v = static_cast<float>(s);
  float* out = k < kNum ? gnum + g * kNum + k
                        : (k < kBase ? gden + g * kDen + (k - kNum) : gcoeff + g * nb * 2 + (k - kBase));
  *out = accumulate ? *out + v : v;
}

// The same reduction with one warp per output: lane l adds chunks l, l+32, ...
// in fp64, then a fixed butterfly combines the lanes (deterministic).
__global__ void __launch_bounds__(256)
reduce_coeff_warp_kernel(const float* __restrict__ partial, int chunks, int groups, float* __restrict__ gnum,
                         float* __restrict__ gden, int accumulate) {
  const int idx = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (idx >= groups * kBase) return;
  const int g = idx / kBase, k = idx % kBase;
  double s = 0.0;
  for (int ch = lane; ch < chunks; ch += 32) s += partial[(static_cast<int64_t>(ch) * groups + g) * kBase + k];
  s = warp_sum_d(s);
  if (lane == 0) {
    const float v = static_cast<float>(s);
    float* out = k < kNum ? gnum + g * kNum + k : gden + g * kDen + (k - kNum);
    *out = accumulate ? *out + v : v;
  }
}

// Affine statistics (reference K9, rational_cuda_kernel.cu:491-573): per
// (row, group) rho, and per group [count, sum t, sum t^2, sum h/rho,
// sum t h/rho] accumulated in fp64 with a deterministic two-stage reduction.
template <typename T, int E, bool CONTIG>
__global__ void __launch_bounds__(kThreads)
affine_stats_kernel(const T* __restrict__ x, const T* __restrict__ feature,
                    float* __restrict__ rho_out, double* __restrict__ partial, int64_t rows,
                    int hidden, int groups, float eps, int rows_per_chunk) {
  __shared__ double red[kWarps][4];
  const int g = blockIdx.y;
  const int w = hidden / groups;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_chunk;
  int64_t r1 = r0 + rows_per_chunk;
  if (r1 > rows) r1 = rows;
  const float inv_w = 1.0f / static_cast<float>(w);
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t r = r0 + warp; r < r1; r += kWarps) {
    if (!span_ok(r, static_cast<int64_t>(g) * w, static_cast<int64_t>(g + 1) * w, rows, hidden, 6)) continue;
    const int64_t off = r * hidden + static_cast<int64_t>(g) * w;
    float z[E], h[E];
    load_seg<T, E, CONTIG>(x + off, w, lane, z);
    load_seg<T, E, CONTIG>(feature + off, w, lane, h);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss = fmaf(z[j], z[j], ss);
    ss = warp_sum(ss);
    const float rho = sqrtf(ss * inv_w + eps);
    if (lane == 0) rho_out[r * groups + g] = rho;
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < E; ++j) {
      if (valid_elem<E, CONTIG>(w, lane, j)) {
        const float t = z[j] / rho;
        const float fn = h[j] / rho;
        s[0] += t;
        s[1] += t * t;
        s[2] += fn;
        s[3] += t * fn;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] += static_cast<double>(s[k]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const double v = warp_sum_d(acc[k]);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < 4) {
    double v = 0.0;
    for (int wi = 0; wi < kWarps; ++wi) v += red[wi][threadIdx.x];
    partial[(static_cast<int64_t>(blockIdx.x) * groups + g) * 4 + threadIdx.x] = v;
  }
}

__global__ void affine_reduce_kernel(const double* __restrict__ partial, int chunks, int groups,
                                     int64_t rows, int width, double* __restrict__ stats) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= groups * 5) return;
  const int g = idx / 5;
  const int k = idx % 5;
  if (k == 0) {
    stats[idx] = static_cast<double>(rows) * static_cast<double>(width);
    return;
  }
  double s = 0.0;
  for (int ch = 0; ch < chunks; ++ch) s += partial[(static_cast<int64_t>(ch) * groups + g) * 4 + (k - 1)];
  stats[idx] = s;
}

// ---------------------------------------------------------------------------
// Legacy ungrouped rational (reference K1-K5): no normalisation, one set of
// coefficients.  SIGNED selects q = 1 + x(b0 + x(b1 + x(b2 + x b3))) (the
// original form); otherwise the absolute "Version A" denominator.
template <bool SIGNED>
__device__ __forceinline__ void legacy_eval(const float* a, const float* braw, float x,
                                            float& f, float& df, float (&part)[kBase]) {
  const float ax = fabsf(x);
  const float x2 = x * x, x3 = x2 * x, x4 = x2 * x2;
  const float p = fmaf(fmaf(fmaf(fmaf(fmaf(a[5], x, a[4]), x, a[3]), x, a[2]), x, a[1]), x, a[0]);
  const float dp = fmaf(fmaf(fmaf(fmaf(5.0f * a[5], x, 4.0f * a[4]), x, 3.0f * a[3]), x, 2.0f * a[2]), x, a[1]);
  float q, dq;
  float dqdb[kDen];
  if constexpr (SIGNED) {
    q = fmaf(fmaf(fmaf(fmaf(braw[3], x, braw[2]), x, braw[1]), x, braw[0]), x, 1.0f);
    dq = fmaf(fmaf(fmaf(4.0f * braw[3], x, 3.0f * braw[2]), x, 2.0f * braw[1]), x, braw[0]);
    dqdb[0] = x; dqdb[1] = x2; dqdb[2] = x3; dqdb[3] = x4;
  } else {
    const float b0 = fabsf(braw[0]), b1 = fabsf(braw[1]), b2 = fabsf(braw[2]), b3 = fabsf(braw[3]);
    q = 1.0f + b0 * ax + b1 * x2 + b2 * ax * x2 + b3 * x4;
    dq = b0 * sign0(x) + 2.0f * b1 * x + 3.0f * b2 * x * ax + 4.0f * b3 * x3;
    dqdb[0] = sign0(braw[0]) * ax; dqdb[1] = sign0(braw[1]) * x2;
    dqdb[2] = sign0(braw[2]) * ax * x2; dqdb[3] = sign0(braw[3]) * x4;
  }
  const float iq = 1.0f / q;
  f = p * iq;
  df = (dp * q - p * dq) * iq * iq;
  part[0] = iq; part[1] = x * iq; part[2] = x2 * iq; part[3] = x3 * iq; part[4] = x4 * iq;
  part[5] = x4 * x * iq;
  const float bsc = -p * iq * iq;
#pragma unroll
  for (int j = 0; j < kDen; ++j) part[kNum + j] = bsc * dqdb[j];
}

template <bool SIGNED>
__global__ void legacy_forward_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                      const float* __restrict__ b, float* __restrict__ y,
                                      int64_t n) {
  float ca[kNum], cb[kDen];
#pragma unroll
  for (int j = 0; j < kNum; ++j) ca[j] = a[j];
#pragma unroll
  for (int j = 0; j < kDen; ++j) cb[j] = b[j];
  const int64_t stride = static_cast<int64_t>(blockDim.x) * gridDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float f, df, part[kBase];
    legacy_eval<SIGNED>(ca, cb, x[i], f, df, part);
    y[i] = f;
  }
}

template <bool SIGNED>
__global__ void __launch_bounds__(256)
legacy_backward_kernel(const float* __restrict__ gy, const float* __restrict__ x,
                       const float* __restrict__ a, const float* __restrict__ b,
                       float* __restrict__ gx, float* __restrict__ partial, int64_t n) {
  __shared__ float red[8][kBase];
  if (!RO_CHECK(blockDim.x <= 256, 7)) return;  // red[] holds 8 warps
  float ca[kNum], cb[kDen];
#pragma unroll
  for (int j = 0; j < kNum; ++j) ca[j] = a[j];
#pragma unroll
  for (int j = 0; j < kDen; ++j) cb[j] = b[j];
  float acc[kBase];
#pragma unroll
  for (int k = 0; k < kBase; ++k) acc[k] = 0.f;
  const int64_t stride = static_cast<int64_t>(blockDim.x) * gridDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float f, df, part[kBase];
    legacy_eval<SIGNED>(ca, cb, x[i], f, df, part);
    const float g = gy[i];
    gx[i] = g * df;
#pragma unroll
    for (int k = 0; k < kBase; ++k) acc[k] = fmaf(g, part[k], acc[k]);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kBase; ++k) {
    const float v = warp_sum(acc[k]);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < kBase) {
    float v = 0.f;
    for (int wi = 0; wi < 8; ++wi) v += red[wi][threadIdx.x];
    partial[static_cast<int64_t>(blockIdx.x) * kBase + threadIdx.x] = v;
  }
}

__global__ void legacy_reduce_kernel(const float* __restrict__ partial, int blocks,
                                     float* __restrict__ ga, float* __restrict__ gb) {
  const int k = threadIdx.x;
  if (k >= kBase) return;
  double s = 0.0;
  for (int bi = 0; bi < blocks; ++bi) s += partial[static_cast<int64_t>(bi) * kBase + k];
  if (k < kNum) ga[k] = static_cast<float>(s);
  else gb[k - kNum] = static_cast<float>(s);
}

// ---------------------------------------------------------------------------
// Host launchers.

inline void plan_chunks(int64_t rows, int groups, int& chunks, int& rows_per_chunk) {
  const int target_blocks = 148 * 8;
  int64_t c = (target_blocks + groups - 1) / groups;
  const int64_t max_chunks = (rows + kWarps - 1) / kWarps;
  if (c > max_chunks) c = max_chunks;
  if (c < 1) c = 1;
  rows_per_chunk = static_cast<int>((rows + c - 1) / c);
  chunks = static_cast<int>((rows + rows_per_chunk - 1) / rows_per_chunk);
}

template <typename F>
inline bool dispatch_layout(int w, bool aligned, F&& f) {
  // Contiguous per-lane vectors when w == 32 * E.
  if (aligned) {
    if (w == 256) { f(std::integral_constant<int, 8>{}, std::true_type{}); return true; }
    if (w == 128) { f(std::integral_constant<int, 4>{}, std::true_type{}); return true; }
    if (w == 64) { f(std::integral_constant<int, 2>{}, std::true_type{}); return true; }
    if (w == 32) { f(std::integral_constant<int, 1>{}, std::true_type{}); return true; }
  }
  if (w <= 32) { f(std::integral_constant<int, 1>{}, std::false_type{}); return true; }
  if (w <= 64) { f(std::integral_constant<int, 2>{}, std::false_type{}); return true; }
  if (w <= 128) { f(std::integral_constant<int, 4>{}, std::false_type{}); return true; }
  if (w <= 256) { f(std::integral_constant<int, 8>{}, std::false_type{}); return true; }
  return false;
}

}  // namespace grain

// Public launch API (called from bindings.cpp).  dtype codes: 0 fp32, 1 bf16.
// Returns 0 on success, a negative code on an unsupported configuration.
int grain_forward(const void* x, int x_dtype, const float* num, const float* den,
                  const float* logits, const float* centers, const float* beta, void* y,
                  int y_dtype, float* rho_out, int64_t rows, int hidden, int groups, int nb,
                  float coeff_limit, float eps, cudaStream_t stream) {
  using namespace grain;
  if (groups <= 0 || hidden % groups || nb < 0 || nb > kMaxBasis) return -1;
  const int w = hidden / groups;
  if (w > 256 || rows <= 0) return rows == 0 ? 0 : -1;
  int chunks, rpc;
  plan_chunks(rows, groups, chunks, rpc);
  dim3 grid(chunks, groups);
  const bool aligned = (hidden % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(y) % 16 == 0);
  bool ok = false;
  const bool packed = nb == 0 && aligned && (w == 256 || w == 128 || w == 64);
  auto go = [&](auto ti, auto to) {
    using TI = decltype(ti);
    using TO = decltype(to);
    if (packed) {
      auto launch = [&](auto e) {
        constexpr int E = decltype(e)::value;
        forward_packed_kernel<TI, TO, E><<<grid, kThreads, 0, stream>>>(
            static_cast<const TI*>(x), num, den, static_cast<TO*>(y), rho_out, rows, hidden, groups,
            eps, rpc);
      };
      if (w == 256) launch(std::integral_constant<int, 8>{});
      else if (w == 128) launch(std::integral_constant<int, 4>{});
      else launch(std::integral_constant<int, 2>{});
      ok = true;
      return;
    }
    ok = dispatch_layout(w, aligned, [&](auto e, auto contig) {
      constexpr int E = decltype(e)::value;
      constexpr bool C = decltype(contig)::value;
      forward_kernel<TI, TO, E, C><<<grid, kThreads, 0, stream>>>(
          static_cast<const TI*>(x), num, den, logits, centers, beta, static_cast<TO*>(y), rho_out,
          rows, hidden, groups, nb, coeff_limit, eps, rpc);
    });
  };
  if (x_dtype == 0 && y_dtype == 0) go(float{}, float{});
  else if (x_dtype == 1 && y_dtype == 1) go(__nv_bfloat16{}, __nv_bfloat16{});
  else if (x_dtype == 1 && y_dtype == 0) go(__nv_bfloat16{}, float{});
  else if (x_dtype == 0 && y_dtype == 1) go(float{}, __nv_bfloat16{});
  else return -2;
  return ok ? static_cast<int>(cudaGetLastError()) : -3;
}

int grain_backward_partial_size(int64_t rows, int groups, int nb) {
  int chunks, rpc;
  grain::plan_chunks(rows, groups, chunks, rpc);
  return chunks * groups * (grain::kBase + 2 * nb);
}

// partial must hold grain_backward_partial_size() floats.
int grain_backward(const void* gy, int gy_dtype, const void* x, int x_dtype, const float* num,
                   const float* den, const float* logits, const float* centers,
                   const float* beta, const float* affine_alpha, const float* affine_beta,
                   float* nonlinear_y, void* gx, int gx_dtype, float* gnum, float* gden,
                   float* gcoeff, float* partial, int64_t rows, int hidden, int groups, int nb,
                   float coeff_limit, float eps, cudaStream_t stream) {
  using namespace grain;
  if (groups <= 0 || hidden % groups || nb < 0 || nb > kMaxBasis) return -1;
  const int w = hidden / groups;
  if (w > 256) return -1;
  if (rows <= 0) return 0;
  int chunks, rpc;
  plan_chunks(rows, groups, chunks, rpc);
  dim3 grid(chunks, groups);
  const bool restrict_ = nonlinear_y != nullptr;
  const bool aligned = (hidden % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(gy) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(gx) % 16 == 0) &&
                       (!restrict_ || reinterpret_cast<uintptr_t>(nonlinear_y) % 16 == 0);
  bool ok = false;
  const bool packed = nb == 0 && !restrict_ && aligned && (w == 256 || w == 128 || w == 64);
  auto go = [&](auto tg, auto ti, auto to) {
    using TG = decltype(tg);
    using TI = decltype(ti);
    using TO = decltype(to);
    if (packed) {
      auto launch = [&](auto e) {
        constexpr int E = decltype(e)::value;
        backward_packed_kernel<TG, TI, TO, E><<<grid, kThreads, 0, stream>>>(
            static_cast<const TG*>(gy), static_cast<const TI*>(x), num, den, static_cast<TO*>(gx),
            partial, rows, hidden, groups, eps, rpc);
      };
      if (w == 256) launch(std::integral_constant<int, 8>{});
      else if (w == 128) launch(std::integral_constant<int, 4>{});
      else launch(std::integral_constant<int, 2>{});
      ok = true;
      return;
    }
    ok = dispatch_layout(w, aligned, [&](auto e, auto contig) {
      constexpr int E = decltype(e)::value;
      constexpr bool C = decltype(contig)::value;
      if (nb == 0 && !restrict_) {
        backward_kernel<TG, TI, TO, E, C, kBase, false><<<grid, kThreads, 0, stream>>>(
            static_cast<const TG*>(gy), static_cast<const TI*>(x), num, den, logits, centers, beta,
            affine_alpha, affine_beta, nonlinear_y, static_cast<TO*>(gx), partial, rows, hidden,
            groups, nb, coeff_limit, eps, rpc);
      } else if (!restrict_) {
        backward_kernel<TG, TI, TO, E, C, kMaxGrad, false><<<grid, kThreads, 0, stream>>>(
            static_cast<const TG*>(gy), static_cast<const TI*>(x), num, den, logits, centers, beta,
            affine_alpha, affine_beta, nonlinear_y, static_cast<TO*>(gx), partial, rows, hidden,
            groups, nb, coeff_limit, eps, rpc);
      } else {
        backward_kernel<TG, TI, TO, E, C, kMaxGrad, true><<<grid, kThreads, 0, stream>>>(
            static_cast<const TG*>(gy), static_cast<const TI*>(x), num, den, logits, centers, beta,
            affine_alpha, affine_beta, nonlinear_y, static_cast<TO*>(gx), partial, rows, hidden,
            groups, nb, coeff_limit, eps, rpc);
      }
    });
  };
  if (gy_dtype == 0 && x_dtype == 0 && gx_dtype == 0) go(float{}, float{}, float{});
  else if (gy_dtype == 1 && x_dtype == 1 && gx_dtype == 1) go(__nv_bfloat16{}, __nv_bfloat16{}, __nv_bfloat16{});
  else if (gy_dtype == 0 && x_dtype == 1 && gx_dtype == 1) go(float{}, __nv_bfloat16{}, __nv_bfloat16{});
  else if (gy_dtype == 1 && x_dtype == 0 && gx_dtype == 0) go(__nv_bfloat16{}, float{}, float{});
  else return -2;
  if (!ok) return -3;
  const int ngrad = kBase + 2 * nb;
  const int total = groups * ngrad;
  reduce_coeff_kernel<<<(total + 127) / 128, 128, 0, stream>>>(partial, chunks, groups, nb, gnum,
                                                              gden, gcoeff);
  return static_cast<int>(cudaGetLastError());
}

// Fixed-order reduction of per-chunk coefficient partials [chunks, groups, 10]
// (the layout of the fused GEMM epilogue) into gnum [groups, 6], gden [groups, 4]
// (added to their contents when `accumulate`).
int grain_reduce_coefficients(const float* partial, int chunks, int groups, float* gnum, float* gden,
                              bool accumulate, cudaStream_t stream) {
  using namespace grain;
  reduce_coeff_warp_kernel<<<(groups * kBase + 7) / 8, 256, 0, stream>>>(partial, chunks, groups, gnum, gden,
                                                                         accumulate ? 1 : 0);
  return static_cast<int>(cudaGetLastError());
}

int grain_affine_partial_size(int64_t rows, int groups) {
  int chunks, rpc;
  grain::plan_chunks(rows, groups, chunks, rpc);
  return chunks * groups * 4;
}

int grain_affine_statistics(const void* x, const void* feature, int dtype, float* rho_out,
                            double* stats, double* partial, int64_t rows, int hidden,
                            int groups, float eps, cudaStream_t stream) {
  using namespace grain;
  if (groups <= 0 || hidden % groups) return -1;
  const int w = hidden / groups;
  if (w > 256) return -1;
  int chunks = 1, rpc = 1;
  if (rows > 0) {
    plan_chunks(rows, groups, chunks, rpc);
    dim3 grid(chunks, groups);
    const bool aligned = (hidden % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(feature) % 16 == 0);
    bool ok = false;
    auto go = [&](auto tv) {
      using T = decltype(tv);
      ok = dispatch_layout(w, aligned, [&](auto e, auto contig) {
        constexpr int E = decltype(e)::value;
        constexpr bool C = decltype(contig)::value;
        affine_stats_kernel<T, E, C><<<grid, kThreads, 0, stream>>>(
            static_cast<const T*>(x), static_cast<const T*>(feature), rho_out, partial, rows, hidden,
            groups, eps, rpc);
      });
    };
    if (dtype == 0) go(float{});
    else if (dtype == 1) go(__nv_bfloat16{});
    else return -2;
    if (!ok) return -3;
  } else {
    chunks = 0;
  }
  affine_reduce_kernel<<<(groups * 5 + 127) / 128, 128, 0, stream>>>(partial, chunks, groups, rows,
                                                                    w, stats);
  return static_cast<int>(cudaGetLastError());
}

int legacy_rational_blocks(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 8) b = 148 * 8;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

int legacy_rational_forward(const float* x, const float* a, const float* b, float* y, int64_t n,
                            bool signed_den, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int blocks = legacy_rational_blocks(n);
  if (signed_den) grain::legacy_forward_kernel<true><<<blocks, 256, 0, stream>>>(x, a, b, y, n);
  else grain::legacy_forward_kernel<false><<<blocks, 256, 0, stream>>>(x, a, b, y, n);
  return static_cast<int>(cudaGetLastError());
}

// partial must hold legacy_rational_blocks(n) * 10 floats.
int legacy_rational_backward(const float* gy, const float* x, const float* a, const float* b,
                             float* gx, float* ga, float* gb, float* partial, int64_t n,
                             bool signed_den, cudaStream_t stream) {
  const int blocks = n > 0 ? legacy_rational_blocks(n) : 0;
  if (n > 0) {
    if (signed_den)
      grain::legacy_backward_kernel<true><<<blocks, 256, 0, stream>>>(gy, x, a, b, gx, partial, n);
    else
      grain::legacy_backward_kernel<false><<<blocks, 256, 0, stream>>>(gy, x, a, b, gx, partial, n);
  }
  grain::legacy_reduce_kernel<<<1, 32, 0, stream>>>(partial, blocks, ga, gb);
  return static_cast<int>(cudaGetLastError());
}

RO_BOUNDS_QUERY(grain_bounds_word)

}  // namespace ro

// ---------------------------------------------------------------------------
// Allocation-free backward (declared and documented in grain_noalloc.h; no
// counterpart in the reference).  Same kernels as grain_backward with fp32
// tensors; the per-block coefficient partials live in a fixed device array.

#include "grain_noalloc.h"

namespace ro {
namespace grain {

constexpr int64_t kNoAllocScratchFloats = 65536;  // 256 KiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];

static float* noalloc_scratch_for_current_device(int* status) {
  static std::mutex lock;
  static float* addr[kNoAllocMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    *status = -3;
    return nullptr;
  }
  std::lock_guard<std::mutex> guard(lock);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_partials) != cudaSuccess || p == nullptr) {
      *status = -3;
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  *status = 0;
  return addr[dev];
}

}  // namespace grain
}  // namespace ro

extern "C" int ro_grain_backward_noalloc(const float* gy, const float* x, const float* num,
                                         const float* den, float* gx, float* grad_num,
                                         float* grad_den, int64_t rows, int hidden, int groups,
                                         float eps, cudaStream_t stream) {
  using namespace ro::grain;
  if (num == nullptr || den == nullptr || grad_num == nullptr || grad_den == nullptr) return -1;
  // empty [0, hidden] tensors may come with null data pointers
  if (rows > 0 && (gy == nullptr || x == nullptr || gx == nullptr)) return -1;
  if (groups <= 0 || hidden <= 0 || hidden % groups || rows < 0) return -1;
  const int w = hidden / groups;
  if (w > 256) return -1;
  int chunks = 0, rpc = 0;
  if (rows > 0) plan_chunks(rows, groups, chunks, rpc);
  if (static_cast<int64_t>(chunks) * groups * kBase > kNoAllocScratchFloats) return -2;
  int setup = 0;
  float* partial = noalloc_scratch_for_current_device(&setup);
  if (partial == nullptr) return setup;
  // Every launch goes through cudaLaunchKernelEx, which returns that launch's
  // own status; an error left pending by some earlier, unrelated call is
  // neither reported as this call's failure nor cleared.
  cudaLaunchConfig_t cfg = {};
  cfg.stream = stream;
  cfg.blockDim = dim3(kThreads);
  cfg.gridDim = dim3(chunks, groups);
  cudaError_t err = cudaSuccess;
  if (rows > 0) {
    const bool aligned = (hidden % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(gy) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(gx) % 16 == 0);
    bool ok = false;
    if (aligned && (w == 256 || w == 128 || w == 64)) {
      // same kernel choice as grain_backward, so both entry points agree bitwise
      auto launch = [&](auto e) {
        constexpr int E = decltype(e)::value;
        err = cudaLaunchKernelEx(&cfg, backward_packed_kernel<float, float, float, E>, gy, x, num,
                                 den, gx, partial, rows, hidden, groups, eps, rpc);
      };
      if (w == 256) launch(std::integral_constant<int, 8>{});
      else if (w == 128) launch(std::integral_constant<int, 4>{});
      else launch(std::integral_constant<int, 2>{});
      ok = true;
    } else {
      ok = dispatch_layout(w, aligned, [&](auto e, auto contig) {
        constexpr int E = decltype(e)::value;
        constexpr bool C = decltype(contig)::value;
        const float* none = nullptr;
        float* none_out = nullptr;
        err = cudaLaunchKernelEx(&cfg, backward_kernel<float, float, float, E, C, kBase, false>,
                                 gy, x, num, den, none, none, none, none, none, none_out, gx,
                                 partial, rows, hidden, groups, 0, 0.0f, eps, rpc);
      });
    }
    if (!ok) return -1;
    if (err != cudaSuccess) return static_cast<int>(err);
  }
  // With rows == 0 there are no partials (chunks == 0) and this writes zeros.
  cfg.blockDim = dim3(128);
  cfg.gridDim = dim3((groups * kBase + 127) / 128);
  err = cudaLaunchKernelEx(&cfg, reduce_coeff_kernel, static_cast<const float*>(partial), chunks,
                           groups, 0, grad_num, grad_den, static_cast<float*>(nullptr), 0);
  return static_cast<int>(err);
}
