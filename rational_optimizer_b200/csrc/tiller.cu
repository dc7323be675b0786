// TILLER direction kernels (sm_100a).
//
// The optimizer works on "grouped" blocks: for a role with L layers and G
// groups, block (l, g) is a [R, C] fp32 matrix.  Router incoming rows:
// R = w (group width), C = d, same memory order as the parameter.  Router
// outgoing: the per-layer transpose of out_proj ([d, H] -> [H, d]) split into
// G blocks of w rows.  Attention: one block per layer, the whole matrix.
// The kernels implement, with deterministic two-stage reductions:
//
//   nesterov      buf <- lerp(buf, g, 1-mu);  m = lerp(g, buf, mu)   (in parameter
//                 layout), plus grouped copies of m (fp32 and bf16 for NS5)
//                 and of g (fp32); per-layer transposes fuse into this pass.
//   g2_stats      row sums of g^2 (complete per CTA) -> row second moment,
//                 column partial sums per row-chunk.
//   moments       column second moment update and per-block row totals.
//   dots          a = m / (sqrt(row*col/row_total/corr) + eps) on the fly and
//                 the 7 block sums p.p, a.a, p.a, g.p, g.a, m.p, m.a plus a
//                 non-finite element count (p = polar * scale).
//   coeffs        the adaptive-tangent chord coefficients per block
//                 (optimizer_design/_tiller/core.py:4209-4247) and the
//                 exact/momentum/budget contractions of the selected direction.
//   apply         param <- decay*param + alpha*c[blk]*(pc*p + ac*a), writing
//                 through the inverse layout map; optionally materialises the
//                 scaled direction for the refresh-step probe scores.
#include "common.cuh"

namespace ro {
namespace tiller {

constexpr int kRowsPerChunk = 32;
constexpr int kMaxLayers = 128;

struct LayerPtrs {
  float* p[kMaxLayers];
};
constexpr int kNumDots = 8;
constexpr float kTiny = 1.17549435e-38f;

__device__ __forceinline__ float lerp_torch(float self, float end, float w) {
  return (fabsf(w) < 0.5f) ? fmaf(w, end - self, self) : end - (end - self) * (1.0f - w);
}

// ---------------------------------------------------------------------------
// Nesterov + layout.  transpose == false: grouped index == parameter index.
// transpose == true: per layer, parameter [P, Q] -> grouped [Q, P].
// One CTA handles a 32 x 32 tile of one layer (smem transpose).
__global__ void __launch_bounds__(256)
nesterov_kernel(const __grid_constant__ LayerPtrs grads, const __grid_constant__ LayerPtrs bufs,
                float* __restrict__ m_out, float* __restrict__ g_out, __nv_bfloat16* __restrict__ m16_out,
                int P, int Q, int transpose, float mu) {
  __shared__ float tm[32][33];
  __shared__ float tg[32][33];
  const int l = blockIdx.z;
  const int64_t layer_off = static_cast<int64_t>(l) * P * Q;
  const float* __restrict__ grad = grads.p[l];
  float* __restrict__ buf = bufs.p[l];
  const int tq = blockIdx.x * 32, tp = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows per pass
  for (int r = ty; r < 32; r += 8) {
    const int pi = tp + r, qi = tq + tx;
    if (pi < P && qi < Q) {
      const int64_t li = static_cast<int64_t>(pi) * Q + qi;
      const int64_t idx = layer_off + li;
      const float g = grad[li];
      float b = buf[li];
      b = lerp_torch(b, g, 1.0f - mu);
      buf[li] = b;
      const float m = lerp_torch(g, b, mu);
      if (!transpose) {
        m_out[idx] = m;
        g_out[idx] = g;
        m16_out[idx] = __float2bfloat16_rn(m);
      } else {
        tm[r][tx] = m;
        tg[r][tx] = g;
      }
    }
  }
  if (!transpose) return;
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int qi = tq + r, pi = tp + tx;   // grouped[qi][pi] = param[pi][qi]
    if (pi < P && qi < Q) {
      const int64_t o = layer_off + static_cast<int64_t>(qi) * P + pi;
      const float m = tm[tx][r];
      m_out[o] = m;
      g_out[o] = tg[tx][r];
      m16_out[o] = __float2bfloat16_rn(m);
    }
  }
}

// Per-layer transpose of a bf16 [P, Q] -> [Q, P] (for the attention output NS layout).
__global__ void __launch_bounds__(256)
transpose_bf16_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int P, int Q) {
  __shared__ __nv_bfloat16 t[32][34];
  const int64_t off = static_cast<int64_t>(blockIdx.z) * P * Q;
  const int tq = blockIdx.x * 32, tp = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8)
    if (tp + r < P && tq + tx < Q) t[r][tx] = in[off + static_cast<int64_t>(tp + r) * Q + tq + tx];
  __syncthreads();
  for (int r = ty; r < 32; r += 8)
    if (tq + r < Q && tp + tx < P) out[off + static_cast<int64_t>(tq + r) * P + tp + tx] = t[tx][r];
}

// ---------------------------------------------------------------------------
// g^2 statistics.  Grid (chunks, nblocks); block b covers rows [R] x cols [C].
// Row moments are updated in place (each row owned by one warp); column
// partial sums go to colpart[b][chunk][C].
__global__ void __launch_bounds__(256)
g2_stats_kernel(const float* __restrict__ g, float* __restrict__ row_m, float* __restrict__ colpart,
                int R, int C, float beta2) {
  extern __shared__ float red[];  // [8][C]
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* gb = g + static_cast<int64_t>(b) * R * C;
  const int r0 = chunk * kRowsPerChunk;
  for (int j = threadIdx.x; j < 8 * C; j += blockDim.x) red[j] = 0.f;
  __syncthreads();
  for (int rr = warp; rr < kRowsPerChunk; rr += 8) {
    const int r = r0 + rr;
    if (r >= R) break;
    float s = 0.f;
    for (int j = lane; j < C; j += 32) {
      const float v = gb[static_cast<int64_t>(r) * C + j];
      const float v2 = v * v;
      s += v2;
      red[warp * C + j] += v2;
    }
    s = warp_sum(s);
    if (lane == 0) {
      float* rm = row_m + static_cast<int64_t>(b) * R + r;
      *rm = fmaf(1.0f - beta2, s, *rm * beta2);
    }
  }
  __syncthreads();
  float* cp = colpart + (static_cast<int64_t>(b) * gridDim.x + chunk) * C;
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w * C + j];
    cp[j] = s;
  }
}

// Column moment update + row totals.  Grid (nblocks); fixed reduction order.
__global__ void __launch_bounds__(256)
moments_kernel(const float* __restrict__ colpart, const float* __restrict__ row_m,
               float* __restrict__ col_m, float* __restrict__ row_total, int R, int C, int chunks,
               float beta2) {
  __shared__ float wsum[8];
  const int b = blockIdx.x;
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.f;
    for (int ch = 0; ch < chunks; ++ch) s += colpart[(static_cast<int64_t>(b) * chunks + ch) * C + j];
    float* c = col_m + static_cast<int64_t>(b) * C + j;
    *c = fmaf(1.0f - beta2, s, *c * beta2);
  }
  float t = 0.f;
  for (int i = threadIdx.x; i < R; i += blockDim.x) t += row_m[static_cast<int64_t>(b) * R + i];
  t = warp_sum(t);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += wsum[w];
    row_total[b] = fmaxf(s, kTiny);
  }
}

__device__ __forceinline__ float adaptive_value(float m, float rm, float cm, float inv_total,
                                                float inv_corr, float eps) {
  const float var = rm * cm * inv_total * inv_corr;
  return m / (sqrtf(var) + eps);
}

// 7 block dot products + nonfinite count, partial per chunk.
__global__ void __launch_bounds__(256)
dots_kernel(const __nv_bfloat16* __restrict__ polar, const float* __restrict__ m,
            const float* __restrict__ g, const float* __restrict__ row_m,
            const float* __restrict__ col_m, const float* __restrict__ row_total,
            float* __restrict__ part, int R, int C, float scale, float inv_corr, float eps) {
  __shared__ float red[8][kNumDots];
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t base = static_cast<int64_t>(b) * R * C;
  const float inv_total = 1.0f / row_total[b];
  float acc[kNumDots] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int r0 = chunk * kRowsPerChunk;
  for (int rr = warp; rr < kRowsPerChunk; rr += 8) {
    const int r = r0 + rr;
    if (r >= R) break;
    const float rm = row_m[static_cast<int64_t>(b) * R + r];
    for (int j = lane; j < C; j += 32) {
      const int64_t idx = base + static_cast<int64_t>(r) * C + j;
      const float p = __bfloat162float(polar[idx]) * scale;
      const float mv = m[idx];
      const float gv = g[idx];
      const float a = adaptive_value(mv, rm, col_m[static_cast<int64_t>(b) * C + j], inv_total, inv_corr, eps);
      acc[0] = fmaf(p, p, acc[0]);
      acc[1] = fmaf(a, a, acc[1]);
      acc[2] = fmaf(p, a, acc[2]);
      acc[3] = fmaf(gv, p, acc[3]);
      acc[4] = fmaf(gv, a, acc[4]);
      acc[5] = fmaf(mv, p, acc[5]);
      acc[6] = fmaf(mv, a, acc[6]);
      if (!isfinite(p) || !isfinite(mv) || !isfinite(gv) || !isfinite(a)) acc[7] += 1.0f;
    }
  }
#pragma unroll
  for (int k = 0; k < kNumDots; ++k) {
    const float v = warp_sum(acc[k]);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < kNumDots) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w][threadIdx.x];
    part[(static_cast<int64_t>(b) * gridDim.x + chunk) * kNumDots + threadIdx.x] = s;
  }
}

// One thread per block: reduce partials (fp64) and evaluate the chord.
// out[b] layout (16 floats): pc, ac, exact, momentum, weight, safe, active,
// cosine, budget, departure, parent_descent, candidate_descent, orientation.
__global__ void coeffs_kernel(const float* __restrict__ part, int chunks, int nblocks,
                              const float* __restrict__ participation,
                              const float* __restrict__ congruence, float adj,
                              float* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  double s[kNumDots] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int ch = 0; ch < chunks; ++ch)
    for (int k = 0; k < kNumDots; ++k) s[k] += part[(static_cast<int64_t>(b) * chunks + ch) * kNumDots + k];
  const float p2 = static_cast<float>(s[0]), a2 = static_cast<float>(s[1]);
  const float pa = static_cast<float>(s[2]), gp = static_cast<float>(s[3]);
  const float ga = static_cast<float>(s[4]), mp = static_cast<float>(s[5]);
  const float ma = static_cast<float>(s[6]);
  const bool all_finite = s[7] == 0.0;
  const float projection = pa / fmaxf(p2, kTiny);
  const float tangent2 = fmaxf(a2 - pa * pa / fmaxf(p2, kTiny), 0.0f);
  const float tangent_descent = ga - projection * gp;
  const float orientation = tangent_descent >= 0.0f ? 1.0f : -1.0f;
  const float info = fminf(fmaxf(participation[b], 0.0f), 1.0f);
  const float align = fminf(fmaxf(congruence[b], 0.0f), 1.0f);
  const float departure = fminf(fmaxf(info * fmaxf(1.0f - align * align, 0.0f), 0.0f), 1.0f);
  const float parent_w = sqrtf(fmaxf(1.0f - departure, 0.0f));
  const float tangent_w = sqrtf(fmaxf(departure, 0.0f));
  float ac = tangent_w * sqrtf(p2 / fmaxf(tangent2, kTiny)) * orientation;
  float pc = parent_w - ac * projection;
  const float cand = pc * gp + ac * ga;
  const bool finite = all_finite && isfinite(pc) && isfinite(ac) && isfinite(cand);
  const bool active = finite && p2 > 0.0f && a2 > 0.0f && tangent2 > kTiny;
  const bool safe = active && gp > 0.0f && cand > 0.0f;
  if (!safe) { pc = 1.0f; ac = 0.0f; }
  const float sel2 = fmaxf(pc * pc * p2 + ac * ac * a2 + 2.0f * pc * ac * pa, 0.0f);
  const float sel_norm = sqrtf(sel2);
  const float p_norm = sqrtf(fmaxf(p2, 0.0f));
  float cosine = (pc * p2 + ac * pa) / fmaxf(sel_norm * p_norm, 1e-8f);
  cosine = fminf(fmaxf(cosine, -1.0f), 1.0f);
  const float budget = fabsf(sel_norm - p_norm) / fmaxf(p_norm, 1.0f);
  float* o = out + static_cast<int64_t>(b) * 16;
  o[0] = pc;
  o[1] = ac;
  o[2] = adj * (pc * gp + ac * ga);           // exact  <g, adj*q>
  o[3] = adj * (pc * mp + ac * ma);           // momentum <m, adj*q>
  o[4] = adj * adj * sel2;                    // ||adj*q||^2
  o[5] = safe ? 1.0f : 0.0f;
  o[6] = active ? 1.0f : 0.0f;
  o[7] = cosine;
  o[8] = budget;
  o[9] = departure;
  o[10] = gp;
  o[11] = cand;
  o[12] = orientation;
}

// Apply.  Grouped element (b, r, c) maps to the parameter through
// (transpose ? per-layer [C_total... ] transpose : identity).  For the
// transposed router outgoing role, grouped layer tensor is [H, d] and the
// parameter layer is [d, H]; blocks_per_layer = G, rows per block = w.
// coef[b]: transaction coefficient (1 for attention).  If sel_out != nullptr,
// the scaled direction adj*(pc p + ac a) is stored in grouped layout.
__global__ void __launch_bounds__(256)
apply_kernel(const __grid_constant__ LayerPtrs params, const __nv_bfloat16* __restrict__ polar,
             const float* __restrict__ m, const float* __restrict__ row_m,
             const float* __restrict__ col_m, const float* __restrict__ row_total,
             const float* __restrict__ chord, const float* __restrict__ coef,
             float* __restrict__ sel_out, int R, int C, int blocks_per_layer, int transpose,
             float scale, float inv_corr, float eps, float decay, float alpha, float adj,
             int update_param) {
  __shared__ float tile[32][33];
  // tile over the layer's grouped matrix [blocks_per_layer*R, C]
  const int l = blockIdx.z;
  const int LR = blocks_per_layer * R;
  const int tc = blockIdx.x * 32, tr = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t layer_off = static_cast<int64_t>(l) * LR * C;
  float* __restrict__ param = params.p[l];
  for (int rr = ty; rr < 32; rr += 8) {
    const int gr = tr + rr, gc = tc + tx;
    if (gr < LR && gc < C) {
      const int blk = l * blocks_per_layer + gr / R;
      const int r = gr % R;
      const int64_t idx = layer_off + static_cast<int64_t>(gr) * C + gc;
      const float p = __bfloat162float(polar[idx]) * scale;
      const float a = adaptive_value(m[idx], row_m[static_cast<int64_t>(blk) * R + r],
                                     col_m[static_cast<int64_t>(blk) * C + gc], 1.0f / row_total[blk],
                                     inv_corr, eps);
      const float* ch = chord + static_cast<int64_t>(blk) * 16;
      const float q = ch[0] * p + ch[1] * a;
      if (sel_out) sel_out[idx] = adj * q;
      if (!update_param) continue;
      const float u = alpha * coef[blk] * q;
      if (!transpose) {
        const int64_t li = static_cast<int64_t>(gr) * C + gc;
        param[li] = fmaf(param[li], decay, u);
      } else {
        tile[rr][tx] = u;
      }
    }
  }
  if (!transpose || !update_param) return;
  __syncthreads();
  // param layer is [C, LR]: param[c][gr] += tile(gr, c)
  for (int rr = ty; rr < 32; rr += 8) {
    const int pc_ = tc + rr, pr = tr + tx;
    if (pc_ < C && pr < LR) {
      const int64_t o = static_cast<int64_t>(pc_) * LR + pr;
      param[o] = fmaf(param[o], decay, tile[tx][rr]);
    }
  }
}


// ---------------------------------------------------------------------------
// Vectorised kernels: each thread owns runs of 8 consecutive elements
// (32-byte fp32 / 16-byte bf16 accesses), so a CTA keeps tens of KB of loads
// in flight.  They are selected when every row length is a multiple of 8
// and every base pointer is 16-byte aligned; the scalar kernels above cover
// the remaining shapes with the same arithmetic.
constexpr int kV = 8;

// Nesterov, identity layout.  Grid (ceil(n / (256 * 8 * 2)), L); n = P * Q.
__global__ void __launch_bounds__(256)
nesterov_vec_kernel(const __grid_constant__ LayerPtrs grads, const __grid_constant__ LayerPtrs bufs,
                    float* __restrict__ m_out, float* __restrict__ g_out,
                    __nv_bfloat16* __restrict__ m16_out, int64_t n, float mu) {
  constexpr int kIter = 2;
  const int l = blockIdx.y;
  const float* __restrict__ grad = grads.p[l];
  float* __restrict__ buf = bufs.p[l];
  const int64_t off = static_cast<int64_t>(l) * n;
  const int64_t i0 = (static_cast<int64_t>(blockIdx.x) * (256 * kIter) + threadIdx.x) * kV;
  float g[kIter][kV], b[kIter][kV];
#pragma unroll
  for (int it = 0; it < kIter; ++it) {
    const int64_t i = i0 + static_cast<int64_t>(it) * 256 * kV;
    if (i < n) {
      load_vec<float, kV>(grad + i, g[it]);
      load_vec<float, kV>(buf + i, b[it]);
    }
  }
#pragma unroll
  for (int it = 0; it < kIter; ++it) {
    const int64_t i = i0 + static_cast<int64_t>(it) * 256 * kV;
    if (i >= n) break;
    float m[kV];
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      b[it][k] = lerp_torch(b[it][k], g[it][k], 1.0f - mu);
      m[k] = lerp_torch(g[it][k], b[it][k], mu);
    }
    store_vec<float, kV>(buf + i, b[it]);
    store_vec<float, kV>(m_out + off + i, m);
    store_vec<float, kV>(g_out + off + i, g[it]);
    store_vec<__nv_bfloat16, kV>(m16_out + off + i, m);
  }
}

// Nesterov with the per-layer transpose [P, Q] -> [Q, P], 64 x 64 tiles.
// Grid (ceil(Q / 64), ceil(P / 64), L).
__global__ void __launch_bounds__(256)
nesterov_t_vec_kernel(const __grid_constant__ LayerPtrs grads, const __grid_constant__ LayerPtrs bufs,
                      float* __restrict__ m_out, float* __restrict__ g_out,
                      __nv_bfloat16* __restrict__ m16_out, int P, int Q, float mu) {
  __shared__ float tm[64][65];
  __shared__ float tg[64][65];
  const int l = blockIdx.z;
  const float* __restrict__ grad = grads.p[l];
  float* __restrict__ buf = bufs.p[l];
  const int64_t layer_off = static_cast<int64_t>(l) * P * Q;
  const int tq = blockIdx.x * 64, tp = blockIdx.y * 64;
  const int sub = threadIdx.x >> 3, c8 = (threadIdx.x & 7) * kV;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int r = sub + pass * 32;
    const int pi = tp + r, qi = tq + c8;
    if (pi < P && qi < Q) {
      const int64_t li = static_cast<int64_t>(pi) * Q + qi;
      float g[kV], b[kV];
      load_vec<float, kV>(grad + li, g);
      load_vec<float, kV>(buf + li, b);
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        b[k] = lerp_torch(b[k], g[k], 1.0f - mu);
        tm[r][c8 + k] = lerp_torch(g[k], b[k], mu);
        tg[r][c8 + k] = g[k];
      }
      store_vec<float, kV>(buf + li, b);
    }
  }
  __syncthreads();
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int q = sub + pass * 32;
    const int qi = tq + q, pi = tp + c8;  // grouped[qi][pi .. pi+8) = param[pi .. pi+8)[qi]
    if (qi < Q && pi < P) {
      float m[kV], g[kV];
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        m[k] = tm[c8 + k][q];
        g[k] = tg[c8 + k][q];
      }
      const int64_t o = layer_off + static_cast<int64_t>(qi) * P + pi;
      store_vec<float, kV>(m_out + o, m);
      store_vec<float, kV>(g_out + o, g);
      store_vec<__nv_bfloat16, kV>(m16_out + o, m);
    }
  }
}

// g^2 statistics (vectorised).  Same grid and outputs as g2_stats_kernel.
// Lane `lane` of every warp owns columns lane*8 + 256*v (v < NV, C = 256*NV),
// so the column sums of the warp's rows stay in registers.
template <int NV>
__global__ void __launch_bounds__(256)
g2_stats_vec_kernel(const float* __restrict__ g, float* __restrict__ row_m, float* __restrict__ colpart,
                    int R, float beta2) {
  constexpr int C = 256 * NV;
  __shared__ __align__(16) float red[8][C];
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* gb = g + static_cast<int64_t>(b) * R * C;
  const int r0 = chunk * kRowsPerChunk;
  float col[NV][kV];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int k = 0; k < kV; ++k) col[v][k] = 0.f;
  for (int rr = warp; rr < kRowsPerChunk; rr += 8) {
    const int r = r0 + rr;
    if (r >= R) break;
    const float* row = gb + static_cast<int64_t>(r) * C + lane * kV;
    float x[NV][kV];
#pragma unroll
    for (int v = 0; v < NV; ++v) load_vec<float, kV>(row + v * 256, x[v]);
    float s = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const float v2 = x[v][k] * x[v][k];
        s += v2;
        col[v][k] += v2;
      }
    s = warp_sum(s);
    if (lane == 0) {
      float* rm = row_m + static_cast<int64_t>(b) * R + r;
      *rm = fmaf(1.0f - beta2, s, *rm * beta2);
    }
  }
#pragma unroll
  for (int v = 0; v < NV; ++v) store_vec<float, kV>(&red[warp][v * 256 + lane * kV], col[v]);
  __syncthreads();
  float* cp = colpart + (static_cast<int64_t>(b) * gridDim.x + chunk) * C;
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][j];
    cp[j] = s;
  }
}

// Block dot products (vectorised).  Same grid and outputs as dots_kernel.
__global__ void __launch_bounds__(256)
dots_vec_kernel(const __nv_bfloat16* __restrict__ polar, const float* __restrict__ m,
                const float* __restrict__ g, const float* __restrict__ row_m,
                const float* __restrict__ col_m, const float* __restrict__ row_total,
                float* __restrict__ part, int R, int C, float scale, float inv_corr, float eps) {
  __shared__ float red[8][kNumDots];
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t base = static_cast<int64_t>(b) * R * C;
  const float* __restrict__ cm = col_m + static_cast<int64_t>(b) * C;
  const float inv_total = 1.0f / row_total[b];
  float acc[kNumDots] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int r0 = chunk * kRowsPerChunk;
  for (int rr = warp; rr < kRowsPerChunk; rr += 8) {
    const int r = r0 + rr;
    if (r >= R) break;
    const float rm = row_m[static_cast<int64_t>(b) * R + r];
    const int64_t rb = base + static_cast<int64_t>(r) * C;
    for (int j = lane * kV; j < C; j += 32 * kV) {
      float pv[kV], mv[kV], gv[kV], cv[kV];
      load_vec<__nv_bfloat16, kV>(polar + rb + j, pv);
      load_vec<float, kV>(m + rb + j, mv);
      load_vec<float, kV>(g + rb + j, gv);
      load_vec<float, kV>(cm + j, cv);
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const float p = pv[k] * scale;
        const float a = adaptive_value(mv[k], rm, cv[k], inv_total, inv_corr, eps);
        acc[0] = fmaf(p, p, acc[0]);
        acc[1] = fmaf(a, a, acc[1]);
        acc[2] = fmaf(p, a, acc[2]);
        acc[3] = fmaf(gv[k], p, acc[3]);
        acc[4] = fmaf(gv[k], a, acc[4]);
        acc[5] = fmaf(mv[k], p, acc[5]);
        acc[6] = fmaf(mv[k], a, acc[6]);
        if (!isfinite(p) || !isfinite(mv[k]) || !isfinite(gv[k]) || !isfinite(a)) acc[7] += 1.0f;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kNumDots; ++k) {
    const float v = warp_sum(acc[k]);
    if (lane == 0) red[warp][k] = v;
  }
  __syncthreads();
  if (threadIdx.x < kNumDots) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w][threadIdx.x];
    part[(static_cast<int64_t>(b) * gridDim.x + chunk) * kNumDots + threadIdx.x] = s;
  }
}

// Apply, identity layout (vectorised).  Grid (ceil(LR / 32), L): each CTA
// covers 32 grouped rows of one layer.
__global__ void __launch_bounds__(256)
apply_vec_kernel(const __grid_constant__ LayerPtrs params, const __nv_bfloat16* __restrict__ polar,
                 const float* __restrict__ m, const float* __restrict__ row_m,
                 const float* __restrict__ col_m, const float* __restrict__ row_total,
                 const float* __restrict__ chord, const float* __restrict__ coef,
                 float* __restrict__ sel_out, int R, int C, int blocks_per_layer, float scale,
                 float inv_corr, float eps, float decay, float alpha, float adj, int update_param) {
  const int l = blockIdx.y;
  const int LR = blocks_per_layer * R;
  const int vecs = C / kV;
  const int64_t layer_off = static_cast<int64_t>(l) * LR * C;
  float* __restrict__ param = params.p[l];
  const int row0 = blockIdx.x * 32;
  for (int v = threadIdx.x; v < 32 * vecs; v += 256) {
    const int gr = row0 + v / vecs;
    if (gr >= LR) break;
    const int gc = (v % vecs) * kV;
    const int blk = l * blocks_per_layer + gr / R;
    const int r = gr - (gr / R) * R;
    const int64_t li = static_cast<int64_t>(gr) * C + gc;
    const int64_t idx = layer_off + li;
    float pv[kV], mv[kV], cv[kV];
    load_vec<__nv_bfloat16, kV>(polar + idx, pv);
    load_vec<float, kV>(m + idx, mv);
    load_vec<float, kV>(col_m + static_cast<int64_t>(blk) * C + gc, cv);
    const float rm = row_m[static_cast<int64_t>(blk) * R + r];
    const float inv_total = 1.0f / row_total[blk];
    const float* ch = chord + static_cast<int64_t>(blk) * 16;
    const float c0 = ch[0], c1 = ch[1];
    float q[kV];
#pragma unroll
    for (int k = 0; k < kV; ++k) {
      const float a = adaptive_value(mv[k], rm, cv[k], inv_total, inv_corr, eps);
      q[k] = c0 * (pv[k] * scale) + c1 * a;
    }
    if (sel_out) {
      float s[kV];
#pragma unroll
      for (int k = 0; k < kV; ++k) s[k] = adj * q[k];
      store_vec<float, kV>(sel_out + idx, s);
    }
    if (!update_param) continue;
    const float cf = alpha * coef[blk];
    float w[kV];
    load_vec<float, kV>(param + li, w);
#pragma unroll
    for (int k = 0; k < kV; ++k) w[k] = fmaf(w[k], decay, cf * q[k]);
    store_vec<float, kV>(param + li, w);
  }
}

// Apply through the per-layer transpose (grouped [LR, C] -> parameter
// [C, LR]), 64 x 64 tiles.  Grid (ceil(C / 64), ceil(LR / 64), L).
__global__ void __launch_bounds__(256)
apply_t_vec_kernel(const __grid_constant__ LayerPtrs params, const __nv_bfloat16* __restrict__ polar,
                   const float* __restrict__ m, const float* __restrict__ row_m,
                   const float* __restrict__ col_m, const float* __restrict__ row_total,
                   const float* __restrict__ chord, const float* __restrict__ coef,
                   float* __restrict__ sel_out, int R, int C, int blocks_per_layer, float scale,
                   float inv_corr, float eps, float decay, float alpha, float adj, int update_param) {
  __shared__ float tile[64][65];
  const int l = blockIdx.z;
  const int LR = blocks_per_layer * R;
  const int tc = blockIdx.x * 64, tr = blockIdx.y * 64;
  const int sub = threadIdx.x >> 3, c8 = (threadIdx.x & 7) * kV;
  const int64_t layer_off = static_cast<int64_t>(l) * LR * C;
  float* __restrict__ param = params.p[l];
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int rr = sub + pass * 32;
    const int gr = tr + rr, gc = tc + c8;
    if (gr < LR && gc < C) {
      const int blk = l * blocks_per_layer + gr / R;
      const int r = gr - (gr / R) * R;
      const int64_t idx = layer_off + static_cast<int64_t>(gr) * C + gc;
      float pv[kV], mv[kV], cv[kV];
      load_vec<__nv_bfloat16, kV>(polar + idx, pv);
      load_vec<float, kV>(m + idx, mv);
      load_vec<float, kV>(col_m + static_cast<int64_t>(blk) * C + gc, cv);
      const float rm = row_m[static_cast<int64_t>(blk) * R + r];
      const float inv_total = 1.0f / row_total[blk];
      const float* ch = chord + static_cast<int64_t>(blk) * 16;
      const float c0 = ch[0], c1 = ch[1];
      const float cf = alpha * coef[blk];
      float q[kV];
#pragma unroll
      for (int k = 0; k < kV; ++k) {
        const float a = adaptive_value(mv[k], rm, cv[k], inv_total, inv_corr, eps);
        q[k] = c0 * (pv[k] * scale) + c1 * a;
        tile[rr][c8 + k] = cf * q[k];
      }
      if (sel_out) {
        float s[kV];
#pragma unroll
        for (int k = 0; k < kV; ++k) s[k] = adj * q[k];
        store_vec<float, kV>(sel_out + idx, s);
      }
    }
  }
  if (!update_param) return;
  __syncthreads();
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
    const int cc = sub + pass * 32;
    const int pc = tc + cc, pr = tr + c8;  // param[pc][pr .. pr+8) += tile[pr-tr+k][cc]
    if (pc < C && pr < LR) {
      const int64_t o = static_cast<int64_t>(pc) * LR + pr;
      float w[kV];
      load_vec<float, kV>(param + o, w);
#pragma unroll
      for (int k = 0; k < kV; ++k) w[k] = fmaf(w[k], decay, tile[c8 + k][cc]);
      store_vec<float, kV>(param + o, w);
    }
  }
}

// Newton-Schulz input normalisation: y = bf16(x / bf16(||x||_F)) per matrix,
// the norm taken in fp32 over the bf16 values and clamped at 1e-7
// (torch.optim.Muon / the reference's batched path).  Two passes over many
// CTAs: per-chunk sums of squares, then each chunk re-reads the partials of
// its matrix in a fixed order (deterministic) and scales.
constexpr int64_t kNsChunk = 16384;

template <bool VEC>
__global__ void __launch_bounds__(256)
ns_sumsq_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ part, int64_t n) {
  __shared__ float red[8];
  const int64_t start = static_cast<int64_t>(blockIdx.x) * kNsChunk;
  const int64_t end = start + kNsChunk < n ? start + kNsChunk : n;
  const __nv_bfloat16* xb = x + static_cast<int64_t>(blockIdx.y) * n;
  float s = 0.f;
  if constexpr (VEC) {
    for (int64_t i = start + threadIdx.x * kV; i < end; i += 256 * kV) {
      float v[kV];
      load_vec<__nv_bfloat16, kV>(xb + i, v);
#pragma unroll
      for (int k = 0; k < kV; ++k) s = fmaf(v[k], v[k], s);
    }
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += 256) {
      const float v = __bfloat162float(xb[i]);
      s = fmaf(v, v, s);
    }
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    part[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = t;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256)
ns_scale_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                const float* __restrict__ part, int64_t n, float clamp_min) {
  __shared__ float s_norm;
  if (threadIdx.x < 32) {
    const float* pb = part + static_cast<int64_t>(blockIdx.y) * gridDim.x;
    float t = 0.f;
    for (int c = threadIdx.x; c < static_cast<int>(gridDim.x); c += 32) t += pb[c];
    t = warp_sum(t);
    if (threadIdx.x == 0) s_norm = __bfloat162float(__float2bfloat16_rn(fmaxf(sqrtf(t), clamp_min)));
  }
  __syncthreads();
  const float nrm = s_norm;
  const int64_t start = static_cast<int64_t>(blockIdx.x) * kNsChunk;
  const int64_t end = start + kNsChunk < n ? start + kNsChunk : n;
  const int64_t off = static_cast<int64_t>(blockIdx.y) * n;
  if constexpr (VEC) {
    for (int64_t i = start + threadIdx.x * kV; i < end; i += 256 * kV) {
      float v[kV];
      load_vec<__nv_bfloat16, kV>(x + off + i, v);
#pragma unroll
      for (int k = 0; k < kV; ++k) v[k] = v[k] / nrm;
      store_vec<__nv_bfloat16, kV>(y + off + i, v);
    }
  } else {
    for (int64_t i = start + threadIdx.x; i < end; i += 256)
      y[off + i] = __float2bfloat16_rn(__bfloat162float(x[off + i]) / nrm);
  }
}

}  // namespace tiller

int64_t ns_normalize_chunks(int64_t n) { return (n + tiller::kNsChunk - 1) / tiller::kNsChunk; }

// part: scratch of batch * ns_normalize_chunks(n) floats.
int ns_normalize(const __nv_bfloat16* x, __nv_bfloat16* y, float* part, int batch, int64_t n,
                 cudaStream_t stream) {
  const int64_t chunks = ns_normalize_chunks(n);
  if (chunks <= 0 || batch <= 0) return 0;
  const dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(batch));
  const bool vec = (n % tiller::kV) == 0 && aligned16(x) && aligned16(y);
  if (vec) {
    tiller::ns_sumsq_kernel<true><<<grid, 256, 0, stream>>>(x, part, n);
    tiller::ns_scale_kernel<true><<<grid, 256, 0, stream>>>(x, y, part, n, 1e-7f);
  } else {
    tiller::ns_sumsq_kernel<false><<<grid, 256, 0, stream>>>(x, part, n);
    tiller::ns_scale_kernel<false><<<grid, 256, 0, stream>>>(x, y, part, n, 1e-7f);
  }
  return static_cast<int>(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Host launchers.

int tiller_nesterov(float* const* grads, float* const* bufs, float* m_out, float* g_out,
                    __nv_bfloat16* m16_out, int L, int P, int Q, bool transpose, float mu,
                    cudaStream_t stream) {
  if (L > tiller::kMaxLayers) return -1;
  tiller::LayerPtrs gp, bp;
  for (int l = 0; l < L; ++l) { gp.p[l] = grads[l]; bp.p[l] = bufs[l]; }
  bool vec = P % tiller::kV == 0 && Q % tiller::kV == 0 && aligned16(m_out) && aligned16(g_out) &&
             aligned16(m16_out);
  for (int l = 0; l < L && vec; ++l) vec = aligned16(grads[l]) && aligned16(bufs[l]);
  if (vec && !transpose) {
    const int64_t n = static_cast<int64_t>(P) * Q;
    dim3 grid(static_cast<unsigned>((n + 256 * 2 * tiller::kV - 1) / (256 * 2 * tiller::kV)), L);
    tiller::nesterov_vec_kernel<<<grid, 256, 0, stream>>>(gp, bp, m_out, g_out, m16_out, n, mu);
  } else if (vec) {
    dim3 grid((Q + 63) / 64, (P + 63) / 64, L);
    tiller::nesterov_t_vec_kernel<<<grid, 256, 0, stream>>>(gp, bp, m_out, g_out, m16_out, P, Q, mu);
  } else {
    dim3 grid((Q + 31) / 32, (P + 31) / 32, L);
    tiller::nesterov_kernel<<<grid, 256, 0, stream>>>(gp, bp, m_out, g_out, m16_out, P, Q,
                                                      transpose ? 1 : 0, mu);
  }
  return static_cast<int>(cudaGetLastError());
}

int tiller_transpose_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, int L, int P, int Q,
                          cudaStream_t stream) {
  dim3 grid((Q + 31) / 32, (P + 31) / 32, L);
  tiller::transpose_bf16_kernel<<<grid, 256, 0, stream>>>(in, out, P, Q);
  return static_cast<int>(cudaGetLastError());
}

int tiller_chunks(int R) { return (R + tiller::kRowsPerChunk - 1) / tiller::kRowsPerChunk; }

// scratch: colpart [nblocks*chunks*C], dotpart [nblocks*chunks*8], row_total [nblocks]
int tiller_chord(const __nv_bfloat16* polar, const float* m, const float* g, float* row_m, float* col_m,
                 float* colpart, float* dotpart, float* row_total, const float* participation,
                 const float* congruence, float* chord_out, int nblocks, int R, int C, float scale,
                 int step, float adj, cudaStream_t stream) {
  const int chunks = tiller_chunks(R);
  const size_t smem = static_cast<size_t>(8) * C * sizeof(float);
  if (smem > 200 * 1024) return -1;
  const bool vec = C % tiller::kV == 0 && aligned16(polar) && aligned16(m) && aligned16(g) &&
                   aligned16(col_m);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(tiller::g2_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  const float beta2 = 0.95f;
  const dim3 sgrid(chunks, nblocks);
  const bool gvec = vec && C % 256 == 0 && C <= 1024;
  if (gvec && C == 256)
    tiller::g2_stats_vec_kernel<1><<<sgrid, 256, 0, stream>>>(g, row_m, colpart, R, beta2);
  else if (gvec && C == 512)
    tiller::g2_stats_vec_kernel<2><<<sgrid, 256, 0, stream>>>(g, row_m, colpart, R, beta2);
  else if (gvec && C == 768)
    tiller::g2_stats_vec_kernel<3><<<sgrid, 256, 0, stream>>>(g, row_m, colpart, R, beta2);
  else if (gvec)
    tiller::g2_stats_vec_kernel<4><<<sgrid, 256, 0, stream>>>(g, row_m, colpart, R, beta2);
  else
    tiller::g2_stats_kernel<<<sgrid, 256, smem, stream>>>(g, row_m, colpart, R, C, beta2);
  tiller::moments_kernel<<<nblocks, 256, 0, stream>>>(colpart, row_m, col_m, row_total, R, C, chunks,
                                                      beta2);
  const double corr = 1.0 - pow(0.95, static_cast<double>(step));
  const float inv_corr = static_cast<float>(1.0 / corr);
  if (vec)
    tiller::dots_vec_kernel<<<dim3(chunks, nblocks), 256, 0, stream>>>(polar, m, g, row_m, col_m, row_total,
                                                                       dotpart, R, C, scale, inv_corr, 1e-8f);
  else
    tiller::dots_kernel<<<dim3(chunks, nblocks), 256, 0, stream>>>(polar, m, g, row_m, col_m, row_total,
                                                                   dotpart, R, C, scale, inv_corr, 1e-8f);
  tiller::coeffs_kernel<<<(nblocks + 127) / 128, 128, 0, stream>>>(dotpart, chunks, nblocks,
                                                                   participation, congruence, adj,
                                                                   chord_out);
  return static_cast<int>(cudaGetLastError());
}

int tiller_apply(float* const* params, const __nv_bfloat16* polar, const float* m, const float* row_m,
                 const float* col_m, const float* row_total, const float* chord, const float* coef,
                 float* sel_out, int L, int blocks_per_layer, int R, int C, bool transpose, float scale,
                 int step, float decay, float alpha, float adj, bool update_param, cudaStream_t stream) {
  const double corr = 1.0 - pow(0.95, static_cast<double>(step));
  const float inv_corr = static_cast<float>(1.0 / corr);
  const int LR = blocks_per_layer * R;
  if (L > tiller::kMaxLayers) return -1;
  tiller::LayerPtrs pp;
  for (int l = 0; l < L; ++l) pp.p[l] = params[l];
  bool vec = C % tiller::kV == 0 && aligned16(polar) && aligned16(m) && aligned16(col_m) &&
             (sel_out == nullptr || aligned16(sel_out)) && (!transpose || LR % tiller::kV == 0);
  for (int l = 0; l < L && vec; ++l) vec = aligned16(params[l]);
  if (vec && !transpose) {
    dim3 grid((LR + 31) / 32, L);
    tiller::apply_vec_kernel<<<grid, 256, 0, stream>>>(pp, polar, m, row_m, col_m, row_total, chord, coef,
                                                       sel_out, R, C, blocks_per_layer, scale, inv_corr,
                                                       1e-8f, decay, alpha, adj, update_param ? 1 : 0);
  } else if (vec) {
    dim3 grid((C + 63) / 64, (LR + 63) / 64, L);
    tiller::apply_t_vec_kernel<<<grid, 256, 0, stream>>>(pp, polar, m, row_m, col_m, row_total, chord, coef,
                                                         sel_out, R, C, blocks_per_layer, scale, inv_corr,
                                                         1e-8f, decay, alpha, adj, update_param ? 1 : 0);
  } else {
    dim3 grid((C + 31) / 32, (LR + 31) / 32, L);
    tiller::apply_kernel<<<grid, 256, 0, stream>>>(pp, polar, m, row_m, col_m, row_total, chord, coef,
                                                   sel_out, R, C, blocks_per_layer, transpose ? 1 : 0,
                                                   scale, inv_corr, 1e-8f, decay, alpha, adj,
                                                   update_param ? 1 : 0);
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro
