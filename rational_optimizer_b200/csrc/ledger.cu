// TILLER loss ledger + equal-budget transaction in ONE single-CTA fp64 kernel.
//
// Replaces hundreds of tiny launches (and two cuSOLVER eigensolves with host
// synchronisation) per optimizer step.  Semantics follow
// optimizer_design/_tiller/core.py:
//   trace-matched surrogate rows ..... core.py:1142-1159  (ordinary steps)
//   functional row norm .............. core.py:1161-1169  (refresh steps)
//   Robust-FD ledger advance ......... core.py:1178-1233
//   diagonal-completed transaction ... core.py:69-232 (Lanczos-32 with full
//                                       re-orthogonalisation, 32x32 eigen-
//                                       solve, 64-round secular bisection,
//                                       acceptance tests)
// Symmetric eigenproblems (the <=96x96 row Gram of the ledger and the 32x32
// Lanczos tridiagonal) use a parallel cyclic Jacobi method (round-robin
// pairing, n/2 independent rotations per round) in shared memory, followed by
// an ascending sort, so eigenvalue order matches torch.linalg.eigh.  Row signs
// and the order of equal eigenvalues may differ from LAPACK; every quantity
// the algorithm consumes is invariant to them (it depends on S^T S).
//
// Launch: one CTA of kThreads threads, dynamic smem = 2*96*97 doubles (+4 KB static).
#include "common.cuh"

namespace ro {
namespace ledger {

constexpr int kThreads = 1024;
constexpr int kCurRows = 32;
constexpr int kPersRows = 64;
constexpr int kMaxSel = 96;
constexpr int kKrylov = 32;
constexpr double kTiny = 2.2250738585072014e-308;
constexpr double kEps = 2.220446049250313e-16;
constexpr float kTinyF = 1.17549435e-38f;

struct Args {
  // inputs
  const float* cur_scores;     // [32, C] functional rows, or nullptr (surrogate)
  const float* cur_decay;      // [32]
  const float* exact;          // [2, C]
  const float* momentum;       // [2, C]
  const float* weights;        // [C]
  const int64_t* layer_ids;    // [C]
  const float* decay_derivative;  // [1] surrogate mode
  // persistent ledger state (fp32, read and written)
  float* pers_scores;          // [64, C] (first prev_rows rows valid)
  float* pers_total_diag;      // [C]
  float* pers_decay_cross;     // [C]
  float* pers_tail;            // [1]
  float* discarded_fraction;   // [1]
  float* shrinkage;            // [1]
  float* ref_row_norm;         // [1]
  // outputs
  float* coefficients;         // [C]
  float* candidate;            // [C]
  float* result;               // [16]
  double* ws;                  // workspace (see ws_doubles)
  unsigned long long* timing;  // optional [16]: %globaltimer at phase ends, sweep counts
  int C, prev_rows, total_layers, functional;
  double eta;
};

__device__ __forceinline__ unsigned long long ledger_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Phase timestamps for the optional timing buffer (diagnostics only).
#define STAMP(k)                                                           \
  do {                                                                     \
    if (a.timing != nullptr && threadIdx.x == 0) a.timing[k] = ledger_clock(); \
  } while (0)

__device__ double block_max(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (warp == 0) {
    t = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmax(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ double block_sum(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (warp == 0) {
    t = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
    t = warp_sum_d(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Parallel cyclic Jacobi on symmetric A (n x n, row-major in smem with leading
// dimension n + 1, so a column walk visits a different bank on every row).  On exit
// A holds eigenvalues on the diagonal, V the eigenvectors (columns); returns
// the number of sweeps that rotated anything.  `rp`/`rq` need n/2+1 ints,
// `rc`/`rs` n/2+1 doubles; `rotated` is a shared flag.
__device__ int jacobi_eigh(double* A, double* V, int n, int* rp, int* rq, double* rc, double* rs,
                           double* red, int* rotated) {
  const int tid = threadIdx.x;
  const int ld = n + 1;
  for (int i = tid; i < n * n; i += blockDim.x) {
    const int r = i / n, c = i - r * n;
    V[r * ld + c] = (r == c) ? 1.0 : 0.0;
  }
  const int m = (n + 1) & ~1;  // even number of players (a dummy if n is odd)
  const int half = m / 2;
  const int nblk = half * half;
  // first item of this thread and the per-item step, as (pair k, pair l) of
  // the A blocks and (pair k, row i) of the V updates
  const int a_k0 = tid / half, a_l0 = tid - a_k0 * half;
  const int a_dk = static_cast<int>(blockDim.x) / half, a_dl = static_cast<int>(blockDim.x) - a_dk * half;
  const int v_k0 = tid / n, v_i0 = tid - v_k0 * n;
  const int v_dk = static_cast<int>(blockDim.x) / n, v_di = static_cast<int>(blockDim.x) - v_dk * n;
  __syncthreads();
  double total = 0.0;
  for (int i = tid; i < n * n; i += blockDim.x) {
    const int r = i / n, c = i - r * n;
    total += A[r * ld + c] * A[r * ld + c];
  }
  const double scale = sqrt(block_sum(total, red));
  // An off-diagonal entry is dropped once it is below 1e-13 of the matrix norm
  // (absolute floor) or at rounding level of its own diagonal pair (relative
  // test).  Dropping changes no eigenvalue by more than n * 1e-13 * ||A||_F,
  // far below the fp32 precision of every output, and it lets sweeps stop:
  // rotations among rounding-level entries of a degenerate (e.g. rank-one
  // surrogate) block only reshuffle noise and never reach zero.
  const double floor_abs = 1e-13 * scale;
  int sweep = 0;
  for (; sweep < 30; ++sweep) {
    if (tid == 0) *rotated = 0;
    __syncthreads();
    for (int round = 0; round < m - 1; ++round) {
      // Round-robin schedule in closed form: player m-1 meets `round`; the
      // others pair as (round+k, round-k) modulo m-1.
      for (int k = tid; k < half; k += blockDim.x) {
        int p, q;
        if (k == 0) {
          p = round;
          q = m - 1;
        } else {
          p = round + k;
          if (p >= m - 1) p -= m - 1;
          q = round - k;
          if (q < 0) q += m - 1;
        }
        if (p > q) { const int t = p; p = q; q = t; }
        double c = 1.0, s = 0.0;
        if (q < n) {
          const double apq = A[p * ld + q];
          const double app = A[p * ld + p], aqq = A[q * ld + q];
          const double aabs = fabs(apq);
          if (aabs > floor_abs && aabs > 0.5 * kEps * fmax(fabs(app), fabs(aqq))) {
            // t = tan of the rotation angle, the smaller root of
            // t^2 + 2 theta t - 1 = 0 with theta = (aqq - app) / (2 apq)
            const double diff = aqq - app;
            const double r = sqrt(fma(diff, diff, 4.0 * apq * apq));
            const double t = 2.0 * apq / (diff + copysign(r, diff));
            c = rsqrt(fma(t, t, 1.0));
            s = t * c;
            *rotated = 1;
          } else if (apq != 0.0) {
            // negligible: drop it so the sweep count reflects real work
            A[p * ld + q] = 0.0;
            A[q * ld + p] = 0.0;
          }
        }
        rp[k] = p;
        rq[k] = q;
        rc[k] = c;
        rs[k] = s;
      }
      __syncthreads();
      // A <- R^T A R and V <- V R.  R is block diagonal over the round's
      // disjoint pairs, so each 2 x 2 block (pair k rows, pair l columns) of A
      // and each (row, pair) of V is updated independently.  A thread's items
      // are tid, tid + blockDim.x, ...; their (k, l) and (pair, row) indices
      // advance by fixed steps instead of being divided out per item.
      {
        int k = a_k0, l = a_l0;
        for (int idx = tid; idx < nblk; idx += blockDim.x) {
          const int p = rp[k], q = rq[k], u = rp[l], w = rq[l];
          const double c = rc[k], sk = rs[k], c2 = rc[l], s2 = rs[l];
          if (sk != 0.0 || s2 != 0.0) {
            const bool qk = q < n, wl = w < n;
            const double apu = A[p * ld + u];
            const double apw = wl ? A[p * ld + w] : 0.0;
            const double aqu = qk ? A[q * ld + u] : 0.0;
            const double aqw = (qk && wl) ? A[q * ld + w] : 0.0;
            // rows (pair k)
            const double bpu = c * apu - sk * aqu, bqu = sk * apu + c * aqu;
            const double bpw = c * apw - sk * aqw, bqw = sk * apw + c * aqw;
            // columns (pair l); the rotated pair's own off-diagonal is zero
            A[p * ld + u] = c2 * bpu - s2 * bpw;
            if (wl) A[p * ld + w] = (k == l) ? 0.0 : s2 * bpu + c2 * bpw;
            if (qk) A[q * ld + u] = (k == l) ? 0.0 : c2 * bqu - s2 * bqw;
            if (qk && wl) A[q * ld + w] = s2 * bqu + c2 * bqw;
          }
          l += a_dl;
          k += a_dk;
          if (l >= half) {
            l -= half;
            ++k;
          }
        }
      }
      {
        int k = v_k0, i = v_i0;
        for (int j = tid; j < n * half; j += blockDim.x) {
          const int p = rp[k], q = rq[k];
          if (q < n && rs[k] != 0.0) {
            const double c = rc[k], sk = rs[k];
            const double vp = V[i * ld + p], vq = V[i * ld + q];
            V[i * ld + p] = c * vp - sk * vq;
            V[i * ld + q] = sk * vp + c * vq;
          }
          i += v_di;
          k += v_dk;
          if (i >= n) {
            i -= n;
            ++k;
          }
        }
      }
      __syncthreads();
    }
    if (*rotated == 0) break;
    __syncthreads();
  }
  return sweep;
}

// Sort eigenpairs ascending: evals[i] from A diag, evecs columns of V -> out (n x n, column i).
// Scratch for arrowhead_eigh (shared memory, sized for n <= kMaxSel).
struct ArrowScratch {
  double d[kMaxSel], z[kMaxSel], tau[kMaxSel], zhat[kMaxSel];
  double rc[kMaxSel], rs[kMaxSel];
  int idx[kMaxSel], org[kMaxSel], rorg[kMaxSel], rot_i[kMaxSel], rot_j[kMaxSel];
  int keep, nrot, ok;
  double alpha, znorm1;
};

// Eigen-decomposition of an arrowhead matrix
//   H = [[D, z], [z^T, alpha]],  D = diag(d_0 .. d_{n-2}),
// stored as A (n x n, leading dimension n + 1) whose leading (n-1) x (n-1)
// block is diagonal up to rounding of its inputs.  This is the shape of the
// ledger's Gram when the persistent rows come from the previous
// decomposition (mutually orthogonal) and the surrogate adds one row.  The
// method is that of Gu and Eisenstat (SIAM J. Matrix Anal. Appl. 15(4),
// 1994): deflate negligible z_i and (Givens) coincident d_i; find each root
// of the secular equation  alpha - lambda + sum_i z_i^2 / (lambda - d_i) = 0
// by bisection in coordinates shifted to the nearer pole; recompute z from
// the computed roots (Loewner's formula) so the eigenvectors
// [z_i / (lambda - d_i); 1] are orthogonal to working precision.  Returns
// false, touching nothing, when the leading block is not diagonal to
// 1e-6 relative (the caller then runs the Jacobi method).  On success the
// eigenvalues are on A's diagonal and V holds the eigenvectors (columns).
__device__ bool arrowhead_eigh(double* A, double* V, int n, ArrowScratch& S, double* red,
                               double* diag = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int ld = n + 1, m = n - 1;
  // 1. the leading block must be diagonal: every off-diagonal entry below 1e-6
  // of its rows' geometric-mean norm, or below 1e-12 of the largest diagonal
  // entry (rows of negligible energy carry rounding-level directions whose
  // relative orthogonality is meaningless; neglecting them changes no output
  // beyond 1e-12 relative)
  double dmax = 0.0;
  for (int i = tid; i < m; i += blockDim.x) dmax = fmax(dmax, fabs(A[i * ld + i]));
  dmax = block_max(dmax, red);
  double off = 0.0, worst = 0.0;
  for (int k = tid; k < m * m; k += blockDim.x) {
    const int i = k / m, j = k - i * m;
    if (i == j) continue;
    const double aij = fabs(A[i * ld + j]);
    const double scale = sqrt(fabs(A[i * ld + i]) * fabs(A[j * ld + j]));
    if (aij > 1e-12 * dmax) worst = fmax(worst, aij / fmax(scale, 1e-300));
    if (aij > 1e-6 * scale && aij > 1e-12 * dmax) off = 1.0;
  }
  worst = block_max(worst, red);
  if (diag != nullptr && threadIdx.x == 0) *diag = worst;
  if (block_sum(off, red) > 0.0) return false;
  // 2. inputs and ranks of d (ascending, ties by index)
  for (int i = tid; i < m; i += blockDim.x) {
    const double di = A[i * ld + i];
    int r = 0;
    for (int j = 0; j < m; ++j) {
      const double dj = A[j * ld + j];
      r += (dj < di) || (dj == di && j < i);
    }
    S.idx[r] = i;
  }
  double zn2 = 0.0, zn1 = 0.0, dn2 = 0.0;
  for (int i = tid; i < m; i += blockDim.x) {
    const double zi = A[i * ld + m], di = A[i * ld + i];
    zn2 += zi * zi;
    zn1 += fabs(zi);
    dn2 += di * di;
  }
  zn2 = block_sum(zn2, red);
  zn1 = block_sum(zn1, red);
  dn2 = block_sum(dn2, red);
  const double alpha = A[m * ld + m];
  const double hnorm = sqrt(dn2 + 2.0 * zn2 + alpha * alpha);
  const double tol = 8.0 * kEps * hnorm;
  // V = I; the deflated coordinates keep their unit vectors
  for (int k = tid; k < n * n; k += blockDim.x) {
    const int r = k / n, c = k - r * n;
    V[r * ld + c] = (r == c) ? 1.0 : 0.0;
  }
  __syncthreads();
  // 3. deflation (one thread, O(m)): sorted order, negligible z and coincident d
  if (tid == 0) {
    int keep = 0, nrot = 0, last = -1;
    for (int r = 0; r < m; ++r) {
      const int i = S.idx[r];
      double zi = A[i * ld + m];
      const double di = A[i * ld + i];
      if (fabs(zi) <= tol) continue;  // eigenpair (d_i, e_i)
      if (last >= 0 && fabs(di - S.d[last]) <= tol) {
        // rotate (kept j, new i) so that z_i vanishes: e_j' = c e_j + s e_i
        const int j = S.org[last];
        const double zj = S.z[last];
        const double rr = sqrt(zj * zj + zi * zi);
        S.rot_i[nrot] = i;
        S.rot_j[nrot] = j;
        S.rc[nrot] = zj / rr;
        S.rs[nrot] = zi / rr;
        ++nrot;
        S.z[last] = rr;
        continue;
      }
      S.d[keep] = di;
      S.z[keep] = zi;
      S.org[keep] = i;
      last = keep;
      ++keep;
    }
    S.keep = keep;
    S.nrot = nrot;
    S.alpha = alpha;
    S.znorm1 = zn1;
  }
  __syncthreads();
  const int K = S.keep;
  // 4. roots: K + 1 of them; root j lies below d_0 (j = 0), in (d_{j-1}, d_j),
  // or above d_{K-1} (j = K).  One warp per root; lanes split the sum.
  const double lower = fmin(K ? S.d[0] : alpha, alpha) - zn1 - tol;
  const double upper = fmax(K ? S.d[K - 1] : alpha, alpha) + zn1 + tol;
  for (int j = warp; j <= K; j += nwarps) {
    if (K == 0) break;
    // bracket (lo, hi) and the pole used as origin
    const double lo_abs = j == 0 ? lower : S.d[j - 1];
    const double hi_abs = j == K ? upper : S.d[j];
    auto secular = [&](int o, double t) {
      const double org = S.d[o];
      double sum = 0.0;
      for (int i = lane; i < K; i += 32) sum += S.z[i] * S.z[i] / ((org - S.d[i]) + t);
      sum = warp_sum_d(sum);
      return S.alpha - (org + t) + sum;
    };
    int o;
    double tlo, thi;
    if (j == 0) {
      o = 0;
      tlo = lower - S.d[0];
      thi = 0.0;
    } else if (j == K) {
      o = K - 1;
      tlo = 0.0;
      thi = upper - S.d[K - 1];
    } else {
      // origin at the pole nearer to the root: sign of f at the midpoint
      const double half = 0.5 * (hi_abs - lo_abs);
      if (secular(j - 1, half) > 0.0) {  // root in the right half
        o = j;
        tlo = -half;
        thi = 0.0;
      } else {
        o = j - 1;
        tlo = 0.0;
        thi = half;
      }
    }
    for (int it = 0; it < 200; ++it) {
      const double mid = 0.5 * (tlo + thi);
      if (mid == tlo || mid == thi) break;
      if (thi - tlo <= 2.0 * kEps * fmax(fabs(tlo), fabs(thi))) break;
      // the open end at the pole (t = 0) is never evaluated: mid != 0 here
      if (secular(o, mid) > 0.0) tlo = mid; else thi = mid;
    }
    if (lane == 0) {
      S.rorg[j] = o;
      S.tau[j] = 0.5 * (tlo + thi);
    }
  }
  __syncthreads();
  // lambda_j - d_i, with the root held as (origin pole, offset)
  auto gap = [&](int j, int i) { return (S.d[S.rorg[j]] - S.d[i]) + S.tau[j]; };
  // 5. Loewner: |zhat_i|^2 = prod_j (lambda_j - d_i) / prod_{k != i} (d_k - d_i),
  // evaluated as bounded ratios; interlacing: lambda_i < d_i < lambda_{i+1}.
  for (int i = tid; i < K; i += blockDim.x) {
    double p = -gap(i, i) * gap(i + 1, i);
    for (int k = 0; k < i; ++k) p *= gap(k, i) / (S.d[k] - S.d[i]);
    for (int k = i + 1; k < K; ++k) p *= gap(k + 1, i) / (S.d[k] - S.d[i]);
    S.zhat[i] = copysign(sqrt(fmax(p, 0.0)), S.z[i]);
  }
  __syncthreads();
  // 6. eigenvectors of the kept block into the columns of the kept
  // coordinates plus the arrow column: column c(j) = org[j] for j < K, m for j = K
  for (int j = warp; j <= K && K > 0; j += nwarps) {
    const int col = j < K ? S.org[j] : m;
    double nrm = 0.0;
    for (int i = lane; i < K; i += 32) {
      const double u = S.zhat[i] / gap(j, i);
      nrm += u * u;
    }
    nrm = warp_sum_d(nrm) + 1.0;  // the arrow component is 1
    const double inv = 1.0 / sqrt(nrm);
    for (int r = lane; r < n; r += 32) V[r * ld + col] = 0.0;
    __syncwarp();
    for (int i = lane; i < K; i += 32) V[S.org[i] * ld + col] = S.zhat[i] / gap(j, i) * inv;
    if (lane == 0) V[m * ld + col] = inv;
    if (lane == 0) A[col * ld + col] = S.d[S.rorg[j]] + S.tau[j];
  }
  __syncthreads();
  if (K == 0 && tid == 0) A[m * ld + m] = alpha;  // every z negligible
  // 7. undo the coincident-d rotations (in reverse order) on the rows of V
  for (int q = S.nrot - 1; q >= 0; --q) {
    const int i = S.rot_i[q], j = S.rot_j[q];
    const double c = S.rc[q], sn = S.rs[q];
    for (int col = tid; col < n; col += blockDim.x) {
      const double vj = V[j * ld + col], vi = V[i * ld + col];
      V[j * ld + col] = c * vj - sn * vi;
      V[i * ld + col] = sn * vj + c * vi;
    }
    __syncthreads();
  }
  return true;
}

__device__ void sort_eigen(const double* A, const double* V, int n, double* evals, double* evecs,
                           int* order) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; ++i) order[i] = i;
    for (int i = 1; i < n; ++i) {
      const int oi = order[i];
      const double v = A[oi * (n + 1) + oi];
      int j = i - 1;
      while (j >= 0 && A[order[j] * (n + 1) + order[j]] > v) {
        order[j + 1] = order[j];
        --j;
      }
      order[j + 1] = oi;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) evals[i] = A[order[i] * (n + 1) + order[i]];
  for (int idx = threadIdx.x; idx < n * n; idx += blockDim.x) {
    const int r = idx / n, col = idx % n;
    evecs[r * n + col] = V[r * (n + 1) + order[col]];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) transaction_kernel(Args a) {
  extern __shared__ double sm[];
  double* A = sm;                       // kMaxSel^2
  double* V = A + kMaxSel * (kMaxSel + 1);  // kMaxSel x (kMaxSel + 1)
  __shared__ double red[40];
  __shared__ double rc[kMaxSel / 2 + 2], rs[kMaxSel / 2 + 2];
  __shared__ int rp[kMaxSel / 2 + 2], rq[kMaxSel / 2 + 2];
  __shared__ int rotated;
  __shared__ int order[kMaxSel + 2];
  __shared__ double evals[kMaxSel];
  __shared__ double sc[64];             // scalars
  __shared__ double alphas[kKrylov], betas[kKrylov], proj[kKrylov], lam[kKrylov];
  __shared__ ArrowScratch arrow_scratch;
  __shared__ double sel_last_scale;  // the collapsed surrogate row's sqrt(32) (else 1)
  __shared__ int sel_last_row;
  const int tid = threadIdx.x;
  const int C = a.C;
  STAMP(0);
  // workspace layout (doubles)
  double* cur = a.ws;                       // [32, C]
  double* sel = cur + kCurRows * C;         // [96, C] selection rows (fp32-rounded values)
  double* decay_cross = sel + kMaxSel * C;  // [C]
  double* Q = decay_cross + C;              // [C, 32] column-major by Krylov index: Q[i*C + c]
  double* rhs = Q + kKrylov * C;            // [C]
  double* vec = rhs + C;                    // [C] current
  double* prv = vec + C;                    // [C]
  double* act = prv + C;                    // [C]
  double* res = act + C;                    // [C]
  double* fb = res + C;                     // [C]
  double* Lv = fb + C;                      // [96]
  double* cand = Lv + kMaxSel;              // [C]
  double* evecT = cand + C;                 // [32*32]
  double* cdec = evecT + kKrylov * kKrylov; // [32] current decay action
  double* evecs = cdec + kCurRows;          // [96*96] sorted ledger eigenvectors
  double* rsw = evecs + kMaxSel * kMaxSel;  // [C] 1/sqrt(w_c)

  // ---- current rows ------------------------------------------------------
  if (!a.functional) {
    double s = 0.0;
    for (int c = tid; c < C; c += blockDim.x) {
      const double g = static_cast<double>(a.exact[c]) + static_cast<double>(a.exact[C + c]);
      s += g * g;
    }
    const double norm = sqrt(block_sum(s, red));
    const double ref = static_cast<double>(a.ref_row_norm[0]);
    const double scale = norm > kTiny ? ref / fmax(norm, kTiny) : 0.0;
    for (int c = tid; c < C; c += blockDim.x) {
      const double g = static_cast<double>(a.exact[c]) + static_cast<double>(a.exact[C + c]);
      const double v = static_cast<double>(static_cast<float>(g * scale));
      for (int r = 0; r < kCurRows; ++r) cur[r * C + c] = v;
    }
    if (tid < kCurRows)
      cdec[tid] = static_cast<double>(static_cast<float>(static_cast<double>(a.decay_derivative[0]) * scale));
    if (tid == 0) a.result[6] = static_cast<float>(scale);
  } else {
    for (int i = tid; i < kCurRows * C; i += blockDim.x) cur[i] = static_cast<double>(a.cur_scores[i]);
    if (tid < kCurRows) cdec[tid] = static_cast<double>(a.cur_decay[tid]);
    if (tid == 0) a.result[6] = 1.0f;
  }
  __syncthreads();
  if (a.functional) {
    double s = 0.0;
    for (int i = tid; i < kCurRows * C; i += blockDim.x) s += cur[i] * cur[i];
    s = block_sum(s, red);
    if (tid == 0) a.ref_row_norm[0] = static_cast<float>(sqrt(s / kCurRows));
  }
  // ---- ledger --------------------------------------------------------------
  const double beta2 = 0.95;
  int nsel;
  double sel_tail;
  if (a.prev_rows == 0) {
    nsel = kCurRows;
    sel_tail = 0.0;
    for (int i = tid; i < kCurRows * C; i += blockDim.x) sel[i] = cur[i];
    for (int c = tid; c < C; c += blockDim.x) {
      double cross = 0.0, rep = 0.0;
      for (int r = 0; r < kCurRows; ++r) {
        cross += cur[r * C + c] * cdec[r];
        rep += cur[r * C + c] * cur[r * C + c];
      }
      decay_cross[c] = static_cast<double>(static_cast<float>(cross / kCurRows));
      a.pers_decay_cross[c] = static_cast<float>(cross / kCurRows);
      a.pers_total_diag[c] = static_cast<float>(rep / kCurRows);
      for (int r = 0; r < kCurRows; ++r) a.pers_scores[r * C + c] = static_cast<float>(cur[r * C + c]);
    }
    if (tid == 0) {
      a.pers_tail[0] = 0.0f;
      a.discarded_fraction[0] = 0.0f;
      a.shrinkage[0] = 0.0f;
      a.result[7] = static_cast<float>(kCurRows);  // persistent rows
    }
    __syncthreads();
  } else {
    const int prev = a.prev_rows;
    // Surrogate rows are 32 copies of one row.  Everything downstream depends
    // on the selection only through sel^T sel, so the copies collapse into a
    // single row scaled by sqrt(32): the eigenproblem shrinks from 96 to 65
    // rows (the 31 removed eigenvalues are exactly zero and always discarded).
    const bool collapse = !a.functional;
    const int cur_rows = collapse ? 1 : kCurRows;
    nsel = prev + cur_rows;
    const float sb = static_cast<float>(sqrt(beta2)), sc1 = static_cast<float>(sqrt(1.0 - beta2));
    const double row_scale = collapse ? sqrt(static_cast<double>(kCurRows)) : 1.0;
    if (tid == 0) {
      sel_last_scale = row_scale;
      sel_last_row = collapse ? prev : -1;
    }
    for (int i = tid; i < prev * C; i += blockDim.x) sel[i] = static_cast<double>(a.pers_scores[i] * sb);
    for (int i = tid; i < cur_rows * C; i += blockDim.x)
      sel[prev * C + i] = static_cast<double>(static_cast<float>(cur[i]) * sc1) * row_scale;
    const double prev_tail = static_cast<double>(a.pers_tail[0]);
    sel_tail = prev_tail * beta2;
    for (int c = tid; c < C; c += blockDim.x) {
      double cross = 0.0;
      for (int r = 0; r < kCurRows; ++r) cross += cur[r * C + c] * cdec[r];
      const double dc = static_cast<double>(a.pers_decay_cross[c]) * beta2 + (cross / kCurRows) * (1.0 - beta2);
      decay_cross[c] = static_cast<double>(static_cast<float>(dc));
    }
    __syncthreads();
    // Gram of the selection rows
    // one warp per (i, j) pair, lanes stride the coordinates (coalesced rows)
    for (int idx = tid >> 5; idx < nsel * nsel; idx += blockDim.x >> 5) {
      const int i = idx / nsel, j = idx - i * nsel;
      if (j < i) continue;
      double s = 0.0;
      for (int c = tid & 31; c < C; c += 32) s += sel[i * C + c] * sel[j * C + c];
      s = warp_sum_d(s);
      if ((tid & 31) == 0) {
        A[i * (nsel + 1) + j] = s;
        A[j * (nsel + 1) + i] = s;
      }
    }
    __syncthreads();
    STAMP(1);
    // surrogate rows over persistent rows from a previous decomposition: the
    // Gram is an arrowhead matrix (orthogonal rows, one new row)
    double worst_ratio = 0.0;
    const bool arrow = collapse && arrowhead_eigh(A, V, nsel, arrow_scratch, red, &worst_ratio);
    if (a.timing != nullptr && tid == 0 && collapse)
      a.timing[14] = static_cast<unsigned long long>(fmin(worst_ratio, 1.0) * 1e15);
    const int gram_sweeps = arrow ? -1 : jacobi_eigh(A, V, nsel, rp, rq, rc, rs, red, &rotated);
    STAMP(2);
    if (a.timing != nullptr && tid == 0) a.timing[12] = gram_sweeps;
    sort_eigen(A, V, nsel, evals, evecs, order);
    // stage the sorted eigenvectors in shared memory (A is free once evals are read)
    for (int i = tid; i < nsel * nsel; i += blockDim.x) A[i] = evecs[i];
    __syncthreads();
    for (int i = tid; i < nsel; i += blockDim.x) evals[i] = fmax(evals[i], 0.0);
    __syncthreads();
    const int retained = nsel < kPersRows ? nsel : kPersRows;
    const int discarded = nsel - retained;
    const double shrink = discarded ? evals[discarded - 1] : 0.0;
    // persistent = mult * (V_kept^T sel)
    for (int idx = tid; idx < retained * C; idx += blockDim.x) {
      const int r = idx / C, c = idx % C;
      const int col = discarded + r;
      double s = 0.0;
      for (int i = 0; i < nsel; ++i) s += A[i * nsel + col] * sel[i * C + c];
      const double kept = evals[col];
      const double mult = sqrt(fmax(kept - shrink, 0.0) / fmax(kept, kTiny));
      a.pers_scores[r * C + c] = static_cast<float>(mult * s);
    }
    // rows of the removed zero eigenvalues (collapsed surrogate only)
    for (int idx = retained * C + tid; idx < kPersRows * C; idx += blockDim.x) a.pers_scores[idx] = 0.0f;
    __syncthreads();
    const double pers_tail = sel_tail + shrink / (2.0 * kCurRows);
    for (int c = tid; c < C; c += blockDim.x) {
      double rep = 0.0;
      for (int r = 0; r < retained; ++r) {
        const double v = static_cast<double>(a.pers_scores[r * C + c]);
        rep += v * v;
      }
      a.pers_total_diag[c] = static_cast<float>(rep / kCurRows + pers_tail);
      a.pers_decay_cross[c] = static_cast<float>(decay_cross[c]);
    }
    double tot = 0.0, disc = 0.0;
    for (int i = tid; i < nsel; i += blockDim.x) {
      tot += evals[i];
      if (i < discarded) disc += evals[i];
    }
    tot = block_sum(tot, red);
    disc = block_sum(disc, red);
    if (tid == 0) {
      a.pers_tail[0] = static_cast<float>(pers_tail);
      a.shrinkage[0] = static_cast<float>(shrink);
      a.discarded_fraction[0] = static_cast<float>(disc / fmax(tot, kTiny));
      const int logical = a.prev_rows + kCurRows;
      a.result[7] = static_cast<float>(logical < kPersRows ? logical : kPersRows);
    }
    __syncthreads();
  }
  const double diag_res = static_cast<double>(static_cast<float>(sel_tail));
  STAMP(3);

  // ---- transaction -----------------------------------------------------------
  const double eta = a.eta;
  // low_rank L[r, c] = sel[r, c] / sqrt(w_c) / sqrt(32): applied on the fly.
  double bsum = 0.0, rn = 0.0;
  for (int c = tid; c < C; c += blockDim.x) {
    const double w = static_cast<double>(a.weights[c]);
    bsum += w;
    const double e = static_cast<double>(a.exact[c]) + static_cast<double>(a.exact[C + c]);
    const double r = (e / eta - decay_cross[c]) / sqrt(w);
    rhs[c] = r;
    rn += r * r;
  }
  for (int c = tid; c < C; c += blockDim.x) rsw[c] = 1.0 / sqrt(static_cast<double>(a.weights[c]));
  const double budget = block_sum(bsum, red);
  const double rhs_norm = sqrt(block_sum(rn, red));
  const int steps = C < kKrylov ? C : kKrylov;
  const double inv_sqrt_m = 1.0 / sqrt(static_cast<double>(kCurRows));
  for (int c = tid; c < C; c += blockDim.x) {
    vec[c] = rhs[c] / fmax(rhs_norm, kTiny);
    prv[c] = 0.0;
  }
  __syncthreads();
  double prev_beta = 0.0;
  STAMP(4);
  // The selection rows are fp32 values (the collapsed surrogate row times
  // sqrt(32)): during the Lanczos iteration they are read from shared memory
  // as floats (the eigenproblem's A/V space is free here), with the row scale
  // applied to the row's coefficient, instead of twice per step from global
  // memory.  Problems too large for shared memory read `sel` as before.
  float* self = reinterpret_cast<float*>(sm);
  const bool sel_smem = static_cast<size_t>(nsel) * C * sizeof(float) <= 2ull * kMaxSel * (kMaxSel + 1) * sizeof(double);
  const int last_row = a.prev_rows == 0 ? -1 : sel_last_row;
  const double last_scale = a.prev_rows == 0 ? 1.0 : sel_last_scale;
  if (sel_smem)
    for (int i2 = tid; i2 < nsel * C; i2 += blockDim.x)
      self[i2] = static_cast<float>(i2 / C == last_row ? sel[i2] / last_scale : sel[i2]);
  __syncthreads();
  for (int i = 0; i < steps; ++i) {
    for (int c = tid; c < C; c += blockDim.x) Q[i * C + c] = vec[c];
    // Lv[r] = sum_c L[r,c] vec[c]  (stored times the row scale for the action)
    for (int r = tid >> 5; r < nsel; r += blockDim.x >> 5) {
      double s = 0.0;
      if (sel_smem) {
        for (int c = tid & 31; c < C; c += 32) s += static_cast<double>(self[r * C + c]) * rsw[c] * vec[c];
        const double rs2 = r == last_row ? last_scale * last_scale : 1.0;
        s *= inv_sqrt_m * rs2;
      } else {
        for (int c = tid & 31; c < C; c += 32) s += sel[r * C + c] * rsw[c] * vec[c];
        s *= inv_sqrt_m;
      }
      s = warp_sum_d(s);
      if ((tid & 31) == 0) Lv[r] = s;
    }
    __syncthreads();
    double adot = 0.0, anorm = 0.0;
    for (int c = tid; c < C; c += blockDim.x) {
      const double rw = rsw[c] * inv_sqrt_m;
      double acc = 0.0;
      if (sel_smem)
        for (int r = 0; r < nsel; ++r) acc += static_cast<double>(self[r * C + c]) * Lv[r];
      else
        for (int r = 0; r < nsel; ++r) acc += sel[r * C + c] * Lv[r];
      double s = diag_res / static_cast<double>(a.weights[c]) * vec[c] + acc * rw;
      act[c] = s;
      adot += vec[c] * s;
      anorm += s * s;
    }
    const double alpha = block_sum(adot, red);
    const double action_norm = sqrt(block_sum(anorm, red));
    for (int c = tid; c < C; c += blockDim.x) res[c] = act[c] - alpha * vec[c] - prev_beta * prv[c];
    __syncthreads();
    for (int pass = 0; pass < 2; ++pass) {
      // coefficients h_j = Q_j . res  (j <= i)
      for (int j = tid >> 5; j <= i; j += blockDim.x >> 5) {
        double s = 0.0;
        for (int c = tid & 31; c < C; c += 32) s += Q[j * C + c] * res[c];
        s = warp_sum_d(s);
        if ((tid & 31) == 0) sc[j] = s;
      }
      __syncthreads();
      for (int c = tid; c < C; c += blockDim.x) {
        double s = res[c];
        for (int j = 0; j <= i; ++j) s -= Q[j * C + c] * sc[j];
        res[c] = s;
      }
      __syncthreads();
    }
    double bn = 0.0;
    for (int c = tid; c < C; c += blockDim.x) bn += res[c] * res[c];
    double beta = sqrt(block_sum(bn, red));
    if (tid == 0) alphas[i] = alpha;
    if (i + 1 < steps) {
      const double threshold = 64.0 * kEps * fmax(action_norm, 1.0);
      const bool broke = beta <= threshold;  // uniform: beta is a block reduction
      double fnorm = 0.0;
      if (broke) {
      // Breakdown: continue from a deterministic cosine vector re-orthogonalised
      // against the basis (used only when it is not itself in the span).
      for (int c = tid; c < C; c += blockDim.x) fb[c] = cos(static_cast<double>(c + 1) * static_cast<double>(i + 1));
      __syncthreads();
      for (int pass = 0; pass < 2; ++pass) {
        for (int j = tid >> 5; j <= i; j += blockDim.x >> 5) {
          double s = 0.0;
          for (int c = tid & 31; c < C; c += 32) s += Q[j * C + c] * fb[c];
          s = warp_sum_d(s);
          if ((tid & 31) == 0) sc[j] = s;
        }
        __syncthreads();
        for (int c = tid; c < C; c += blockDim.x) {
          double s = fb[c];
          for (int j = 0; j <= i; ++j) s -= Q[j * C + c] * sc[j];
          fb[c] = s;
        }
        __syncthreads();
      }
      double fn = 0.0;
      for (int c = tid; c < C; c += blockDim.x) fn += fb[c] * fb[c];
      fnorm = sqrt(block_sum(fn, red));
      }
      const bool use_fb = broke && (fnorm > threshold);
      for (int c = tid; c < C; c += blockDim.x) {
        const double nxt = use_fb ? fb[c] / fmax(fnorm, kTiny) : res[c] / fmax(beta, kTiny);
        prv[c] = vec[c];
        vec[c] = nxt;
      }
      if (broke) beta = 0.0;
      if (tid == 0) betas[i] = beta;
      prev_beta = beta;
      __syncthreads();
    }
  }
  // tridiagonal -> A (steps x steps), Jacobi
  for (int idx = tid; idx < steps * steps; idx += blockDim.x) {
    const int i = idx / steps, j = idx % steps;
    double v = 0.0;
    if (i == j) v = alphas[i];
    else if (j == i + 1) v = betas[i];
    else if (i == j + 1) v = betas[j];
    A[i * (steps + 1) + j] = v;
  }
  __syncthreads();
  STAMP(6);
  const int tri_sweeps = jacobi_eigh(A, V, steps, rp, rq, rc, rs, red, &rotated);
  if (a.timing != nullptr && tid == 0) a.timing[13] = tri_sweeps;
  STAMP(7);
  sort_eigen(A, V, steps, lam, evecT, order);
  for (int i = tid; i < steps; i += blockDim.x) lam[i] = fmax(lam[i], 0.0);
  __syncthreads();
  // proj = E^T (Q^T rhs)
  for (int j = tid >> 5; j < steps; j += blockDim.x >> 5) {
    double s = 0.0;
    for (int c = tid & 31; c < C; c += 32) s += Q[j * C + c] * rhs[c];
    s = warp_sum_d(s);
    if ((tid & 31) == 0) sc[j] = s;
  }
  __syncthreads();
  if (tid < steps) {
    double s = 0.0;
    for (int j = 0; j < steps; ++j) s += evecT[j * steps + tid] * sc[j];
    proj[tid] = s;
  }
  __syncthreads();
  if (tid < 32) {
    // One warp: lane j owns Krylov term j (steps <= 32), sums by shuffle.
    const int lane = tid;
    const bool own = lane < steps;
    const double pj = own ? proj[lane] : 0.0, lj = own ? lam[lane] : 0.0;
    const double lower = kEps * static_cast<double>(C);
    double lmax = own ? lj : 0.0;
    for (int o = 16; o > 0; o >>= 1) lmax = fmax(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    const double upper = rhs_norm / sqrt(budget) + lmax + lower;
    auto secular = [&](double mu) {
      const double v = own ? pj / (lj + mu) : 0.0;
      return warp_sum_d(v * v);
    };
    const bool hard = secular(lower) < budget;
    double lo = lower, hi = upper;
    for (int r = 0; r < 64; ++r) {
      const double mid = 0.5 * (lo + hi);
      if (secular(mid) > budget) lo = mid; else hi = mid;
    }
    if (own) sc[lane] = pj / (lj + hi);
    if (lane == 0) {
      sc[40] = hi;
      sc[41] = hard ? 1.0 : 0.0;
    }
  }
  __syncthreads();
  STAMP(8);
  // y = E * sc  -> in the Krylov basis; cand = Q y / sqrt(w)
  if (tid < steps) {
    double s = 0.0;
    for (int j = 0; j < steps; ++j) s += evecT[tid * steps + j] * sc[j];
    proj[tid] = s;  // reuse as y
  }
  __syncthreads();
  double cb = 0.0;
  for (int c = tid; c < C; c += blockDim.x) {
    double y = 0.0;
    for (int j = 0; j < steps; ++j) y += Q[j * C + c] * proj[j];
    const double w = static_cast<double>(a.weights[c]);
    const double cc = y / sqrt(w);
    cand[c] = cc;
    cb += w * cc * cc;
  }
  const double cand_budget = block_sum(cb, red);
  const double budget_res = fabs(cand_budget - budget) / fmax(budget, 1.0);
  // scores: actions per selection row
  double pa2 = 0.0, ca2 = 0.0;
  for (int r = tid >> 5; r < nsel; r += blockDim.x >> 5) {
    double sp = 0.0, sc_ = 0.0;
    for (int c = tid & 31; c < C; c += 32) {
      sp += sel[r * C + c];
      sc_ += sel[r * C + c] * cand[c];
    }
    sp = warp_sum_d(sp);
    sc_ = warp_sum_d(sc_);
    if ((tid & 31) == 0) {
      pa2 += sp * sp;
      ca2 += sc_ * sc_;
    }
  }
  pa2 = block_sum(pa2, red);
  ca2 = block_sum(ca2, red);
  double pe = 0.0, ce = 0.0, pdiag = 0.0, cdiag = 0.0, pdec = 0.0, cdec2 = 0.0;
  bool finite = true;
  for (int c = tid; c < C; c += blockDim.x) {
    const double e = static_cast<double>(a.exact[c]) + static_cast<double>(a.exact[C + c]);
    pe += e;
    ce += e * cand[c];
    pdiag += diag_res;
    cdiag += diag_res * cand[c] * cand[c];
    pdec += decay_cross[c];
    cdec2 += decay_cross[c] * cand[c];
    if (!isfinite(cand[c])) finite = false;
  }
  pe = block_sum(pe, red);
  ce = block_sum(ce, red);
  pdiag = block_sum(pdiag, red);
  cdiag = block_sum(cdiag, red);
  pdec = block_sum(pdec, red);
  cdec2 = block_sum(cdec2, red);
  const double nonfinite = block_sum(finite ? 0.0 : 1.0, red);
  const double m = static_cast<double>(kCurRows);
  const double parent_score = -eta * pe + 0.5 * eta * eta * (pa2 / m + pdiag + 2.0 * pdec);
  const double cand_score = -eta * ce + 0.5 * eta * eta * (ca2 / m + cdiag + 2.0 * cdec2);
  // per-layer contractions (both roles): parent exact/momentum and candidate
  // versions must all be positive.  One warp per layer.
  __shared__ int layer_ok;
  if (tid == 0) layer_ok = 1;
  __syncthreads();
  for (int l = tid >> 5; l < a.total_layers; l += blockDim.x >> 5) {
    double v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = tid & 31; c < C; c += 32) {
      if (a.layer_ids[c] != l) continue;
      for (int role = 0; role < 2; ++role) {
        const double ex = a.exact[role * C + c], mo = a.momentum[role * C + c];
        v[role * 4 + 0] += ex;
        v[role * 4 + 1] += mo;
        v[role * 4 + 2] += ex * cand[c];
        v[role * 4 + 3] += mo * cand[c];
      }
    }
    for (int k = 0; k < 8; ++k) {
      const double t = warp_sum_d(v[k]);
      if ((tid & 31) == 0 && !(t > 0.0)) atomicExch(&layer_ok, 0);
    }
  }
  __syncthreads();
  const bool hard = sc[41] != 0.0;
  const bool accepted = nonfinite == 0.0 && isfinite(cand_score) && isfinite(budget_res) && !hard &&
                        cand_score < parent_score && budget_res <= 1e-8 && layer_ok;
  for (int c = tid; c < C; c += blockDim.x) {
    const float cf = static_cast<float>(cand[c]);
    a.candidate[c] = cf;
    a.coefficients[c] = accepted ? cf : 1.0f;
  }
  if (tid == 0) {
    a.result[0] = accepted ? 1.0f : 0.0f;
    a.result[1] = hard ? 0.0f : static_cast<float>(sc[40]);
    a.result[2] = hard ? 1.0f : 0.0f;
    a.result[3] = static_cast<float>(budget_res);
    a.result[4] = static_cast<float>(parent_score);
    a.result[5] = static_cast<float>(cand_score);
    a.result[8] = static_cast<float>(a.prev_rows == 0 || a.functional ? nsel : nsel + kCurRows - 1);
  }
  STAMP(9);
}

}  // namespace ledger

int64_t ledger_workspace_doubles(int C) {
  using namespace ledger;
  return static_cast<int64_t>(kCurRows) * C + static_cast<int64_t>(kMaxSel) * C + C +
         static_cast<int64_t>(kKrylov) * C + 7LL * C + kMaxSel + C + kKrylov * kKrylov + kCurRows +
         static_cast<int64_t>(kMaxSel) * kMaxSel + C;
}

int ledger_transaction(const float* cur_scores, const float* cur_decay, const float* exact,
                       const float* momentum, const float* weights, const int64_t* layer_ids,
                       const float* decay_derivative, float* pers_scores, float* pers_total_diag,
                       float* pers_decay_cross, float* pers_tail, float* discarded_fraction,
                       float* shrinkage, float* ref_row_norm, float* coefficients, float* candidate,
                       float* result, double* ws, int C, int prev_rows, int total_layers,
                       bool functional, double eta, unsigned long long* timing,
                       cudaStream_t stream) {
  using namespace ledger;
  if (C < 2 || (prev_rows != 0 && prev_rows != kCurRows && prev_rows != kPersRows)) return -1;
  Args a{cur_scores, cur_decay, exact, momentum, weights, layer_ids, decay_derivative, pers_scores,
         pers_total_diag, pers_decay_cross, pers_tail, discarded_fraction, shrinkage, ref_row_norm,
         coefficients, candidate, result, ws, timing, C, prev_rows, total_layers,
         functional ? 1 : 0, eta};
  const size_t smem = 2ull * kMaxSel * (kMaxSel + 1) * sizeof(double);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(transaction_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    configured = true;
  }
  transaction_kernel<<<1, kThreads, smem, stream>>>(a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro
