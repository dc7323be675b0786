// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores
// (tcgen05.mma, accumulator in TMEM), operands streamed by TMA.
//
//   C[b] (M x N) = alpha * A[b] (M x K) . B[b]^T (K x N) + beta * D[b]
//
// A is K-major ([M, K] rows) or M-major ([K, M] rows); B is K-major
// ([N, K] rows, i.e. an nn.Linear weight) or N-major ([K, N] rows).  These
// four layouts cover y = x W^T, dx = dy W, dW = dy^T x and the three
// products of a Newton-Schulz iteration without any transpose pass.
//
// CTA layout (192 threads, one CTA per SM, grid = #SMs, persistent over tiles):
//   warp 0      TMA producer (one elected lane), 128B-swizzled tiles,
//               kStages-deep smem ring guarded by full/empty mbarriers;
//   warp 1      TMEM allocator and MMA issuer (one elected lane):
//               tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN, K=16;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, alpha/beta/convert,
//               direct 16-byte stores (rows/columns masked at the edges).
// The accumulator is double-buffered in TMEM (2 x BN columns) so the
// epilogue of tile t overlaps the main loop of tile t+1.
//
// Every mbarrier wait is bounded by a wall-clock limit; on expiry the waiting
// role records an error code in `err`, stops, and the CTA still releases its
// TMEM and returns, so a broken invariant cannot hang the GPU.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

#include "common.cuh"

namespace ro {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;          // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

struct Params {
  int M, N, K, batch;
  void* C;
  int64_t ldc, strideC;
  const __nv_bfloat16* D;
  int64_t ldd, strideD;
  float alpha, beta;
  int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase does not
// complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 32 lanes x 32 columns of 32-bit accumulator per warp.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor for a 128B-swizzled tile (version 1).
//   K-major:  8 rows of 128 B per core group, SBO = 1024 B between groups.
//   MN-major: 64-element (128 B) MN blocks at LBO, 8-row K groups at SBO.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, bf16 x bf16 -> f32, M=128, N=BN.
template <int BN, bool A_MN, bool B_MN>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
  return (1u << 4)                      // C format f32
         | (1u << 7)                    // A bf16
         | (1u << 10)                   // B bf16
         | ((A_MN ? 1u : 0u) << 15)     // A major
         | ((B_MN ? 1u : 0u) << 16)     // B major
         | (static_cast<uint32_t>(BN >> 3) << 17)
         | (static_cast<uint32_t>(BM >> 4) << 24);
}

template <int BN>
struct Config {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kTmemCols = 2 * BN;   // double-buffered accumulator
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& b, int& m, int& n) {
  // Grouped ordering: 8 M-tiles share each sweep over N for L2 reuse of B.
  constexpr int kGroup = 8;
  const int per_batch = num_m * num_n;
  b = tile / per_batch;
  int t = tile % per_batch;
  const int group_span = kGroup * num_n;
  const int g = t / group_span;
  const int first_m = g * kGroup;
  int gm = num_m - first_m;
  if (gm > kGroup) gm = kGroup;
  const int r = t % group_span;
  m = first_m + r % gm;
  n = r / gm;
}

template <int BN, bool A_MN, bool B_MN, bool OUT_F32, bool HAS_D>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            Params p) {
  using Cfg = Config<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + Cfg::kStages;
  uint64_t* acc_full = bars + 2 * Cfg::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_k = (p.K + BK - 1) / BK;
  const int tiles = num_m * num_n * p.batch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(Cfg::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        int b, tm, tn;
        tile_coords(tile, num_m, num_n, b, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, p.err, 1)) { ok = false; break; }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_expect_tx(fb, Cfg::kStageBytes);
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d(sa, &tmA, fb, k0, m0, b);
          } else {
            tma_load_3d(sa, &tmA, fb, m0, k0, b);
            tma_load_3d(sa + 64 * 128, &tmA, fb, m0 + 64, k0, b);
          }
          if constexpr (!B_MN) {
            tma_load_3d(sb, &tmB, fb, k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(sb + j * 64 * 128, &tmB, fb, n0 + 64 * j, k0, b);
          }
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<BN, A_MN, B_MN>();
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, p.err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if constexpr (!A_MN) ad = smem_desc(sa + k * 32, 16, 1024);
            else ad = smem_desc(sa + k * 16 * 128, 64 * 128, 1024);
            if constexpr (!B_MN) bd = smem_desc(sb + k * 32, 16, 1024);
            else bd = smem_desc(sb + k * 16 * 128, 64 * 128, 1024);
            tc_mma(tmem_d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&empty[stage]));
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(smem_u32(&acc_full[acc]));
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int local = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      int b, tm, tn;
      tile_coords(tile, num_m, num_n, b, tm, tn);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(&acc_full[acc]), acc_phase, p.err, 4)) break;
      tc_fence_after();
      const int row = tm * BM + quarter * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tbase + c, r);
        const int col0 = tn * BN + c;
        if (!row_ok || col0 >= p.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
        const bool full_cols = col0 + 32 <= p.N;
        if constexpr (HAS_D) {
          const __nv_bfloat16* dp = p.D + b * p.strideD + static_cast<int64_t>(row) * p.ldd + col0;
          if (full_cols && (reinterpret_cast<uintptr_t>(dp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float dv[8];
              load_vec<__nv_bfloat16, 8>(dp + j, dv);
#pragma unroll
              for (int q = 0; q < 8; ++q) v[j + q] = fmaf(p.beta, dv[q], v[j + q]);
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) v[j] = fmaf(p.beta, __bfloat162float(dp[j]), v[j]);
          }
        }
        if constexpr (OUT_F32) {
          float* cp = static_cast<float*>(p.C) + b * p.strideC + static_cast<int64_t>(row) * p.ldc + col0;
          if (full_cols && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(cp + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) cp[j] = v[j];
          }
        } else {
          __nv_bfloat16* cp = static_cast<__nv_bfloat16*>(p.C) + b * p.strideC +
                              static_cast<int64_t>(row) * p.ldc + col0;
          if (full_cols && (reinterpret_cast<uintptr_t>(cp) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float w8[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) w8[q] = v[j + q];
              store_vec<__nv_bfloat16, 8>(cp + j, w8);
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) cp[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&acc_empty[acc]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Cfg::kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no libcuda link).

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                              CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// 3-D bf16 map: inner (contiguous) extent, outer extent, batch; row stride and
// batch stride in elements; box = {64, box_outer, 1}, 128B swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t batch,
              int64_t row_stride, int64_t batch_stride, int box_outer) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2),
                           static_cast<cuuint64_t>((batch > 1 ? batch_stride : outer * row_stride) * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_outer), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, bool OUT_F32, bool HAS_D>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, cudaStream_t stream) {
  using Cfg = Config<BN>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, OUT_F32, HAS_D>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    configured = true;
  }
  const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN) * p.batch;
  int grid = num_sms();
  if (tiles < grid) grid = tiles;
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ma, mb, p);
  return static_cast<int>(cudaGetLastError());
}

template <int BN, bool A_MN, bool B_MN>
int dispatch_out(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, bool out_f32,
                 cudaStream_t s) {
  if (out_f32) return p.D ? launch<BN, A_MN, B_MN, true, true>(ma, mb, p, s)
                          : launch<BN, A_MN, B_MN, true, false>(ma, mb, p, s);
  return p.D ? launch<BN, A_MN, B_MN, false, true>(ma, mb, p, s)
             : launch<BN, A_MN, B_MN, false, false>(ma, mb, p, s);
}

}  // namespace gemm

// C[b] = alpha * op(A[b]) op(B[b])^T + beta * D[b], bf16 inputs.
//   a_mn == false: A is [M, K] with row stride lda;  true: A is [K, M] (stride lda).
//   b_mn == false: B is [N, K] with row stride ldb;  true: B is [K, N] (stride ldb).
// Batch strides are in elements.  Returns 0 on success, negative when the
// configuration is unsupported (caller falls back), positive CUDA error codes.
int gemm_bf16_tn(const void* A, int64_t lda, int64_t strideA, bool a_mn, const void* B, int64_t ldb,
                 int64_t strideB, bool b_mn, void* C, int64_t ldc, int64_t strideC, bool out_f32,
                 const void* D, int64_t ldd, int64_t strideD, float alpha, float beta, int M, int N,
                 int K, int batch, int* err, cudaStream_t stream) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return -1;
  // TMA: 16-byte aligned base and row strides; inner extents multiples of 8.
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al16(A) || !al16(B) || (lda % 8) || (ldb % 8)) return -2;
  if (batch > 1 && ((strideA % 8) || (strideB % 8))) return -2;
  if ((a_mn ? M : K) % 8 || (b_mn ? N : K) % 8) return -2;
  const int BNsel = (N >= 256 || b_mn) ? 256 : 128;
  CUtensorMap ma, mb;
  bool ok = a_mn ? make_map(&ma, A, M, K, batch, lda, strideA, 64)
                 : make_map(&ma, A, K, M, batch, lda, strideA, BM);
  ok = ok && (b_mn ? make_map(&mb, B, N, K, batch, ldb, strideB, 64)
                   : make_map(&mb, B, K, N, batch, ldb, strideB, BNsel));
  if (!ok) return -3;
  Params p{M, N, K, batch, C, ldc, strideC, static_cast<const __nv_bfloat16*>(D), ldd, strideD,
           alpha, beta, err};
  if (BNsel == 256) {
    if (!a_mn && !b_mn) return dispatch_out<256, false, false>(ma, mb, p, out_f32, stream);
    if (!a_mn && b_mn) return dispatch_out<256, false, true>(ma, mb, p, out_f32, stream);
    if (a_mn && !b_mn) return dispatch_out<256, true, false>(ma, mb, p, out_f32, stream);
    return dispatch_out<256, true, true>(ma, mb, p, out_f32, stream);
  }
  if (!a_mn) return dispatch_out<128, false, false>(ma, mb, p, out_f32, stream);
  return dispatch_out<128, true, false>(ma, mb, p, out_f32, stream);
}

}  // namespace ro
