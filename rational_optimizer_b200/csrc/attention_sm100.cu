// Causal flash attention, forward, on the 5th-generation tensor cores.
//
//   O = softmax(Q K^T * scale + causal mask) V,     LSE2 = log2 of the row sums
//
// Layout: q, k, v and o are token-major bf16 planes [B, S, ld] (row = token,
// head h at columns [h*HD, (h+1)*HD)), exactly what the fused q/k/v + RoPE
// projection writes and what the output projection reads, so no transposes
// are needed.  lse2 is fp32 [B, H, S] in log2 units of the scaled scores:
// lse2 = m + log2(l) with m the row max of s*scale*log2(e) and l the sum of
// exp2 of the shifted scores; the backward recomputes P = exp2(s' - lse2).
//
// Tiles: 128 queries x 128 keys, head_dim HD = 64 or 128.  A persistent CTA
// (192 threads, one per SM) walks (query tile, head, batch) work items,
// heaviest causal tiles first:
//   warp 0      TMA producer: Q tile once per item, then K/V tiles into a
//               3-stage ring (2 stages for HD = 128);
//   warp 1      TMEM allocation and the MMA issuer: S_j = Q K_j^T into one of
//               two TMEM score buffers, and O_j = P_j V_j into one of two TMEM
//               output buffers, with S_{j+1} issued before O_j so the tensor
//               core works on the next scores while softmax runs;
//   warps 2..5  softmax and epilogue: the thread of TMEM lane r owns query
//               row r: row max (first pass over S_j), exp2 / row sum / bf16 P
//               (second pass) written in the UMMA K-major 128B-swizzled
//               layout, and the running output o = o * alpha + O_{j-1} kept
//               in registers (the PV product of each tile is not accumulated
//               in TMEM, so no TMEM read-modify-write is needed for the
//               rescale); finally o / l is stored through a swizzled staging
//               tile by a 3-D TMA store (rows past S are clipped by TMA).
//
// Every mbarrier wait is bounded (2 s wall clock); on expiry the role records
// an error code and stops, every role drains what it issued, TMEM is freed
// and the kernel returns: a broken invariant cannot hang the GPU.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

#include "common.cuh"

namespace ro {
namespace attn {

constexpr int kBM = 128;   // queries per tile
constexpr int kBN = 128;   // keys per tile
constexpr int kThreads = 192;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint64_t kDrainNs = 2000000ull;         // 2 ms

template <int HD>
struct Cfg {
  static constexpr int kAtoms = HD / 64;                  // 64-column swizzle atoms per row
  static constexpr int kQBytes = kBM * HD * 2;
  static constexpr int kKBytes = kBN * HD * 2;
  static constexpr int kStageBytes = 2 * kKBytes;         // K and V
  static constexpr int kStages = HD == 64 ? 3 : 2;
  static constexpr int kPBytes = kBM * kBN * 2;           // 32 KB
  // epilogue staging: its own buffer for HD = 64; for HD = 128 it reuses the
  // P buffers (free once the item's last PV product has completed)
  static constexpr bool kOutInP = HD > 64;
  static constexpr int kOutBytes = kOutInP ? 0 : kBM * HD * 2;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes =
      kQBytes + kStages * kStageBytes + 2 * kPBytes + kOutBytes + kBarBytes + 1024;
  static constexpr int kTmemS = 0;                        // 2 x 128 columns
  static constexpr int kTmemO = 2 * kBN;                  // 2 x HD columns
  static constexpr int kTmemCols = 512;
  static_assert(kTmemO + 2 * HD <= kTmemCols, "TMEM");
};

struct Params {
  int B, H, S;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  float* lse2;       // [B, H, S]
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
// Bounded wait: false when the error word is set or the limit expires (then
// `code` is recorded).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code,
                                          uint64_t limit = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (global_ns() - t0 > limit) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
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
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
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
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// UMMA shared-memory descriptor, 128B swizzle (sm_100 version bit).
//   K-major:  rows of 128 B, 8-row groups SBO = 1024 B apart.
//   MN-major: 64-element MN blocks LBO apart, 8-row K groups SBO = 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}
// kind::f16, bf16 x bf16 -> f32, M = 128.
template <int N, bool B_MN>
__device__ __forceinline__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((B_MN ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

// 2^x with the MUFU instruction (approximate, flush-to-zero; 2^-inf = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Issue `N` 32-column TMEM loads (lanes of this warp) and wait once for all of them.
template <int N>
__device__ __forceinline__ void tmem_ld32xN(uint32_t taddr, float (&v)[32 * N]) {
  uint32_t r[32 * N];
#pragma unroll
  for (int c = 0; c < N; ++c)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[32 * c + 0]), "=r"(r[32 * c + 1]), "=r"(r[32 * c + 2]), "=r"(r[32 * c + 3]),
          "=r"(r[32 * c + 4]), "=r"(r[32 * c + 5]), "=r"(r[32 * c + 6]), "=r"(r[32 * c + 7]),
          "=r"(r[32 * c + 8]), "=r"(r[32 * c + 9]), "=r"(r[32 * c + 10]), "=r"(r[32 * c + 11]),
          "=r"(r[32 * c + 12]), "=r"(r[32 * c + 13]), "=r"(r[32 * c + 14]), "=r"(r[32 * c + 15]),
          "=r"(r[32 * c + 16]), "=r"(r[32 * c + 17]), "=r"(r[32 * c + 18]), "=r"(r[32 * c + 19]),
          "=r"(r[32 * c + 20]), "=r"(r[32 * c + 21]), "=r"(r[32 * c + 22]), "=r"(r[32 * c + 23]),
          "=r"(r[32 * c + 24]), "=r"(r[32 * c + 25]), "=r"(r[32 * c + 26]), "=r"(r[32 * c + 27]),
          "=r"(r[32 * c + 28]), "=r"(r[32 * c + 29]), "=r"(r[32 * c + 30]), "=r"(r[32 * c + 31])
        : "r"(taddr + 32 * c));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32 * N; ++i) v[i] = __uint_as_float(r[i]);
}

// AND of `v` over the 128 softmax threads (named barrier 1): every one of them
// takes the same branch afterwards, so the named barriers that follow cannot
// be left with a missing participant.
__device__ __forceinline__ bool group_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "barrier.cta.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p) {
  using C = Cfg<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + C::kQBytes;
  uint8_t* sP = sKV + C::kStages * C::kStageBytes;
  uint8_t* sOut = C::kOutInP ? sP : sP + 2 * C::kPBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::kPBytes + C::kOutBytes);
  // barrier slots
  const uint32_t q_full = smem_u32(bars + 0), q_empty = smem_u32(bars + 1);
  auto kv_full = [&](int s) { return smem_u32(bars + 2 + s); };
  auto kv_empty = [&](int s) { return smem_u32(bars + 5 + s); };
  auto s_full = [&](int i) { return smem_u32(bars + 8 + i); };
  auto s_empty = [&](int i) { return smem_u32(bars + 10 + i); };
  auto p_full = [&](int i) { return smem_u32(bars + 12 + i); };
  auto o_full = [&](int i) { return smem_u32(bars + 14 + i); };
  auto o_empty = [&](int i) { return smem_u32(bars + 16 + i); };
  const uint32_t done_bar = smem_u32(bars + 18);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_qt = (p.S + kBM - 1) / kBM;
  const int items = num_qt * p.H * p.B;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_empty(i), 128);
      mbar_init(p_full(i), 128);
      mbar_init(o_full(i), 1);
      mbar_init(o_empty(i), 128);
    }
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Work items: index t -> query tile qt = num_qt - 1 - t / (H * B) (heaviest first),
  // then head-major within one query-tile index.
  auto coords = [&](int t, int& qt, int& h, int& b) {
    const int hb = p.H * p.B;
    qt = num_qt - 1 - t / hb;
    const int r = t % hb;
    b = r / p.H;
    h = r % p.H;
  };
  auto kv_tiles = [&](int qt) {
    if (!p.causal) return (p.S + kBN - 1) / kBN;
    const int last_row = min(qt * kBM + kBM - 1, p.S - 1);
    return last_row / kBN + 1;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      int issued = 0;  // K/V loads issued (for the drain)
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        if (!mbar_wait(q_empty, (local & 1) ^ 1, p.err, 1)) { ok = false; break; }
        mbar_expect_tx(q_full, C::kQBytes);
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a)
          tma_load_3d(smem_u32(sQ) + a * kBM * 128, &tmQ, q_full, h * HD + 64 * a, qt * kBM, b);
        const int n = kv_tiles(qt);
        for (int j = 0; j < n; ++j) {
          if (!mbar_wait(kv_empty(stage), phase ^ 1, p.err, 2)) { ok = false; break; }
          const uint32_t fb = kv_full(stage);
          mbar_expect_tx(fb, C::kStageBytes);
          const uint32_t sk = smem_u32(sKV) + stage * C::kStageBytes;
          const uint32_t sv = sk + C::kKBytes;
#pragma unroll
          for (int a = 0; a < C::kAtoms; ++a) {
            tma_load_3d(sk + a * kBN * 128, &tmK, fb, h * HD + 64 * a, j * kBN, b);
            tma_load_3d(sv + a * kBN * 128, &tmV, fb, h * HD + 64 * a, j * kBN, b);
          }
          ++issued;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // let the loads already issued land before the CTA can exit
        int s = stage, ph = phase;
        for (int i = 0; i < C::kStages && i < issued; ++i) {
          if (--s < 0) { s = C::kStages - 1; ph ^= 1; }
          mbar_wait(kv_full(s), ph, p.err, 0, kDrainNs);
        }
        mbar_wait(q_full, (local & 1), p.err, 0, kDrainNs);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc<kBN, false>();
      constexpr uint32_t idesc_o = instr_desc<HD, true>();
      int stage = 0;
      uint32_t phase = 0;
      int g = 0;  // kv-tile counter over all items: buffer g % 2, parity (g / 2) & 1
      int local = 0;
      bool ok = true;
      const uint32_t sq = smem_u32(sQ);
      const uint32_t sp = smem_u32(sP);
      // O_j = P_j V_j for kv tile counter gj held in `stage_j`
      auto issue_o = [&](int gj, int stage_j) -> bool {
        const int buf = gj & 1;
        const uint32_t par = (gj >> 1) & 1;
        if (!mbar_wait(p_full(buf), par, p.err, 5)) return false;
        if (!mbar_wait(o_empty(buf), par ^ 1, p.err, 6)) return false;
        tc_fence_after();
        const uint32_t tmem_o = tmem_base + C::kTmemO + buf * HD;
        const uint32_t pa = sp + buf * C::kPBytes;
        const uint32_t vb = smem_u32(sKV) + stage_j * C::kStageBytes + C::kKBytes;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          // A = P (K-major over keys: two 64-key atoms of [128 rows x 128 B])
          const uint64_t ad = smem_desc(pa + (k >> 2) * (kBM * 128) + (k & 3) * 32, 16, 1024);
          // B = V (MN-major: keys are K, head_dim is N; 64-wide N blocks kBN * 128 B apart)
          const uint64_t bd = smem_desc(vb + k * 16 * 128, kBN * 128, 1024);
          tc_mma(tmem_o, ad, bd, idesc_o, k != 0 ? 1u : 0u);
        }
        tc_commit(o_full(buf));
        tc_commit(kv_empty(stage_j));
        return true;
      };
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        (void)h;
        (void)b;
        const int n = kv_tiles(qt);
        if (!mbar_wait(q_full, local & 1, p.err, 3)) { ok = false; break; }
        int prev_stage = -1;
        for (int j = 0; j < n; ++j, ++g) {
          const int buf = g & 1;
          const uint32_t par = (g >> 1) & 1;
          if (!mbar_wait(kv_full(stage), phase, p.err, 4)) { ok = false; break; }
          if (!mbar_wait(s_empty(buf), par ^ 1, p.err, 7)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tmem_s = tmem_base + C::kTmemS + buf * kBN;
          const uint32_t kb = smem_u32(sKV) + stage * C::kStageBytes;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * (kBM * 128) + (k & 3) * 32;
            const uint64_t ad = smem_desc(sq + off, 16, 1024);
            const uint64_t bd = smem_desc(kb + (k >> 2) * (kBN * 128) + (k & 3) * 32, 16, 1024);
            tc_mma(tmem_s, ad, bd, idesc_s, k != 0 ? 1u : 0u);
          }
          tc_commit(s_full(buf));
          if (j == n - 1) tc_commit(q_empty);
          if (j > 0 && !issue_o(g - 1, prev_stage)) { ok = false; break; }
          prev_stage = stage;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (!issue_o(g - 1, prev_stage)) { ok = false; break; }
      }
      // every MMA issued so far completes before TMEM can be released
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, 0, kDrainNs);
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;             // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;      // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sp = smem_u32(sP);
    const uint32_t so = smem_u32(sOut);
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < items && ok; t += gridDim.x) {
      int qt, h, b;
      coords(t, qt, h, b);
      const int n = kv_tiles(qt);
      const int q_index = qt * kBM + row;
      float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
      float o[HD];
#pragma unroll
      for (int c = 0; c < HD; ++c) o[c] = 0.f;
      // accumulate O of kv counter gj into o with factor a
      auto take_o = [&](int gj, float a) -> bool {
        const int buf = gj & 1;
        if (!mbar_wait(o_full(buf), (gj >> 1) & 1, p.err, 9)) return false;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          float v[64];
          tmem_ld32xN<2>(tmem_base + lane_off + C::kTmemO + buf * HD + 64 * c, v);
#pragma unroll
          for (int i = 0; i < 64; ++i) o[64 * c + i] = fmaf(o[64 * c + i], a, v[i]);
        }
        tc_fence_before();
        mbar_arrive(o_empty(buf));
        return true;
      };
      if constexpr (C::kOutInP) {
        // the previous item's output store reads the P buffers: wait for it
        if (threadIdx.x == 64) bulk_wait_read_all();
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      bool good = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int buf = g & 1;
        if (!mbar_wait(s_full(buf), (g >> 1) & 1, p.err, 8)) { good = false; break; }
        tc_fence_after();
        const uint32_t ts = tmem_base + lane_off + C::kTmemS + buf * kBN;
        const int kv0 = j * kBN;
        // keys at column >= limit are masked for this row
        int limit = kBN;
        if (p.causal) limit = min(limit, q_index - kv0 + 1);
        limit = min(limit, p.S - kv0);
        const bool full = limit >= kBN;  // no masked column in this tile for this row
        const uint32_t prow = sp + buf * C::kPBytes + row * 128;
        float mx = -INFINITY, sum = 0.f, m_new, alpha;
        // P = exp2(s' - m_new) of columns [32c, 32c+32) as bf16 into the swizzled A-operand tile
        auto emit = [&](const float* v, int c) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = fast_exp2(fmaf(v[i], p.scale_log2, -m_new));
            const float p1 = fast_exp2(fmaf(v[i + 1], p.scale_log2, -m_new));
            sum += p0 + p1;
            packed[i / 2] = pack_bf16(p0, p1);
          }
          const uint32_t atom = prow + (c >> 1) * (kBM * 128);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t chunk = static_cast<uint32_t>(((c & 1) * 4 + q) ^ (row & 7));
            st_shared_v4(atom + chunk * 16, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          }
        };
        if constexpr (HD == 64) {
          // the whole score row fits in registers next to o[64]: one TMEM read
          float sv[kBN];
          tmem_ld32xN<4>(ts, sv);
          if (!full) {
#pragma unroll
            for (int i = 0; i < kBN; ++i)
              if (i >= limit) sv[i] = -INFINITY;
          }
#pragma unroll
          for (int i = 0; i < kBN; ++i) mx = fmaxf(mx, sv[i]);
          m_new = fmaxf(m, mx * p.scale_log2);
          alpha = fast_exp2(m - m_new);
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c) emit(sv + 32 * c, c);
        } else {
          // two passes over TMEM (o[128] leaves no room for the row)
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float v[64];
            tmem_ld32xN<2>(ts + 64 * h2, v);
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (full || 64 * h2 + i < limit) mx = fmaxf(mx, v[i]);
          }
          m_new = fmaxf(m, mx * p.scale_log2);
          alpha = fast_exp2(m - m_new);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float v[64];
            tmem_ld32xN<2>(ts + 64 * h2, v);
            if (!full) {
#pragma unroll
              for (int i = 0; i < 64; ++i)
                if (64 * h2 + i >= limit) v[i] = -INFINITY;
            }
            emit(v, 2 * h2);
            emit(v + 32, 2 * h2 + 1);
          }
        }
        tc_fence_before();
        mbar_arrive(s_empty(buf));  // this S buffer may be overwritten by S_{g+2}
        fence_async_smem();         // P (generic-proxy stores) visible to the tensor core
        mbar_arrive(p_full(buf));
        l = fmaf(l, alpha, sum);
        if (j > 0 && !take_o(g - 1, alpha_prev)) { good = false; break; }
        alpha_prev = alpha;
        m = m_new;
      }
      if (good) good = take_o(g - 1, alpha_prev);
      ok = group_all(good);
      if (!ok) break;
      // ---- epilogue: o / l -> bf16 staging (128B swizzle per 64-column atom) -> TMA store
      const float inv = l > 0.f ? 1.f / l : 0.f;
      // previous item's store must have read the staging tile
      if (threadIdx.x == 64) bulk_wait_read_all();
      asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
      for (int a = 0; a < C::kAtoms; ++a) {
        const uint32_t base = so + a * (kBM * 128) + row * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int c0 = 64 * a + 8 * q;
          const uint32_t chunk = static_cast<uint32_t>(q ^ (row & 7));
          st_shared_v4(base + chunk * 16, pack_bf16(o[c0] * inv, o[c0 + 1] * inv),
                       pack_bf16(o[c0 + 2] * inv, o[c0 + 3] * inv), pack_bf16(o[c0 + 4] * inv, o[c0 + 5] * inv),
                       pack_bf16(o[c0 + 6] * inv, o[c0 + 7] * inv));
        }
      }
      if (q_index < p.S)
        p.lse2[(static_cast<int64_t>(b) * p.H + h) * p.S + q_index] = m + log2f(l);
      fence_async_smem();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) tma_store_3d(&tmO, so + a * (kBM * 128), h * HD + 64 * a, qt * kBM, b);
        bulk_commit();
      }
    }
    if (threadIdx.x == 64) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols));
}

// ---------------------------------------------------------------------------
// Forward with eight softmax warps (two per TMEM lane quarter).  The warp
// pair of a lane quarter splits every 128-column score row into two 64-column
// halves: each half keeps its own running sum and the output columns
// [half * HD/2, (half + 1) * HD/2) in registers, and the two halves agree on
// the row maximum through shared memory once per tile.  Twice the warps of
// the four-warp kernel and half the work per warp: the softmax, which bounds
// this kernel, hides its latencies with two warps per SM sub-partition.
// Waits that gate a whole tile are done by one thread and published with a
// barrier reduction, so every softmax thread leaves a tile loop at the same
// point and the named barriers that follow always see all 256 threads.
constexpr int kThreads8 = 320;

__device__ __forceinline__ bool group256_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "barrier.cta.red.and.pred p, 1, 256, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group256_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int HD>
__global__ void __launch_bounds__(kThreads8, 1)
    attn_fwd8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p) {
  using C = Cfg<HD>;
  constexpr int kHalfO = HD / 2;  // output columns per warp of a pair
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + C::kQBytes;
  uint8_t* sP = sKV + C::kStages * C::kStageBytes;
  uint8_t* sOut = C::kOutInP ? sP : sP + 2 * C::kPBytes;
  // row maxima / sums exchanged by the two halves: [2 buffers][2 halves][128 rows]
  float* sX = reinterpret_cast<float*>(sP + 2 * C::kPBytes + C::kOutBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + 2 * 2 * 128);
  const uint32_t q_full = smem_u32(bars + 0), q_empty = smem_u32(bars + 1);
  auto kv_full = [&](int s) { return smem_u32(bars + 2 + s); };
  auto kv_empty = [&](int s) { return smem_u32(bars + 5 + s); };
  auto s_full = [&](int i) { return smem_u32(bars + 8 + i); };
  auto s_empty = [&](int i) { return smem_u32(bars + 10 + i); };
  auto p_full = [&](int i) { return smem_u32(bars + 12 + i); };
  auto o_full = [&](int i) { return smem_u32(bars + 14 + i); };
  auto o_empty = [&](int i) { return smem_u32(bars + 16 + i); };
  const uint32_t done_bar = smem_u32(bars + 18);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_qt = (p.S + kBM - 1) / kBM;
  const int items = num_qt * p.H * p.B;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_empty(i), 256);
      mbar_init(p_full(i), 256);
      mbar_init(o_full(i), 1);
      mbar_init(o_empty(i), 256);
    }
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto coords = [&](int t, int& qt, int& h, int& b) {
    const int hb = p.H * p.B;
    qt = num_qt - 1 - t / hb;
    const int r = t % hb;
    b = r / p.H;
    h = r % p.H;
  };
  auto kv_tiles = [&](int qt) {
    if (!p.causal) return (p.S + kBN - 1) / kBN;
    const int last_row = min(qt * kBM + kBM - 1, p.S - 1);
    return last_row / kBN + 1;
  };

  if (warp == 0) {
    // ---------------- TMA producer (as in attn_fwd_kernel) ----------------
    if (lane == 0) {
      int stage = 0, local = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        if (!mbar_wait(q_empty, (local & 1) ^ 1, p.err, 1)) { ok = false; break; }
        mbar_expect_tx(q_full, C::kQBytes);
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a)
          tma_load_3d(smem_u32(sQ) + a * kBM * 128, &tmQ, q_full, h * HD + 64 * a, qt * kBM, b);
        const int n = kv_tiles(qt);
        for (int j = 0; j < n; ++j) {
          if (!mbar_wait(kv_empty(stage), phase ^ 1, p.err, 2)) { ok = false; break; }
          const uint32_t fb = kv_full(stage);
          mbar_expect_tx(fb, C::kStageBytes);
          const uint32_t sk = smem_u32(sKV) + stage * C::kStageBytes;
          const uint32_t sv = sk + C::kKBytes;
#pragma unroll
          for (int a = 0; a < C::kAtoms; ++a) {
            tma_load_3d(sk + a * kBN * 128, &tmK, fb, h * HD + 64 * a, j * kBN, b);
            tma_load_3d(sv + a * kBN * 128, &tmV, fb, h * HD + 64 * a, j * kBN, b);
          }
          ++issued;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < C::kStages && i < issued; ++i) {
          if (--s < 0) { s = C::kStages - 1; ph ^= 1; }
          mbar_wait(kv_full(s), ph, p.err, 0, kDrainNs);
        }
        mbar_wait(q_full, local & 1, p.err, 0, kDrainNs);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (as in attn_fwd_kernel) ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc<kBN, false>();
      constexpr uint32_t idesc_o = instr_desc<HD, true>();
      int stage = 0, g = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t sq = smem_u32(sQ);
      const uint32_t sp = smem_u32(sP);
      auto issue_o = [&](int gj, int stage_j) -> bool {
        const int buf = gj & 1;
        const uint32_t par = (gj >> 1) & 1;
        if (!mbar_wait(p_full(buf), par, p.err, 5)) return false;
        if (!mbar_wait(o_empty(buf), par ^ 1, p.err, 6)) return false;
        tc_fence_after();
        const uint32_t tmem_o = tmem_base + C::kTmemO + buf * HD;
        const uint32_t pa = sp + buf * C::kPBytes;
        const uint32_t vb = smem_u32(sKV) + stage_j * C::kStageBytes + C::kKBytes;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          const uint64_t ad = smem_desc(pa + (k >> 2) * (kBM * 128) + (k & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc(vb + k * 16 * 128, kBN * 128, 1024);
          tc_mma(tmem_o, ad, bd, idesc_o, k != 0 ? 1u : 0u);
        }
        tc_commit(o_full(buf));
        tc_commit(kv_empty(stage_j));
        return true;
      };
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        const int n = kv_tiles(qt);
        if (!mbar_wait(q_full, local & 1, p.err, 3)) { ok = false; break; }
        int prev_stage = -1;
        for (int j = 0; j < n; ++j, ++g) {
          const int buf = g & 1;
          const uint32_t par = (g >> 1) & 1;
          if (!mbar_wait(kv_full(stage), phase, p.err, 4)) { ok = false; break; }
          if (!mbar_wait(s_empty(buf), par ^ 1, p.err, 7)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tmem_s = tmem_base + C::kTmemS + buf * kBN;
          const uint32_t kb = smem_u32(sKV) + stage * C::kStageBytes;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint32_t off = (k >> 2) * (kBM * 128) + (k & 3) * 32;
            tc_mma(tmem_s, smem_desc(sq + off, 16, 1024), smem_desc(kb + (k >> 2) * (kBN * 128) + (k & 3) * 32, 16, 1024),
                   idesc_s, k != 0 ? 1u : 0u);
          }
          tc_commit(s_full(buf));
          if (j == n - 1) tc_commit(q_empty);
          if (j > 0 && !issue_o(g - 1, prev_stage)) { ok = false; break; }
          prev_stage = stage;
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (!issue_o(g - 1, prev_stage)) { ok = false; break; }
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, 0, kDrainNs);
    }
  } else {
    // ---------------- softmax (warps 2..9) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;             // warps 2..5: columns 0..63, warps 6..9: 64..127
    const int row = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;             // 0..255
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sp = smem_u32(sP);
    const uint32_t so = smem_u32(sOut);
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < items && ok; t += gridDim.x) {
      int qt, h, b;
      coords(t, qt, h, b);
      const int n = kv_tiles(qt);
      const int q_index = qt * kBM + row;
      float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
      float o[kHalfO];
#pragma unroll
      for (int c = 0; c < kHalfO; ++c) o[c] = 0.f;
      if constexpr (C::kOutInP) {
        if (tid == 0) bulk_wait_read_all();
        group256_sync();
      }
      // o = o * a + (this half's columns of O_gj)
      auto take_o = [&](int gj, float a) {
        const int buf = gj & 1;
        float v[kHalfO];
        tmem_ld32xN<kHalfO / 32>(tmem_base + lane_off + C::kTmemO + buf * HD + half * kHalfO, v);
#pragma unroll
        for (int i = 0; i < kHalfO; ++i) o[i] = fmaf(o[i], a, v[i]);
        tc_fence_before();
        mbar_arrive(o_empty(buf));
      };
      bool good = true;
      for (int j = 0; j < n; ++j, ++g) {
        const int buf = g & 1;
        // one thread waits for S_g (and for O_{g-1}, issued right after S_g)
        bool w = true;
        if (tid == 0) {
          w = mbar_wait(s_full(buf), (g >> 1) & 1, p.err, 8);
          if (w && j > 0) w = mbar_wait(o_full((g - 1) & 1), ((g - 1) >> 1) & 1, p.err, 9);
        }
        if (!group256_all(w)) { good = false; break; }
        tc_fence_after();
        if (j > 0) take_o(g - 1, alpha_prev);
        const uint32_t ts = tmem_base + lane_off + C::kTmemS + buf * kBN + half * 64;
        const int kv0 = j * kBN + half * 64;
        int limit = 64;
        if (p.causal) limit = min(limit, q_index - kv0 + 1);
        limit = min(limit, p.S - kv0);
        float sv[64];
        tmem_ld32xN<2>(ts, sv);
        if (limit < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= limit) sv[i] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) mx = fmaxf(mx, sv[i]);
        // buffer g % 2: the write two tiles later comes after the consensus barrier
        // that every thread passes only once it has read this one
        float* xb = sX + buf * 256;
        xb[half * 128 + row] = mx;
        group256_sync();
        mx = fmaxf(mx, xb[(half ^ 1) * 128 + row]);
        const float m_new = fmaxf(m, mx * p.scale_log2);
        const float alpha = fast_exp2(m - m_new);
        float sum = 0.f;
        const uint32_t atom = sp + buf * C::kPBytes + half * (kBM * 128) + row * 128;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = fast_exp2(fmaf(sv[32 * c + i], p.scale_log2, -m_new));
            const float p1 = fast_exp2(fmaf(sv[32 * c + i + 1], p.scale_log2, -m_new));
            sum += p0 + p1;
            packed[i / 2] = pack_bf16(p0, p1);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t chunk = static_cast<uint32_t>((c * 4 + q) ^ (row & 7));
            st_shared_v4(atom + chunk * 16, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(s_empty(buf));
        fence_async_smem();
        mbar_arrive(p_full(buf));
        l = fmaf(l, alpha, sum);
        alpha_prev = alpha;
        m = m_new;
      }
      if (!good) { ok = false; break; }
      bool w = true;
      if (tid == 0) w = mbar_wait(o_full((g - 1) & 1), ((g - 1) >> 1) & 1, p.err, 9);
      if (!group256_all(w)) { ok = false; break; }
      tc_fence_after();
      take_o(g - 1, alpha_prev);
      // ---- epilogue: the row sum is the sum of the halves' sums
      sX[half * 128 + row] = l;
      if constexpr (!C::kOutInP) {
        if (tid == 0) bulk_wait_read_all();
      }
      group256_sync();
      const float l_all = l + sX[(half ^ 1) * 128 + row];
      const float inv = l_all > 0.f ? 1.f / l_all : 0.f;
      // this half's HD/2 columns: atom (half * HD/2) / 64, chunks (half * HD/2 % 64) / 8 ...
#pragma unroll
      for (int c0 = 0; c0 < kHalfO; c0 += 8) {
        const int col = half * kHalfO + c0;
        const uint32_t base = so + (col / 64) * (kBM * 128) + row * 128;
        const uint32_t chunk = static_cast<uint32_t>(((col % 64) / 8) ^ (row & 7));
        st_shared_v4(base + chunk * 16, pack_bf16(o[c0] * inv, o[c0 + 1] * inv),
                     pack_bf16(o[c0 + 2] * inv, o[c0 + 3] * inv), pack_bf16(o[c0 + 4] * inv, o[c0 + 5] * inv),
                     pack_bf16(o[c0 + 6] * inv, o[c0 + 7] * inv));
      }
      if (half == 0 && q_index < p.S)
        p.lse2[(static_cast<int64_t>(b) * p.H + h) * p.S + q_index] = m + log2f(l_all);
      fence_async_smem();
      group256_sync();
      if (tid == 0) {
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) tma_store_3d(&tmO, so + a * (kBM * 128), h * HD + 64 * a, qt * kBM, b);
        bulk_commit();
      }
    }
    if (tid == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols));
}

// ---------------------------------------------------------------------------
// Backward.  Deterministic (no atomics): two passes that each own their output
// tile, with the usual recomputation of P from lse2.
//
//   D        = rowsum(dO * O)                     (attn_bwd_prep_kernel)
//   P        = exp2(s * scale * log2e - lse2),   dS = P * (dP - D),  dP = dO V^T
//   dQ       = scale * dS K                       (query-stationary pass)
//   dK, dV   = scale * dS^T Q,  P^T dO            (key-stationary pass)
//
// Both passes are persistent one-CTA-per-SM kernels with the forward's warp
// roles: warp 0 TMA, warp 1 TMEM + MMA issuer, warps 2..5 the elementwise
// work on the rows of their TMEM lane quarter.  The recomputed scores and dP
// of the current tile share one TMEM buffer each; the next tile's products
// are issued as soon as the compute warps have read the current ones.

struct BwdParams {
  int B, H, S;
  float scale_log2;   // softmax scale * log2(e)
  float scale;        // softmax scale (gradient of the raw scores)
  int causal;
  const float* lse2;  // [B, H, S]
  const float* delta; // [B, H, S]
  int* err;
};

template <int HD>
struct BwdCfg {
  static constexpr int kAtoms = HD / 64;
  static constexpr int kTileBytes = 128 * HD * 2;       // one 128-row operand tile
  static constexpr int kStagesDQ = HD == 64 ? 3 : 2;    // streamed (K, V) pairs, dQ pass
  static constexpr int kStagesKV = HD == 64 ? 3 : 1;    // streamed (Q, dO) pairs, dK/dV pass
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kPBytes = 128 * 128 * 2;
  static constexpr int kBarBytes = 256;
  static constexpr int kStatBytes = 2 * 2 * 128 * 4;    // lse2 / delta of two query tiles
  static constexpr int kTmemS = 0, kTmemDP = 128, kTmemAcc = 256;
  static constexpr int kTmemCols = 512;
};

// D[b, h, s] = sum_c dO[b, s, h*hd + c] * O[b, s, h*hd + c]; one thread per (b, s, h).
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                     float* __restrict__ delta, int B, int S, int H, int hd, int64_t ldo,
                                     int64_t lddo) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(B) * S * H) return;
  const int h = static_cast<int>(idx % H);
  const int64_t bs = idx / H;
  const int s = static_cast<int>(bs % S);
  const int b = static_cast<int>(bs / S);
  const __nv_bfloat16* po = o + bs * ldo + static_cast<int64_t>(h) * hd;
  const __nv_bfloat16* pd = dout + bs * lddo + static_cast<int64_t>(h) * hd;
  float acc = 0.f;
  for (int c = 0; c < hd; c += 8) {
    float a[8], d[8];
    load_vec<__nv_bfloat16, 8>(po + c, a);
    load_vec<__nv_bfloat16, 8>(pd + c, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fmaf(a[i], d[i], acc);
  }
  delta[(static_cast<int64_t>(b) * H + h) * S + s] = acc;
}

// Store a 128 x HD fp32 accumulator row set (this thread's row, already
// scaled, in `v`) as bf16 into a 128B-swizzled staging tile.
template <int HD>
__device__ __forceinline__ void stage_row(uint32_t staging, int row, const float (&v)[HD]) {
#pragma unroll
  for (int a = 0; a < HD / 64; ++a) {
    const uint32_t base = staging + a * (128 * 128) + row * 128;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int c0 = 64 * a + 8 * q;
      const uint32_t chunk = static_cast<uint32_t>(q ^ (row & 7));
      st_shared_v4(base + chunk * 16, pack_bf16(v[c0], v[c0 + 1]), pack_bf16(v[c0 + 2], v[c0 + 3]),
                   pack_bf16(v[c0 + 4], v[c0 + 5]), pack_bf16(v[c0 + 6], v[c0 + 7]));
    }
  }
}

// The HD/2 columns [half * HD/2, (half + 1) * HD/2) of `row` (values in `v`)
// as bf16 into a 128B-swizzled staging tile.
template <int HD>
__device__ __forceinline__ void stage_row_half(uint32_t staging, int row, int half, const float (&v)[HD / 2]) {
#pragma unroll
  for (int c0 = 0; c0 < HD / 2; c0 += 8) {
    const int col = half * (HD / 2) + c0;
    const uint32_t base = staging + (col / 64) * (128 * 128) + row * 128;
    const uint32_t chunk = static_cast<uint32_t>(((col % 64) / 8) ^ (row & 7));
    st_shared_v4(base + chunk * 16, pack_bf16(v[c0], v[c0 + 1]), pack_bf16(v[c0 + 2], v[c0 + 3]),
                 pack_bf16(v[c0 + 4], v[c0 + 5]), pack_bf16(v[c0 + 6], v[c0 + 7]));
  }
}

// Write 32 bf16 values (16 packed words) of columns [32c, 32c+32) of `row`
// into a [128 x 128] K-major 128B-swizzled operand tile.
__device__ __forceinline__ void store_operand_chunk(uint32_t tile, int row, int c, const uint32_t (&w)[16]) {
  const uint32_t atom = tile + (c >> 1) * (128 * 128) + row * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t chunk = static_cast<uint32_t>(((c & 1) * 4 + q) ^ (row & 7));
    st_shared_v4(atom + chunk * 16, w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
}

template <int HD>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float (&v)[HD]) {
#pragma unroll
  for (int c = 0; c < HD / 32; ++c) {
    float t[32];
    tmem_ld32(taddr + 32 * c, t);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[32 * c + i] = t[i];
  }
}

// ---- dQ: query-stationary ------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kThreads8, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, BwdParams p) {
  using C = BwdCfg<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + C::kTileBytes;
  uint8_t* sKV = sDO + C::kTileBytes;
  uint8_t* sDS = sKV + C::kStagesDQ * C::kStageBytes;   // dS [128 q][128 keys]; also the output staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + C::kPBytes);
  const uint32_t q_full = smem_u32(bars + 0), q_empty = smem_u32(bars + 1);
  auto kv_full = [&](int s) { return smem_u32(bars + 2 + s); };
  auto kv_empty = [&](int s) { return smem_u32(bars + 5 + s); };
  const uint32_t st_full = smem_u32(bars + 8), st_empty = smem_u32(bars + 9);
  const uint32_t ds_full = smem_u32(bars + 10), ds_empty = smem_u32(bars + 11);
  const uint32_t acc_full = smem_u32(bars + 12), acc_empty = smem_u32(bars + 13);
  const uint32_t done_bar = smem_u32(bars + 14);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_qt = (p.S + 127) / 128;
  const int items = num_qt * p.H * p.B;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::kStagesDQ; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_empty, 256);
    mbar_init(ds_full, 256);
    mbar_init(ds_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto coords = [&](int t, int& qt, int& h, int& b) {
    const int hb = p.H * p.B;
    qt = num_qt - 1 - t / hb;
    const int r = t % hb;
    b = r / p.H;
    h = r % p.H;
  };
  auto kv_tiles = [&](int qt) {
    if (!p.causal) return (p.S + 127) / 128;
    return min(qt * 128 + 127, p.S - 1) / 128 + 1;
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, issued = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        if (!mbar_wait(q_empty, (local & 1) ^ 1, p.err, 21)) { ok = false; break; }
        mbar_expect_tx(q_full, 2 * C::kTileBytes);
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) {
          tma_load_3d(smem_u32(sQ) + a * 16384, &tmQ, q_full, h * HD + 64 * a, qt * 128, b);
          tma_load_3d(smem_u32(sDO) + a * 16384, &tmDO, q_full, h * HD + 64 * a, qt * 128, b);
        }
        const int n = kv_tiles(qt);
        for (int j = 0; j < n; ++j) {
          if (!mbar_wait(kv_empty(stage), phase ^ 1, p.err, 22)) { ok = false; break; }
          const uint32_t fb = kv_full(stage);
          mbar_expect_tx(fb, C::kStageBytes);
          const uint32_t sk = smem_u32(sKV) + stage * C::kStageBytes;
#pragma unroll
          for (int a = 0; a < C::kAtoms; ++a) {
            tma_load_3d(sk + a * 16384, &tmK, fb, h * HD + 64 * a, j * 128, b);
            tma_load_3d(sk + C::kTileBytes + a * 16384, &tmV, fb, h * HD + 64 * a, j * 128, b);
          }
          ++issued;
          if (++stage == C::kStagesDQ) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < C::kStagesDQ && i < issued; ++i) {
          if (--s < 0) { s = C::kStagesDQ - 1; ph ^= 1; }
          mbar_wait(kv_full(s), ph, p.err, 0, kDrainNs);
        }
        mbar_wait(q_full, local & 1, p.err, 0, kDrainNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc<128, false>();
      constexpr uint32_t idesc_dq = instr_desc<HD, true>();
      const uint32_t sq = smem_u32(sQ), sdo = smem_u32(sDO), sds = smem_u32(sDS);
      int stage = 0, local = 0, g = 0;
      uint32_t phase = 0;
      bool ok = true;
      // S = Q K^T and dP = dO V^T of the K/V pair in `st` (g: tile counter for st_empty parity)
      auto issue_s = [&](int st, int gg) -> bool {
        if (!mbar_wait(kv_full(st), (gg / C::kStagesDQ) & 1, p.err, 23)) return false;
        if (!mbar_wait(st_empty, (gg & 1) ^ 1, p.err, 24)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(sKV) + st * C::kStageBytes;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          tc_mma(tmem_base + C::kTmemS, smem_desc(sq + off, 16, 1024), smem_desc(kb + off, 16, 1024), idesc_s,
                 k != 0 ? 1u : 0u);
          tc_mma(tmem_base + C::kTmemDP, smem_desc(sdo + off, 16, 1024),
                 smem_desc(kb + C::kTileBytes + off, 16, 1024), idesc_s, k != 0 ? 1u : 0u);
        }
        tc_commit(st_full);
        return true;
      };
      (void)phase;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int qt, h, b;
        coords(t, qt, h, b);
        (void)h;
        (void)b;
        const int n = kv_tiles(qt);
        if (!mbar_wait(q_full, local & 1, p.err, 25)) { ok = false; break; }
        if (!mbar_wait(acc_empty, (local & 1) ^ 1, p.err, 26)) { ok = false; break; }
        int st_j = stage;
        if (!issue_s(stage, g)) { ok = false; break; }
        for (int j = 0; j < n; ++j, ++g) {
          const int st_next = (st_j + 1) % C::kStagesDQ;
          if (j + 1 < n && !issue_s(st_next, g + 1)) { ok = false; break; }
          if (j + 1 == n) tc_commit(q_empty);
          // dQ += dS_j K_j  (A = dS K-major over keys; B = K_j MN-major, N = head_dim)
          if (!mbar_wait(ds_full, g & 1, p.err, 27)) { ok = false; break; }
          tc_fence_after();
          const uint32_t kb = smem_u32(sKV) + st_j * C::kStageBytes;
#pragma unroll
          for (int k = 0; k < 128 / 16; ++k) {
            const uint64_t ad = smem_desc(sds + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc(kb + k * 16 * 128, 128 * 128, 1024);
            tc_mma(tmem_base + C::kTmemAcc, ad, bd, idesc_dq, (j | k) != 0 ? 1u : 0u);
          }
          tc_commit(ds_empty);
          tc_commit(kv_empty(st_j));
          st_j = st_next;
        }
        stage = st_j;
        if (!ok) break;
        tc_commit(acc_full);
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, 0, kDrainNs);
    }
  } else {
    // eight compute warps: the pair of a lane quarter splits the 128 key columns
    // (and the head_dim columns of dQ) into two halves
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int tid = threadIdx.x - 64;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sds = smem_u32(sDS);
    int g = 0, local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
      int qt, h, b;
      coords(t, qt, h, b);
      const int n = kv_tiles(qt);
      const int q_index = qt * 128 + row;
      const int64_t stat = (static_cast<int64_t>(b) * p.H + h) * p.S + min(q_index, p.S - 1);
      const float lse = q_index < p.S ? p.lse2[stat] : INFINITY;
      const float dlt = q_index < p.S ? p.delta[stat] : 0.f;
      // the previous item's dQ store reads the dS buffer (it doubles as staging)
      if (tid == 0) bulk_wait_read_all();
      group256_sync();
      bool good = true;
      for (int j = 0; j < n; ++j, ++g) {
        bool w = true;
        if (tid == 0) w = mbar_wait(st_full, g & 1, p.err, 28) && mbar_wait(ds_empty, (g & 1) ^ 1, p.err, 29);
        if (!group256_all(w)) { good = false; break; }
        tc_fence_after();
        const int kv0 = j * 128 + half * 64;
        int limit = 64;
        if (p.causal) limit = min(limit, q_index - kv0 + 1);
        limit = min(limit, p.S - kv0);
        const bool full = limit >= 64;
        float s[64], dp[64];
        tmem_ld32xN<2>(tmem_base + lane_off + C::kTmemS + half * 64, s);
        tmem_ld32xN<2>(tmem_base + lane_off + C::kTmemDP + half * 64, dp);
        tc_fence_before();
        mbar_arrive(st_empty);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t w2[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int col = 32 * c + i;
            float p0 = fast_exp2(fmaf(s[col], p.scale_log2, -lse));
            float p1 = fast_exp2(fmaf(s[col + 1], p.scale_log2, -lse));
            if (!full) {
              p0 = col < limit ? p0 : 0.f;
              p1 = col + 1 < limit ? p1 : 0.f;
            }
            w2[i / 2] = pack_bf16(p0 * (dp[col] - dlt), p1 * (dp[col + 1] - dlt));
          }
          store_operand_chunk(sds, row, 2 * half + c, w2);
        }
        fence_async_smem();
        mbar_arrive(ds_full);
      }
      if (!good) { ok = false; break; }
      // epilogue: dQ = scale * acc -> bf16 -> staging (the dS buffer) -> TMA store;
      // the last dQ product read dS, and it has completed once acc_full fired
      bool w = true;
      if (tid == 0) w = mbar_wait(acc_full, local & 1, p.err, 30);
      if (!group256_all(w)) { ok = false; break; }
      tc_fence_after();
      float v[HD / 2];
      tmem_ld32xN<HD / 64>(tmem_base + lane_off + C::kTmemAcc + half * (HD / 2), v);
      tc_fence_before();
      mbar_arrive(acc_empty);
#pragma unroll
      for (int c = 0; c < HD / 2; ++c) v[c] *= p.scale;
      stage_row_half<HD>(sds, row, half, v);
      fence_async_smem();
      group256_sync();
      if (tid == 0) {
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) tma_store_3d(&tmDQ, sds + a * 16384, h * HD + 64 * a, qt * 128, b);
        bulk_commit();
      }
    }
    if (tid == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols));
}

// ---- dK, dV: key-stationary ----------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kThreads8, 1)
    attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                         const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                         BwdParams p) {
  using C = BwdCfg<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::kTileBytes;
  uint8_t* sQD = sV + C::kTileBytes;                  // ring of (Q, dO) pairs
  uint8_t* sPT = sQD + C::kStagesKV * C::kStageBytes;   // P^T  [128 keys][128 queries]; staging for dV
  uint8_t* sDST = sPT + C::kPBytes;                    // dS^T [128 keys][128 queries]; staging for dK
  float* sStat = reinterpret_cast<float*>(sDST + C::kPBytes);  // [2][lse2 128 | delta 128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sStat) + C::kStatBytes);
  const uint32_t kv_full = smem_u32(bars + 0), kv_empty = smem_u32(bars + 1);
  auto qd_full = [&](int s) { return smem_u32(bars + 2 + s); };
  auto qd_empty = [&](int s) { return smem_u32(bars + 5 + s); };
  const uint32_t st_full = smem_u32(bars + 8), st_empty = smem_u32(bars + 9);
  const uint32_t pd_full = smem_u32(bars + 10), pd_empty = smem_u32(bars + 11);
  const uint32_t acc_full = smem_u32(bars + 12), acc_empty = smem_u32(bars + 13);
  const uint32_t done_bar = smem_u32(bars + 14);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_t = (p.S + 127) / 128;
  const int items = num_t * p.H * p.B;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < C::kStagesKV; ++s) {
      mbar_init(qd_full(s), 1);
      mbar_init(qd_empty(s), 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_empty, 256);
    mbar_init(pd_full, 256);
    mbar_init(pd_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(done_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_async_smem();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // items: key tile kt, lightest-last (key tile 0 sees every query tile under the causal mask)
  auto coords = [&](int t, int& kt, int& h, int& b) {
    const int hb = p.H * p.B;
    kt = t / hb;
    const int r = t % hb;
    b = r / p.H;
    h = r % p.H;
  };
  auto first_qt = [&](int kt) { return p.causal ? kt : 0; };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, issued = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int kt, h, b;
        coords(t, kt, h, b);
        if (!mbar_wait(kv_empty, (local & 1) ^ 1, p.err, 41)) { ok = false; break; }
        mbar_expect_tx(kv_full, 2 * C::kTileBytes);
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) {
          tma_load_3d(smem_u32(sK) + a * 16384, &tmK, kv_full, h * HD + 64 * a, kt * 128, b);
          tma_load_3d(smem_u32(sV) + a * 16384, &tmV, kv_full, h * HD + 64 * a, kt * 128, b);
        }
        for (int i = first_qt(kt); i < num_t; ++i) {
          if (!mbar_wait(qd_empty(stage), phase ^ 1, p.err, 42)) { ok = false; break; }
          const uint32_t fb = qd_full(stage);
          mbar_expect_tx(fb, C::kStageBytes);
          const uint32_t sq = smem_u32(sQD) + stage * C::kStageBytes;
#pragma unroll
          for (int a = 0; a < C::kAtoms; ++a) {
            tma_load_3d(sq + a * 16384, &tmQ, fb, h * HD + 64 * a, i * 128, b);
            tma_load_3d(sq + C::kTileBytes + a * 16384, &tmDO, fb, h * HD + 64 * a, i * 128, b);
          }
          ++issued;
          if (++stage == C::kStagesKV) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < C::kStagesKV && i < issued; ++i) {
          if (--s < 0) { s = C::kStagesKV - 1; ph ^= 1; }
          mbar_wait(qd_full(s), ph, p.err, 0, kDrainNs);
        }
        mbar_wait(kv_full, local & 1, p.err, 0, kDrainNs);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc<128, false>();
      constexpr uint32_t idesc_acc = instr_desc<HD, true>();
      const uint32_t sk = smem_u32(sK), sv = smem_u32(sV), spt = smem_u32(sPT), sdst = smem_u32(sDST);
      int stage = 0, local = 0, g = 0;
      bool ok = true;
      // S^T = K Q_i^T and dP^T = V dO_i^T of the (Q, dO) pair in `st`
      auto issue_s = [&](int st, int gg) -> bool {
        if (!mbar_wait(qd_full(st), (gg / C::kStagesKV) & 1, p.err, 43)) return false;
        if (!mbar_wait(st_empty, (gg & 1) ^ 1, p.err, 44)) return false;
        tc_fence_after();
        const uint32_t qb = smem_u32(sQD) + st * C::kStageBytes;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          tc_mma(tmem_base + C::kTmemS, smem_desc(sk + off, 16, 1024), smem_desc(qb + off, 16, 1024), idesc_s,
                 k != 0 ? 1u : 0u);
          tc_mma(tmem_base + C::kTmemDP, smem_desc(sv + off, 16, 1024),
                 smem_desc(qb + C::kTileBytes + off, 16, 1024), idesc_s, k != 0 ? 1u : 0u);
        }
        tc_commit(st_full);
        return true;
      };
      for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
        int kt, h, b;
        coords(t, kt, h, b);
        (void)h;
        (void)b;
        const int i0 = first_qt(kt);
        const int n = num_t - i0;
        if (!mbar_wait(kv_full, local & 1, p.err, 45)) { ok = false; break; }
        if (!mbar_wait(acc_empty, (local & 1) ^ 1, p.err, 46)) { ok = false; break; }
        int st_i = stage;
        if (!issue_s(stage, g)) { ok = false; break; }
        for (int i = 0; i < n; ++i, ++g) {
          const int st_next = (st_i + 1) % C::kStagesKV;
          // with two or more stages the next pair's products go first; with one
          // stage the next pair can only land after this pair's products
          if (C::kStagesKV > 1 && i + 1 < n && !issue_s(st_next, g + 1)) { ok = false; break; }
          // dV += P^T dO_i, dK += dS^T Q_i  (A K-major over queries; B MN-major, N = head_dim)
          if (!mbar_wait(pd_full, g & 1, p.err, 47)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qb = smem_u32(sQD) + st_i * C::kStageBytes;
#pragma unroll
          for (int k = 0; k < 128 / 16; ++k) {
            const uint32_t aoff = (k >> 2) * 16384 + (k & 3) * 32;
            const uint32_t boff = k * 16 * 128;
            const uint32_t acc = (i | k) != 0 ? 1u : 0u;
            tc_mma(tmem_base + C::kTmemAcc, smem_desc(spt + aoff, 16, 1024),
                   smem_desc(qb + C::kTileBytes + boff, 128 * 128, 1024), idesc_acc, acc);
            tc_mma(tmem_base + C::kTmemAcc + HD, smem_desc(sdst + aoff, 16, 1024),
                   smem_desc(qb + boff, 128 * 128, 1024), idesc_acc, acc);
          }
          tc_commit(pd_empty);
          tc_commit(qd_empty(st_i));
          if (C::kStagesKV == 1 && i + 1 < n && !issue_s(st_next, g + 1)) { ok = false; break; }
          st_i = st_next;
        }
        stage = st_i;
        if (!ok) break;
        tc_commit(kv_empty);
        tc_commit(acc_full);
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, 0, kDrainNs);
    }
  } else {
    // eight compute warps: the pair of a lane quarter splits the 128 query
    // columns (and the head_dim columns of dK and dV) into two halves
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;          // key row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int tid = threadIdx.x - 64;             // 0..255
    const uint32_t spt = smem_u32(sPT), sdst = smem_u32(sDST);
    int g = 0, local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < items && ok; t += gridDim.x, ++local) {
      int kt, h, b;
      coords(t, kt, h, b);
      const int i0 = first_qt(kt);
      const int n = num_t - i0;
      const int k_index = kt * 128 + row;
      const int64_t stat_row = (static_cast<int64_t>(b) * p.H + h) * p.S;
      // the previous item's dK / dV stores read the P^T and dS^T buffers
      if (tid == 0) bulk_wait_read_all();
      group256_sync();
      bool good = true;
      for (int i = 0; i < n; ++i, ++g) {
        const int q0 = (i0 + i) * 128;
        // lse2 / delta of this query tile (buffer g % 2); masked columns get lse = inf
        float* st = sStat + (g & 1) * 256;
        if (tid < 128) {
          const int qi = q0 + tid;
          st[tid] = qi < p.S ? p.lse2[stat_row + qi] : INFINITY;
          st[128 + tid] = qi < p.S ? p.delta[stat_row + qi] : 0.f;
        }
        // one thread waits for the products and the free operand buffers; the
        // group barrier publishes the statistics and the outcome to all 256
        bool w = true;
        if (tid == 0) w = mbar_wait(st_full, g & 1, p.err, 48) && mbar_wait(pd_empty, (g & 1) ^ 1, p.err, 49);
        if (!group256_all(w)) { good = false; break; }
        tc_fence_after();
        float s2[64], dp[64];
        tmem_ld32xN<2>(tmem_base + lane_off + C::kTmemS + half * 64, s2);
        tmem_ld32xN<2>(tmem_base + lane_off + C::kTmemDP + half * 64, dp);
        tc_fence_before();
        mbar_arrive(st_empty);
        // query column c (of this half) is allowed for this key when q0 + c >= k_index
        const int lo = p.causal ? k_index - q0 - half * 64 : 0;
        const float* lse = st + half * 64;
        const float* dlt = st + 128 + half * 64;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t wp[16], wd[16];
#pragma unroll
          for (int i2 = 0; i2 < 32; i2 += 2) {
            const int col = 32 * c + i2;
            float p0 = fast_exp2(fmaf(s2[col], p.scale_log2, -lse[col]));
            float p1 = fast_exp2(fmaf(s2[col + 1], p.scale_log2, -lse[col + 1]));
            if (lo > 0) {
              p0 = col >= lo ? p0 : 0.f;
              p1 = col + 1 >= lo ? p1 : 0.f;
            }
            wp[i2 / 2] = pack_bf16(p0, p1);
            wd[i2 / 2] = pack_bf16(p0 * (dp[col] - dlt[col]), p1 * (dp[col + 1] - dlt[col + 1]));
          }
          store_operand_chunk(spt, row, 2 * half + c, wp);
          store_operand_chunk(sdst, row, 2 * half + c, wd);
        }
        fence_async_smem();
        mbar_arrive(pd_full);
      }
      if (!good) { ok = false; break; }
      bool w = true;
      if (tid == 0) w = mbar_wait(acc_full, local & 1, p.err, 50);
      if (!group256_all(w)) { ok = false; break; }
      tc_fence_after();
      float v[HD / 2];
      tmem_ld32xN<HD / 64>(tmem_base + lane_off + C::kTmemAcc + half * (HD / 2), v);        // dV
      stage_row_half<HD>(spt, row, half, v);
      tmem_ld32xN<HD / 64>(tmem_base + lane_off + C::kTmemAcc + HD + half * (HD / 2), v);   // dK
      tc_fence_before();
      mbar_arrive(acc_empty);
#pragma unroll
      for (int c = 0; c < HD / 2; ++c) v[c] *= p.scale;
      stage_row_half<HD>(sdst, row, half, v);
      fence_async_smem();
      group256_sync();
      if (tid == 0) {
#pragma unroll
        for (int a = 0; a < C::kAtoms; ++a) {
          tma_store_3d(&tmDV, spt + a * 16384, h * HD + 64 * a, kt * 128, b);
          tma_store_3d(&tmDK, sdst + a * 16384, h * HD + 64 * a, kt * 128, b);
        }
        bulk_commit();
      }
    }
    if (tid == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::kTmemCols));
}

// ---------------------------------------------------------------------------
// Host side.

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                              CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
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

// 3-D bf16 map over [B, S, ld] token-major planes (inner extent `cols`);
// box = {64, 128, 1}, 128B swizzle; rows past S read as zero / are not written.
static bool make_plane_map(CUtensorMap* map, const void* base, int B, int S, int64_t cols, int64_t ld) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(ld * 2 * S)};
  cuuint32_t box[3] = {64u, 128u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int HD>
static int launch_fwd(const void* q, const void* k, const void* v, void* o, int64_t ld, int64_t ldo, Params p,
                      cudaStream_t stream) {
  using C = Cfg<HD>;
  CUtensorMap mq, mk, mv, mo;
  const int64_t cols = static_cast<int64_t>(p.H) * HD;
  if (!make_plane_map(&mq, q, p.B, p.S, cols, ld) || !make_plane_map(&mk, k, p.B, p.S, cols, ld) ||
      !make_plane_map(&mv, v, p.B, p.S, cols, ld) || !make_plane_map(&mo, o, p.B, p.S, cols, ldo))
    return -3;
  static_assert(C::kSmemBytes <= 232448, "exceeds the 227 KB per-CTA shared memory of sm_100");
  // the eight-softmax-warp kernel needs 2 KB more shared memory (row exchange);
  // RO_ATTN_FWD_WARPS=8 selects it (measured slower than the four-warp kernel
  // at the 18-layer shape: 0.270 against 0.207 ms)
  // (head_dim 128 leaves no room for it: that size runs the four-warp kernel)
  constexpr int kSmem8 = C::kSmemBytes + 2 * 2 * 128 * 4;
  constexpr bool kHas8 = HD == 64;
  static_assert(!kHas8 || kSmem8 <= 232448, "exceeds the 227 KB per-CTA shared memory of sm_100");
  static const bool four_warps = [] {
    const char* v = std::getenv("RO_ATTN_FWD_WARPS");
    return !(v != nullptr && v[0] == '8');
  }();
  static int configured = 0;
  if (configured == 0) {
    const bool a = cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::kSmemBytes) == cudaSuccess;
    const bool b = !kHas8 || cudaFuncSetAttribute(attn_fwd8_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  kSmem8) == cudaSuccess;
    configured = a && b ? 1 : -1;
    cudaGetLastError();
  }
  if (configured < 0) return -4;
  const int items = ((p.S + kBM - 1) / kBM) * p.H * p.B;
  int grid = num_sms();
  if (items < grid) grid = items;
  if constexpr (kHas8) {
    if (!four_warps) {
      attn_fwd8_kernel<HD><<<grid, kThreads8, kSmem8, stream>>>(mq, mk, mv, mo, p);
      return static_cast<int>(cudaGetLastError());
    }
  }
  attn_fwd_kernel<HD><<<grid, kThreads, C::kSmemBytes, stream>>>(mq, mk, mv, mo, p);
  return static_cast<int>(cudaGetLastError());
}

template <int HD>
static int launch_bwd(const void* q, const void* k, const void* v, int64_t ld, const void* o, const void* dout,
                      void* dq, void* dk, void* dv, int64_t ld2, float* delta, BwdParams p, cudaStream_t stream) {
  using C = BwdCfg<HD>;
  const int64_t cols = static_cast<int64_t>(p.H) * HD;
  CUtensorMap mq, mk, mv, mdo, mdq, mdk, mdv;
  if (!make_plane_map(&mq, q, p.B, p.S, cols, ld) || !make_plane_map(&mk, k, p.B, p.S, cols, ld) ||
      !make_plane_map(&mv, v, p.B, p.S, cols, ld) || !make_plane_map(&mdo, dout, p.B, p.S, cols, ld2) ||
      !make_plane_map(&mdq, dq, p.B, p.S, cols, ld2) || !make_plane_map(&mdk, dk, p.B, p.S, cols, ld2) ||
      !make_plane_map(&mdv, dv, p.B, p.S, cols, ld2))
    return -3;
  constexpr int kSmemDQ = 2 * C::kTileBytes + C::kStagesDQ * C::kStageBytes + C::kPBytes + C::kBarBytes + 1024;
  constexpr int kSmemKV = 2 * C::kTileBytes + C::kStagesKV * C::kStageBytes + 2 * C::kPBytes + C::kStatBytes +
                          C::kBarBytes + 1024;
  static_assert(kSmemDQ <= 232448 && kSmemKV <= 232448, "exceeds the 227 KB per-CTA shared memory of sm_100");
  static int configured = 0;
  if (configured == 0) {
    const bool a = cudaFuncSetAttribute(attn_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmemDQ) == cudaSuccess;
    const bool b = cudaFuncSetAttribute(attn_bwd_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmemKV) == cudaSuccess;
    configured = a && b ? 1 : -1;
    cudaGetLastError();
  }
  if (configured < 0) return -4;
  const int64_t rows = static_cast<int64_t>(p.B) * p.S * p.H;
  attn_bwd_prep_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(dout), delta, p.B, p.S, p.H, HD, ld2,
      ld2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  p.delta = delta;
  const int items = ((p.S + 127) / 128) * p.H * p.B;
  int grid = num_sms();
  if (items < grid) grid = items;
  attn_bwd_dkdv_kernel<HD><<<grid, kThreads8, kSmemKV, stream>>>(mq, mk, mv, mdo, mdk, mdv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  attn_bwd_dq_kernel<HD><<<grid, kThreads8, kSmemDQ, stream>>>(mq, mk, mv, mdo, mdq, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace attn

// Backward of attention_forward: dq, dk, dv [B, S, ld2] bf16 from q, k, v
// [B, S, ld] and o, dout [B, S, ld2] (ld2 >= H*hd), lse2 [B, H, S] from the
// forward; delta is fp32 [B, H, S] scratch.  Deterministic.  Returns 0 on
// success, negative for unsupported arguments, or a CUDA error.
int attention_backward(const void* q, const void* k, const void* v, int64_t ld, const void* o, const void* dout,
                       const float* lse2, void* dq, void* dk, void* dv, int64_t ld2, float* delta, int B, int S,
                       int H, int hd, float scale, bool causal, int* err, cudaStream_t stream) {
  using namespace attn;
  if (B <= 0 || S <= 0 || H <= 0 || (hd != 64 && hd != 128)) return -1;
  if (ld < static_cast<int64_t>(H) * hd || ld % 8 || ld2 < static_cast<int64_t>(H) * hd || ld2 % 8) return -1;
  for (const void* t : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (!aligned16(t)) return -2;
  BwdParams p{B, H, S, scale * 1.4426950408889634f, scale, causal ? 1 : 0, lse2, nullptr, err};
  if (hd == 64) return launch_bwd<64>(q, k, v, ld, o, dout, dq, dk, dv, ld2, delta, p, stream);
  return launch_bwd<128>(q, k, v, ld, o, dout, dq, dk, dv, ld2, delta, p, stream);
}

// Causal (or full) attention forward over token-major bf16 planes q, k, v
// [B, S, ld] and o [B, S, ldo] with H heads of width hd (64 or 128) at columns
// h*hd; lse2 fp32 [B, H, S] (log2 units of the scaled scores).  Returns 0 on
// success, negative for unsupported arguments (the caller falls back), or a
// CUDA error.
int attention_forward(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int S, int H,
                      int hd, int64_t ld, int64_t ldo, float scale, bool causal, int* err, cudaStream_t stream) {
  using namespace attn;
  if (B <= 0 || S <= 0 || H <= 0 || (hd != 64 && hd != 128)) return -1;
  if (ld < static_cast<int64_t>(H) * hd || ld % 8 || ldo < static_cast<int64_t>(H) * hd || ldo % 8) return -1;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return -2;
  if (static_cast<int64_t>(B) * S > (1ll << 31) - 1) return -1;
  Params p{B, H, S, scale * 1.4426950408889634f, causal ? 1 : 0, lse2, err};
  if (hd == 64) return launch_fwd<64>(q, k, v, o, ld, ldo, p, stream);
  return launch_fwd<128>(q, k, v, o, ld, ldo, p, stream);
}

}  // namespace ro
