// 2-SM GEMM (tcgen05.mma.cta_group::2) with fused epilogues.
//
//   acc (M x N) = A (M x K) . B (N x K)^T          bf16 operands, fp32 accumulator
//
// A and B are K-major (an activation [M, K] and an nn.Linear weight [N, K]).
// A CTA pair (a cluster of 2) owns a 256 x 256 output tile: each CTA stages
// 128 rows of A and 128 rows of B per 64-wide K block, the leader issues
// M=256 N=256 K=16 MMAs that read both CTAs' shared memory, and each CTA's
// tensor memory receives its own 128 rows of the accumulator.
//
// Per CTA (320 threads; 576 for the GRAIN backward; one CTA per SM).  The
// grid has one cluster per output tile; a running cluster takes over the
// tiles of clusters that have not started (cluster launch control) and
// passes each tile index to both CTAs through a small shared-memory ring, so
// the clusters that run do all the work whatever SMs other kernels hold.
//   warp 0      TMA producer: loads into this CTA's ring; the completion
//               bytes of both CTAs land on the leader's `full` barrier; the
//               leader's producer thread is also the tile scheduler;
//   warp 1      TMEM allocation (both CTAs) and, in the leader, the MMA
//               issuer; each K block is released to both producers with a
//               multicast tcgen05.commit (no multicast loads are used);
//   warps 2..9  epilogue: 8 warps, two per TMEM lane quarter, each owning 32
//               rows x 128 columns of the tile; results go through a
//               128B-swizzled staging buffer to TMA bulk stores.
// The accumulator is double-buffered in TMEM (2 x 256 columns = all 512), so
// the epilogue of tile t overlaps the main loop of tile t+1.
//
// Epilogues:
//   kStore      C = bf16(acc)
//   kGrainFwd   GRAIN activation fused behind the in-projection (group width
//               256 = one tile width): H = bf16(acc) is stored, rho per row is
//               the RMS of H over the group, Y = rho * P(t)/Q(|t|) with
//               t = H / rho is stored (the arithmetic of
//               ro::grain::forward_packed_kernel).
//   kGrainBwd   GRAIN backward fused behind the out-projection's input
//               gradient: gy stays in TMEM, the forward H slice is fetched by
//               TMA, dH is stored and per-tile coefficient partials written.
//   kQkvRope    q/k/v projection with RoPE applied to q and k, stored as
//               three token-major planes through a 3-D TMA store.
//
// Every mbarrier wait is bounded by a wall-clock limit; on expiry the waiting
// role records an error code in `err` and stops.  Every thread of both CTAs
// reaches the final cluster barrier exactly once, TMEM is released, and the
// kernel returns, so a broken invariant cannot hang the GPU.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "packed.cuh"

namespace ro {
namespace gemm2 {

constexpr int kBM = 256;         // rows per CTA pair
constexpr int kBN = 256;         // columns per tile
constexpr int kBK = 64;          // 64 bf16 = 128 B = one swizzle row
constexpr int kHalfM = 128;      // rows per CTA
constexpr int kHalfN = 128;      // B rows staged per CTA
constexpr int kStagesMax = 5;
constexpr int kABytes = kHalfM * kBK * 2;          // 16 KB
constexpr int kBBytes = kHalfN * kBK * 2;          // 16 KB
constexpr int kStageBytes = kABytes + kBBytes;     // 32 KB per CTA
constexpr int kStageOut = 32 * 128;                // one 32 x 64 bf16 staging tile
constexpr int kOutBytes = 64 * 1024;               // output staging per CTA
constexpr int kBarBytes = 512;   // mbarriers, TMEM slot, tile scheduler ring
constexpr int kSched = 4;        // tile scheduler ring depth

enum Epilogue : int { kStore = 0, kGrainFwd = 1, kGrainBwd = 2, kQkvRope = 3 };

// Per-epilogue shape: the GRAIN backward's epilogue is the heaviest (the
// whole activation backward runs there), so it gets 16 warps (four per TMEM
// lane quarter, 64 columns each, one staging tile each) and a 4-stage ring.
template <int EPI>
struct Traits {
  static constexpr int kWarps = EPI == kGrainBwd ? 16 : 8;
  static constexpr int kThreads = 64 + 32 * kWarps;
  static constexpr int kSlice = 256 / (kWarps / 4);     // columns per warp
  static constexpr int kStages = EPI == kGrainBwd ? 4 : kStagesMax;
  static constexpr int kBuffers = kOutBytes / (kWarps * kStageOut);
  static constexpr int kExchBytes = kWarps * 32 * 4 + kWarps * 10 * 4;  // row sums, coefficient partials
  // dynamic shared memory only (no static __shared__), 1 KB of alignment slack
  static constexpr int kSmemBytes = kStages * kStageBytes + kOutBytes + kBarBytes + kExchBytes + 1024;
    static_assert(kBuffers >= 1, "staging");
};
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint64_t kDrainNs = 2000000ull;         // 2 ms for in-flight copies after an error

struct Params {
  int M, N, K;
  int* err;
  // GRAIN epilogues
  const float* num;   // [groups, 6]
  const float* den;   // [groups, 4]
  float eps;
  // GRAIN backward: the forward pre-activation h [M, N] (row stride ldh) and
  // the coefficient partials [2 * num_m_tiles, groups, 10]
  const __nv_bfloat16* h;
  int64_t ldh;
  float* partial;
  // q/k/v projection with RoPE: fp32 tables [seq, hd/2]; output planes of width N/3
  const float* cos_t;
  const float* sin_t;
  int seq, hd;
  // tile schedule: 0 = cluster launch control over one cluster per tile;
  // n > 0 = static round robin over a persistent grid of n clusters
  int static_clusters;
  // 1: readers free ring slots with release-ordered arrivals (comparison)
  int ordered_release;
  // 1: epilogue warps free accumulator buffers with cluster-scope releases
  int acc_release_cluster;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, code);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Arrive on an mbarrier anywhere in the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Cluster launch control: ask the hardware to cancel the launch of a cluster
// of this grid that has not started yet.  The 16-byte response is written to
// `resp` (this CTA) and completes 16 transaction bytes on `bar`.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];"
               ::"r"(resp), "r"(bar)
               : "memory");
}

// x index of the first CTA of the cluster a response cancelled; -1 when the
// request failed (every cluster of the grid has started).
__device__ __forceinline__ int clc_first_cta_x(uint32_t resp) {
  int x;
  asm volatile(
      "{\n\t.reg .b128 r;\n\t.reg .pred p;\n\t"
      "ld.shared.b128 r, [%1];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n\t"
      "@!p mov.s32 %0, -1;\n\t}"
      : "=r"(x)
      : "r"(resp)
      : "memory");
  return x;
}

// Tile scheduler ring (per CTA).  The leader's producer thread obtains tile
// i+1 through cluster launch control while it loads tile i, then writes it
// into slot i % kSched of both CTAs and arrives on both `full` barriers.
// Every other role reads the slot and arrives on the leader's `empty`
// barrier, which gates the slot's reuse.
struct Sched {
  uint32_t base;  // shared::cta address: responses [kSched x 16 B], then the CLC,
                  // full and empty barriers [kSched each], then the tile slots
  __device__ __forceinline__ uint32_t resp(uint32_t s) const { return base + 16 * s; }
  __device__ __forceinline__ uint32_t clc(uint32_t s) const { return base + 16 * kSched + 8 * s; }
  __device__ __forceinline__ uint32_t full(uint32_t s) const { return base + 24 * kSched + 8 * s; }
  __device__ __forceinline__ uint32_t empty(uint32_t s) const { return base + 32 * kSched + 8 * s; }
  __device__ __forceinline__ uint32_t tile(uint32_t s) const { return base + 40 * kSched + 4 * s; }
  // tile i+1 travels through slot i % kSched, in that slot's use i / kSched
  __device__ __forceinline__ uint32_t slot_of(int i) const { return static_cast<uint32_t>(i % kSched); }
  __device__ __forceinline__ uint32_t parity_of(int i) const { return static_cast<uint32_t>((i / kSched) & 1); }
};

// Read tile i+1 from the ring (one thread); -1: no more tiles, -2: wait gave up.
__device__ __forceinline__ int sched_next(const Sched& sc, int i, int* err, int code, bool ordered = false) {
  const uint32_t slot = sc.slot_of(i);
  if (!mbar_wait(sc.full(slot), sc.parity_of(i), err, code)) return -2;
  int t;
  asm volatile("ld.shared.s32 %0, [%1];" : "=r"(t) : "r"(sc.tile(slot)) : "memory");
  // Free the slot with a relaxed arrival (no cluster-scope fence per reader
  // and tile).  Its address is made to depend on the value read, so the read
  // has completed before the arrival that lets the leader overwrite the slot.
  // (tile indices are >= -2, so `dep` is always 0, but the assembler cannot
  // know that and keeps the dependency)
  uint32_t dep;
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.lt.s32 q, %1, -2;\n\tselp.u32 %0, 8, 0, q;\n\t}"
      : "=r"(dep)
      : "r"(t));
  if (ordered)
    mbar_arrive_cluster(map_to_rank(sc.empty(slot), 0));
  else
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                     map_to_rank(sc.empty(slot), 0) + dep)
                 : "memory");
  return t;
}

// Leader producer: publish tile i+1 to both CTAs of the pair.
__device__ __forceinline__ void sched_publish(const Sched& sc, int i, int t) {
  const uint32_t slot = sc.slot_of(i);
#pragma unroll
  for (uint32_t r = 0; r < 2; ++r) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(map_to_rank(sc.tile(slot), r)), "r"(t) : "memory");
    mbar_arrive_cluster(map_to_rank(sc.full(slot), r));
  }
}

// Release an accumulator buffer to the leader's MMA issuer (remote arrive).
// After tcgen05.wait::ld and tcgen05.fence::before_thread_sync the TMEM reads
// are complete, so the arrival needs no cluster-scope fence: the default
// (CTA-scope release) form is used, the cluster-scope release on request.
__device__ __forceinline__ void acc_release(uint32_t cluster_addr, bool cluster_scope) {
  if (cluster_scope)
    mbar_arrive_cluster(cluster_addr);
  else
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; the transaction bytes are
// counted on `bar`, which may live in the peer CTA (cta_group::2).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completion on a local barrier.
__device__ __forceinline__ void tma_load_2d_local(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0,
                                                  int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive on the barrier at the same offset in both CTAs once every MMA
// issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

__device__ __forceinline__ void tc_mma2(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
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

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// The same store without waiting for it: a later tcgen05.wait::st (before
// any read of those columns) completes every store issued so far.
__device__ __forceinline__ void tmem_st16_async(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Split load: issue without waiting, then wait with the destination
// registers as operands, so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// UMMA shared-memory descriptor, 128B swizzle, K-major (8-row core groups
// 1024 B apart).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(16 >> 4) << 16;    // leading byte offset (unused for K-major swizzle)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;  // stride byte offset
  d |= 1ull << 46;                              // descriptor version (sm_100)
  d |= 2ull << 61;                              // SWIZZLE_128B
  return d;
}

// kind::f16, bf16 x bf16 -> f32, both K-major, M = 256, N = 256.
__device__ __forceinline__ constexpr uint32_t instr_desc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kBN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& tm, int& tn) {
  // 8 M-tiles share each sweep over N (L2 reuse of the weight tiles)
  constexpr int kGroup = 8;
  const int span = kGroup * num_n;
  const int g = tile / span;
  const int first = g * kGroup;
  int gm = num_m - first;
  if (gm > kGroup) gm = kGroup;
  const int r = tile - g * span;
  tm = first + r % gm;
  tn = r / gm;
}

// Write 32 fp32 values of one row (lane = row) as bf16 into a 32 x 64 staging
// tile laid out for a 128B-swizzled TMA store; `c0` selects the 32-column half.
__device__ __forceinline__ void stage_row32(uint8_t* stage, int lane, int c0, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = v[q * 8 + j];
    const int chunk = (c0 / 8 + q) ^ (lane & 7);
    store_vec<__nv_bfloat16, 8>(reinterpret_cast<__nv_bfloat16*>(stage + lane * 128 + chunk * 16), w);
  }
}

// 16 values of one row into the swizzled 32 x 64 staging tile at column c0.
__device__ __forceinline__ void stage_row16(uint8_t* stage, int lane, int c0, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = v[q * 8 + k];
    const int chunk = (c0 / 8 + q) ^ (lane & 7);
    store_vec<__nv_bfloat16, 8>(reinterpret_cast<__nv_bfloat16*>(stage + lane * 128 + chunk * 16), w);
  }
}

// GRAIN coefficients of one group, splatted to fp32 pairs.
struct GrainCoeffs {
  float2 a[6];  // numerator
  float2 b[4];  // |denominator|
};

__device__ __forceinline__ void load_grain_coeffs(GrainCoeffs& c, int g, const float* __restrict__ num,
                                                  const float* __restrict__ den) {
#pragma unroll
  for (int j = 0; j < 6; ++j) c.a[j] = splat2(num[g * 6 + j]);
#pragma unroll
  for (int j = 0; j < 4; ++j) c.b[j] = splat2(fabsf(den[g * 4 + j]));
}

// GRAIN backward behind the out-projection's input-gradient GEMM.  The
// accumulator holds gy = dL/dy for one 128-row x 256-column tile (one group).
// Sixteen epilogue warps: four per TMEM lane quarter (32 rows), each owning
// 64 columns; row reductions combine the four slices through shared memory.
// The warp's 32 x 64 slice of h arrives in its staging tile by TMA (issued one
// tile ahead).  Per row, with z = h, rho = sqrt(mean z^2 + eps), t = z / rho,
// f = P(t)/Q(|t|):
//   pass 1  sum z^2 over the slice -> rho;
//   pass 2  gy from TMEM, rounded to bf16 as the unfused GEMM output is;
//           coefficient partials (the factored form of
//           ro::grain::backward_packed_kernel), the row sum of gy (f - t f'),
//           and gy f' written back over gy in TMEM;
//   pass 3  gx = gy f' + t * (row sum) / 256 -> bf16, written over z in the
//           staging tile -> one TMA store.
// The 10 coefficient partials of the CTA's 128 rows go to
// partial[(2 * tm + crank) * groups + tn][k] (reduced later in a fixed order).
template <int W>
__device__ __forceinline__ void grain_bwd_epilogue(const Params& p, uint32_t tbase, uint8_t* stage, int tm, int tn,
                                                   uint32_t crank, int quarter, int e, int lane, int row0, int col0,
                                                   const CUtensorMap* tmC, float (*rho_part)[32],
                                                   float (*coef_part)[10]) {
  constexpr int kSlices = W / 4;
  constexpr int kCols = 256 / kSlices;   // 64
  constexpr int kChunks = kCols / 16;
  const int mate0 = e & 3;               // warps mate0 + 4j share these TMEM lanes
  // z (the pre-activation h) arrived in the warp's staging tile by TMA: row
  // `lane`, 16-byte chunk k of the row at ((k ^ (lane & 7)) * 16)
  auto load_z = [&](int ch, uint32_t (&zc)[8]) {
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const int chunk = (ch * 2 + v) ^ (lane & 7);
      const uint4 raw = *reinterpret_cast<const uint4*>(stage + lane * 128 + chunk * 16);
      zc[4 * v] = raw.x;
      zc[4 * v + 1] = raw.y;
      zc[4 * v + 2] = raw.z;
      zc[4 * v + 3] = raw.w;
    }
  };
  auto quarter_sum = [&](float v) {
    rho_part[e][lane] = v;
    asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "n"(32 * kSlices) : "memory");
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < kSlices; ++j) t += rho_part[mate0 + 4 * j][lane];
    asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "n"(32 * kSlices) : "memory");
    return t;
  };
  // pass 1
  float ss = 0.f;
#pragma unroll
  for (int ch = 0; ch < kChunks; ++ch) {
    uint32_t zc[8];
    load_z(ch, zc);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 z = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zc[i]));
      ss = fmaf(z.x, z.x, ss);
      ss = fmaf(z.y, z.y, ss);
    }
  }
  const float rho = sqrtf(quarter_sum(ss) * (1.0f / 256.0f) + p.eps);
  const float2 ir = splat2(__fdividef(1.0f, rho));
  GrainCoeffs c;
  load_grain_coeffs(c, tn, p.num, p.den);
  const float2 one = splat2(1.0f);
  float2 acc[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) acc[k] = splat2(0.0f);
  float2 sacc = splat2(0.0f);
  // pass 2: chunk ch+1's TMEM load is in flight while chunk ch is processed
  // (two register sets; the loop body covers two chunks so neither set is
  // indexed dynamically)
  static_assert(kChunks % 2 == 0, "pass 2 walks the chunks in pairs");
  auto pass2_chunk = [&](int ch, uint32_t (&r)[16]) {
    uint32_t zc[8];
    load_z(ch, zc);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // gy rounded to bf16 as the unfused GEMM output is (one paired conversion)
      const float2 g2 = __bfloat1622float2(__floats2bfloat162_rn(__uint_as_float(r[2 * j]),
                                                                 __uint_as_float(r[2 * j + 1])));
      const float2 z = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zc[j]));
      const float2 t = mul2(z, ir);
      const float2 at = abs2(t);
      const float2 t2 = mul2(t, t);
      // P(t) by Horner's rule with P'(t) carried along (synthetic division:
      // each derivative step folds in the running value of P)
      float2 pp = fma2(c.a[5], t, c.a[4]);
      float2 dp = fma2(c.a[5], t, pp);
      pp = fma2(pp, t, c.a[3]);
      dp = fma2(dp, t, pp);
      pp = fma2(pp, t, c.a[2]);
      dp = fma2(dp, t, pp);
      pp = fma2(pp, t, c.a[1]);
      dp = fma2(dp, t, pp);
      pp = fma2(pp, t, c.a[0]);
      // Q(x) = 1 + |b0| x + |b1| x^2 + |b2| x^3 + |b3| x^4 at x = |t|, with
      // dQ/dx the same way; dQ/dt = sign0(t) dQ/dx
      float2 q = fma2(c.b[3], at, c.b[2]);
      float2 hq = fma2(c.b[3], at, q);
      q = fma2(q, at, c.b[1]);
      hq = fma2(hq, at, q);
      q = fma2(q, at, c.b[0]);
      const float2 dq = mul2(fma2(hq, at, q), sign02(t));
      q = fma2(q, at, one);
      const float2 iq = rcp2(q);
      const float2 f = mul2(pp, iq);
      const float2 df = mul2(fma2(neg2(f), dq, dp), iq);
      sacc = fma2(g2, fma2(neg2(t), df, f), sacc);
      // the row's rho multiplies every coefficient partial of the row: it is
      // applied once to the row's sums below instead of per element
      const float2 s1 = mul2(g2, iq);
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
      const float2 gd = mul2(g2, df);
      r[2 * j] = __float_as_uint(gd.x);
      r[2 * j + 1] = __float_as_uint(gd.y);
    }
    tmem_st16_async(tbase + ch * 16, r);
  };
  uint32_t ra[16], rb[16];
  tmem_ld16_issue(tbase, ra);
#pragma unroll 1
  for (int ch = 0; ch < kChunks; ch += 2) {
    tmem_ld16_wait(ra);
    tmem_ld16_issue(tbase + (ch + 1) * 16, rb);
    pass2_chunk(ch, ra);
    tmem_ld16_wait(rb);
    if (ch + 2 < kChunks) tmem_ld16_issue(tbase + (ch + 2) * 16, ra);
    pass2_chunk(ch + 1, rb);
  }
  tmem_wait_st();  // pass 3 reads these columns back
  const float2 sw = splat2(quarter_sum(sacc.x + sacc.y) * (1.0f / 256.0f));
  // pass 3: gx over z in the staging tile (each lane rewrites its own row) ->
  // one bulk store; chunk ch+1's TMEM load is in flight while chunk ch is formed
  uint32_t rr[2][16];
  tmem_ld16_issue(tbase, rr[0]);
#pragma unroll
  for (int ch = 0; ch < kChunks; ++ch) {
    uint32_t (&r)[16] = rr[ch & 1];
    tmem_ld16_wait(r);
    if (ch + 1 < kChunks) tmem_ld16_issue(tbase + (ch + 1) * 16, rr[(ch + 1) & 1]);
    uint32_t zc[8];
    load_z(ch, zc);
    float out[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 z = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zc[j]));
      const float2 t = mul2(z, ir);
      const float2 gx = fma2(t, sw, make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])));
      out[2 * j] = gx.x;
      out[2 * j + 1] = gx.y;
    }
    stage_row16(stage, lane, ch * 16, out);
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmC, smem_u32(stage), col0, row0);
    bulk_commit();
  }
  // coefficient partials of the CTA's rows (fixed-order reduction)
#pragma unroll
  for (int k = 0; k < 10; ++k) {
    float v = (acc[k].x + acc[k].y) * rho;
    if (k >= 6) {
      const float b = p.den[tn * 4 + (k - 6)];
      v *= b > 0.f ? -1.f : (b < 0.f ? 1.f : 0.f);
    }
    v = warp_sum(v);
    if (lane == 0) coef_part[e][k] = v;
  }
  asm volatile("bar.sync 5, %0;" ::"n"(W * 32) : "memory");
  if (e == 0 && lane < 10) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) v += coef_part[w][lane];
    const int groups = p.N / kBN;
    p.partial[(static_cast<int64_t>(2 * tm + static_cast<int>(crank)) * groups + tn) * 10 + lane] = v;
  }
  asm volatile("bar.sync 5, %0;" ::"n"(W * 32) : "memory");
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Traits<EPI>::kThreads, 1)
gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
             const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmY, Params p) {
  constexpr int kStages = Traits<EPI>::kStages;
  constexpr int kW = Traits<EPI>::kWarps;
  constexpr int kSlice = Traits<EPI>::kSlice;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_stage = smem + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + kOutBytes);
  uint64_t* full = bars;                   // [kStages]  (used in the leader)
  uint64_t* empty = bars + kStages;        // [kStages]  (both CTAs)
  uint64_t* acc_full = empty + kStages;    // [2]        (both CTAs)
  uint64_t* acc_empty = acc_full + 2;      // [2]        (used in the leader)
  uint64_t* hbar = acc_empty + 2;         // [kW]       (GRAIN backward: h slice per warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(hbar + kW);
  const Sched sc{smem_u32(bars) + 256};  // tile scheduler ring (bars + 256 B)
  float (*rho_part)[32] = reinterpret_cast<float (*)[32]>(out_stage + kOutBytes + kBarBytes);
  float (*coef_part)[10] = reinterpret_cast<float (*)[10]>(out_stage + kOutBytes + kBarBytes + kW * 32 * 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_rank();
  const bool leader = crank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + kBN - 1) / kBN;
  const int num_k = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&acc_full[a]), 1);
      mbar_init(smem_u32(&acc_empty[a]), 2 * kW);
    }
    for (int w = 0; w < kW; ++w) mbar_init(smem_u32(&hbar[w]), 1);
    for (int s = 0; s < kSched; ++s) {
      mbar_init(sc.clc(s), 1);
      mbar_init(sc.full(s), 1);
      // readers: leader MMA + epilogue warps, peer producer + epilogue warps
      mbar_init(sc.empty(s), 2 + 2 * kW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int tile = cluster_id;
      for (int i = 0; tile >= 0 && ok; ++i) {
        if (leader) {
          if (!mbar_wait(sc.empty(sc.slot_of(i)), sc.parity_of(i) ^ 1, p.err, 6)) break;
          if (p.static_clusters == 0) {
            // ask for the next tile now; the answer is read after this tile's loads
            mbar_expect_tx(sc.clc(sc.slot_of(i)), 16);
            clc_try_cancel(sc.resp(sc.slot_of(i)), sc.clc(sc.slot_of(i)));
          }
        }
        int tm, tn;
        tile_coords(tile, num_m, num_n, tm, tn);
        const int m0 = tm * kBM + static_cast<int>(crank) * kHalfM;
        const int n0 = tn * kBN + static_cast<int>(crank) * kHalfN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, p.err, 1)) { ok = false; break; }
          const uint32_t fb_local = smem_u32(&full[stage]);
          if (leader) mbar_expect_tx(fb_local, 2 * kStageBytes);
          const uint32_t fb = map_to_rank(fb_local, 0);
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          tma_load_2d(sa, &tmA, fb, kb * kBK, m0);
          tma_load_2d(sa + kABytes, &tmB, fb, kb * kBK, n0);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (leader) {
          if (p.static_clusters == 0) {
            if (!mbar_wait(sc.clc(sc.slot_of(i)), sc.parity_of(i), p.err, 7)) break;
            const int x = clc_first_cta_x(sc.resp(sc.slot_of(i)));
            tile = x < 0 ? -1 : (x >> 1);
          } else {
            tile += p.static_clusters;
            if (tile >= num_m * num_n) tile = -1;
          }
          sched_publish(sc, i, tile);
        } else {
          tile = sched_next(sc, i, p.err, 8, p.ordered_release != 0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = instr_desc();
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = cluster_id; tile >= 0 && ok; ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&acc_empty[acc]), acc_phase ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * kBN;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, p.err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            tc_mma2(tmem_d, smem_desc(sa + k * 32), smem_desc(sb + k * 32), idesc, (kb | k) != 0 ? 1u : 0u);
          tc_commit_both(smem_u32(&empty[stage]));
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit_both(smem_u32(&acc_full[acc]));
        tile = sched_next(sc, local, p.err, 9, p.ordered_release != 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int e = warp - 2;              // 0 .. kW-1
    const int quarter = warp & 3;        // TMEM lanes [32*quarter, +32)
    const int chalf = e >> 2;            // column slice: [kSlice*chalf, +kSlice)
    uint8_t* stage_buf = out_stage + e * Traits<EPI>::kBuffers * kStageOut;
    int buf = 0;
    const uint32_t empty_leader = map_to_rank(smem_u32(&acc_empty[0]), 0);
    // GRAIN backward: TMA the warp's slice of h for a tile into its staging tile
    auto fetch_h = [&](int tile) {
      if constexpr (EPI == kGrainBwd) {
        if (tile >= 0 && lane == 0) {
          int fm, fn;
          tile_coords(tile, num_m, num_n, fm, fn);
          bulk_wait_read<0>();  // the previous bulk store has read the tile
          const uint32_t hb = smem_u32(&hbar[e]);
          mbar_expect_tx(hb, kStageOut);
          tma_load_2d_local(smem_u32(stage_buf), &tmY, hb, fn * kBN + chalf * kSlice,
                            fm * kBM + static_cast<int>(crank) * kHalfM + quarter * 32);
        }
        __syncwarp();
      }
    };
    fetch_h(cluster_id);
    GrainCoeffs gc;
    float2 one2 = splat2(1.0f);
    int local = 0;
    // tile i+1 of this CTA pair, read by lane 0 and shared with the warp
    auto next_tile = [&](int i) {
      int t = 0;
      if (lane == 0) t = sched_next(sc, i, p.err, 10, p.ordered_release != 0);
      return __shfl_sync(0xffffffffu, t, 0);
    };
    for (int tile = cluster_id; tile >= 0; ++local) {
      int tm, tn;
      tile_coords(tile, num_m, num_n, tm, tn);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(smem_u32(&acc_full[acc]), acc_phase, p.err, 4)) break;
      tc_fence_after();
      const int row0 = tm * kBM + static_cast<int>(crank) * kHalfM + quarter * 32;
      const int col0 = tn * kBN + chalf * kSlice;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kBN + chalf * kSlice;
      float rho = 1.0f;
      if constexpr (EPI == kGrainFwd) {
        // pass 1: sum of squares of bf16(acc) over this warp's 128 columns,
        // combined with the partner warp's half (same rows) through smem
        float ss = 0.f;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float h = __bfloat162float(__float2bfloat16_rn(__uint_as_float(r[j])));
            ss = fmaf(h, h, ss);
          }
        }
        rho_part[e][lane] = ss;
        // named barrier per lane quarter: warps e and e^4
        asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
        const float tot = rho_part[e][lane] + rho_part[e ^ 4][lane];
        asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
        rho = sqrtf(tot * (1.0f / 256.0f) + p.eps);
        load_grain_coeffs(gc, tn, p.num, p.den);
      }
      if constexpr (EPI == kGrainBwd) {
        if (!mbar_wait(smem_u32(&hbar[e]), local & 1, p.err, 5)) break;
        grain_bwd_epilogue<kW>(p, tbase, stage_buf, tm, tn, crank, quarter, e, lane, row0, col0, &tmC, rho_part,
                               coef_part);
        const int next = next_tile(local);
        fetch_h(next);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) acc_release(empty_leader + acc * 8, p.acc_release_cluster != 0);
        tile = next;
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < 128; c += 64) {
        uint8_t* st = stage_buf + buf * kStageOut;
        // the staging buffer's previous bulk store must have read it
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        float hv[2][32];
        {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) hv[0][j] = __uint_as_float(r[j]);
          tmem_ld32(tbase + c + 32, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) hv[1][j] = __uint_as_float(r[j]);
        }
        int plane = 0, pcol = col0 + c;
        if constexpr (EPI == kQkvRope) {
          // plane 0/1/2 = q/k/v; q and k are rotated (interleaved pairs, fp32
          // tables, applied to the bf16-rounded projection like ro::nn's RoPE kernel)
          const int width = p.N / 3;
          plane = (col0 + c) / width;
          pcol = (col0 + c) - plane * width;
          if (plane < 2) {
            const int row = row0 + lane;
            const int pos = (row < p.M ? row : 0) % p.seq;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int pair0 = ((pcol + hh * 32) % p.hd) / 2;
              const float4* cp = reinterpret_cast<const float4*>(p.cos_t + static_cast<int64_t>(pos) * (p.hd / 2) + pair0);
              const float4* sp = reinterpret_cast<const float4*>(p.sin_t + static_cast<int64_t>(pos) * (p.hd / 2) + pair0);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                const float4 cv = __ldg(cp + q4), sv = __ldg(sp + q4);
                const float cs[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const int j = (q4 * 4 + u) * 2;
                  const float ev = __bfloat162float(__float2bfloat16_rn(hv[hh][j]));
                  const float ov = __bfloat162float(__float2bfloat16_rn(hv[hh][j + 1]));
                  hv[hh][j] = ev * cs[u] - ov * sn[u];
                  hv[hh][j + 1] = ev * sn[u] + ov * cs[u];
                }
              }
            }
          }
        }
        stage_row32(st, lane, 0, hv[0]);
        stage_row32(st, lane, 32, hv[1]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (EPI == kQkvRope) tma_store_3d(&tmC, smem_u32(st), pcol, row0, plane);
          else tma_store_2d(&tmC, smem_u32(st), col0 + c, row0);
          bulk_commit();
        }
        buf ^= 1;
        if constexpr (EPI == kGrainFwd) {
          uint8_t* sy = stage_buf + buf * kStageOut;
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
          const float2 ir = splat2(__fdividef(1.0f, rho)), rh = splat2(rho);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              float2 t = make_float2(__bfloat162float(__float2bfloat16_rn(hv[hh][j])),
                                     __bfloat162float(__float2bfloat16_rn(hv[hh][j + 1])));
              t = mul2(t, ir);
              const float2 at = abs2(t);
              float2 pp = fma2(gc.a[5], t, gc.a[4]);
              pp = fma2(pp, t, gc.a[3]);
              pp = fma2(pp, t, gc.a[2]);
              pp = fma2(pp, t, gc.a[1]);
              pp = fma2(pp, t, gc.a[0]);
              float2 q = fma2(gc.b[3], at, gc.b[2]);
              q = fma2(q, at, gc.b[1]);
              q = fma2(q, at, gc.b[0]);
              q = fma2(q, at, one2);
              const float2 y = mul2(mul2(pp, rh), rcp2(q));
              hv[hh][j] = y.x;
              hv[hh][j + 1] = y.y;
            }
          }
          stage_row32(sy, lane, 0, hv[0]);
          stage_row32(sy, lane, 32, hv[1]);
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmY, smem_u32(sy), col0 + c, row0);
            bulk_commit();
          }
          buf ^= 1;
        }
      }
      // accumulator buffer drained: release it to the leader's MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) acc_release(empty_leader + acc * 8, p.acc_release_cluster != 0);
      tile = next_tile(local);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  if (*reinterpret_cast<volatile int*>(p.err) != 0) {
    // a wait gave up: TMA loads already issued into this pair's shared memory
    // (operand stages, the GRAIN-backward h slices) complete without any
    // further action, so give them a bounded interval to land before the
    // shared memory is handed to the next cluster
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < kDrainNs) __nanosleep(1000);
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Host side.

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

// 2-D bf16 map over a row-major [rows, cols] matrix with row stride `ld`
// (elements); box = {64, box_rows}, 128B swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D bf16 map over planes of a [planes, rows, cols] tensor (row-major planes);
// box = {64, 32, 1}, 128B swizzle.
bool make_map_planes(CUtensorMap* map, const void* base, int64_t planes, int64_t rows, int64_t cols) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2), static_cast<cuuint64_t>(rows * cols * 2)};
  cuuint32_t box[3] = {64u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

template <int EPI>
int launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, void* Y, int64_t ldy,
           Params p, cudaStream_t stream) {
  CUtensorMap ma, mb, mc, my;
  if (!make_map(&ma, A, p.M, p.K, lda, kHalfM) || !make_map(&mb, B, p.N, p.K, ldb, kHalfN)) return -3;
  if constexpr (EPI == kQkvRope) {
    if (!make_map_planes(&mc, C, 3, p.M, p.N / 3)) return -3;
  } else {
    if (!make_map(&mc, C, p.M, p.N, ldc, 32)) return -3;
  }
  if constexpr (EPI == kGrainBwd) {
    if (!make_map(&my, p.h, p.M, p.N, p.ldh, 32)) return -3;
  } else if constexpr (EPI == kGrainFwd) {
    if (!make_map(&my, Y, p.M, p.N, ldy, 32)) return -3;
  } else {
    my = mc;
  }
  static_assert(Traits<EPI>::kSmemBytes <= 232448, "exceeds the 227 KB per-CTA shared memory of sm_100");
  auto kern = gemm2_kernel<EPI>;
  static int configured = 0;  // 1 ok, -1 this configuration cannot run
  if (configured == 0) {
    configured = -1;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Traits<EPI>::kSmemBytes) ==
        cudaSuccess) {
      // a cluster of two CTAs of this size must fit on the device
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(Traits<EPI>::kThreads, 1, 1);
      cfg.dynamicSmemBytes = Traits<EPI>::kSmemBytes;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int active = 0;
      if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) == cudaSuccess && active > 0) configured = 1;
    }
    cudaGetLastError();  // clear a failed query
  }
  if (configured < 0) return -4;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + kBN - 1) / kBN);
  // default: one cluster per tile; the clusters that start first take over
  // the tiles of clusters that have not started (cluster launch control), so
  // SMs held by other kernels (collectives on another stream) delay no tile.
  // RO_GEMM2_STATIC=1: a persistent grid of one cluster per SM pair.
  static const bool static_sched = [] {
    const char* v = std::getenv("RO_GEMM2_STATIC");
    return v != nullptr && v[0] == '1';
  }();
  static const bool ordered = [] {
    const char* v = std::getenv("RO_GEMM2_ORDERED_RELEASE");
    return v != nullptr && v[0] == '1';
  }();
  p.ordered_release = ordered ? 1 : 0;
  static const bool acc_cluster = [] {
    const char* v = std::getenv("RO_GEMM2_ACC_CLUSTER_RELEASE");
    return v != nullptr && v[0] == '1';
  }();
  p.acc_release_cluster = acc_cluster ? 1 : 0;
  int clusters = tiles;
  if (static_sched) {
    clusters = num_sms() / 2;
    if (tiles < clusters) clusters = tiles;
    p.static_clusters = clusters;
  }
  kern<<<2 * clusters, Traits<EPI>::kThreads, Traits<EPI>::kSmemBytes, stream>>>(ma, mb, mc, my, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace gemm2

// C[M, N] = bf16(A[M, K] . B[N, K]^T), both K-major, on the 2-SM path.
// Returns 0 on success, negative when the configuration is unsupported (the
// caller falls back), positive CUDA error codes.
int gemm2_bf16_nt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int M, int N,
                  int K, int* err, cudaStream_t stream) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0) return -1;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C) || (lda % 8) || (ldb % 8) || (ldc % 8) || (K % 8) ||
      (N % 8))
    return -2;
  Params p{M, N, K, err, nullptr, nullptr, 0.f, nullptr, 0, nullptr, nullptr, nullptr, 1, 64};
  return launch<kStore>(A, lda, B, ldb, C, ldc, nullptr, 0, p, stream);
}

// GRAIN forward fused behind the in-projection: H = bf16(X W^T) and
// Y = GRAIN(H) with groups of 256 columns (N = 256 * groups).  num [groups, 6],
// den [groups, 4] fp32 (no local-basis atoms, no affine restriction).
int gemm2_grain_forward(const void* X, int64_t ldx, const void* W, int64_t ldw, void* H, void* Y, int M, int N,
                        int K, const float* num, const float* den, float eps, int* err, cudaStream_t stream) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0 || N % kBN) return -1;
  if (!aligned16(X) || !aligned16(W) || !aligned16(H) || !aligned16(Y) || (ldx % 8) || (ldw % 8) || (K % 8))
    return -2;
  Params p{M, N, K, err, num, den, eps, nullptr, 0, nullptr, nullptr, nullptr, 1, 64};
  return launch<kGrainFwd>(X, ldx, W, ldw, H, N, Y, N, p, stream);
}

int gemm2_grain_partial_rows(int M) { return 2 * ((M + gemm2::kBM - 1) / gemm2::kBM); }

// GRAIN backward fused behind the out-projection's input gradient:
//   gy = bf16(dO W_out) (dO [M, K], W_out^T given K-major as wt [N, K]),
//   gx = dGRAIN(h, gy) -> GX [M, N] (bf16), coefficient partials ->
//   partial [gemm2_grain_partial_rows(M), N / 256, 10].
int gemm2_grain_backward(const void* dO, int64_t ldo, const void* wt, int64_t ldw, const void* h, int64_t ldh,
                         void* GX, float* partial, int M, int N, int K, const float* num, const float* den,
                         float eps, int* err, cudaStream_t stream) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0 || N % kBN) return -1;
  if (!aligned16(dO) || !aligned16(wt) || !aligned16(h) || !aligned16(GX) || (ldo % 8) || (ldw % 8) ||
      (ldh % 8) || (K % 8))
    return -2;
  Params p{M, N, K, err, num, den, eps, static_cast<const __nv_bfloat16*>(h), ldh, partial, nullptr, nullptr,
           1, 64};
  return launch<kGrainBwd>(dO, ldo, wt, ldw, GX, N, nullptr, 0, p, stream);
}

// q, k, v = RoPE(bf16(x W_qkv^T)) split into three [M, N/3] planes of QKV
// (token-major: row = token, columns = heads x head_dim); positions are
// row % seq; cos/sin fp32 [seq, hd/2].  hd must be a multiple of 32.
int gemm2_qkv_rope(const void* X, int64_t ldx, const void* W, int64_t ldw, void* QKV, int M, int N, int K,
                   const float* cos_t, const float* sin_t, int seq, int hd, int* err, cudaStream_t stream) {
  using namespace gemm2;
  if (M <= 0 || N <= 0 || K <= 0 || N % 3 || (N / 3) % kBN || hd % 32 || (N / 3) % hd || seq <= 0) return -1;
  if (!aligned16(X) || !aligned16(W) || !aligned16(QKV) || !aligned16(cos_t) || !aligned16(sin_t) || (ldx % 8) ||
      (ldw % 8) || (K % 8))
    return -2;
  Params p{M, N, K, err, nullptr, nullptr, 0.f, nullptr, 0, nullptr, cos_t, sin_t, seq, hd};
  return launch<kQkvRope>(X, ldx, W, ldw, QKV, N / 3, nullptr, 0, p, stream);
}

}  // namespace ro
