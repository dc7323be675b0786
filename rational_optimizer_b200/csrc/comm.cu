// In-kernel NVLink collectives over peer memory (CUDA IPC), one process per GPU.
//
// Every rank owns one communication buffer (cudaMalloc'd here so its IPC
// handle covers it from offset 0) and a small flag array.  Peers map both
// with cudaIpcOpenMemHandle; kernels then read peer data with ordinary
// 16-byte global loads that travel over NVLink/NVSwitch, and signal each
// other with release/acquire stores and loads at system scope on the flag
// arrays.  No TMA and no multicast is used on peer memory.
//
// All-reduce (mean) of a fp32 buffer, in place, as three launches:
//   rs     signal "ready(epoch)" to every peer; wait for every peer's ready;
//          reduce this rank's shard over all ranks in rank order (identical
//          summation order on every rank -> bitwise-identical replicas) and
//          scale by 1/W, writing the shard in place;
//   ag     signal "reduced(epoch)"; wait; copy every other rank's reduced
//          shard from its owner;
//   fence  signal "gathered(epoch)"; wait - afterwards no peer will read
//          this rank's buffer again for this epoch, so the next backward may
//          overwrite it.
// Variants: bf16 transport (peer loads of a bf16 copy) and int8 transport
// with one fp32 scale per 256-element block (quantise locally, reduce the
// dequantised values in rank order, requantise the reduced shard; every rank,
// the owner included, ends with the same dequantised values).
//
// Waits are bounded by a caller-given time limit; on expiry the kernel writes
// an error code (1 = ready, 2 = reduced, 3 = gathered wait) to `err` and skips
// its data movement, so a dead peer cannot hang the GPU.
#include "common.cuh"

namespace ro {
namespace comm {

constexpr int kMaxRanks = 16;
constexpr int kQuantBlock = 256;

struct Peers {
  const void* data[kMaxRanks];     // peer communication buffers (own rank included)
  unsigned int* flags[kMaxRanks];  // peer flag arrays [3][kMaxRanks]
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Block 0 publishes `epoch` into slot [phase][rank] of every peer's flags;
// every block then waits (thread 0, bounded) until all peers published into
// this rank's own flags.  Returns false on timeout.
__device__ bool cross_rank_barrier(const Peers& peers, int rank, int world, int phase,
                                   unsigned int epoch, int* err, uint64_t timeout_ns) {
  __shared__ int ok;
  if (blockIdx.x == 0 && threadIdx.x < world && static_cast<int>(threadIdx.x) != rank) {
    __threadfence_system();
    store_release_sys(peers.flags[threadIdx.x] + phase * kMaxRanks + rank, epoch);
  }
  if (threadIdx.x == 0) {
    ok = 1;
    const unsigned int* mine = peers.flags[rank] + phase * kMaxRanks;
    const uint64_t t0 = now_ns();
    for (int p = 0; p < world && ok; ++p) {
      if (p == rank) continue;
      while (static_cast<int>(load_acquire_sys(mine + p) - epoch) < 0) {
        if (*reinterpret_cast<volatile int*>(err) != 0 || now_ns() - t0 > timeout_ns) {
          atomicCAS(err, 0, phase + 1);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ void shard_range(int64_t n, int world, int s, int64_t& lo, int64_t& hi) {
  // shards are multiples of 4 elements (16 bytes) except the tail
  int64_t per = (n + world - 1) / world;
  per = (per + 3) & ~int64_t(3);
  lo = per * s;
  hi = lo + per;
  if (lo > n) lo = n;
  if (hi > n) hi = n;
}

// ---------------------------------------------------------------------------
// fp32 transport

__global__ void __launch_bounds__(512)
rs_f32_kernel(const __grid_constant__ Peers peers, float* mine, int rank, int world, int64_t n,
              float scale, unsigned int epoch, int* err, uint64_t timeout_ns) {
  if (!cross_rank_barrier(peers, rank, world, 0, epoch, err, timeout_ns)) return;
  int64_t lo, hi;
  shard_range(n, world, rank, lo, hi);
  const int64_t nvec = (hi - lo) / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    const int64_t i = lo + v * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < world; ++p) {
      const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(peers.data[p]) + i);
      acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    *reinterpret_cast<float4*>(mine + i) = acc;
  }
  // tail (fewer than 4 elements)
  if (blockIdx.x == 0 && threadIdx.x < (hi - lo) % 4) {
    const int64_t i = lo + nvec * 4 + threadIdx.x;
    float acc = 0.f;
    for (int p = 0; p < world; ++p) acc += static_cast<const float*>(peers.data[p])[i];
    mine[i] = acc * scale;
  }
}

__global__ void __launch_bounds__(512)
ag_f32_kernel(const __grid_constant__ Peers peers, float* mine, int rank, int world, int64_t n,
              unsigned int epoch, int* err, uint64_t timeout_ns) {
  if (!cross_rank_barrier(peers, rank, world, 1, epoch, err, timeout_ns)) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int k = 1; k < world; ++k) {
    const int p = (rank + k) % world;  // stagger sources across ranks
    int64_t lo, hi;
    shard_range(n, world, p, lo, hi);
    const int64_t nvec = (hi - lo) / 4;
    const float* src = static_cast<const float*>(peers.data[p]);
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
      const int64_t i = lo + v * 4;
      *reinterpret_cast<float4*>(mine + i) = *reinterpret_cast<const float4*>(src + i);
    }
    if (blockIdx.x == 0 && threadIdx.x < (hi - lo) % 4) {
      const int64_t i = lo + nvec * 4 + threadIdx.x;
      mine[i] = src[i];
    }
  }
}

__global__ void fence_kernel(const __grid_constant__ Peers peers, int rank, int world, unsigned int epoch,
                             int* err, uint64_t timeout_ns) {
  cross_rank_barrier(peers, rank, world, 2, epoch, err, timeout_ns);
}

// ---------------------------------------------------------------------------
// int8 transport.  Layout of a rank's communication buffer for n elements:
//   [n int8 values][nb fp32 scales]   (nb = ceil(n / 256)), rounded to 16 B.
// quantise: local fp32 -> (int8, scale) for all blocks (own buffer).
// rs: owner dequantises its shard blocks from every rank in rank order, sums,
//     scales, requantises the reduced blocks into its own buffer and also
//     writes the dequantised result into its fp32 output.
// ag: every rank dequantises the other owners' reduced blocks into fp32.

__global__ void __launch_bounds__(256)
quantize_kernel(const float* __restrict__ src, int8_t* __restrict__ q, float* __restrict__ scales,
                int64_t n) {
  const int64_t nb = (n + kQuantBlock - 1) / kQuantBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * 8 + warp; b < nb; b += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t base = b * kQuantBlock;
    float v[8];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = base + lane * 8 + j;
      v[j] = i < n ? src[i] : 0.f;
      amax = fmaxf(amax, fabsf(v[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax > 0.f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = base + lane * 8 + j;
      if (i < n) q[i] = static_cast<int8_t>(__float2int_rn(fminf(fmaxf(v[j] * inv, -127.f), 127.f)));
    }
    if (lane == 0) scales[b] = s;
  }
}

__device__ __forceinline__ int64_t qblock_lo(int64_t nb, int world, int s) {
  return (nb * s) / world;
}

__global__ void __launch_bounds__(256)
rs_i8_kernel(const __grid_constant__ Peers peers, int8_t* my_q, float* my_scales, float* out, int rank,
             int world, int64_t n, int64_t scale_off, float scale, unsigned int epoch, int* err,
             uint64_t timeout_ns) {
  if (!cross_rank_barrier(peers, rank, world, 0, epoch, err, timeout_ns)) return;
  const int64_t nb = (n + kQuantBlock - 1) / kQuantBlock;
  const int64_t b_lo = qblock_lo(nb, world, rank), b_hi = qblock_lo(nb, world, rank + 1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = b_lo + static_cast<int64_t>(blockIdx.x) * 8 + warp; b < b_hi;
       b += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t base = b * kQuantBlock;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int p = 0; p < world; ++p) {
      const int8_t* q = static_cast<const int8_t*>(peers.data[p]);
      const float s = reinterpret_cast<const float*>(static_cast<const int8_t*>(peers.data[p]) + scale_off)[b];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t i = base + lane * 8 + j;
        if (i < n) acc[j] += s * static_cast<float>(q[i]);
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[j] *= scale;
      amax = fmaxf(amax, fabsf(acc[j]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax > 0.f ? amax / 127.0f : 1.0f;
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t i = base + lane * 8 + j;
      if (i < n) {
        const int8_t qv = static_cast<int8_t>(__float2int_rn(fminf(fmaxf(acc[j] * inv, -127.f), 127.f)));
        my_q[i] = qv;
        out[i] = s * static_cast<float>(qv);
      }
    }
    if (lane == 0) my_scales[b] = s;
  }
}

__global__ void __launch_bounds__(256)
ag_i8_kernel(const __grid_constant__ Peers peers, float* out, int rank, int world, int64_t n,
             int64_t scale_off, unsigned int epoch, int* err, uint64_t timeout_ns) {
  if (!cross_rank_barrier(peers, rank, world, 1, epoch, err, timeout_ns)) return;
  const int64_t nb = (n + kQuantBlock - 1) / kQuantBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int k = 1; k < world; ++k) {
    const int p = (rank + k) % world;
    const int64_t b_lo = qblock_lo(nb, world, p), b_hi = qblock_lo(nb, world, p + 1);
    const int8_t* q = static_cast<const int8_t*>(peers.data[p]);
    const float* sc = reinterpret_cast<const float*>(q + scale_off);
    for (int64_t b = b_lo + static_cast<int64_t>(blockIdx.x) * 8 + warp; b < b_hi;
         b += static_cast<int64_t>(gridDim.x) * 8) {
      const float s = sc[b];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t i = b * kQuantBlock + lane * 8 + j;
        if (i < n) out[i] = s * static_cast<float>(q[i]);
      }
    }
  }
}

}  // namespace comm

// ---------------------------------------------------------------------------
// Host API.

int comm_ipc_handle(const void* base, void* handle_out) {
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
  if (e != cudaSuccess) return static_cast<int>(e);
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

int comm_ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int comm_ipc_close(void* ptr) { return static_cast<int>(cudaIpcCloseMemHandle(ptr)); }

static comm::Peers make_peers(void* const* data, unsigned int* const* flags, int world) {
  comm::Peers p;
  for (int i = 0; i < comm::kMaxRanks; ++i) {
    p.data[i] = i < world ? data[i] : nullptr;
    p.flags[i] = i < world ? flags[i] : nullptr;
  }
  return p;
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 4) g = 148 * 4;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

// data[r]/flags[r]: every rank's buffer / flags as mapped in this process.
int comm_allreduce_f32(void* const* data, unsigned int* const* flags, int rank, int world, int64_t n,
                       float scale, unsigned int epoch, int* err, uint64_t timeout_ns,
                       cudaStream_t stream) {
  if (world < 1 || world > comm::kMaxRanks) return -1;
  if (reinterpret_cast<uintptr_t>(data[rank]) % 16) return -2;
  comm::Peers peers = make_peers(data, flags, world);
  float* mine = static_cast<float*>(data[rank]);
  const int g = grid_for(n / world / 4 + 1, 512);
  comm::rs_f32_kernel<<<g, 512, 0, stream>>>(peers, mine, rank, world, n, scale, epoch, err, timeout_ns);
  comm::ag_f32_kernel<<<g, 512, 0, stream>>>(peers, mine, rank, world, n, epoch, err, timeout_ns);
  comm::fence_kernel<<<1, 32, 0, stream>>>(peers, rank, world, epoch, err, timeout_ns);
  return static_cast<int>(cudaGetLastError());
}

int64_t comm_i8_scale_offset(int64_t n) { return (n + 15) & ~int64_t(15); }
int64_t comm_i8_bytes(int64_t n) {
  const int64_t nb = (n + comm::kQuantBlock - 1) / comm::kQuantBlock;
  return comm_i8_scale_offset(n) + ((nb * 4 + 15) & ~int64_t(15));
}

// src (fp32, n) -> every rank's `out` holds the mean; data[r] are int8 comm buffers
// of comm_i8_bytes(n) bytes.
int comm_allreduce_i8(const float* src, float* out, void* const* data, unsigned int* const* flags, int rank,
                      int world, int64_t n, float scale, unsigned int epoch, int* err,
                      uint64_t timeout_ns, cudaStream_t stream) {
  if (world < 1 || world > comm::kMaxRanks) return -1;
  comm::Peers peers = make_peers(data, flags, world);
  int8_t* q = static_cast<int8_t*>(data[rank]);
  const int64_t soff = comm_i8_scale_offset(n);
  float* sc = reinterpret_cast<float*>(q + soff);
  const int64_t nb = (n + comm::kQuantBlock - 1) / comm::kQuantBlock;
  comm::quantize_kernel<<<grid_for(nb, 8), 256, 0, stream>>>(src, q, sc, n);
  const int g = grid_for(nb / world + 1, 8);
  comm::rs_i8_kernel<<<g, 256, 0, stream>>>(peers, q, sc, out, rank, world, n, soff, scale, epoch, err,
                                            timeout_ns);
  comm::ag_i8_kernel<<<g, 256, 0, stream>>>(peers, out, rank, world, n, soff, epoch, err, timeout_ns);
  comm::fence_kernel<<<1, 32, 0, stream>>>(peers, rank, world, epoch, err, timeout_ns);
  return static_cast<int>(cudaGetLastError());
}

// Bounded wait on a flag nobody sets (used by the failure-detection test):
// waits on slot [phase][peer] of this rank's flags for `epoch`.
int comm_wait_only(void* const* data, unsigned int* const* flags, int rank, int world, unsigned int epoch,
                   int* err, uint64_t timeout_ns, cudaStream_t stream) {
  comm::Peers peers = make_peers(data, flags, world);
  comm::fence_kernel<<<1, 32, 0, stream>>>(peers, rank, world, epoch, err, timeout_ns);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro
