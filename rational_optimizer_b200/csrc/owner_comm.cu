// Reduce-to-owner of layer gradients over NVLink peer memory.
//
// With layer-sharded optimizers only the owner of a layer needs that layer's
// averaged gradient.  Instead of an all-reduce (every rank receives every
// layer), each rank sends its gradient of a layer straight into a slot of
// the owner's receive buffer, and the owner sums the slots:
//
//   send   (every non-owner, per layer, on the communication stream as soon
//          as backward has produced the layer's gradient): read the fp32
//          gradient, convert to the transport type (bf16 or fp32), store it
//          into slot [sender rank] of the owner's receive buffer with plain
//          16-byte peer stores, then per CTA: __syncthreads, a system-scope
//          fence and one atomic increment of the owner's counter for the layer;
//   reduce (owner, after backward): wait until every sender CTA of every owned
//          layer has arrived (bounded; on expiry an error code is recorded and
//          the reduction is skipped), then sum the slots in rank order with its
//          own fp32 gradient in its rank position, scale by 1/world, write the
//          fp32 result over its own gradient, return each counter to zero for
//          the next step and emit per-CTA sums of squares of the result (the
//          owned part of the global gradient norm).
//
// The next step's sends into a slot cannot start before the owner has
// consumed it: a sender's next backward follows its next forward, which waits
// for the owner's updated weights, which the owner publishes after this
// reduction.  Nothing here uses TMA or multicast on peer memory.
#include "common.cuh"

namespace ro {
namespace owner {

constexpr int kThreads = 512;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads)
send_kernel(const float* __restrict__ src, void* __restrict__ dst, int64_t n, unsigned int* counter) {
  const int64_t nvec = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    float x[8];
    load_vec<float, 8>(src + v * 8, x);
    if constexpr (BF16) store_vec<__nv_bfloat16, 8>(static_cast<__nv_bfloat16*>(dst) + v * 8, x);
    else store_vec<float, 8>(static_cast<float*>(dst) + v * 8, x);
  }
  if (blockIdx.x == 0 && threadIdx.x < n - nvec * 8) {
    const int64_t i = nvec * 8 + threadIdx.x;
    if constexpr (BF16) static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(src[i]);
    else static_cast<float*>(dst)[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    atomicAdd_system(counter, 1u);
  }
}

struct ReduceArgs {
  float* grad;             // this rank's flat gradient buffer
  const void* recv;        // this rank's receive buffer: [layer][world][elems] in transport type
  unsigned int* counters;  // [owned layers]
  const int64_t* offsets;  // [owned layers] element offset of the layer in `grad`
  const int64_t* sizes;    // [owned layers] elements
  const int64_t* recv_offsets;  // [owned layers] element offset of the layer's slots in `recv`
  float* sumsq;            // [gridDim.x] partial sums of squares of the reduced gradient
  int layers, rank, world;
  unsigned int expected;   // arrivals per layer: (world - 1) * sender CTAs
  float scale;
  int* err;
  uint64_t timeout_ns;
};

template <bool BF16>
__global__ void __launch_bounds__(kThreads) reduce_kernel(const __grid_constant__ ReduceArgs a) {
  __shared__ int ok;
  __shared__ float red[kThreads / 32];
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = now_ns();
    for (int l = 0; l < a.layers && ok; ++l) {
      while (load_acquire_sys(a.counters + l) < a.expected) {
        if (*reinterpret_cast<volatile int*>(a.err) != 0 || now_ns() - t0 > a.timeout_ns) {
          atomicCAS(a.err, 0, 11);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  float acc = 0.f;
  if (ok) {
    for (int l = 0; l < a.layers; ++l) {
      const int64_t n = a.sizes[l];
      float* g = a.grad + a.offsets[l];
      const int64_t nvec = n / 8;
      const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
      for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        float s[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          float x[8];
          if (r == a.rank) {
            load_vec<float, 8>(g + v * 8, x);
          } else if constexpr (BF16) {
            load_vec<__nv_bfloat16, 8>(static_cast<const __nv_bfloat16*>(a.recv) + a.recv_offsets[l] + r * n + v * 8, x);
          } else {
            load_vec<float, 8>(static_cast<const float*>(a.recv) + a.recv_offsets[l] + r * n + v * 8, x);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) s[i] += x[i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          s[i] *= a.scale;
          acc = fmaf(s[i], s[i], acc);
        }
        store_vec<float, 8>(g + v * 8, s);
      }
      if (blockIdx.x == 0 && threadIdx.x < n - nvec * 8) {
        const int64_t i = nvec * 8 + threadIdx.x;
        float s = 0.f;
        for (int r = 0; r < a.world; ++r) {
          float x;
          if (r == a.rank) x = g[i];
          else if constexpr (BF16) x = __bfloat162float(static_cast<const __nv_bfloat16*>(a.recv)[a.recv_offsets[l] + r * n + i]);
          else x = static_cast<const float*>(a.recv)[a.recv_offsets[l] + r * n + i];
          s += x;
        }
        s *= a.scale;
        acc = fmaf(s, s, acc);
        g[i] = s;
      }
    }
  }
  // fixed-order block reduction of the squares
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    a.sumsq[blockIdx.x] = t;
  }
}

// Counters return to zero once every CTA of the reduction has read its slots.
__global__ void release_kernel(unsigned int* counters, int layers, unsigned int expected) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l < layers) atomicSub_system(counters + l, expected);
}

}  // namespace owner

int owner_send(const float* src, void* dst, int64_t n, bool bf16, unsigned int* counter, int ctas,
               cudaStream_t stream) {
  using namespace owner;
  if (n <= 0 || ctas <= 0) return -1;
  if (!aligned16(src) || !aligned16(dst)) return -2;
  if (bf16) send_kernel<true><<<ctas, kThreads, 0, stream>>>(src, dst, n, counter);
  else send_kernel<false><<<ctas, kThreads, 0, stream>>>(src, dst, n, counter);
  return static_cast<int>(cudaGetLastError());
}

int owner_reduce(float* grad, const void* recv, unsigned int* counters, const int64_t* offsets,
                 const int64_t* sizes, const int64_t* recv_offsets, float* sumsq, int ctas, int layers,
                 int rank, int world, unsigned int expected, float scale, bool bf16, int* err,
                 uint64_t timeout_ns, cudaStream_t stream) {
  using namespace owner;
  if (layers <= 0) return 0;
  if (ctas <= 0 || world < 2) return -1;
  ReduceArgs a{grad, recv, counters, offsets, sizes, recv_offsets, sumsq, layers, rank, world, expected,
               scale, err, timeout_ns};
  if (bf16) reduce_kernel<true><<<ctas, kThreads, 0, stream>>>(a);
  else reduce_kernel<false><<<ctas, kThreads, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  release_kernel<<<(layers + 31) / 32, 32, 0, stream>>>(counters, layers, expected);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro

// ---------------------------------------------------------------------------
// All-gather of the owners' updated weights, pulled by every other rank.
//
//   publish   (owner, after its optimizer step, main stream): one thread
//             fences at system scope and increments the owner's `published`
//             counter (release).
//   wait      (puller, one thread): spin (bounded) until the owner's
//             published counter has reached the puller's own - every rank
//             publishes once per step, so the owner has finished the same
//             step; the copy that follows on the same stream reads its weights.
//             Waiting again before the next publish returns at once (pulls
//             are idempotent).
//   copy      (puller): 16-byte loads from the owner's weight buffer (peer
//             memory), stores into the local buffer; optionally also the
//             bf16 rounding of the same values into a second local buffer.
//
// An owner overwrites its weights only after it received this rank's next
// gradients, which this rank produces after the forward that waited for the
// copy, so a copy never reads a half-written update.

namespace ro {
namespace owner {

__global__ void publish_kernel(unsigned int* published) {
  __threadfence_system();
  atomicAdd_system(published, 1u);
}

__global__ void wait_kernel(const unsigned int* published, const unsigned int* mine, int* err, uint64_t timeout_ns) {
  const unsigned int want = *reinterpret_cast<const volatile unsigned int*>(mine);
  const uint64_t t0 = now_ns();
  while (static_cast<int>(load_acquire_sys(published) - want) < 0) {
    if (*reinterpret_cast<volatile int*>(err) != 0 || now_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, 12);
      return;  // the copy that follows is skipped (err set)
    }
  }
}

__global__ void __launch_bounds__(kThreads)
copy_kernel(const float* __restrict__ src, float* __restrict__ dst, __nv_bfloat16* __restrict__ dst16, int64_t n,
            const int* err) {
  if (*reinterpret_cast<const volatile int*>(err) != 0) return;
  const int64_t nvec = n / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    float x[8];
    load_vec<float, 8>(src + v * 8, x);
    store_vec<float, 8>(dst + v * 8, x);
    if (dst16 != nullptr) store_vec<__nv_bfloat16, 8>(dst16 + v * 8, x);
  }
  if (blockIdx.x == 0 && threadIdx.x < n - nvec * 8) {
    const int64_t i = nvec * 8 + threadIdx.x;
    dst[i] = src[i];
    if (dst16 != nullptr) dst16[i] = __float2bfloat16_rn(src[i]);
  }
}

}  // namespace owner

int owner_publish(unsigned int* published, cudaStream_t stream) {
  owner::publish_kernel<<<1, 1, 0, stream>>>(published);
  return static_cast<int>(cudaGetLastError());
}

int owner_pull(const float* src, float* dst, __nv_bfloat16* dst16, int64_t n, const unsigned int* published,
               const unsigned int* mine, int* err, uint64_t timeout_ns, int ctas, cudaStream_t stream) {
  using namespace owner;
  if (n <= 0 || ctas <= 0) return -1;
  if (!aligned16(src) || !aligned16(dst) || (dst16 != nullptr && !aligned16(dst16))) return -2;
  wait_kernel<<<1, 1, 0, stream>>>(published, mine, err, timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  copy_kernel<<<ctas, kThreads, 0, stream>>>(src, dst, dst16, n, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace ro
