// Reduce-to-owner of layer gradients over NVLink peer memory.
//
// With layer-sharded optimizers only the owner of a layer needs that layer's
// averaged gradient.  Instead of an all-reduce (every rank receives every
// layer), each rank sends its gradient of a layer straight into a slot of
// the owner's receive buffer, and the owner sums the slots:
//
//   send   (every non-owner, per layer, on the communication stream as soon
//          as backward has produced the layer's gradient): read the fp32
//          gradient, convert to the transport format, store it into slot
//          [sender rank] of the owner's receive buffer with plain peer stores,
//          then per CTA: __syncthreads, a system-scope fence and one atomic
//          increment of the owner's counter for the layer.  Formats: fp32,
//          bf16, or int8 with one fp32 scale per 256-element block (a warp
//          quantises one block: scale = max|g| / 127, q = round(g / scale)
//          clamped to [-127, 127]; the slot holds the n int8 values, padded
//          to 16 bytes, then the block scales);
//          A sender may instead let the layer's weight-gradient GEMMs store
//          their fp32 tiles straight into the slot (peer stores from the GEMM
//          epilogue, tile by tile) and then signal the arrivals (signal_kernel);
//   reduce (owner, after backward): wait until every sender CTA of every owned
//          layer has arrived (bounded; on expiry an error code is recorded and
//          the reduction is skipped), then sum the slots (int8: dequantised,
//          q * scale) in rank order with its own fp32 gradient in its rank
//          position, scale by 1/world, write the
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
constexpr int kUnroll = 4;  // 8-element vectors per thread per pass in the copy loops
constexpr int kF32 = 0, kBF16 = 1, kI8 = 2;  // transport formats
constexpr int kQBlock = 256;                   // int8: elements per fp32 scale

__host__ __device__ __forceinline__ int64_t round16(int64_t bytes) { return (bytes + 15) / 16 * 16; }

// Bytes of one sender's slot of an n-element layer (n a multiple of 8).
__host__ __device__ __forceinline__ int64_t slot_bytes(int64_t n, int mode) {
  if (mode == kF32) return 4 * n;
  if (mode == kBF16) return 2 * n;
  return round16(n) + round16(4 * ((n + kQBlock - 1) / kQBlock));
}

__device__ __forceinline__ uint32_t pack_i8x4(const float* q) {
  return (static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q[0])))) |
         (static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q[1]))) << 8) |
         (static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q[2]))) << 16) |
         (static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q[3]))) << 24);
}

__device__ __forceinline__ void unpack_i8x8(uint2 raw, float scale, float (&x)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = static_cast<float>(static_cast<int8_t>((raw.x >> (8 * i)) & 0xffu)) * scale;
    x[4 + i] = static_cast<float>(static_cast<int8_t>((raw.y >> (8 * i)) & 0xffu)) * scale;
  }
}

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

template <int MODE>
__global__ void __launch_bounds__(kThreads)
send_kernel(const float* __restrict__ src, void* __restrict__ dst, int64_t n, unsigned int* counter) {
  const int64_t nvec = n / 8;
  if constexpr (MODE == kI8) {
    // one warp per 256-element block; lane l owns elements [8l, 8l + 8)
    int8_t* q8 = static_cast<int8_t*>(dst);
    float* scales = reinterpret_cast<float*>(q8 + round16(n));
    const int lane = threadIdx.x & 31;
    const int64_t blocks = (n + kQBlock - 1) / kQBlock;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    // kUnroll blocks per warp per pass, loads first (bytes in flight)
    for (int64_t b0 = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5); b0 < blocks;
         b0 += warps * kUnroll) {
      float x[kUnroll][8];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t e0 = (b0 + u * warps) * kQBlock + lane * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) x[u][i] = 0.f;
        // n is a multiple of 8: a lane's 8 elements are all in or all out
        if (b0 + u * warps < blocks && e0 < n) load_vec<float, 8>(src + e0, x[u]);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t b = b0 + u * warps;
        if (b >= blocks) break;  // uniform across the warp
        const int64_t e0 = b * kQBlock + lane * 8;
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[u][i]));
        amax = warp_max(amax);
        const float inv = amax > 0.f ? 127.0f / amax : 0.f;
        float q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = fminf(fmaxf(rintf(x[u][i] * inv), -127.f), 127.f);
        if (e0 < n) *reinterpret_cast<uint2*>(q8 + e0) = make_uint2(pack_i8x4(q), pack_i8x4(q + 4));
        if (lane == 0) scales[b] = amax / 127.0f;
      }
    }
  } else {
    // kUnroll vectors per thread per pass: their loads are all issued before
    // the first peer store, so a few CTAs keep enough bytes in flight
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t v0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v0 < nvec;
         v0 += stride * kUnroll) {
      float x[kUnroll][8];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (v0 + u * stride < nvec) load_vec<float, 8>(src + (v0 + u * stride) * 8, x[u]);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = v0 + u * stride;
        if (v >= nvec) break;
        if constexpr (MODE == kBF16) store_vec<__nv_bfloat16, 8>(static_cast<__nv_bfloat16*>(dst) + v * 8, x[u]);
        else store_vec<float, 8>(static_cast<float*>(dst) + v * 8, x[u]);
      }
    }
    if (blockIdx.x == 0 && threadIdx.x < n - nvec * 8) {
      const int64_t i = nvec * 8 + threadIdx.x;
      if constexpr (MODE == kBF16) static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(src[i]);
      else static_cast<float*>(dst)[i] = src[i];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && counter != nullptr) {
    __threadfence_system();
    atomicAdd_system(counter, 1u);
  }
}

// Arrival for data that reached the owner's slot by other kernels earlier on
// this stream (a weight-gradient GEMM storing its tiles there, sends without
// a counter): the system-scope fence orders those stores (stream order makes
// them precede this kernel) before the counter increment the owner acquires.
__global__ void signal_kernel(unsigned int* counter, unsigned int count) {
  __threadfence_system();
  atomicAdd_system(counter, count);
}

struct ReduceArgs {
  float* grad;             // this rank's flat gradient buffer
  const void* recv;        // this rank's receive buffer: [layer][world][elems] in transport type
  unsigned int* counters;  // [owned layers]
  const int64_t* offsets;  // [owned layers] element offset of the layer in `grad`
  const int64_t* sizes;    // [owned layers] elements
  const int64_t* recv_offsets;  // [owned layers] byte offset of the layer's slots in `recv`
  float* sumsq;            // [gridDim.x] partial sums of squares of the reduced gradient
  int layers, rank, world;
  unsigned int expected;   // arrivals per layer: (world - 1) * sender CTAs
  float scale;
  int* err;
  uint64_t timeout_ns;
};

template <int MODE>
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
      const int64_t slot = slot_bytes(n, MODE);
      const uint8_t* base = static_cast<const uint8_t*>(a.recv) + a.recv_offsets[l];
      const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
      for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        float s[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          float x[8];
          const uint8_t* from = base + r * slot;
          if (r == a.rank) {
            load_vec<float, 8>(g + v * 8, x);
          } else if constexpr (MODE == kI8) {
            const float scale = reinterpret_cast<const float*>(from + round16(n))[v / (kQBlock / 8)];
            unpack_i8x8(*reinterpret_cast<const uint2*>(from + v * 8), scale, x);
          } else if constexpr (MODE == kBF16) {
            load_vec<__nv_bfloat16, 8>(reinterpret_cast<const __nv_bfloat16*>(from) + v * 8, x);
          } else {
            load_vec<float, 8>(reinterpret_cast<const float*>(from) + v * 8, x);
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
      if (MODE != kI8 && blockIdx.x == 0 && threadIdx.x < n - nvec * 8) {
        const int64_t i = nvec * 8 + threadIdx.x;
        float s = 0.f;
        for (int r = 0; r < a.world; ++r) {
          const uint8_t* from = base + r * slot;
          float x;
          if (r == a.rank) x = g[i];
          else if constexpr (MODE == kBF16) x = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(from)[i]);
          else x = reinterpret_cast<const float*>(from)[i];
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

int64_t owner_slot_bytes(int64_t n, int mode) { return owner::slot_bytes(n, mode); }

int owner_signal(unsigned int* counter, unsigned int count, cudaStream_t stream) {
  owner::signal_kernel<<<1, 1, 0, stream>>>(counter, count);
  return static_cast<int>(cudaGetLastError());
}

// fp32 send by a copy engine: one device-to-device copy into the owner's
// slot (peer memory through the IPC mapping), so no SM works on the send.
// The arrival is a separate owner_signal after it on the same stream: stream
// order makes the copy complete before that kernel fences and increments.
int owner_copy(const float* src, void* dst, int64_t n, cudaStream_t stream) {
  if (n <= 0) return -1;
  if (!aligned16(src) || !aligned16(dst)) return -2;
  return static_cast<int>(cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * sizeof(float),
                                          cudaMemcpyDeviceToDevice, stream));
}

int owner_send(const float* src, void* dst, int64_t n, int mode, unsigned int* counter, int ctas,
               cudaStream_t stream) {
  using namespace owner;
  if (n <= 0 || ctas <= 0 || mode < kF32 || mode > kI8) return -1;
  if (!aligned16(src) || !aligned16(dst) || (mode == kI8 && n % 8 != 0)) return -2;
  if (mode == kI8) send_kernel<kI8><<<ctas, kThreads, 0, stream>>>(src, dst, n, counter);
  else if (mode == kBF16) send_kernel<kBF16><<<ctas, kThreads, 0, stream>>>(src, dst, n, counter);
  else send_kernel<kF32><<<ctas, kThreads, 0, stream>>>(src, dst, n, counter);
  return static_cast<int>(cudaGetLastError());
}

int owner_reduce(float* grad, const void* recv, unsigned int* counters, const int64_t* offsets,
                 const int64_t* sizes, const int64_t* recv_offsets, float* sumsq, int ctas, int layers,
                 int rank, int world, unsigned int expected, float scale, int mode, int* err,
                 uint64_t timeout_ns, cudaStream_t stream) {
  using namespace owner;
  if (layers <= 0) return 0;
  if (ctas <= 0 || world < 2 || mode < kF32 || mode > kI8) return -1;
  ReduceArgs a{grad, recv, counters, offsets, sizes, recv_offsets, sumsq, layers, rank, world, expected,
               scale, err, timeout_ns};
  if (mode == kI8) reduce_kernel<kI8><<<ctas, kThreads, 0, stream>>>(a);
  else if (mode == kBF16) reduce_kernel<kBF16><<<ctas, kThreads, 0, stream>>>(a);
  else reduce_kernel<kF32><<<ctas, kThreads, 0, stream>>>(a);
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
  // kUnroll peer loads in flight per thread before the first store (remote
  // latency is several times local latency)
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v0 < nvec;
       v0 += stride * kUnroll) {
    float x[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (v0 + u * stride < nvec) load_vec<float, 8>(src + (v0 + u * stride) * 8, x[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = v0 + u * stride;
      if (v >= nvec) break;
      store_vec<float, 8>(dst + v * 8, x[u]);
      if (dst16 != nullptr) store_vec<__nv_bfloat16, 8>(dst16 + v * 8, x[u]);
    }
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
