// GRAIN backward entry point that allocates no memory.
//
// This entry point has no counterpart in the reference implementation.
//
// Who needs it: a caller that must not allocate device memory during the
// call - C or C++ code that links only this shared library and owns no
// allocator, or a caller that has planned its whole device-memory budget in
// advance and cannot let a library call take more.  The regular entry point
// (`grain_backward` in the Python extension) asks PyTorch's allocator for a
// per-call partial-sum buffer; this one keeps those partials in a fixed
// 256 KiB array in the library's own device memory instead.
//
// Contract:
//   * fp32 tensors only, contiguous, 16-byte aligned for the vector path:
//       gy, x, gx : [rows, hidden]   (may be null when rows == 0)
//       num       : [groups, 6]     den : [groups, 4]
//       grad_num  : [groups, 6]     grad_den : [groups, 4]   (overwritten)
//     with hidden % groups == 0 and hidden / groups <= 256.
//   * Scratch limit: the per-block coefficient partials
//     (blocks x groups x 10 floats, blocks chosen for ~1184 CTAs) must fit in
//     65536 floats; larger problems are rejected with -2 before anything is
//     launched.  At most ~6500 groups fit.
//   * Nothing has to start at zero: every partial that is read is written
//     first by the same call, and grad_num / grad_den are always written
//     (zeros when rows == 0).
//   * Set-up: the first call on each device looks up that device's address
//     of the scratch array (cudaGetSymbolAddress, with that device current)
//     and keeps it for the life of the process.  Make the first call on a
//     device before any stream capture begins.  The kept address belongs to
//     the device's context at that time: after cudaDeviceReset (or anything
//     else that destroys the primary context) it is stale, so do not call
//     this entry point again in that process.
//   * Calls that overlap in time on the same device (two streams, two host
//     threads) share the scratch array and race; serialise them.
//   * Work is enqueued on `stream` (0 = legacy default stream); the call does
//     not synchronise.
//
// Returns 0 on success, -1 for unsupported shapes or pointers, -2 when the
// partials exceed the scratch limit, -3 when the set-up lookup failed, or the
// positive cudaError_t of the first launch that failed (each launch reports
// its own status; an error pending from an earlier, unrelated call is not
// reported here and is left pending).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int ro_grain_backward_noalloc(const float* gy, const float* x, const float* num, const float* den,
                              float* gx, float* grad_num, float* grad_den, int64_t rows,
                              int hidden, int groups, float eps, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
