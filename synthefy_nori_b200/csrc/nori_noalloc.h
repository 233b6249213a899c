// Allocation-free entry point of the attention backward pass.
//
// This entry point has no counterpart in the reference implementation. It exists for
// callers that cannot call cudaMalloc: engines that reserve all device memory in a fixed
// pool at start-up and forbid any later allocation, and plain C / FFI hosts that link
// this library without PyTorch's caching allocator (so a per-call scratch buffer has
// nowhere to come from). The regular entry point
// (`nori::attn_bwd`, Python `ops.attention_bwd`) allocates a per-call scratch vector for
// the row dot products dO . O; this variant keeps that scratch in a fixed file-scope
// device array instead.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest BH * Nq (query rows over all heads) accepted: the scratch array holds one
// float per row, 4 MiB per device that loads the library, held until the process exits.
#define NORI_NOALLOC_MAX_ROWS (1u << 20)

// Flash-attention backward without any allocation.
//
//   q, k, v, o, dout : bf16 device pointers; a layout is six int64 values
//                      (s0, s1, s2, row_stride, d1, d2): head bh decomposes as
//                      i2 = bh % d2, i1 = (bh / d2) % d1, i0 = bh / (d1 * d2) and row r
//                      of head bh starts at element i0*s0 + i1*s1 + i2*s2 + r*row_stride.
//   lse              : fp32 [BH, Nq] natural-log row log-sum-exp from the forward pass.
//   dq               : fp32 [BH, Nq, 64] head-major; this function zeroes it, then
//                      accumulates the (scaled) query gradient into it.
//   dk, dv           : bf16 outputs written through their layouts.
//   stream           : the stream to run on (0 = legacy default stream).
//
// Returns cudaSuccess, or cudaErrorInvalidValue when BH * Nq exceeds
// NORI_NOALLOC_MAX_ROWS or an argument is malformed: a null or misaligned pointer (the
// bf16 tensors and dq 16-byte aligned, lse 4-byte aligned), a layout stride that is
// negative or not a multiple of 8 elements, or a layout d1 / d2 that is not positive
// (nori_attention_bwd_noalloc_error() then gives a one-line reason). Every check runs
// before any work is queued, so a rejected call leaves dq, dk, dv and the scratch alone.
// The first call on each device looks up the scratch array's device address with
// cudaGetSymbolAddress (once per device; later calls reuse it). Every call on a device
// shares the one scratch array and overwrites it, so calls that may overlap on the GPU
// (different streams without ordering) race.
cudaError_t nori_attention_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                       const float* lse, float* dq, void* dk, void* dv, const int64_t* lq,
                                       const int64_t* lk, const int64_t* lv, const int64_t* lo, const int64_t* ldo,
                                       const int64_t* ldk, const int64_t* ldv, int64_t BH, int64_t Nq, int64_t Nk,
                                       int64_t d_valid, double scale, cudaStream_t stream);

// Reason for the last cudaErrorInvalidValue returned on this thread (empty if none).
const char* nori_attention_bwd_noalloc_error(void);

#ifdef __cplusplus
}
#endif
