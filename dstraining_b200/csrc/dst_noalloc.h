// C entry point of dstraining_b200 that allocates no device memory.
//
// This entry point has no counterpart in the reference implementation
// (mohamadmsalman82/dstraining is pure PyTorch and exposes no C API); it is
// an addition of this library.
//
// Who it is for: callers that cannot allocate device memory themselves. A
// plugin or custom operator hosted by another runtime usually has to take
// every byte of device memory from its host's allocator (the host owns the
// memory pool and its budget), and a caller on a latency-critical path may
// not afford cudaMalloc/cudaFree, which can synchronise the whole device.
// Those callers pass their own input and output buffers; the scratch space
// this operation needs lives in a fixed array inside the library.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of dst_layernorm_bwd_noalloc.
#define DST_NOALLOC_OK 0
#define DST_NOALLOC_ERR_TOO_LARGE 1   // hidden size above DST_NOALLOC_MAX_HIDDEN
#define DST_NOALLOC_ERR_BAD_ARG 2     // null or misaligned pointer, rows < 1, hidden not a multiple of 8
#define DST_NOALLOC_ERR_CUDA 3        // a CUDA call failed (set-up or launch)

// Largest hidden size (last dimension) the fixed scratch array supports.
#define DST_NOALLOC_MAX_HIDDEN 4096
// Number of partial rows the scratch array holds (two per CTA: dgamma and
// dbeta), which caps the CTAs of the first pass; any row count is accepted.
#define DST_NOALLOC_MAX_CTAS 296

// LayerNorm backward over the last dimension, bf16 tensors, fp32 statistics,
// without allocating device memory:
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = w * dy,
//   xhat = (x - mean) * rstd,  dw = sum_rows(dy * xhat),  db = sum_rows(dy)
//
//   dy, x, dx : [rows, hidden] bf16, row-major, contiguous
//   w, dw, db : [hidden] bf16
//   mean, rstd: [rows] fp32 (as saved by the forward pass)
//   alignment : dy, x, w and dx start on a 16-byte boundary (they are moved
//               in 16-byte vectors), mean and rstd on 4 bytes, dw and db on 2;
//               a misaligned pointer returns DST_NOALLOC_ERR_BAD_ARG
//   stream    : the stream the work is queued on (0 = legacy default stream)
//
// Any hidden size from 8 to DST_NOALLOC_MAX_HIDDEN (a multiple of 8) is
// handled in full.
//
// Scratch: a static device array of 2 * DST_NOALLOC_MAX_CTAS *
// DST_NOALLOC_MAX_HIDDEN floats (9.25 MiB) compiled into the library; every
// GPU that loads the library holds it until the process exits. Each call
// overwrites every scratch element it reads, so no clearing is needed between
// calls, but all calls share the one array: calls whose work overlaps on the
// GPU (different streams, or different host threads, on the same device)
// race on it and must be serialised by the caller.
//
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current; make that first call
// before any stream capture on the device.
//
// Returns DST_NOALLOC_OK once the kernels are queued (errors inside the
// kernels surface at the next synchronisation), or one of the codes above;
// on DST_NOALLOC_ERR_TOO_LARGE / DST_NOALLOC_ERR_BAD_ARG nothing is queued.
int dst_layernorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* mean, const float* rstd,
                              void* dx, void* dw, void* db, int rows, int hidden, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
