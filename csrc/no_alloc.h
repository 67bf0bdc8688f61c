// Allocation-free C entry point for the RMSNorm backward kernel.
//
// No counterpart in the reference: it has no native code at all, and its
// RMSNorm backward is PyTorch autograd. This entry exists for callers that
// must not allocate device memory - a C or C++ host program that drives the
// kernel without PyTorch's caching allocator, or code that runs while another
// runtime owns nearly all of the device memory, or a latency-critical path
// that cannot afford cudaMalloc's implicit device-wide synchronisation. The
// PyTorch binding (rmsnorm_bwd) allocates its partial-sum scratch per call;
// this entry instead uses a fixed scratch array that lives in the module's
// static device memory.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest hidden size accepted (the scratch holds 128 partial rows of this width, 2 MiB of fp32;
// the kernel runs at most 128 CTAs, one partial row each).
#define NTB_NOALLOC_RMSNORM_MAX_H 4096

// dx[rows, H] = d/dx of y = h * rstd * w given dy (bf16, row-major, contiguous), plus dres when
// dres is non-null (gradient arriving along the residual stream). dw[H] (fp32) receives the full
// weight gradient; it is overwritten, so nothing has to start at zero, and neither does the scratch.
// rstd[rows] is the fp32 reciprocal RMS saved by the forward pass. All pointers are device pointers;
// the work is queued on `stream` and the call returns without synchronising.
//
// Returns 0 on success, or a non-zero code with a message from ntb_noalloc_last_error():
//   1  H is not in [1, NTB_NOALLOC_RMSNORM_MAX_H] or rows < 0
//   2  a CUDA call failed (set-up or launch)
//   3  an error from earlier, unrelated CUDA work was already pending on this thread; nothing was
//      launched and the error is left pending (cudaPeekAtLastError) for the code that caused it
// The first call on each device does the set-up (it looks up the scratch address with
// cudaGetSymbolAddress, which can load the module), so make it before any stream capture. The
// set-up belongs to the context that was current when it ran: the address is looked up again
// when a call finds a different context current on that device (after cudaDeviceReset, or once
// the primary context was released and re-created), so that first call of a new context should
// also come before any capture.
// Calls on one device share one scratch array: calls that overlap in time on that device (other
// streams, other host threads) race on it and must be ordered by the caller.
int ntb_rmsnorm_bwd_bf16_noalloc(const void* dy, const void* h, const void* w, const float* rstd,
                                 const void* dres, void* dx, float* dw, int64_t rows, int H, cudaStream_t stream);

// Message of the last failed call from this host thread ("" after a success).
const char* ntb_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
