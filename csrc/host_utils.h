// Host-side helpers shared by the extension's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>

#define NTB_CUDA_CHECK(expr)                                                                 \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, \
                ":", __LINE__, " in ", #expr);                                               \
  } while (0)

namespace ntb {

// Count of kernels this extension has launched (process-wide), for the
// benchmark's launch accounting.
void note_launches(int n);
long long launch_count();

#define NTB_LAUNCH_CHECK(n)          \
  do {                               \
    ::ntb::note_launches(n);         \
    NTB_CUDA_CHECK(cudaGetLastError()); \
  } while (0)

// Number of SMs of a device (cached).
int num_sms(int device);

// Per-device status word that kernels raise on a bounded-wait timeout or a
// rejected shape (see StatusCode in common.cuh). Allocated once per device.
int* device_status(int device);

// Reads and clears the status word of a device (synchronises the device).
int read_and_clear_status(int device);

// Tensor maps are written into caller-provided storage that must be 64-byte
// aligned (the driver stores them with aligned vector writes). Host code
// keeps them in thread-local aligned slots (TmaSlots) and launches kernels
// with cudaLaunchKernel by pointer, never copying a CUtensorMap through an
// ordinary stack frame whose alignment is not guaranteed.
struct alignas(128) TmaSlots {
  CUtensorMap m[4];
};
TmaSlots& tls_tma_slots();

// Makes the current device's primary context current on this thread.
void bind_current_context();

// 2-D TMA descriptor for a bf16 matrix with inner extent d0 (contiguous),
// outer extent d1, row pitch ld (elements), box box0 x box1, 128-byte swizzle.
void make_tma_2d_bf16(CUtensorMap* out, void* base, int64_t d0, int64_t d1, int64_t ld, int box0, int box1);
// bf16, 128-byte swizzle; dims innermost first, strides (in elements) of dims 1..3.
void make_tma_4d_bf16(CUtensorMap* out, const void* base, const int64_t (&dims)[4], const int64_t (&strides)[3],
                      const int (&box)[4]);

// Same for an arbitrary element size in bytes with a chosen swizzle.
void make_tma_2d(CUtensorMap* out, void* base, CUtensorMapDataType dtype, int elem_bytes, int64_t d0, int64_t d1,
                 int64_t ld, int box0, int box1, CUtensorMapSwizzle swz);

}  // namespace ntb
