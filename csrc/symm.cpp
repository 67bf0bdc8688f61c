// Symmetric memory for one node: every rank cudaMalloc's a buffer of the
// same size, exports a CUDA IPC handle, and opens its peers' handles, so each
// rank's kernels can address every peer buffer directly over NVLink.
// Handles are exchanged by the Python layer through the process group.
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <string>

#include "host_utils.h"

namespace ntb {

// Allocates `bytes` of zeroed device memory on the current device and returns
// (address, IPC handle bytes).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t bytes) {
  TORCH_CHECK(bytes > 0, "symm_alloc: size must be positive");
  bind_current_context();
  void* p = nullptr;
  NTB_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  NTB_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  NTB_CUDA_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  NTB_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return {reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  bind_current_context();
  void* p = nullptr;
  NTB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t peer_ptr) { NTB_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(peer_ptr))); }

void symm_free(int64_t ptr) { NTB_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

// Tensor view of this rank's OWN symmetric buffer (never of a peer's), so
// ordinary torch ops can fill or read local slots.
at::Tensor symm_local_view(int64_t ptr, int64_t offset_bytes, std::vector<int64_t> sizes, at::ScalarType dtype,
                           int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<int>(device));
  return at::from_blob(reinterpret_cast<char*>(ptr) + offset_bytes, sizes, opts);
}

}  // namespace ntb
