#include "host_utils.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace ntb {

namespace {
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices] = {0};
int* g_status[kMaxDevices] = {nullptr};
std::mutex g_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    NTB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}
std::atomic<long long> g_launches{0};
}  // namespace

void note_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

int num_sms(int device) {
  if (device < 0 || device >= kMaxDevices) device = 0;
  if (!g_sms[device]) {
    int v = 0;
    NTB_CUDA_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
    g_sms[device] = v;
  }
  return g_sms[device];
}

int* device_status(int device) {
  TORCH_CHECK(device >= 0 && device < kMaxDevices, "bad device");
  if (!g_status[device]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status[device]) {
      int prev;
      NTB_CUDA_CHECK(cudaGetDevice(&prev));
      NTB_CUDA_CHECK(cudaSetDevice(device));
      int* p = nullptr;
      NTB_CUDA_CHECK(cudaMalloc(&p, sizeof(int) * 4));
      NTB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int) * 4));
      NTB_CUDA_CHECK(cudaDeviceSynchronize());
      NTB_CUDA_CHECK(cudaSetDevice(prev));
      g_status[device] = p;
    }
  }
  return g_status[device];
}

int read_and_clear_status(int device) {
  int* p = device_status(device);
  int prev;
  NTB_CUDA_CHECK(cudaGetDevice(&prev));
  NTB_CUDA_CHECK(cudaSetDevice(device));
  NTB_CUDA_CHECK(cudaDeviceSynchronize());
  int v = 0;
  NTB_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) NTB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  NTB_CUDA_CHECK(cudaSetDevice(prev));
  return v;
}

void bind_current_context() {
  static thread_local int bound_device = -1;
  int dev = 0;
  NTB_CUDA_CHECK(cudaGetDevice(&dev));
  if (bound_device != dev) {
    NTB_CUDA_CHECK(cudaSetDevice(dev));
    bound_device = dev;
  }
}

TmaSlots& tls_tma_slots() {
  static thread_local TmaSlots slots;
  return slots;
}

void make_tma_2d(CUtensorMap* out, void* base, CUtensorMapDataType dtype, int elem_bytes, int64_t d0, int64_t d1,
                 int64_t ld, int box0, int box1, CUtensorMapSwizzle swz) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out) & 63) == 0, "tensor map storage must be 64-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1)};
  cuuint32_t estr[2] = {1, 1};
  // The driver call needs a current context; a thread that has not made a
  // runtime call yet (e.g. autograd's device thread) has none.
  bind_current_context();
  CUresult r = encode_fn()(out, dtype, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ") dims=", d0, "x", d1,
              " ld=", ld, " box=", box0, "x", box1);
}

void make_tma_4d_bf16(CUtensorMap* out, const void* base, const int64_t (&dims)[4], const int64_t (&strides)[3],
                      const int (&box)[4]) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out) & 63) == 0, "tensor map storage must be 64-byte aligned");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "tensor map base must be 16-byte aligned");
  cuuint64_t d[4], st[3];
  cuuint32_t bx[4], estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 4; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    bx[i] = static_cast<cuuint32_t>(box[i]);
  }
  for (int i = 0; i < 3; ++i) {
    TORCH_CHECK((strides[i] * 2) % 16 == 0, "tensor map strides must be multiples of 16 bytes");
    st[i] = static_cast<cuuint64_t>(strides[i] * 2);
  }
  bind_current_context();
  CUresult r = encode_fn()(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), d, st, bx, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (4-D) failed (", static_cast<int>(r), ")");
}

void make_tma_2d_bf16(CUtensorMap* out, void* base, int64_t d0, int64_t d1, int64_t ld, int box0, int box1) {
  make_tma_2d(out, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d0, d1, ld, box0, box1, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace ntb
