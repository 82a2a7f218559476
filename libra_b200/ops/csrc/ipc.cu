// CUDA IPC helpers for peer-memory kernels.
//
// A peer buffer must be mapped into the context of the device whose kernels
// read it: opening the handle with that device current and
// cudaIpcMemLazyEnablePeerAccess gives a pointer those kernels can
// dereference over NVLink.  (Rebuilding a shared torch tensor maps it on the
// exporting device's index instead, which a kernel on another device cannot
// dereference without separately enabled peer access.)
#include <torch/extension.h>

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace libra {
namespace ipc {

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetRangeFn get_range() {
  static GetRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    LIBRA_CHECK(cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess && p,
                "ipc: cuMemGetAddressRange is unavailable");
    fn = reinterpret_cast<GetRangeFn>(p);
  }
  return fn;
}

// Returns (handle bytes of the allocation that contains t, byte offset of t in it).
std::tuple<py::bytes, int64_t> ipc_export(torch::Tensor t) {
  LIBRA_CHECK(t.is_cuda(), "ipc_export: CUDA tensor required");
  cudaFree(nullptr);  // bind the device's primary context on this thread
  CUdeviceptr base = 0;
  size_t size = 0;
  LIBRA_CHECK(get_range()(&base, &size, (CUdeviceptr)(uintptr_t)t.data_ptr()) == CUDA_SUCCESS,
              "ipc_export: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>((uintptr_t)base));
  LIBRA_CHECK(e == cudaSuccess, "ipc_export: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  return {py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)),
          (int64_t)((uintptr_t)t.data_ptr() - (uintptr_t)base)};
}

// Maps a peer allocation into the current device's context; returns its base address.
int64_t ipc_open(py::bytes handle) {
  std::string s = handle;
  LIBRA_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  LIBRA_CHECK(e == cudaSuccess, "ipc_open: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
  return (int64_t)(uintptr_t)p;
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>((uintptr_t)ptr)); }

}  // namespace ipc
}  // namespace libra
