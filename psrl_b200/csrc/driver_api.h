// Driver-API entry points resolved at run time through the CUDA runtime
// (cudaGetDriverEntryPointByVersion at the older of the cuda.h this file is
// compiled against and the runtime loaded in the process, which may be the
// one PyTorch ships), so the extension does not link libcuda: it imports on a
// host without an NVIDIA driver (a build machine) and a driver call fails with
// an exception only when it is made.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace psrl {
namespace drv {

inline void* entry(const char* name) {
  void* fn = nullptr;
  int rt = 0;
  if (cudaRuntimeGetVersion(&rt) != cudaSuccess || rt <= 0 || rt > CUDA_VERSION) rt = CUDA_VERSION;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &fn, (unsigned)rt, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
    throw std::runtime_error(std::string("CUDA driver entry point unavailable: ") + name + " (" +
                             cudaGetErrorString(e) + ")");
  return fn;
}

}  // namespace drv
}  // namespace psrl

// PSRL_DRV(cuMemCreate)(...) calls the driver function; the pointer is looked
// up once per call site.  The string keeps the unversioned API name; the
// pointer type follows cuda.h's (possibly versioned) declaration.
#define PSRL_DRV(name)                                                                   \
  ([]() {                                                                                \
    static const auto fn_ = reinterpret_cast<decltype(&::name)>(::psrl::drv::entry(#name)); \
    return fn_;                                                                          \
  }())
