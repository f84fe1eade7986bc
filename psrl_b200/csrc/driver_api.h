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

// Driver-API calls act on the calling thread's current context, which the
// runtime binds to a host thread only lazily.  A thread that has not made a
// runtime call needing the context yet (a fresh worker thread, the autograd
// engine's device thread) would call the driver with no current context, and
// some entry points (cuTensorMapEncodeTiled among them) do not survive that.
// cudaFree(nullptr) binds the current device's primary context; once per
// thread and device.
inline void bind_thread_context() {
  thread_local int bound_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (dev != bound_dev) {
    cudaFree(nullptr);
    bound_dev = dev;
  }
}

}  // namespace drv
}  // namespace psrl

// PSRL_DRV(cuMemCreate)(...) calls the driver function; the pointer is looked
// up once per call site.  The string keeps the unversioned API name; the
// pointer type follows cuda.h's (possibly versioned) declaration.
#define PSRL_DRV(name)                                                                   \
  ([]() {                                                                                \
    ::psrl::drv::bind_thread_context();                                                  \
    static const auto fn_ = reinterpret_cast<decltype(&::name)>(::psrl::drv::entry(#name)); \
    return fn_;                                                                          \
  }())
