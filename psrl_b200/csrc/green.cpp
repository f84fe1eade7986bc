// Spatial SM partitions for a trainer and a rollout engine that share one GPU.
//
// Overlapped colocation runs training kernels and decode kernels at the same
// time.  Large training GEMMs are persistent (one CTA per SM, looping over
// tiles), so a decode kernel queued behind one waits for the whole GEMM even on
// a high-priority stream.  A CUDA green context owns a disjoint subset of the
// SMs: the trainer's stream lives in one that leaves `reserve` SMs out, so a
// decode kernel always finds those SMs free (and still uses every SM when the
// trainer is idle, since the rollout engine stays on an ordinary stream).
//
// green_partition(device, reserve_sms, priority) splits the device's SMs into
// aligned groups (cuDevSmResourceSplitByCount), keeps the first groups covering
// at least `reserve_sms` out, builds one green context from the remaining
// groups plus the split's remainder, and returns a stream of that context.
// Contexts and streams live until process exit.
#include <cuda.h>

#include "driver_api.h"
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include <mutex>
#include <vector>

namespace py = pybind11;

namespace psrl {

namespace {
struct Partition {
  CUgreenCtx gctx = nullptr;
  CUstream stream = nullptr;
  unsigned sms = 0, reserved = 0, total = 0;
};
std::mutex g_mu;
std::vector<Partition> g_parts;   // kept alive until exit

void check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* msg = nullptr;
    PSRL_DRV(cuGetErrorString)(r, &msg);
    TORCH_CHECK(false, what, " failed: ", msg ? msg : "unknown", " (", (int)r, ")");
  }
}
}  // namespace

py::dict green_partition(int64_t device, int64_t reserve_sms, int64_t priority) {
  std::lock_guard<std::mutex> lk(g_mu);
  CUdevice dev;
  check(PSRL_DRV(cuDeviceGet)(&dev, (int)device), "cuDeviceGet");
  CUdevResource all;
  check(PSRL_DRV(cuDeviceGetDevResource)(dev, &all, CU_DEV_RESOURCE_TYPE_SM), "cuDeviceGetDevResource");
  const unsigned total = all.sm.smCount;
  TORCH_CHECK(reserve_sms > 0 && (unsigned)reserve_sms < total, "reserve_sms must be in (0, ", total, ")");
  // groups of 8 SMs (the split's alignment on this architecture)
  unsigned n = 0;
  check(PSRL_DRV(cuDevSmResourceSplitByCount)(nullptr, &n, &all, nullptr, 0, 8), "cuDevSmResourceSplitByCount(query)");
  TORCH_CHECK(n >= 2, "cannot split the SMs into groups");
  std::vector<CUdevResource> groups(n);
  CUdevResource rest{};
  check(PSRL_DRV(cuDevSmResourceSplitByCount)(groups.data(), &n, &all, &rest, 0, 8), "cuDevSmResourceSplitByCount");
  unsigned reserved = 0, k = 0;
  while (k < n && reserved < (unsigned)reserve_sms) reserved += groups[k++].sm.smCount;
  TORCH_CHECK(k < n, "reserve_sms leaves no SM group for the trainer");
  std::vector<CUdevResource> mine(groups.begin() + k, groups.begin() + n);
  if (rest.sm.smCount > 0) mine.push_back(rest);
  unsigned sms = 0;
  for (auto& g : mine) sms += g.sm.smCount;
  CUdevResourceDesc desc;
  check(PSRL_DRV(cuDevResourceGenerateDesc)(&desc, mine.data(), (unsigned)mine.size()), "cuDevResourceGenerateDesc");
  Partition p;
  check(PSRL_DRV(cuGreenCtxCreate)(&p.gctx, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM), "cuGreenCtxCreate");
  check(PSRL_DRV(cuGreenCtxStreamCreate)(&p.stream, p.gctx, CU_STREAM_NON_BLOCKING, (int)priority), "cuGreenCtxStreamCreate");
  p.sms = sms;
  p.reserved = reserved;
  p.total = total;
  g_parts.push_back(p);
  py::dict d;
  d["stream"] = (int64_t)(uintptr_t)p.stream;
  d["sms"] = (int64_t)sms;
  d["reserved_sms"] = (int64_t)reserved;
  d["total_sms"] = (int64_t)total;
  return d;
}

}  // namespace psrl
