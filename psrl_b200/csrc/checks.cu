// Host side of the debug-build bounds checks (checks.cuh): whether this build
// has them, and the first failure recorded by any kernel on the current
// device since the last clear.
#include "checks.cuh"

namespace psrl {

bool kernel_checks_enabled() { return chk::kOn; }

// [code, a, b, c, d, failures] of the first translation unit whose record is
// set (all zeros when no check failed or the build has no checks); `clear`
// resets every record.  Synchronises the device.
std::vector<int64_t> kernel_check_status(bool clear) {
  std::vector<int64_t> first(chk::REC, 0);
  if constexpr (chk::kOn) {
    PSRL_CHECK_CUDA(cudaDeviceSynchronize());
    for (chk::Reader r : chk::readers()) {
      int rec[chk::REC];
      r(rec, clear);
      if (first[0] == 0 && rec[0] != 0)
        for (int i = 0; i < chk::REC; ++i) first[i] = rec[i];
    }
  }
  return first;
}

}  // namespace psrl
