// Virtual-memory regions with releasable physical backing (N9 / N10).
//
// A region reserves a virtual address range once (cuMemAddressReserve) and
// maps physical memory into it (cuMemCreate + cuMemMap + cuMemSetAccess).
// sleep() optionally copies the contents to pinned host memory, then unmaps
// and releases the physical pages (the VA stays reserved, so tensors viewing
// it keep their addresses); wake() maps fresh physical memory at the same VA
// and restores the backup.  This is how rollout weights / KV caches and
// training state are paused to share a GPU between roles.  Physical handles
// are created as POSIX-fd exportable so peers can map them.
#include <cuda.h>

#include "driver_api.h"
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <memory>

namespace psrl {

#define CU_CHECK(x)                                                                  \
  do {                                                                               \
    CUresult _r = (x);                                                               \
    if (_r != CUDA_SUCCESS) {                                                        \
      const char* msg = nullptr;                                                     \
      PSRL_DRV(cuGetErrorString)(_r, &msg);                                                    \
      TORCH_CHECK(false, "CUDA driver error ", (int)_r, " (", msg ? msg : "?", ") at ", #x); \
    }                                                                                \
  } while (0)

class VmmRegion {
 public:
  VmmRegion(int64_t bytes, int64_t device) : device_((int)device) {
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device_;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    CU_CHECK(PSRL_DRV(cuMemGetAllocationGranularity)(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    size_ = ((size_t)bytes + gran - 1) / gran * gran;
    prop_ = prop;
    CU_CHECK(PSRL_DRV(cuMemAddressReserve)(&va_, size_, gran, 0, 0));
    map_();
  }
  ~VmmRegion() {
    if (mapped_) {
      PSRL_DRV(cuMemUnmap)(va_, size_);
      PSRL_DRV(cuMemRelease)(handle_);
    }
    if (va_) PSRL_DRV(cuMemAddressFree)(va_, size_);
    if (host_) cudaFreeHost(host_);
  }
  int64_t ptr() const { return (int64_t)va_; }
  int64_t size() const { return (int64_t)size_; }
  bool awake() const { return mapped_; }

  void sleep(bool backup) {
    TORCH_CHECK(mapped_, "region is already asleep");
    TORCH_CHECK(cudaDeviceSynchronize() == cudaSuccess, "device sync failed before sleep");
    if (backup) {
      if (!host_) TORCH_CHECK(cudaMallocHost(&host_, size_) == cudaSuccess, "pinned backup alloc failed");
      TORCH_CHECK(cudaMemcpy(host_, (void*)va_, size_, cudaMemcpyDeviceToHost) == cudaSuccess, "backup copy failed");
      has_backup_ = true;
    } else {
      has_backup_ = false;
    }
    CU_CHECK(PSRL_DRV(cuMemUnmap)(va_, size_));
    CU_CHECK(PSRL_DRV(cuMemRelease)(handle_));
    mapped_ = false;
  }

  void wake() {
    TORCH_CHECK(!mapped_, "region is awake");
    map_();
    if (has_backup_) {
      TORCH_CHECK(cudaMemcpy((void*)va_, host_, size_, cudaMemcpyHostToDevice) == cudaSuccess, "restore failed");
    } else {
      TORCH_CHECK(cudaMemset((void*)va_, 0, size_) == cudaSuccess, "zero fill failed");
    }
    TORCH_CHECK(cudaDeviceSynchronize() == cudaSuccess, "device sync failed after wake");
  }

 private:
  void map_() {
    CU_CHECK(PSRL_DRV(cuMemCreate)(&handle_, size_, &prop_, 0));
    CU_CHECK(PSRL_DRV(cuMemMap)(va_, size_, 0, handle_, 0));
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device_;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    CU_CHECK(PSRL_DRV(cuMemSetAccess)(va_, size_, &acc, 1));
    mapped_ = true;
  }
  int device_;
  size_t size_ = 0;
  CUdeviceptr va_ = 0;
  CUmemGenericAllocationHandle handle_{};
  CUmemAllocationProp prop_{};
  bool mapped_ = false;
  bool has_backup_ = false;
  void* host_ = nullptr;
};

void register_vmm(pybind11::module& m) {
  pybind11::class_<VmmRegion, std::shared_ptr<VmmRegion>>(m, "VmmRegion")
      .def(pybind11::init<int64_t, int64_t>())
      .def("ptr", &VmmRegion::ptr)
      .def("size", &VmmRegion::size)
      .def("awake", &VmmRegion::awake)
      .def("sleep", &VmmRegion::sleep)
      .def("wake", &VmmRegion::wake);
}

}  // namespace psrl
