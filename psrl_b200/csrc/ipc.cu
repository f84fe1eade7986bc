// Peer-memory plumbing for the trainer -> rollout weight sync (K17).
//
//  ipc_handle / ipc_open : export a device allocation with cudaIpcGetMemHandle
//    (the handle names the whole cudaMalloc'd range, so the tensor's offset
//    inside it travels with the handle) and map it in another process with
//    cudaIpcMemLazyEnablePeerAccess.  Mappings are cached per process.
//  copy_segments : ONE kernel that gathers up to 16 byte ranges from local or
//    peer device pointers into one destination buffer with 16-byte vector
//    loads/stores; when a source is another GPU's memory the loads travel over
//    NVLink (no copy engine, no staging, no TMA multicast).
#include <cuda.h>

#include "driver_api.h"
#include <pybind11/pybind11.h>

#include <map>
#include <mutex>
#include <string>

#include "checks.cuh"
#include "common.cuh"

namespace py = pybind11;

namespace psrl {

std::tuple<py::bytes, int64_t> ipc_handle(at::Tensor t) {
  CHECK_CUDA_TENSOR(t);
  at::cuda::CUDAGuard g(t.device());
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = PSRL_DRV(cuMemGetAddressRange)(&base, &size, (CUdeviceptr)t.data_ptr());
  TORCH_CHECK(r == CUDA_SUCCESS, "cuMemGetAddressRange failed (", (int)r, ")");
  cudaIpcMemHandle_t h;
  PSRL_CHECK_CUDA(cudaIpcGetMemHandle(&h, (void*)base));
  const int64_t off = (int64_t)((CUdeviceptr)t.data_ptr() - base);
  return {py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)), off};
}

static std::mutex g_ipc_mu;
static std::map<std::string, void*> g_ipc_open;

at::Tensor ipc_open(py::bytes handle, int64_t offset, int64_t numel, at::ScalarType dtype, int64_t src_device) {
  std::string key = handle;
  TORCH_CHECK(key.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_ipc_mu);
    auto it = g_ipc_open.find(key);
    if (it != g_ipc_open.end()) {
      base = it->second;
    } else {
      cudaIpcMemHandle_t h;
      memcpy(&h, key.data(), sizeof(h));
      PSRL_CHECK_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
      g_ipc_open[key] = base;
    }
  }
  // The mapping lives until process exit; the tensor only views it.  In the
  // importing process the mapped pointer belongs to the current device (peer
  // access makes the exporting GPU's memory addressable from here).
  (void)src_device;
  int cur = 0;
  PSRL_CHECK_CUDA(cudaGetDevice(&cur));
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, cur);
  return at::from_blob(static_cast<char*>(base) + offset, {numel}, [](void*) {}, opts);
}

void enable_peer_access(int64_t peer) {
  int dev;
  cudaGetDevice(&dev);
  if (dev == peer) return;
  int can = 0;
  cudaDeviceCanAccessPeer(&can, dev, (int)peer);
  TORCH_CHECK(can, "device ", dev, " cannot access peer ", peer);
  cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return;
  }
  PSRL_CHECK_CUDA(e);
}

constexpr int MAX_SEG = 16;
struct SegTable {
  const uint4* src[MAX_SEG];
  int64_t dst_off[MAX_SEG];  // in 16 B units
  int64_t len[MAX_SEG];      // in 16 B units
  int64_t start[MAX_SEG + 1];  // prefix sums of len
  int64_t dst_total;           // destination size in 16 B units (bounds checks)
  int n;
};

__global__ void __launch_bounds__(512) copy_segments_kernel(uint4* __restrict__ dst, SegTable t) {
  const int64_t total = t.start[t.n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int seg = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride * 4) {
    uint4 v[4];
    int64_t idx[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      idx[u] = i + u * stride;
      if (idx[u] < total) {
        while (seg + 1 < t.n && idx[u] >= t.start[seg + 1]) ++seg;
        while (seg > 0 && idx[u] < t.start[seg]) --seg;
        v[u] = t.src[seg][idx[u] - t.start[seg]];
        idx[u] = t.dst_off[seg] + (idx[u] - t.start[seg]);
        if (!chk::in_range(idx[u], t.dst_total, 65, seg, 0)) idx[u] = -1;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u * stride < total && (!chk::kOn || idx[u] >= 0)) dst[idx[u]] = v[u];
  }
}

// dst: destination tensor (bytes are what matter); srcs: tensors (local or IPC-mapped peer views);
// dst_offsets_bytes / lengths_bytes per source (multiples of 16).
void copy_segments(at::Tensor dst, std::vector<at::Tensor> srcs, std::vector<int64_t> dst_offsets_bytes,
                   std::vector<int64_t> src_offsets_bytes, std::vector<int64_t> lengths_bytes) {
  CHECK_CUDA_TENSOR(dst);
  const int n = srcs.size();
  TORCH_CHECK(n <= MAX_SEG && n == (int)dst_offsets_bytes.size() && n == (int)lengths_bytes.size() &&
                  n == (int)src_offsets_bytes.size(),
              "bad segment lists");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0, "dst must be 16-byte aligned");
  SegTable t{};
  t.n = n;
  t.start[0] = 0;
  t.dst_total = dst.numel() * dst.element_size() / 16;
  const int64_t dst_bytes = dst.numel() * dst.element_size();
  for (int i = 0; i < n; ++i) {
    const char* sp = static_cast<const char*>(srcs[i].data_ptr()) + src_offsets_bytes[i];
    TORCH_CHECK(reinterpret_cast<uintptr_t>(sp) % 16 == 0, "source ", i, " not 16-byte aligned");
    TORCH_CHECK(lengths_bytes[i] % 16 == 0 && dst_offsets_bytes[i] % 16 == 0, "lengths/offsets must be x16");
    TORCH_CHECK(dst_offsets_bytes[i] + lengths_bytes[i] <= dst_bytes, "segment ", i, " overflows dst");
    TORCH_CHECK(src_offsets_bytes[i] + lengths_bytes[i] <= srcs[i].numel() * srcs[i].element_size(),
                "segment ", i, " overflows its source");
    t.src[i] = reinterpret_cast<const uint4*>(sp);
    t.dst_off[i] = dst_offsets_bytes[i] / 16;
    t.len[i] = lengths_bytes[i] / 16;
    t.start[i + 1] = t.start[i] + t.len[i];
  }
  if (t.start[n] == 0) return;
  at::cuda::CUDAGuard g(dst.device());
  const int grid = std::min<int64_t>(num_sms() * 4, (t.start[n] + 511) / 512);
  copy_segments_kernel<<<grid, 512, 0, stream()>>>(reinterpret_cast<uint4*>(dst.data_ptr()), t);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl

// ---------------------------------------------------------------------------
// scatter_segments: the mirror of copy_segments for one source and up to 16
// destinations (local or peer device pointers): segment i copies len[i] bytes
// from src + src_off[i] to dsts[i] + dst_off[i] with 16-byte vector loads and
// stores.  The peer all-to-all of expert parallelism (parallel/ep_p2p.py)
// writes each destination rank's rows straight into that rank's receive
// buffer this way: the stores travel over NVLink, no copy engine, no staging.
namespace psrl {

struct ScatterTable {
  uint4* dst[MAX_SEG];
  int64_t src_off[MAX_SEG];    // in 16 B units
  int64_t start[MAX_SEG + 1];  // prefix sums of lengths (16 B units)
  int64_t dst_total[MAX_SEG];  // destination size in 16 B units (bounds checks)
  int n;
};

__global__ void __launch_bounds__(512) scatter_segments_kernel(const uint4* __restrict__ src, ScatterTable t) {
  const int64_t total = t.start[t.n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int seg = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride * 4) {
    uint4 v[4];
    int64_t at[4];
    int sg[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t idx = i + u * stride;
      sg[u] = -1;
      if (idx < total) {
        while (seg + 1 < t.n && idx >= t.start[seg + 1]) ++seg;
        while (seg > 0 && idx < t.start[seg]) --seg;
        const int64_t w = idx - t.start[seg];
        v[u] = src[t.src_off[seg] + w];
        at[u] = w;
        sg[u] = chk::in_range(w, t.dst_total[seg], 65, seg, 1) ? seg : -1;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (sg[u] >= 0) t.dst[sg[u]][at[u]] = v[u];
  }
  __threadfence_system();  // peer stores visible before the barrier that follows
}

// src: source tensor; dsts: destination views (each segment writes from the
// start of its view, so pass the view at the destination offset); src offsets
// and lengths in bytes (multiples of 16).
void scatter_segments(at::Tensor src, std::vector<at::Tensor> dsts, std::vector<int64_t> src_offsets_bytes,
                      std::vector<int64_t> lengths_bytes) {
  CHECK_CUDA_TENSOR(src);
  const int n = dsts.size();
  TORCH_CHECK(n <= MAX_SEG && n == (int)src_offsets_bytes.size() && n == (int)lengths_bytes.size(),
              "bad segment lists");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "src must be 16-byte aligned");
  const int64_t src_bytes = src.numel() * src.element_size();
  ScatterTable t{};
  t.n = n;
  t.start[0] = 0;
  for (int i = 0; i < n; ++i) {
    TORCH_CHECK(reinterpret_cast<uintptr_t>(dsts[i].data_ptr()) % 16 == 0, "destination ", i, " not 16-byte aligned");
    TORCH_CHECK(lengths_bytes[i] % 16 == 0 && src_offsets_bytes[i] % 16 == 0, "lengths/offsets must be x16");
    TORCH_CHECK(src_offsets_bytes[i] + lengths_bytes[i] <= src_bytes, "segment ", i, " overflows the source");
    const int64_t db = dsts[i].numel() * dsts[i].element_size();
    TORCH_CHECK(lengths_bytes[i] <= db, "segment ", i, " overflows its destination");
    t.dst[i] = reinterpret_cast<uint4*>(dsts[i].data_ptr());
    t.src_off[i] = src_offsets_bytes[i] / 16;
    t.dst_total[i] = db / 16;
    t.start[i + 1] = t.start[i] + lengths_bytes[i] / 16;
  }
  if (t.start[n] == 0) return;
  at::cuda::CUDAGuard g(src.device());
  const int grid = std::min<int64_t>(num_sms() * 4, (t.start[n] + 511) / 512);
  scatter_segments_kernel<<<grid, 512, 0, stream()>>>(reinterpret_cast<const uint4*>(src.data_ptr()), t);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl

// ---------------------------------------------------------------------------
// copy_rows: one kernel for any number of 2-D byte blocks gathered into one
// destination buffer (the layout-transforming weight pull): block k copies
// `rows` rows of `row_vecs` 16-byte vectors from src_ptr (local or peer device
// memory; row stride src_stride bytes) to dst + dst_off (row stride dst_stride
// bytes).  A tensor-parallel shard of a row-parallel weight (columns of the
// full matrix) is one block; a contiguous range is a block of one row.  The
// table (int64 [n, 6]) and the prefix sums of rows * row_vecs (int64 [n + 1])
// live on the device, built once per pull plan.
namespace psrl {

__global__ void __launch_bounds__(512) copy_rows_kernel(uint8_t* __restrict__ dst, const int64_t* __restrict__ tab,
                                                        const int64_t* __restrict__ start, int n, int64_t dst_bytes) {
  const int64_t total = start[n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += stride) {
    int lo = 0, hi = n;  // block k holds vectors [start[k], start[k + 1])
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (start[mid] <= v) lo = mid;
      else hi = mid;
    }
    const int64_t* t = tab + 6 * lo;
    const int64_t local = v - start[lo];
    const int64_t rv = t[3];
    const int64_t row = local / rv, col = local - row * rv;
    const uint4* s = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(t[0]) + row * t[4]) + col;
    const int64_t d = t[1] + row * t[5] + col * 16;
    if (!chk::in_range(d + 15, dst_bytes, 65, lo, 2)) continue;
    *reinterpret_cast<uint4*>(dst + d) = *s;
  }
}

void copy_rows(at::Tensor dst, at::Tensor table, at::Tensor start) {
  CHECK_CUDA_TENSOR(dst);
  TORCH_CHECK(table.is_cuda() && start.is_cuda() && table.scalar_type() == at::kLong &&
                  start.scalar_type() == at::kLong && table.dim() == 2 && table.size(1) == 6 &&
                  start.numel() == table.size(0) + 1 && table.is_contiguous() && start.is_contiguous(),
              "table: int64 [n, 6] and start: int64 [n + 1] on the device");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0, "dst must be 16-byte aligned");
  const int n = (int)table.size(0);
  if (n == 0) return;
  at::cuda::CUDAGuard g(dst.device());
  const int grid = num_sms() * 4;
  copy_rows_kernel<<<grid, 512, 0, stream()>>>(reinterpret_cast<uint8_t*>(dst.data_ptr()), table.data_ptr<int64_t>(),
                                               start.data_ptr<int64_t>(), n, dst.numel() * dst.element_size());
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
