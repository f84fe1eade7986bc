// Cross-GPU pieces of the fused tensor-parallel GEMMs (csrc/gemm_2sm.cu,
// OUT_F32_ADD2):
//
//  peer_barrier   a one-thread kernel per rank: it publishes the call's epoch
//                 into its slot of every peer's flag array (system-scope
//                 release store through the NVLink mapping of the peer's
//                 memory) and waits until every peer has published the same
//                 epoch into its own array (acquire loads).  Stream order puts
//                 it after the fused GEMM, so when it returns every rank's
//                 epilogue writes into this rank's accumulator are complete and
//                 visible.  Epochs only grow, so the flags never need a reset.
//                 The wait is bounded by a timeout in nanoseconds of the global
//                 timer; on expiry it records an error code (and the epochs it
//                 saw) and returns, so the host learns of a missing peer
//                 without a hung GPU.
//  acc_finalize   out = bf16(acc + bias); acc = 0 (ready for the next call).
//
// The two ranks are separate processes on separate GPUs, so the waiting
// kernels always run concurrently.
#include "common.cuh"

namespace psrl {
namespace tpf {

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerFlags {
  int* slot_in_peer[8];  // this rank's slot in each rank's flag array (own array included)
  const int* own[8];     // every rank's slot in this rank's flag array
  int world;
};

__global__ void peer_barrier_kernel(PeerFlags f, int epoch, unsigned long long timeout_ns, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  for (int r = 0; r < f.world; ++r) st_release_sys(f.slot_in_peer[r], epoch);
  const uint64_t t0 = now_ns();
  for (int r = 0; r < f.world; ++r) {
    int seen;
    while ((seen = ld_acquire_sys(f.own[r])) < epoch) {
      if (now_ns() - t0 > timeout_ns) {
        if (atomicCAS(err, 0, 51) == 0) {
          err[1] = r;      // the rank that did not arrive
          err[2] = seen;   // its last epoch
          err[3] = epoch;  // the epoch waited for
        }
        return;
      }
    }
  }
}

__global__ void acc_finalize_kernel(float* __restrict__ acc, bf16* __restrict__ out, int64_t n4,
                                    const bf16* __restrict__ bias, int N) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 v = reinterpret_cast<float4*>(acc)[i];
  reinterpret_cast<float4*>(acc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (bias != nullptr) {
    const int n = (int)((4 * i) % N);
    v.x += __bfloat162float(bias[n]);
    v.y += __bfloat162float(bias[n + 1]);
    v.z += __bfloat162float(bias[n + 2]);
    v.w += __bfloat162float(bias[n + 3]);
  }
  bf162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  reinterpret_cast<bf162*>(out)[2 * i] = lo;
  reinterpret_cast<bf162*>(out)[2 * i + 1] = hi;
}

}  // namespace tpf

using namespace tpf;

// flags_in_peer[r]: int32 tensor view of this rank's slot in rank r's flag
// array (own and peer memory); own_slots[r]: rank r's slot in this rank's
// array.  Returns immediately after launching; errors land in `err`.
void peer_barrier(std::vector<at::Tensor> flags_in_peer, std::vector<at::Tensor> own_slots, int64_t epoch,
                  double timeout_s, at::Tensor err) {
  TORCH_CHECK(flags_in_peer.size() == own_slots.size() && !own_slots.empty() && own_slots.size() <= 8,
              "one slot per rank, at most 8 ranks");
  PeerFlags f{};
  f.world = (int)own_slots.size();
  for (int r = 0; r < f.world; ++r) {
    TORCH_CHECK(flags_in_peer[r].scalar_type() == at::kInt && own_slots[r].scalar_type() == at::kInt, "int32 flags");
    f.slot_in_peer[r] = flags_in_peer[r].data_ptr<int>();
    f.own[r] = own_slots[r].data_ptr<int>();
  }
  at::cuda::CUDAGuard g(err.device());
  peer_barrier_kernel<<<1, 32, 0, stream()>>>(f, (int)epoch, (unsigned long long)(timeout_s * 1e9),
                                              err.data_ptr<int>());
  PSRL_CHECK_LAUNCH();
}

// out (bf16, same shape [.., N]) = acc (+ bias [N]); acc = 0.
void acc_finalize(at::Tensor acc, at::Tensor out, c10::optional<at::Tensor> bias) {
  CHECK_DTYPE(acc, at::kFloat);
  CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(acc.is_contiguous() && out.is_contiguous() && acc.numel() == out.numel() && acc.numel() % 4 == 0,
              "contiguous fp32 / bf16 pair, size a multiple of 4");
  const int N = (int)out.size(-1);
  const bf16* bp = nullptr;
  if (bias.has_value()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous() && N % 4 == 0, "bias must be bf16 [N], N % 4 == 0");
    bp = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  at::cuda::CUDAGuard g(acc.device());
  const int64_t n4 = acc.numel() / 4;
  if (n4 == 0) return;
  acc_finalize_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, stream()>>>(
      acc.data_ptr<float>(), reinterpret_cast<bf16*>(out.data_ptr()), n4, bp, N);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
