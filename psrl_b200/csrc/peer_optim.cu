// Fused data-parallel optimizer step over NVLink peer memory (the gradient
// reduce-scatter fused with the cast/scale and the sharded AdamW update, and
// the parameter all-gather fused into the update's store).
//
// Every rank's fp32 main-gradient buffer and bf16 parameter buffer are mapped
// into every other rank (CUDA IPC).  Rank r owns, in every bucket b, the shard
// [base_b + r * S_b, base_b + (r + 1) * S_b) of the flat buffers; its shards
// are concatenated in its contiguous shard buffers (master, m, v, reduced
// gradient), with bucket b starting at start[b].
//
//  peer_reduce_kernel   red[i] = sum over ranks of grad_rank[src(i)] with
//                       16-byte peer loads, plus per-CTA sums of red^2 (the
//                       squared gradient norm, finished by a one-CTA pass);
//  peer_adamw_kernel    AdamW on the master shard with the clipped, scaled
//                       reduced gradient; the bf16 result is stored into the
//                       parameter buffer of EVERY rank (8-byte peer stores).
//
// No kernel waits on another rank: the host orders the steps with NCCL
// collectives on the same stream (a one-element all-reduce before the reduce,
// the norm all-reduce between the kernels, a one-element all-reduce after the
// update), so every peer buffer a kernel touches is quiescent while it runs.
// No TMA and no multicast: plain loads and stores through the IPC mappings.
#include "checks.cuh"
#include "common.cuh"

namespace psrl {

constexpr int MAX_PEERS = 16;

struct PeerSet {
  const float* grad[MAX_PEERS];   // each rank's flat fp32 gradient (local pointer for this rank)
  bf16* flat[MAX_PEERS];          // each rank's flat bf16 parameters
  int64_t numel;                  // elements in each flat buffer (bounds checks)
  int n;
};

// bucket of shard element i (start: prefix of shard lengths, nb + 1 entries)
__device__ __forceinline__ int seg_of(const int64_t* start, int nb, int64_t i) {
  int lo = 0, hi = nb;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (start[mid] <= i) lo = mid;
    else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(256) peer_reduce_kernel(PeerSet ps, const int64_t* __restrict__ start,
                                                          const int64_t* __restrict__ src_off, int nb,
                                                          int64_t total, float* __restrict__ red,
                                                          float* __restrict__ partial) {
  __shared__ float sh[32];
  float acc = 0.f;
  const int64_t nv = total >> 2;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = v << 2;
    const int b = seg_of(start, nb, i);
    const int64_t g = src_off[b] + (i - start[b]);
    if (!chk::in_range(g + 3, ps.numel, 66, b, 0)) continue;
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < ps.n; ++r) {   // fixed rank order: the sum does not depend on timing
      const float4 t = *reinterpret_cast<const float4*>(ps.grad[r] + g);
      s.x += t.x;
      s.y += t.y;
      s.z += t.z;
      s.w += t.w;
    }
    reinterpret_cast<float4*>(red)[v] = s;
    acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

__global__ void peer_sum_finish_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) out[0] = acc;
}

__global__ void __launch_bounds__(256) peer_adamw_kernel(PeerSet ps, const int64_t* __restrict__ start,
                                                         const int64_t* __restrict__ src_off, int nb, int64_t total,
                                                         float* __restrict__ p, const float* __restrict__ g,
                                                         float* __restrict__ m, float* __restrict__ v, float lr,
                                                         float b1, float b2, float eps, float wd, float bc1, float bc2,
                                                         const float* __restrict__ coef, float gscale) {
  const float gs = gscale * coef[0];
  const int64_t nv = total >> 2;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[q];
    float4 mm = reinterpret_cast<float4*>(m)[q];
    float4 vv = reinterpret_cast<float4*>(v)[q];
    const float4 gg4 = reinterpret_cast<const float4*>(g)[q];
    const float gg[4] = {gg4.x, gg4.y, gg4.z, gg4.w};
    float* pa = &pp.x;
    float* ma = &mm.x;
    float* va = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = gg[k] * gs;
      ma[k] = b1 * ma[k] + (1.f - b1) * gk;
      va[k] = b2 * va[k] + (1.f - b2) * gk * gk;
      const float upd = (ma[k] / bc1) / (sqrtf(va[k] / bc2) + eps);
      pa[k] = pa[k] - lr * (wd * pa[k] + upd);
    }
    reinterpret_cast<float4*>(p)[q] = pp;
    reinterpret_cast<float4*>(m)[q] = mm;
    reinterpret_cast<float4*>(v)[q] = vv;
    bf162 o[2] = {__floats2bfloat162_rn(pp.x, pp.y), __floats2bfloat162_rn(pp.z, pp.w)};
    const uint2 word = *reinterpret_cast<const uint2*>(o);
    const int64_t i = q << 2;
    const int b = seg_of(start, nb, i);
    const int64_t dst = src_off[b] + (i - start[b]);
    if (!chk::in_range(dst + 3, ps.numel, 66, b, 1)) continue;
    for (int r = 0; r < ps.n; ++r) *reinterpret_cast<uint2*>(ps.flat[r] + dst) = word;
  }
  // make the peer stores visible system-wide before the kernel retires
  __threadfence_system();
}

static PeerSet make_set(const std::vector<at::Tensor>& grads, const std::vector<at::Tensor>& flats) {
  TORCH_CHECK(grads.size() == flats.size() && !grads.empty() && (int)grads.size() <= MAX_PEERS, "bad peer lists");
  PeerSet ps{};
  ps.n = (int)grads.size();
  ps.numel = grads[0].numel();
  for (int r = 0; r < ps.n; ++r) {
    TORCH_CHECK(grads[r].numel() == ps.numel && flats[r].numel() == ps.numel, "peer buffers differ in size");
    TORCH_CHECK(grads[r].scalar_type() == at::kFloat && flats[r].scalar_type() == at::kBFloat16, "peer dtypes");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(grads[r].data_ptr()) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(flats[r].data_ptr()) % 16 == 0,
                "peer buffers must be 16-byte aligned");
    ps.grad[r] = grads[r].data_ptr<float>();
    ps.flat[r] = reinterpret_cast<bf16*>(flats[r].data_ptr());
  }
  return ps;
}

// red (fp32 [total]) <- sum of every rank's gradient over this rank's shards;
// sq (fp32 [1]) <- ||red||^2.  start: int64 [nb + 1], src_off: int64 [nb]
// (device); every segment length is a multiple of 4.
void peer_reduce(std::vector<at::Tensor> grads, std::vector<at::Tensor> flats, at::Tensor start, at::Tensor src_off,
                 at::Tensor red, at::Tensor sq, at::Tensor partial) {
  CHECK_CUDA_TENSOR(red);
  const int64_t total = red.numel();
  TORCH_CHECK(total % 4 == 0, "shard total must be a multiple of 4");
  const int nb = src_off.numel();
  PeerSet ps = make_set(grads, flats);
  at::cuda::CUDAGuard g(red.device());
  const int grid = (int)std::min<int64_t>(partial.numel(), std::max<int64_t>(1, (total / 4 + 255) / 256));
  peer_reduce_kernel<<<grid, 256, 0, stream()>>>(ps, start.data_ptr<int64_t>(), src_off.data_ptr<int64_t>(), nb,
                                                 total, red.data_ptr<float>(), partial.data_ptr<float>());
  PSRL_CHECK_LAUNCH();
  peer_sum_finish_kernel<<<1, 1024, 0, stream()>>>(partial.data_ptr<float>(), grid, sq.data_ptr<float>());
  PSRL_CHECK_LAUNCH();
}

void peer_adamw(std::vector<at::Tensor> grads, std::vector<at::Tensor> flats, at::Tensor start, at::Tensor src_off,
                at::Tensor master, at::Tensor red, at::Tensor m, at::Tensor v, double lr, double b1, double b2,
                double eps, double wd, int64_t step, at::Tensor coef, double gscale) {
  CHECK_CUDA_TENSOR(master);
  const int64_t total = master.numel();
  TORCH_CHECK(total % 4 == 0 && red.numel() == total && m.numel() == total && v.numel() == total, "shard sizes");
  const int nb = src_off.numel();
  PeerSet ps = make_set(grads, flats);
  at::cuda::CUDAGuard g(master.device());
  const float bc1 = 1.f - powf((float)b1, (float)step), bc2 = 1.f - powf((float)b2, (float)step);
  const int grid = (int)std::min<int64_t>(4 * num_sms(), std::max<int64_t>(1, (total / 4 + 255) / 256));
  peer_adamw_kernel<<<grid, 256, 0, stream()>>>(ps, start.data_ptr<int64_t>(), src_off.data_ptr<int64_t>(), nb, total,
                                                master.data_ptr<float>(), red.data_ptr<float>(), m.data_ptr<float>(),
                                                v.data_ptr<float>(), (float)lr, (float)b1, (float)b2, (float)eps,
                                                (float)wd, bc1, bc2, coef.data_ptr<float>(), (float)gscale);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
