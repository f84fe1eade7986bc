// Mixture-of-experts token routing kernels (router top-k, permutation, gather,
// weighted combine).  The expert MLPs between gather and combine run as
// grouped tcgen05 GEMMs (gemm_sm100.cu, tc_grouped_gemm).
//
//  moe_route    one warp per token: softmax over E <= 256 router logits (+ an
//               optional per-expert log-prior), top-k by k warp arg-max rounds
//               (ties -> lower expert id), optional renormalisation of the k
//               weights, and a per-expert token count (shared-memory histogram
//               per CTA, then one global atomic per expert and CTA).
//  moe_permute  exclusive scan of the counts into expert segment offsets and
//               tile offsets for the grouped GEMM (one CTA), then a scatter
//               that gives every (token, slot) its row in expert-sorted order.
//               Rows inside one expert's segment are ordered by atomics; every
//               row is computed independently and the combine gathers per
//               token in slot order, so results do not depend on that order.
//  moe_gather   xs[row] = x[token_of_row[row]] with 16-byte vector copies.
//  moe_combine  y[t] = sum_j w[t, j] * ys[pos[t, j]] in fp32 (gather form:
//               deterministic, no atomics).
// Reference behaviour: Qwen3-MoE routing as served by vLLM fused_moe and
// Megatron's router (psrl/utils/megatron_converter.py maps the same weights).
#include "common.cuh"

namespace psrl {

constexpr int ROUTE_WARPS = 8;
constexpr int MAX_E = 256;

__global__ void __launch_bounds__(ROUTE_WARPS * 32)
    moe_route_kernel(const float* __restrict__ logits, const float* __restrict__ prior, int T, int E, int k,
                     bool renorm, float* __restrict__ w_out, int* __restrict__ id_out, int* __restrict__ counts) {
  __shared__ int hist[MAX_E];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * ROUTE_WARPS + warp;
  if (t < T) {
    constexpr int PER = MAX_E / 32;
    float v[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? logits[(int64_t)t * E + e] + (prior ? prior[e] : 0.f) : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      v[i] = (lane + 32 * i < E) ? __expf(v[i] - mx) : -1.f;   // probabilities (unnormalised); -1 = absent
      sum += fmaxf(v[i], 0.f);
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    float picked = 0.f, my_w = 0.f;
    int my_id = 0;
    for (int j = 0; j < k; ++j) {
      float bv = -1.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (v[i] > bv) {   // strictly greater: the lower id wins among this lane's equal values
          bv = v[i];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      // the owner lane retires the winner
      if ((bi & 31) == lane) v[bi >> 5] = -1.f;
      const float p = bv * inv;
      picked += p;
      if (lane == j) {
        my_w = p;
        my_id = bi;
      }
    }
    if (lane < k) {
      w_out[(int64_t)t * k + lane] = renorm ? my_w / picked : my_w;
      id_out[(int64_t)t * k + lane] = my_id;
      atomicAdd(&hist[my_id], 1);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

// One CTA: exclusive scans of counts -> seg [E+1] (row offsets) and
// tile_off [E+1] (grouped-GEMM tile offsets, tiles of bm rows x tiles_n);
// cursor [E] is reset to seg.
__global__ void moe_offsets_kernel(const int* __restrict__ counts, int E, int bm, int tiles_n, int* __restrict__ seg,
                                   int* __restrict__ tile_off, int* __restrict__ cursor) {
  __shared__ int sc[MAX_E], st[MAX_E];
  const int e = threadIdx.x;
  const int c = e < E ? counts[e] : 0;
  sc[e] = c;
  st[e] = e < E ? (c + bm - 1) / bm * tiles_n : 0;
  __syncthreads();
  // Hillis-Steele inclusive scans over MAX_E entries
  for (int o = 1; o < MAX_E; o <<= 1) {
    const int a = e >= o ? sc[e - o] : 0, b = e >= o ? st[e - o] : 0;
    __syncthreads();
    sc[e] += a;
    st[e] += b;
    __syncthreads();
  }
  if (e < E) {
    seg[e + 1] = sc[e];
    tile_off[e + 1] = st[e];
    cursor[e] = sc[e] - c;
  }
  if (e == 0) {
    seg[0] = 0;
    tile_off[0] = 0;
  }
}

__global__ void moe_scatter_kernel(const int* __restrict__ ids, int n, int k, int* __restrict__ cursor,
                                   int* __restrict__ pos, int* __restrict__ token_of_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = atomicAdd(&cursor[ids[i]], 1);
  pos[i] = r;
  token_of_row[r] = i / k;
}

__global__ void moe_gather_kernel(const bf16* __restrict__ x, int64_t ldx, const int* __restrict__ token_of_row,
                                  int R, int h8, bf16* __restrict__ xs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)R * h8) return;
  const int r = i / h8, c = i % h8;
  reinterpret_cast<bf16x8*>(xs)[(int64_t)r * h8 + c] =
      reinterpret_cast<const bf16x8*>(x + (int64_t)token_of_row[r] * ldx)[c];
}

__global__ void moe_combine_kernel(const bf16* __restrict__ ys, const int* __restrict__ pos,
                                   const float* __restrict__ w, int k, int h8, bf16* __restrict__ y) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x; c < h8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const float wj = w[(int64_t)t * k + j];
      float v[8];
      unpack8(reinterpret_cast<const bf16x8*>(ys)[(int64_t)pos[(int64_t)t * k + j] * h8 + c], v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wj * v[q];
    }
    reinterpret_cast<bf16x8*>(y)[(int64_t)t * h8 + c] = pack8(acc);
  }
}

// ------------------------------------------------------------------ host
// Returns {weights fp32 [T,k], ids int32 [T,k], counts int32 [E]}.
std::vector<at::Tensor> moe_route(at::Tensor logits, c10::optional<at::Tensor> prior, int64_t k, bool renorm) {
  CHECK_CUDA_TENSOR(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == at::kFloat && logits.is_contiguous(),
              "logits must be contiguous fp32 [T, E]");
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= MAX_E && k >= 1 && k <= 32 && k <= E, "E <= 256 and 1 <= k <= min(32, E)");
  at::cuda::CUDAGuard g(logits.device());
  auto w = at::empty({T, k}, logits.options());
  auto ids = at::empty({T, k}, logits.options().dtype(at::kInt));
  auto counts = at::zeros({E}, logits.options().dtype(at::kInt));
  const float* pp = nullptr;
  if (prior.has_value()) {
    TORCH_CHECK(prior->numel() == E && prior->scalar_type() == at::kFloat && prior->is_contiguous(), "bad prior");
    pp = prior->data_ptr<float>();
  }
  if (T == 0) return {w, ids, counts};
  moe_route_kernel<<<(T + ROUTE_WARPS - 1) / ROUTE_WARPS, ROUTE_WARPS * 32, 0, stream()>>>(
      logits.data_ptr<float>(), pp, T, E, (int)k, renorm, w.data_ptr<float>(), ids.data_ptr<int>(),
      counts.data_ptr<int>());
  PSRL_CHECK_LAUNCH();
  return {w, ids, counts};
}

// Returns {pos int32 [T,k], token_of_row int32 [T*k], seg int32 [E+1], tile_off int32 [E+1]}.
std::vector<at::Tensor> moe_permute(at::Tensor ids, at::Tensor counts, int64_t bm, int64_t tiles_n) {
  CHECK_CUDA_TENSOR(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 2, "ids int32 [T, k]");
  const int T = ids.size(0), k = ids.size(1), E = counts.numel();
  TORCH_CHECK(E <= MAX_E, "E <= 256");
  at::cuda::CUDAGuard g(ids.device());
  auto o = ids.options();
  auto pos = at::empty({T, k}, o);
  auto tor = at::empty({(int64_t)T * k}, o);
  auto seg = at::empty({E + 1}, o);
  auto toff = at::empty({E + 1}, o);
  auto cursor = at::empty({E}, o);
  moe_offsets_kernel<<<1, MAX_E, 0, stream()>>>(counts.data_ptr<int>(), E, (int)bm, (int)tiles_n, seg.data_ptr<int>(),
                                                toff.data_ptr<int>(), cursor.data_ptr<int>());
  PSRL_CHECK_LAUNCH();
  const int n = T * k;
  if (n > 0) {
    moe_scatter_kernel<<<(n + 255) / 256, 256, 0, stream()>>>(ids.data_ptr<int>(), n, k, cursor.data_ptr<int>(),
                                                              pos.data_ptr<int>(), tor.data_ptr<int>());
    PSRL_CHECK_LAUNCH();
  }
  return {pos, tor, seg, toff};
}

at::Tensor moe_gather(at::Tensor x, at::Tensor token_of_row) {
  CHECK_CUDA_TENSOR(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) % 8 == 0 && x.stride(0) % 8 == 0 &&
                  x.scalar_type() == at::kBFloat16 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "x must be bf16 [T, h] with 16-byte aligned rows, h % 8 == 0");
  const int R = token_of_row.numel(), h = x.size(1);
  at::cuda::CUDAGuard g(x.device());
  auto xs = at::empty({R, h}, x.options());
  const int64_t n = (int64_t)R * (h / 8);
  if (n > 0) {
    moe_gather_kernel<<<(n + 255) / 256, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0),
                                                             token_of_row.data_ptr<int>(), R, h / 8,
                                                             reinterpret_cast<bf16*>(xs.data_ptr()));
    PSRL_CHECK_LAUNCH();
  }
  return xs;
}

at::Tensor moe_combine(at::Tensor ys, at::Tensor pos, at::Tensor w) {
  CHECK_CUDA_TENSOR(ys);
  TORCH_CHECK(ys.dim() == 2 && ys.is_contiguous() && ys.size(1) % 8 == 0 && ys.scalar_type() == at::kBFloat16,
              "ys must be contiguous bf16 [R, h], h % 8 == 0");
  TORCH_CHECK(pos.is_contiguous() && w.is_contiguous() && w.scalar_type() == at::kFloat, "pos/w layout");
  const int T = pos.size(0), k = pos.size(1), h = ys.size(1);
  at::cuda::CUDAGuard g(ys.device());
  auto y = at::empty({T, h}, ys.options());
  if (T > 0) {
    moe_combine_kernel<<<T, 128, 0, stream()>>>(reinterpret_cast<const bf16*>(ys.data_ptr()), pos.data_ptr<int>(),
                                                w.data_ptr<float>(), k, h / 8, reinterpret_cast<bf16*>(y.data_ptr()));
    PSRL_CHECK_LAUNCH();
  }
  return y;
}

}  // namespace psrl
