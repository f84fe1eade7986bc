// Vocabulary-wide softmax statistics for RL:
//  * logprob_fwd: per row of logits z (scaled by 1/T): log-softmax of the label
//    token, entropy, and the log-sum-exp (saved for backward) in ONE pass over
//    the row using an online (max, sum, weighted-sum) recurrence.
//  * logprob_bwd: d logits = (g_lp * (onehot - p) - g_ent * p * (log p + H)) / T,
//    written in place over the logits (so the LM-head backward GEMMs consume it).
//  * sample: Gumbel-max sampling (argmax(z/T - log(-log u))) fused with the
//    sampled token's log-probability; u from a counter-based hash (seed, row, j).
#include "common.cuh"

namespace psrl {

constexpr int LP_THREADS = 1024;

struct OnlineStat {
  float m, s, t;  // running max, sum exp(z-m), sum exp(z-m)*z
};

__device__ __forceinline__ void ostat_add(OnlineStat& a, float z) {
  if (z > a.m) {
    const float c = __expf(a.m - z);
    a.s = a.s * c + 1.f;
    a.t = a.t * c + z;
    a.m = z;
  } else {
    const float e = __expf(z - a.m);
    a.s += e;
    a.t += e * z;
  }
}

__device__ __forceinline__ OnlineStat ostat_merge(OnlineStat a, OnlineStat b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  const float ca = __expf(a.m - m), cb = __expf(b.m - m);
  return {m, a.s * ca + b.s * cb, a.t * ca + b.t * cb};
}

__device__ __forceinline__ OnlineStat ostat_block(OnlineStat v, OnlineStat* sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    OnlineStat w{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o),
                 __shfl_xor_sync(0xffffffffu, v.t, o)};
    v = ostat_merge(v, w);
  }
  if (lane == 0) sm[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? sm[lane] : OnlineStat{-INFINITY, 0.f, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      OnlineStat w{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o),
                   __shfl_xor_sync(0xffffffffu, v.t, o)};
      v = ostat_merge(v, w);
    }
    if (lane == 0) sm[0] = v;
  }
  __syncthreads();
  return sm[0];
}

template <typename T>
__global__ void __launch_bounds__(LP_THREADS)
    logprob_fwd_kernel(const T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels, int V,
                       float inv_temp, float* __restrict__ lp, float* __restrict__ ent, float* __restrict__ lse_out) {
  __shared__ OnlineStat sm[32];
  const int64_t row = blockIdx.x;
  const T* z = logits + row * ld;
  OnlineStat st{-INFINITY, 0.f, 0.f};
  if constexpr (std::is_same<T, bf16>::value) {
    const int nv = V >> 3;
    const bf16x8* zv = reinterpret_cast<const bf16x8*>(z);
    for (int i = threadIdx.x; i < nv; i += LP_THREADS) {
      float f[8];
      unpack8(zv[i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) ostat_add(st, f[k] * inv_temp);
    }
    for (int i = nv * 8 + threadIdx.x; i < V; i += LP_THREADS) ostat_add(st, to_f(z[i]) * inv_temp);
  } else {
    for (int i = threadIdx.x; i < V; i += LP_THREADS) ostat_add(st, to_f(z[i]) * inv_temp);
  }
  st = ostat_block(st, sm);
  if (threadIdx.x == 0) {
    const float lse = st.m + __logf(st.s);
    const int64_t lab = labels[row];
    const float zl = (lab >= 0 && lab < V) ? to_f(z[lab]) * inv_temp : 0.f;
    lp[row] = (lab >= 0 && lab < V) ? zl - lse : 0.f;
    if (ent) ent[row] = lse - st.t / st.s;
    lse_out[row] = lse;
  }
}

std::vector<at::Tensor> logprob_fwd(at::Tensor logits, at::Tensor labels, double temperature, bool want_entropy) {
  CHECK_CUDA_TENSOR(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [rows, V] with unit column stride");
  CHECK_DTYPE(labels, at::kLong);
  const int64_t rows = logits.size(0);
  const int V = logits.size(1);
  at::cuda::CUDAGuard g(logits.device());
  auto opts = logits.options().dtype(at::kFloat);
  auto lp = at::empty({rows}, opts), lse = at::empty({rows}, opts);
  auto ent = want_entropy ? at::empty({rows}, opts) : at::Tensor();
  if (rows == 0) return {lp, ent, lse};
  const float it = 1.f / (float)temperature;
  if (logits.scalar_type() == at::kBFloat16) {
    TORCH_CHECK(logits.stride(0) % 8 == 0 && V % 8 == 0, "bf16 logits rows must be 16-byte aligned");
    logprob_fwd_kernel<bf16><<<rows, LP_THREADS, 0, stream()>>>(
        reinterpret_cast<const bf16*>(logits.data_ptr()), logits.stride(0), labels.data_ptr<int64_t>(), V, it,
        lp.data_ptr<float>(), want_entropy ? ent.data_ptr<float>() : nullptr, lse.data_ptr<float>());
  } else {
    CHECK_DTYPE(logits, at::kFloat);
    logprob_fwd_kernel<float><<<rows, LP_THREADS, 0, stream()>>>(
        logits.data_ptr<float>(), logits.stride(0), labels.data_ptr<int64_t>(), V, it, lp.data_ptr<float>(),
        want_entropy ? ent.data_ptr<float>() : nullptr, lse.data_ptr<float>());
  }
  PSRL_CHECK_LAUNCH();
  return {lp, ent, lse};
}

// In place: logits <- d loss / d logits.
template <typename T>
__global__ void __launch_bounds__(LP_THREADS)
    logprob_bwd_kernel(T* __restrict__ logits, int64_t ld, const int64_t* __restrict__ labels, int V, float inv_temp,
                       const float* __restrict__ glp, const float* __restrict__ gent, const float* __restrict__ lse,
                       const float* __restrict__ ent) {
  const int64_t row = blockIdx.x;
  T* z = logits + row * ld;
  const float L = lse[row];
  const int64_t lab0 = labels[row];
  // rows without a label contribute no log-prob term (forward wrote lp = 0)
  const float gl = (glp && lab0 >= 0 && lab0 < V) ? glp[row] : 0.f;
  const float ge = gent ? gent[row] : 0.f;
  const float H = (gent && ent) ? ent[row] : 0.f;
  const int64_t lab = labels[row];
  for (int i = threadIdx.x; i < V; i += LP_THREADS) {
    const float zi = to_f(z[i]) * inv_temp;
    const float logp = zi - L;
    const float p = __expf(logp);
    float d = -gl * p - ge * p * (logp + H);
    if (i == lab) d += gl;
    z[i] = from_f<T>(d * inv_temp);
  }
}

void logprob_bwd_(at::Tensor logits, at::Tensor labels, double temperature, c10::optional<at::Tensor> glp,
                  c10::optional<at::Tensor> gent, at::Tensor lse, c10::optional<at::Tensor> ent) {
  const int64_t rows = logits.size(0);
  const int V = logits.size(1);
  if (rows == 0) return;
  at::cuda::CUDAGuard g(logits.device());
  const float it = 1.f / (float)temperature;
  const float* gl = glp.has_value() ? glp->data_ptr<float>() : nullptr;
  const float* ge = gent.has_value() ? gent->data_ptr<float>() : nullptr;
  const float* en = ent.has_value() ? ent->data_ptr<float>() : nullptr;
  if (logits.scalar_type() == at::kBFloat16)
    logprob_bwd_kernel<bf16><<<rows, LP_THREADS, 0, stream()>>>(reinterpret_cast<bf16*>(logits.data_ptr()),
                                                                logits.stride(0), labels.data_ptr<int64_t>(), V, it,
                                                                gl, ge, lse.data_ptr<float>(), en);
  else
    logprob_bwd_kernel<float><<<rows, LP_THREADS, 0, stream()>>>(logits.data_ptr<float>(), logits.stride(0),
                                                                 labels.data_ptr<int64_t>(), V, it, gl, ge,
                                                                 lse.data_ptr<float>(), en);
  PSRL_CHECK_LAUNCH();
}

// ---------------------------------------------------------------- sampling ---
struct ArgMax {
  float key;
  int idx;
};

__device__ __forceinline__ ArgMax amax(ArgMax a, ArgMax b) {
  return (b.key > a.key || (b.key == a.key && b.idx < a.idx)) ? b : a;
}

// Gumbel key of one element and its contribution to the running statistics.
struct SampleAcc {
  OnlineStat st;
  ArgMax best;
};

// Add 8 scaled logits z[0..7] (indices i0..i0+7) to the accumulator: one
// rescale of the running sum per group instead of one per element.
__device__ __forceinline__ void sample_add8(SampleAcc& a, const float* z, int i0, bool greedy, uint64_t key) {
  float m8 = z[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) m8 = fmaxf(m8, z[j]);
  if (m8 == -INFINITY) return;               // fully masked group: no mass, never sampled
  if (m8 > a.st.m) {
    const float c = (a.st.m == -INFINITY) ? 0.f : __expf(a.st.m - m8);
    a.st.s *= c;
    a.st.t *= c;
    a.st.m = m8;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float e = __expf(z[j] - a.st.m);
    a.st.s += e;
    a.st.t += e * z[j];
    float k = z[j];
    if (!greedy) k = z[j] - __logf(-__logf(uniform01_k(key, (uint32_t)(i0 + j))));
    if (k > a.best.key) a.best = ArgMax{k, i0 + j};   // ascending indices: first max wins
  }
}

template <typename T>
__global__ void __launch_bounds__(LP_THREADS)
    sample_kernel(const T* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temps,
                  const int64_t* __restrict__ seeds, const int* __restrict__ streams, int64_t* __restrict__ out_tok,
                  float* __restrict__ out_lp) {
  __shared__ OnlineStat sm[32];
  __shared__ ArgMax am[32];
  const int64_t row = blockIdx.x;
  const T* z = logits + row * ld;
  const float tmp = temps ? temps[row] : 1.f;
  const bool greedy = tmp <= 0.f;
  const float it = greedy ? 1.f : 1.f / tmp;
  const uint64_t seed = seeds ? (uint64_t)seeds[row] : 0ull;
  const uint64_t step = streams ? (uint64_t)streams[row] : 0ull;
  // per-row key: the request's randomness depends only on (seed, position)
  const uint64_t key = mix64(seed ^ mix64(step * 0x632be59bd9b4e019ull));
  SampleAcc acc{{-INFINITY, 0.f, 0.f}, {-INFINITY, 0x7fffffff}};
  constexpr int VEC = 16 / (int)sizeof(T);   // elements per 16-byte load
  const bool vec_ok = (reinterpret_cast<uintptr_t>(z) % 16 == 0);
  const int nvec = vec_ok ? V / 8 : 0;       // groups of 8 elements
  for (int g = threadIdx.x; g < nvec; g += LP_THREADS) {
    float v[8];
    if constexpr (VEC == 8) {
      const bf16x8 p = *reinterpret_cast<const bf16x8*>(z + (int64_t)g * 8);
      unpack8(p, v);
    } else {
      const float4 p0 = *reinterpret_cast<const float4*>(z + (int64_t)g * 8);
      const float4 p1 = *reinterpret_cast<const float4*>(z + (int64_t)g * 8 + 4);
      v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
      v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= it;
    sample_add8(acc, v, g * 8, greedy, key);
  }
  // ragged tail (or the whole row when it is not 16-byte aligned)
  for (int i = nvec * 8 + threadIdx.x; i < V; i += LP_THREADS) {
    const float zi = to_f(z[i]) * it;
    ostat_add(acc.st, zi);
    float k = zi;
    if (!greedy) k = zi - __logf(-__logf(uniform01_k(key, (uint32_t)i)));
    acc.best = amax(acc.best, ArgMax{k, i});
  }
  OnlineStat st = ostat_block(acc.st, sm);
  ArgMax best = acc.best;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax w{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
    best = amax(best, w);
  }
  if (lane == 0) am[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (LP_THREADS / 32) ? am[lane] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax w{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
      best = amax(best, w);
    }
    if (lane == 0) {
      const float lse = st.m + __logf(st.s);
      out_tok[row] = best.idx;
      out_lp[row] = to_f(z[best.idx]) * it - lse;
    }
  }
}

// streams: per-row RNG stream (the sequence position of the sampled token), so a
// request's randomness depends only on (seed, position) and the launch is
// graph-capturable.
std::vector<at::Tensor> sample(at::Tensor logits, c10::optional<at::Tensor> temps, c10::optional<at::Tensor> seeds,
                               c10::optional<at::Tensor> streams) {
  CHECK_CUDA_TENSOR(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits must be [rows, V]");
  const int64_t rows = logits.size(0);
  const int V = logits.size(1);
  at::cuda::CUDAGuard g(logits.device());
  auto tok = at::empty({rows}, logits.options().dtype(at::kLong));
  auto lp = at::empty({rows}, logits.options().dtype(at::kFloat));
  if (rows == 0) return {tok, lp};
  const float* tp = temps.has_value() ? temps->data_ptr<float>() : nullptr;
  const int64_t* sp = seeds.has_value() ? seeds->data_ptr<int64_t>() : nullptr;
  const int* st = streams.has_value() ? streams->data_ptr<int>() : nullptr;
  if (logits.scalar_type() == at::kBFloat16)
    sample_kernel<bf16><<<rows, LP_THREADS, 0, stream()>>>(reinterpret_cast<const bf16*>(logits.data_ptr()),
                                                           logits.stride(0), V, tp, sp, st, tok.data_ptr<int64_t>(),
                                                           lp.data_ptr<float>());
  else
    sample_kernel<float><<<rows, LP_THREADS, 0, stream()>>>(logits.data_ptr<float>(), logits.stride(0), V, tp, sp,
                                                            st, tok.data_ptr<int64_t>(), lp.data_ptr<float>());
  PSRL_CHECK_LAUNCH();
  return {tok, lp};
}

}  // namespace psrl
