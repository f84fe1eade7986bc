// Elementwise / reduction kernels: SwiGLU fwd+bwd, fused AdamW over flat fp32
// shards (with bf16 param write-back), squared-norm reduction, scaled casts.
#include "common.cuh"

namespace psrl {

// ---------------------------------------------------------------- SwiGLU ---
// gu: [rows, 2*I] = [gate | up]; out: [rows, I] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int64_t rows, int I) {
  const int nv = I >> 3;
  const int64_t total = rows * nv;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nv;
    const int c = idx % nv;
    const bf16x8* g = reinterpret_cast<const bf16x8*>(gu + r * 2 * I);
    const bf16x8* u = reinterpret_cast<const bf16x8*>(gu + r * 2 * I + I);
    float gf[8], uf[8], o[8];
    unpack8(g[c], gf);
    unpack8(u[c], uf);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = gf[k] / (1.f + __expf(-gf[k])) * uf[k];
    reinterpret_cast<bf16x8*>(out + r * I)[c] = pack8(o);
  }
}

// dgu[:, :I] = dout * up * silu'(gate); dgu[:, I:] = dout * silu(gate)
__global__ void swiglu_bwd_kernel(const bf16* __restrict__ gu, const bf16* __restrict__ dout,
                                  bf16* __restrict__ dgu, int64_t rows, int I) {
  const int nv = I >> 3;
  const int64_t total = rows * nv;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / nv;
    const int c = idx % nv;
    float gf[8], uf[8], df[8], dg[8], du[8];
    unpack8(reinterpret_cast<const bf16x8*>(gu + r * 2 * I)[c], gf);
    unpack8(reinterpret_cast<const bf16x8*>(gu + r * 2 * I + I)[c], uf);
    unpack8(reinterpret_cast<const bf16x8*>(dout + r * I)[c], df);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = 1.f / (1.f + __expf(-gf[k]));
      const float silu = gf[k] * s;
      du[k] = df[k] * silu;
      dg[k] = df[k] * uf[k] * s * (1.f + gf[k] * (1.f - s));
    }
    reinterpret_cast<bf16x8*>(dgu + r * 2 * I)[c] = pack8(dg);
    reinterpret_cast<bf16x8*>(dgu + r * 2 * I + I)[c] = pack8(du);
  }
}

static int elem_grid(int64_t work) {
  int64_t g = (work + 255) / 256;
  int64_t cap = (int64_t)num_sms() * 16;
  return (int)std::max<int64_t>(1, std::min(g, cap));
}

at::Tensor swiglu_fwd(at::Tensor gu) {
  CHECK_CUDA_TENSOR(gu);
  CHECK_CONTIG(gu);
  CHECK_DTYPE(gu, at::kBFloat16);
  const int I = gu.size(-1) / 2;
  TORCH_CHECK(I % 8 == 0, "intermediate size must be a multiple of 8");
  const int64_t rows = gu.numel() / (2 * I);
  auto sizes = gu.sizes().vec();
  sizes.back() = I;
  auto out = at::empty(sizes, gu.options());
  if (rows == 0) return out;
  at::cuda::CUDAGuard g(gu.device());
  swiglu_fwd_kernel<<<elem_grid(rows * I / 8), 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(gu.data_ptr()), reinterpret_cast<bf16*>(out.data_ptr()), rows, I);
  PSRL_CHECK_LAUNCH();
  return out;
}

at::Tensor swiglu_bwd(at::Tensor gu, at::Tensor dout) {
  CHECK_CONTIG(gu);
  CHECK_CONTIG(dout);
  const int I = gu.size(-1) / 2;
  const int64_t rows = gu.numel() / (2 * I);
  auto dgu = at::empty_like(gu);
  if (rows == 0) return dgu;
  at::cuda::CUDAGuard g(gu.device());
  swiglu_bwd_kernel<<<elem_grid(rows * I / 8), 256, 0, stream()>>>(
      reinterpret_cast<const bf16*>(gu.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()),
      reinterpret_cast<bf16*>(dgu.data_ptr()), rows, I);
  PSRL_CHECK_LAUNCH();
  return dgu;
}

// ----------------------------------------------------------------- AdamW ---
// Decoupled weight decay (Loshchilov & Hutter): p -= lr * (wd * p + mhat / (sqrt(vhat) + eps)).
// Gradients are multiplied by `gscale` (1/world, clip coefficient) first.
// Optionally writes a bf16 copy of the updated fp32 master.
template <typename GT>
__global__ void adamw_kernel(float* __restrict__ p, const GT* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, bf16* __restrict__ p16, int64_t n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ gscale_ptr,
                             float gscale) {
  const float gs = gscale_ptr ? gscale * gscale_ptr[0] : gscale;
  const int64_t nv = n >> 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float gg[4];
    if constexpr (std::is_same<GT, float>::value) {
      float4 t = reinterpret_cast<const float4*>(g)[i];
      gg[0] = t.x; gg[1] = t.y; gg[2] = t.z; gg[3] = t.w;
    } else {
      const bf162* gp = reinterpret_cast<const bf162*>(g) + 2 * i;
      float2 a = __bfloat1622float2(gp[0]), b = __bfloat1622float2(gp[1]);
      gg[0] = a.x; gg[1] = a.y; gg[2] = b.x; gg[3] = b.y;
    }
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
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16) {
      bf162* o = reinterpret_cast<bf162*>(p16) + 2 * i;
      o[0] = __floats2bfloat162_rn(pp.x, pp.y);
      o[1] = __floats2bfloat162_rn(pp.z, pp.w);
    }
  }
}

void adamw_(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p16, double lr,
            double b1, double b2, double eps, double wd, int64_t step, c10::optional<at::Tensor> gscale_t,
            double gscale) {
  CHECK_CUDA_TENSOR(p);
  CHECK_CONTIG(p);
  CHECK_CONTIG(g);
  CHECK_DTYPE(p, at::kFloat);
  const int64_t n = p.numel();
  TORCH_CHECK(n % 4 == 0, "flat shard length must be a multiple of 4");
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "size mismatch");
  if (n == 0) return;
  at::cuda::CUDAGuard gd(p.device());
  const float bc1 = 1.f - powf((float)b1, (float)step), bc2 = 1.f - powf((float)b2, (float)step);
  bf16* o = p16.has_value() ? reinterpret_cast<bf16*>(p16->data_ptr()) : nullptr;
  const float* gsp = gscale_t.has_value() ? gscale_t->data_ptr<float>() : nullptr;
  const int grid = elem_grid(n / 4);
  if (g.scalar_type() == at::kFloat)
    adamw_kernel<float><<<grid, 256, 0, stream()>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                                    v.data_ptr<float>(), o, n, lr, b1, b2, eps, wd, bc1, bc2, gsp,
                                                    gscale);
  else {
    CHECK_DTYPE(g, at::kBFloat16);
    adamw_kernel<bf16><<<grid, 256, 0, stream()>>>(p.data_ptr<float>(), reinterpret_cast<const bf16*>(g.data_ptr()),
                                                   m.data_ptr<float>(), v.data_ptr<float>(), o, n, lr, b1, b2, eps, wd,
                                                   bc1, bc2, gsp, gscale);
  }
  PSRL_CHECK_LAUNCH();
}

// ------------------------------------------------------- squared L2 norm ---
// Two-pass reduction: per-CTA partial sums (scratch) then a single-CTA finish.
template <typename T>
__global__ void sqnorm_partial_kernel(const T* __restrict__ x, int64_t n, float* __restrict__ partial) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float f = to_f(x[i]);
    acc += f * f;
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

__global__ void sum_finish_kernel(const float* __restrict__ partial, int n, float* __restrict__ out, int accumulate) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) out[0] = accumulate ? out[0] + acc : acc;
}

// Adds sum(x^2) into out[0] (fp32 device scalar); `partial` is caller scratch of >= grid floats.
void sqnorm_accumulate_(at::Tensor x, at::Tensor out, at::Tensor partial) {
  CHECK_CONTIG(x);
  const int64_t n = x.numel();
  if (n == 0) return;
  at::cuda::CUDAGuard g(x.device());
  const int grid = std::min<int64_t>(partial.numel(), std::max<int64_t>(1, (n + 255) / 256));
  if (x.scalar_type() == at::kFloat)
    sqnorm_partial_kernel<float><<<grid, 256, 0, stream()>>>(x.data_ptr<float>(), n, partial.data_ptr<float>());
  else
    sqnorm_partial_kernel<bf16><<<grid, 256, 0, stream()>>>(reinterpret_cast<const bf16*>(x.data_ptr()), n,
                                                            partial.data_ptr<float>());
  sum_finish_kernel<<<1, 1024, 0, stream()>>>(partial.data_ptr<float>(), grid, out.data_ptr<float>(), 1);
  PSRL_CHECK_LAUNCH();
}

// clip coefficient from a squared norm: coef = min(1, max_norm / (sqrt(sq) + 1e-6)), written to coef[0]
__global__ void clip_coef_kernel(const float* sq, float max_norm, float* coef, float* norm_out) {
  const float nrm = sqrtf(sq[0]);
  if (norm_out) norm_out[0] = nrm;
  coef[0] = (max_norm > 0.f) ? fminf(1.f, max_norm / (nrm + 1e-6f)) : 1.f;
}

void clip_coef_(at::Tensor sq, double max_norm, at::Tensor coef, at::Tensor norm_out) {
  at::cuda::CUDAGuard g(sq.device());
  clip_coef_kernel<<<1, 1, 0, stream()>>>(sq.data_ptr<float>(), (float)max_norm, coef.data_ptr<float>(),
                                          norm_out.data_ptr<float>());
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
