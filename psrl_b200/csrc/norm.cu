// Fused residual-add + RMSNorm forward / backward (bf16 activations, fp32 math).
//
// Forward:  s = x (+ residual);  y = s * rsqrt(mean(s^2) + eps) * w
//           writes y, s (the new residual stream) and rstd per row.
// Backward: ds = dres + rstd * (w*dy) - s * rstd^3 * mean(w*dy*s)
//           dw += sum_rows dy * s * rstd  (per-block register partials, one
//           fp32 atomicAdd per element per block).
//
// One CTA of 256 threads per row; each thread owns up to MAXV 16-byte vectors of
// the row in registers, so a row is read exactly once.
#include "common.cuh"

namespace psrl {

constexpr int NORM_THREADS = 256;

template <int MAXV>
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_fwd_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ res, const bf16* __restrict__ w,
    bf16* __restrict__ y, bf16* __restrict__ res_out, float* __restrict__ rstd_out, int h,
    float eps) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = h >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (size_t)row * h);
  const bf16x8* rr = res ? reinterpret_cast<const bf16x8*>(res + (size_t)row * h) : nullptr;
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    int i = threadIdx.x + j * NORM_THREADS;
    if (i < nvec) {
      unpack8(xr[i], v[j]);
      if (rr) {
        float r8[8];
        unpack8(rr[i], r8);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[j][k] += r8[k];
        // the residual stream is kept in bf16: round before normalising
        bf16x8 p = pack8(v[j]);
        unpack8(p, v[j]);
        reinterpret_cast<bf16x8*>(res_out + (size_t)row * h)[i] = p;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[j][k] * v[j][k];
    }
  }
  ss = block_sum(ss, red);
  const float rstd = rsqrtf(ss / (float)h + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = rstd;
  const bf16x8* wv = reinterpret_cast<const bf16x8*>(w);
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + (size_t)row * h);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    int i = threadIdx.x + j * NORM_THREADS;
    if (i < nvec) {
      float w8[8], o[8];
      unpack8(wv[i], w8);
#pragma unroll
      for (int k = 0; k < 8; ++k) o[k] = v[j][k] * rstd * w8[k];
      yr[i] = pack8(o);
    }
  }
}

template <int MAXV>
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_bwd_kernel(
    const bf16* __restrict__ dy, const bf16* __restrict__ s, const bf16* __restrict__ w,
    const float* __restrict__ rstd, const bf16* __restrict__ dres, bf16* __restrict__ ds,
    float* __restrict__ dw_acc, int rows, int h) {
  __shared__ float red[32];
  const int nvec = h >> 3;
  const bf16x8* wv = reinterpret_cast<const bf16x8*>(w);
  float wreg[MAXV][8];
  float dwp[MAXV][8];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    int i = threadIdx.x + j * NORM_THREADS;
#pragma unroll
    for (int k = 0; k < 8; ++k) dwp[j][k] = 0.f;
    if (i < nvec) unpack8(wv[i], wreg[j]);
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const bf16x8* dyr = reinterpret_cast<const bf16x8*>(dy + (size_t)row * h);
    const bf16x8* sr = reinterpret_cast<const bf16x8*>(s + (size_t)row * h);
    const float r = rstd[row];
    float sv[MAXV][8], gv[MAXV][8];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      int i = threadIdx.x + j * NORM_THREADS;
      if (i < nvec) {
        float d8[8];
        unpack8(dyr[i], d8);
        unpack8(sr[i], sv[j]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          gv[j][k] = d8[k] * wreg[j][k];
          dot += gv[j][k] * sv[j][k];
          dwp[j][k] += d8[k] * sv[j][k] * r;
        }
      }
    }
    dot = block_sum(dot, red);
    const float c = dot * r * r * r / (float)h;
    bf16x8* dsr = reinterpret_cast<bf16x8*>(ds + (size_t)row * h);
    const bf16x8* drr = dres ? reinterpret_cast<const bf16x8*>(dres + (size_t)row * h) : nullptr;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      int i = threadIdx.x + j * NORM_THREADS;
      if (i < nvec) {
        float o[8], a[8];
        if (drr) unpack8(drr[i], a);
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = r * gv[j][k] - c * sv[j][k] + (drr ? a[k] : 0.f);
        dsr[i] = pack8(o);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    int i = threadIdx.x + j * NORM_THREADS;
    if (i < nvec) {
#pragma unroll
      for (int k = 0; k < 8; ++k) atomicAdd(dw_acc + i * 8 + k, dwp[j][k]);
    }
  }
}

#define NORM_DISPATCH(MAXV_EXPR, ...)                              \
  do {                                                             \
    int _mv = (MAXV_EXPR);                                         \
    if (_mv <= 1) { constexpr int MAXV = 1; __VA_ARGS__; }         \
    else if (_mv <= 2) { constexpr int MAXV = 2; __VA_ARGS__; }    \
    else if (_mv <= 4) { constexpr int MAXV = 4; __VA_ARGS__; }    \
    else TORCH_CHECK(false, "hidden size too large for rmsnorm");  \
  } while (0)

// returns {y, residual_out (or empty), rstd}
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, c10::optional<at::Tensor> residual, at::Tensor w,
                                    double eps) {
  CHECK_CUDA_TENSOR(x);
  CHECK_CONTIG(x);
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_DTYPE(w, at::kBFloat16);
  const int h = x.size(-1);
  TORCH_CHECK(h % 8 == 0, "hidden size must be a multiple of 8");
  const int rows = x.numel() / h;
  at::cuda::CUDAGuard g(x.device());
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor rout;
  const bf16* rp = nullptr;
  if (residual.has_value()) {
    auto r = residual.value();
    CHECK_CONTIG(r);
    CHECK_DTYPE(r, at::kBFloat16);
    rp = reinterpret_cast<const bf16*>(r.data_ptr());
    rout = at::empty_like(x);
  }
  if (rows == 0) return {y, rout, rstd};
  NORM_DISPATCH((h / 8 + NORM_THREADS - 1) / NORM_THREADS,
                rmsnorm_fwd_kernel<MAXV><<<rows, NORM_THREADS, 0, stream()>>>(
                    reinterpret_cast<const bf16*>(x.data_ptr()), rp,
                    reinterpret_cast<const bf16*>(w.data_ptr()), reinterpret_cast<bf16*>(y.data_ptr()),
                    rp ? reinterpret_cast<bf16*>(rout.data_ptr()) : nullptr, rstd.data_ptr<float>(), h,
                    (float)eps));
  PSRL_CHECK_LAUNCH();
  return {y, rout, rstd};
}

// returns {ds, dw(fp32)}
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor s, at::Tensor w, at::Tensor rstd,
                                    c10::optional<at::Tensor> dres) {
  CHECK_CONTIG(dy);
  CHECK_CONTIG(s);
  CHECK_DTYPE(dy, at::kBFloat16);
  const int h = s.size(-1);
  const int rows = s.numel() / h;
  at::cuda::CUDAGuard g(s.device());
  auto ds = at::empty_like(s);
  auto dw = at::zeros({h}, s.options().dtype(at::kFloat));
  const bf16* drp = nullptr;
  if (dres.has_value()) {
    CHECK_CONTIG(dres.value());
    drp = reinterpret_cast<const bf16*>(dres.value().data_ptr());
  }
  if (rows == 0) return {ds, dw};
  const int grid = std::min(rows, num_sms() * 4);
  NORM_DISPATCH((h / 8 + NORM_THREADS - 1) / NORM_THREADS,
                rmsnorm_bwd_kernel<MAXV><<<grid, NORM_THREADS, 0, stream()>>>(
                    reinterpret_cast<const bf16*>(dy.data_ptr()), reinterpret_cast<const bf16*>(s.data_ptr()),
                    reinterpret_cast<const bf16*>(w.data_ptr()), rstd.data_ptr<float>(), drp,
                    reinterpret_cast<bf16*>(ds.data_ptr()), dw.data_ptr<float>(), rows, h));
  PSRL_CHECK_LAUNCH();
  return {ds, dw};
}

// Per-head RMSNorm applied in place on q/k heads (Qwen3 q_norm/k_norm): x is a
// [rows, heads, d] strided view with unit stride on d; one warp per (row, head).
__global__ void head_rmsnorm_kernel(bf16* __restrict__ x, const bf16* __restrict__ w, float* __restrict__ rstd_out,
                                    int rows, int heads, int d, int64_t row_stride, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows * heads) return;
  const int row = warp / heads, hd = warp % heads;
  bf16* p = x + row * row_stride + (int64_t)hd * d;
  float v[8];
  float ss = 0.f;
  const int per = d / 32;  // d <= 256
  for (int k = 0; k < per; ++k) {
    v[k] = to_f(p[lane * per + k]);
    ss += v[k] * v[k];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / d + eps);
  if (lane == 0 && rstd_out) rstd_out[warp] = r;
  for (int k = 0; k < per; ++k) p[lane * per + k] = __float2bfloat16(v[k] * r * to_f(w[lane * per + k]));
}

at::Tensor head_rmsnorm_(at::Tensor x, at::Tensor w, double eps) {
  // x: [rows, heads, d] view (last dim contiguous)
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.stride(1) == x.size(2), "bad head view");
  const int rows = x.size(0), heads = x.size(1), d = x.size(2);
  TORCH_CHECK(d % 32 == 0 && d <= 256, "head_dim must be a multiple of 32, <= 256");
  at::cuda::CUDAGuard g(x.device());
  auto rstd = at::empty({rows, heads}, x.options().dtype(at::kFloat));
  const int warps = rows * heads;
  if (warps == 0) return rstd;
  head_rmsnorm_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream()>>>(
      reinterpret_cast<bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(w.data_ptr()), rstd.data_ptr<float>(),
      rows, heads, d, x.stride(0), (float)eps);
  PSRL_CHECK_LAUNCH();
  return rstd;
}

}  // namespace psrl
