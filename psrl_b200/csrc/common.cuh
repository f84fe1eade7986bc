// Shared helpers for the psrl_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <utility>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#define PSRL_CHECK_CUDA(expr)                                                        \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ",    \
                __FILE__, ":", __LINE__);                                            \
  } while (0)

#define PSRL_CHECK_LAUNCH() PSRL_CHECK_CUDA(cudaGetLastError())

#define CHECK_CUDA_TENSOR(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_DTYPE(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has wrong dtype")

namespace psrl {

using bf16 = __nv_bfloat16;
using bf162 = __nv_bfloat162;

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Raise a kernel's dynamic shared-memory limit on the current device, once
// per (kernel, device): the attribute is per device, so a process that
// launches the kernel on several GPUs sets it on each of them.
template <typename Kernel>
inline void ensure_smem_attr(Kernel* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  PSRL_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(fn), dev);
  if (done.count(key)) return;
  PSRL_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert(key);
}

__device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float x) { return __float2bfloat16(x); }
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ half from_f<half>(float x) { return __float2half(x); }

// 16-byte vector of 8 bf16 values.
struct alignas(16) bf16x8 {
  bf162 v[4];
};

__device__ __forceinline__ void unpack8(const bf16x8& p, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p.v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bf16x8 pack8(const float* f) {
  bf16x8 p;
#pragma unroll
  for (int i = 0; i < 4; ++i) p.v[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return p;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `smem` needs one float per warp. Result broadcast to all threads.
__device__ __forceinline__ float block_sum(float v, float* smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float r = (threadIdx.x < nwarps) ? smem[threadIdx.x] : 0.f;
  if (warp == 0) r = warp_sum(r);
  if (threadIdx.x == 0) smem[0] = r;
  __syncthreads();
  r = smem[0];
  return r;
}

__device__ __forceinline__ float block_max(float v, float* smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) smem[warp] = v;
  __syncthreads();
  float r = (threadIdx.x < nwarps) ? smem[threadIdx.x] : -INFINITY;
  if (warp == 0) r = warp_max(r);
  if (threadIdx.x == 0) smem[0] = r;
  __syncthreads();
  r = smem[0];
  return r;
}

// Counter-based uniform random numbers: a 64-bit mix (SplitMix64 finaliser,
// Steele et al. 2014) of (seed, stream, index). Returns a float in (0, 1).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t stream, uint64_t idx) {
  uint64_t h = mix64(seed ^ mix64(stream * 0x632be59bd9b4e019ull + idx));
  // 24 random mantissa bits, shifted off zero.
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

// 32-bit integer hash "lowbias32" (C. Wellons, hash-prospector, public
// domain): xorshift-multiply rounds with low avalanche bias.  Used for
// per-element random bits once a 64-bit per-row key has been mixed.
__device__ __forceinline__ uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// uniform (0, 1) from a per-row 64-bit key and a 32-bit element index
__device__ __forceinline__ float uniform01_k(uint64_t key, uint32_t idx) {
  const uint32_t h = hash32(hash32(idx ^ (uint32_t)key) + (uint32_t)(key >> 32));
  return ((float)(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

}  // namespace psrl
