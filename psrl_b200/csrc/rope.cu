// Rotary position embedding (rotate-half convention, as in Qwen2/Qwen3) applied
// in place to the q and k heads of a fused qkv activation, optionally fused with
// the paged KV-cache write used by the rollout engine.
//
// qkv: [T, (nq + 2*nkv) * d] bf16 (row stride may exceed the width)
// cos/sin: [max_pos, d/2] fp32 tables; positions: [T] int32
// k_cache/v_cache: [num_blocks, nkv, block_size, d] bf16; slots: [T] int32 (-1 = skip)
//
// One warp per (token, head); lane l owns rotary pairs (2l, 2l+1) and their
// partners at +d/2 (d = 128: 4 bf16 per lane, fully coalesced).
#include "common.cuh"

namespace psrl {

template <int D>
__global__ void rope_kernel(bf16* __restrict__ qkv, int64_t row_stride, const int* __restrict__ pos,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, int T, int nq,
                            int nkv, float sign, bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                            const int* __restrict__ slots, int block_size) {
  constexpr int HALF = D / 2;
  constexpr int PER = HALF / 32;  // pairs per lane (2 for D=128)
  const int heads = nq + 2 * nkv;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (int64_t)T * heads) return;
  const int t = warp / heads, hd = warp % heads;
  bf16* p = qkv + t * row_stride + (int64_t)hd * D;
  const bool is_v = hd >= nq + nkv;
  const bool is_k = !is_v && hd >= nq;
  int slot = -1;
  if (slots) slot = slots[t];
  bf16* cache_dst = nullptr;
  if (slot >= 0 && (is_k || is_v)) {
    const int kvh = is_k ? hd - nq : hd - nq - nkv;
    const int blk = slot / block_size, off = slot % block_size;
    cache_dst = (is_k ? k_cache : v_cache) + (((int64_t)blk * nkv + kvh) * block_size + off) * D;
  }
  if (is_v) {
    if (cache_dst) {
      // copy 128 bf16 = 256 B: 8 B per lane
      const uint2* s = reinterpret_cast<const uint2*>(p);
      uint2* d = reinterpret_cast<uint2*>(cache_dst);
      for (int i = lane; i < D / 4; i += 32) d[i] = s[i];
    }
    return;
  }
  const int ps = pos[t];
  const float* cr = cos_t + (int64_t)ps * HALF;
  const float* sr = sin_t + (int64_t)ps * HALF;
  if constexpr (PER % 2 == 0) {
#pragma unroll
    for (int k = 0; k < PER; k += 2) {
      const int i = lane * PER + k;
      bf162 a = *reinterpret_cast<const bf162*>(p + i);
      bf162 b = *reinterpret_cast<const bf162*>(p + i + HALF);
      float2 af = __bfloat1622float2(a), bf = __bfloat1622float2(b);
      float c0 = cr[i], c1 = cr[i + 1], s0 = sign * sr[i], s1 = sign * sr[i + 1];
      float2 oa = make_float2(af.x * c0 - bf.x * s0, af.y * c1 - bf.y * s1);
      float2 ob = make_float2(bf.x * c0 + af.x * s0, bf.y * c1 + af.y * s1);
      bf162 ra = __floats2bfloat162_rn(oa.x, oa.y), rb = __floats2bfloat162_rn(ob.x, ob.y);
      *reinterpret_cast<bf162*>(p + i) = ra;
      *reinterpret_cast<bf162*>(p + i + HALF) = rb;
      if (cache_dst) {
        *reinterpret_cast<bf162*>(cache_dst + i) = ra;
        *reinterpret_cast<bf162*>(cache_dst + i + HALF) = rb;
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = lane * PER + k;
      float a = to_f(p[i]), b = to_f(p[i + HALF]);
      float c = cr[i], sn = sign * sr[i];
      bf16 ra = __float2bfloat16(a * c - b * sn), rb = __float2bfloat16(b * c + a * sn);
      p[i] = ra;
      p[i + HALF] = rb;
      if (cache_dst) {
        cache_dst[i] = ra;
        cache_dst[i + HALF] = rb;
      }
    }
  }
}

void rope_(at::Tensor qkv, at::Tensor positions, at::Tensor cos_t, at::Tensor sin_t, int64_t nq, int64_t nkv,
           int64_t d, bool inverse, c10::optional<at::Tensor> k_cache, c10::optional<at::Tensor> v_cache,
           c10::optional<at::Tensor> slots) {
  CHECK_CUDA_TENSOR(qkv);
  CHECK_DTYPE(qkv, at::kBFloat16);
  CHECK_DTYPE(positions, at::kInt);
  TORCH_CHECK(qkv.stride(-1) == 1, "qkv last dim must be contiguous");
  TORCH_CHECK(d == 128 || d == 64, "head_dim must be 64 or 128");
  const int T = qkv.size(0);
  if (T == 0) return;
  at::cuda::CUDAGuard g(qkv.device());
  bf16 *kc = nullptr, *vc = nullptr;
  const int* sl = nullptr;
  int block_size = 1;
  if (k_cache.has_value()) {
    TORCH_CHECK(v_cache.has_value() && slots.has_value(), "cache write needs k, v caches and slots");
    kc = reinterpret_cast<bf16*>(k_cache->data_ptr());
    vc = reinterpret_cast<bf16*>(v_cache->data_ptr());
    sl = slots->data_ptr<int>();
    block_size = k_cache->size(2);
    TORCH_CHECK(k_cache->size(1) == nkv && k_cache->size(3) == d, "k_cache must be [blocks, nkv, bs, d]");
  }
  const int64_t warps = (int64_t)T * (nq + 2 * nkv);
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (d == 128)
    rope_kernel<128><<<blocks, threads, 0, stream()>>>(
        reinterpret_cast<bf16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int>(), cos_t.data_ptr<float>(),
        sin_t.data_ptr<float>(), T, nq, nkv, inverse ? -1.f : 1.f, kc, vc, sl, block_size);
  else
    rope_kernel<64><<<blocks, threads, 0, stream()>>>(
        reinterpret_cast<bf16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int>(), cos_t.data_ptr<float>(),
        sin_t.data_ptr<float>(), T, nq, nkv, inverse ? -1.f : 1.f, kc, vc, sl, block_size);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
