// Weight-streaming tcgen05 GEMM for decode (few rows, large weights):
//   Y[b, n] = sum_k X[b, k] W[n, k]  (+ bias[n]),  b < B <= 256.
//
// The roles of the operands are swapped so that the weight fills the MMA's M
// dimension: each CTA computes D[128 weight rows, NB tokens] = W_tile X^T with
// tcgen05.mma (M = 128, N = NB, K = 16) into NB fp32 TMEM columns, streaming its
// 128-row weight slab through a 4-stage TMA ring.  A decode step's GEMMs have
// too few 128-row slabs to occupy every SM (QKV of a 3B model: 20), so the K
// loop is split across CTAs; split partial sums are added into an fp32
// workspace with TMA reduce-add tiles and a finalize kernel converts to bf16,
// adds the bias and zeroes the workspace for the next call.  With one split the
// epilogue stores bf16 directly.
//
// Per CTA: 192 threads: warp 0 TMA producer, warp 1 MMA issuer (one thread),
// warps 2..5 epilogue (TMEM lane quadrant = 32 weight rows each; the tile is
// transposed through shared memory so every store is a [tokens, features]
// box).  Waits are bounded; a timeout records an error code and the kernel
// leaves after releasing its TMEM.  Tile loads are plain per-CTA TMA copies.
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"
#include "tcgen05.cuh"

namespace psrl {
namespace gsk {

using namespace tc5;

constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int NTHREADS = 192;
constexpr int STG_BYTES = 4096;  // per warp and buffer: 32 tokens x 128 B

template <int NB>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = NB * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STG_OFF + 4 * 2 * STG_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 128 + 1024;
  static constexpr int TMEM_COLS = NB < 32 ? 32 : NB;
};

struct Args {
  int B, N, K;
  int tiles_n, kblocks, splits;
  const bf16* bias;  // bf16 output only
  int* err;
};

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

template <int NB, bool F32_RED>
__global__ void __launch_bounds__(NTHREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmY, Args a) {
  using C = Cfg<NB>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES, accf = empty0 + 8 * STAGES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x % a.tiles_n, split = blockIdx.x / a.tiles_n;
  const int n0 = tile * BM;
  const int kb_lo = (int)((int64_t)split * a.kblocks / a.splits);
  const int kb_hi = (int)((int64_t)(split + 1) * a.kblocks / a.splits);
  __shared__ volatile int s_abort;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    mbar_init(accf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc_1cta(smem_u32(tmem_slot), C::TMEM_COLS);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1)) {
          set_err(a.err, 41);
          s_abort = 1;
          break;
        }
        const uint32_t fb = full0 + 8 * stage;
        mbar_expect_tx(fb, C::STAGE_BYTES);
        const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
        tma_load_2d(sa, &tmW, kb * BK, n0, fb);
        tma_load_2d(sa + C::A_BYTES, &tmX, kb * BK, 0, fb);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, NB, false, false);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!mbar_wait(full0 + 8 * stage, phase) || s_abort) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES), sb = sa + C::A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          mma_1cta(tmem, desc_sw128(sa + k * 32, 16, 1024), desc_sw128(sb + k * 32, 16, 1024), idesc,
                   (kb > kb_lo || k > 0) ? 1u : 0u);
        commit_1cta(empty0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        set_err(a.err, 42);
        s_abort = 1;
      }
      commit_1cta(accf);
    }
  } else {
    // epilogue: this warp's 32 weight rows (output features) x NB tokens
    const int quad = warp & 3;
    const int feat0 = n0 + quad * 32;
    uint8_t* stg = smem + C::STG_OFF + (warp - 2) * 2 * STG_BYTES;
    int next = 0;
    if (!mbar_wait(accf, 0)) set_err(a.err, 43);
    fence_after();
    const bool ok = !s_abort;
    const float bias = (!F32_RED && a.bias != nullptr && feat0 + lane < a.N) ? __bfloat162float(a.bias[feat0 + lane]) : 0.f;
    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < NB / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);  // r[t] = D[feature = lane][token = 32 c + t]
      tmem_wait_ld();
      if (!ok || c * 32 >= a.B) continue;
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
      uint8_t* buf = stg + next * STG_BYTES;
      if constexpr (F32_RED) {
        float* t = reinterpret_cast<float*>(buf);  // [32 tokens][32 features]
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i * 32 + lane] = __uint_as_float(r[i]);
      } else {
        bf16* t = reinterpret_cast<bf16*>(buf);    // [32 tokens][32 features]
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i * 32 + lane] = __float2bfloat16(__uint_as_float(r[i]) + bias);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (F32_RED) tma_reduce_add_2d(&tmY, smem_u32(buf), feat0, c * 32);
        else tma_store_2d(&tmY, smem_u32(buf), feat0, c * 32);
        bulk_commit();
      }
      next ^= 1;
    }
    if (lane == 0) bulk_wait_all();
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_free_1cta(tmem, C::TMEM_COLS);
  }
}

// y = bf16(ws + bias); ws = 0 (ready for the next accumulation)
__global__ void skinny_finalize(float* __restrict__ ws, bf16* __restrict__ y, const bf16* __restrict__ bias,
                                int64_t total, int N) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= total) return;
  float4 v = *reinterpret_cast<float4*>(ws + i);
  *reinterpret_cast<float4*>(ws + i) = make_float4(0.f, 0.f, 0.f, 0.f);
  float f[4] = {v.x, v.y, v.z, v.w};
  if (bias != nullptr) {
    const int n = (int)(i % N);
#pragma unroll
    for (int j = 0; j < 4; ++j) f[j] += __bfloat162float(bias[n + j]);
  }
  bf162 lo = __floats2bfloat162_rn(f[0], f[1]), hi = __floats2bfloat162_rn(f[2], f[3]);
  *reinterpret_cast<bf162*>(y + i) = lo;
  *reinterpret_cast<bf162*>(y + i + 2) = hi;
}

}  // namespace gsk

using namespace gsk;

static CUtensorMap skinny_map(const at::Tensor& t, uint32_t box_cols, uint32_t box_rows, bool swizzle) {
  const bool f32 = t.scalar_type() == at::kFloat;
  const int esz = f32 ? 4 : 2;
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && (t.stride(0) * esz) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "operand rows must start on 16-byte boundaries with unit inner stride");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * esz};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = PSRL_DRV(cuTensorMapEncodeTiled)(
      &m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides,
      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

template <int NB, bool F32_RED>
static void skinny_launch(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty, const Args& a) {
  ensure_smem_attr(skinny_kernel<NB, F32_RED>, Cfg<NB>::SMEM_BYTES);
  skinny_kernel<NB, F32_RED><<<a.tiles_n * a.splits, NTHREADS, Cfg<NB>::SMEM_BYTES, stream()>>>(tw, tx, ty, a);
  PSRL_CHECK_LAUNCH();
}

template <bool F32_RED>
static void skinny_dispatch(int nb, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty,
                            const Args& a) {
  switch (nb) {
    case 32: skinny_launch<32, F32_RED>(tw, tx, ty, a); break;
    case 64: skinny_launch<64, F32_RED>(tw, tx, ty, a); break;
    case 128: skinny_launch<128, F32_RED>(tw, tx, ty, a); break;
    default: skinny_launch<256, F32_RED>(tw, tx, ty, a); break;
  }
}

// Decode GEMM y = x w^T (+ bias): x [B, K] bf16 with B <= 256, w [N, K] bf16.
// splits > 1 splits the K loop across CTAs and needs `ws`, an fp32 workspace of
// at least B * N elements that is all zero on entry (it is zero again on
// return).  Returns y [B, N] bf16.
at::Tensor tc_gemm_skinny(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, int64_t splits,
                          c10::optional<at::Tensor> ws, at::Tensor err) {
  CHECK_CUDA_TENSOR(x);
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "x [B, K] and w [N, K]");
  const int64_t B = x.size(0), N = w.size(0), K = x.size(1);
  TORCH_CHECK(B <= 256, "at most 256 rows");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "N and K must be multiples of 8");
  at::cuda::CUDAGuard g(x.device());
  auto y = at::empty({B, N}, x.options());
  if (B == 0 || N == 0) return y;
  const int nb = B <= 32 ? 32 : B <= 64 ? 64 : B <= 128 ? 128 : 256;
  Args a{};
  a.B = (int)B;
  a.N = (int)N;
  a.K = (int)K;
  a.tiles_n = (int)((N + BM - 1) / BM);
  a.kblocks = (int)((K + BK - 1) / BK);
  a.splits = (int)std::max<int64_t>(1, std::min<int64_t>(splits, a.kblocks));
  a.err = err.data_ptr<int>();
  const bf16* bptr = nullptr;
  if (bias.has_value()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "bias must be a contiguous bf16 [N]");
    bptr = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  const CUtensorMap tw = skinny_map(w, 64, BM, true), tx = skinny_map(x, 64, (uint32_t)nb, true);
  if (a.splits == 1) {
    a.bias = bptr;
    const CUtensorMap ty = skinny_map(y, 32, 32, false);
    skinny_dispatch<false>(nb, tw, tx, ty, a);
    return y;
  }
  TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat && ws->is_contiguous() && ws->numel() >= B * N,
              "split-K needs a zeroed fp32 workspace of at least B * N elements");
  auto acc = ws->narrow(0, 0, B * N).view({B, N});
  const CUtensorMap ty = skinny_map(acc, 32, 32, false);
  skinny_dispatch<true>(nb, tw, tx, ty, a);
  const int64_t total = B * N;
  skinny_finalize<<<(unsigned)((total / 4 + 255) / 256), 256, 0, stream()>>>(
      acc.data_ptr<float>(), reinterpret_cast<bf16*>(y.data_ptr()), bptr, total, (int)N);
  PSRL_CHECK_LAUNCH();
  return y;
}

}  // namespace psrl
