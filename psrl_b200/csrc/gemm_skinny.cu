// Weight-streaming tcgen05 GEMM for decode (few rows, large weights):
//   Y[b, n] = sum_k X[b, k] W[n, k] (+ bias[n])                        (ACT_NONE)
//   H[b, i] = silu(G[b, i]) * U[b, i],  G / U = X W[i] / X W[I + i]     (ACT_SWIGLU)
// for b < B <= 256.
//
// The roles of the operands are swapped so that the weight fills the MMA's M
// dimension: a tile is 128 weight rows (output features) x NB tokens, computed
// as D = W_tile X^T with tcgen05.mma (M = 128, N = NB, K = 16) into NB fp32 TMEM
// columns (two accumulators, gate and up, for ACT_SWIGLU), the weight slab
// streaming through a TMA ring.  A decode step's GEMMs have too few tiles to
// occupy 148 SMs (QKV of a 3B model: 20, O and down: 16), so the K loop of a
// tile is split over the S CTAs of one thread-block cluster (S = 1, 2, 4 or 8,
// chosen on the host so that tiles x S fits one wave): each CTA accumulates its
// K slice in TMEM and writes the fp32 partial tile into its own shared memory
// (the drained TMA ring), one cluster barrier publishes the partials, and CTA r
// sums rows [r NB / S, (r + 1) NB / S) of all S partials with distributed
// shared-memory loads, applies bias or SwiGLU and stores bf16 -- no global
// workspace, no atomics, no second launch.  With S = 1 the epilogue stores the
// tile from TMEM directly (TMA store of bf16 boxes).
//
// Per CTA: 192 threads: warp 0 TMA producer, warp 1 MMA issuer (one thread),
// warps 2..5 epilogue (TMEM lane quadrant = 32 weight rows each).  Waits are
// bounded; a timeout records an error code, and every thread still reaches
// both cluster barriers, so the cluster's peers are never left waiting.  Tile
// loads are plain per-CTA TMA copies (no multicast).
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"
#include "tcgen05.cuh"

namespace psrl {
namespace gsk {

using namespace tc5;

constexpr int BM = 128, BK = 64;
constexpr int NTHREADS = 192;
constexpr int STG_BYTES = 4096;  // per warp and buffer: 32 tokens x 32 bf16 features
constexpr int RING_BUDGET = 193 * 1024;
enum { ACT_NONE = 0, ACT_SWIGLU = 1 };

template <int NB, int ACT>
struct Cfg {
  static constexpr int NACC = ACT == ACT_SWIGLU ? 2 : 1;            // accumulators per tile
  static constexpr int A_BYTES = BM * BK * 2;                        // one 128-row weight slab
  static constexpr int B_BYTES = NB * BK * 2;
  static constexpr int STAGE_BYTES = NACC * A_BYTES + B_BYTES;
  static constexpr int STAGES = RING_BUDGET / STAGE_BYTES > 8 ? 8 : RING_BUDGET / STAGE_BYTES;
  static constexpr int ACC_COLS = NACC * NB;                         // TMEM columns per tile
  static constexpr int TMEM_COLS = ACC_COLS < 32 ? 32 : ACC_COLS;
  static constexpr int PART_BYTES = NACC * NB * BM * 4;              // fp32 partial tile (split K)
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr bool CAN_SPLIT = PART_BYTES <= STG_OFF;           // partials fit the drained ring
  static constexpr int BAR_OFF = STG_OFF + 4 * 2 * STG_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
};

struct Args {
  int B, N, K;          // N: output features (I for ACT_SWIGLU)
  int up_off;           // ACT_SWIGLU: row of W where the up half starts (= I)
  int kblocks;
  int S;                // CTAs per cluster splitting one tile's K loop
  const bf16* bias;     // ACT_NONE only (may be null)
  bf16* y;              // [B, N]
  int* err;
};

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int NB, int ACT>
__global__ void __launch_bounds__(NTHREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmY, Args a) {
  using C = Cfg<NB, ACT>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES, accf = empty0 + 8 * STAGES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.S;
  const int rank = S > 1 ? (int)cluster_ctarank() : 0;
  const int tile = blockIdx.x / S;
  const int n0 = tile * BM;
  const int kb_lo = (int)((int64_t)rank * a.kblocks / S), kb_hi = (int)((int64_t)(rank + 1) * a.kblocks / S);
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
        if constexpr (ACT == ACT_SWIGLU) tma_load_2d(sa + C::A_BYTES, &tmW, kb * BK, a.up_off + n0, fb);
        tma_load_2d(sa + C::NACC * C::A_BYTES, &tmX, kb * BK, 0, fb);
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
        const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES), sb = sa + C::NACC * C::A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint32_t accum = (kb > kb_lo || k > 0) ? 1u : 0u;
          const uint64_t db = desc_sw128(sb + k * 32, 16, 1024);
          mma_1cta(tmem, desc_sw128(sa + k * 32, 16, 1024), db, idesc, accum);
          if constexpr (ACT == ACT_SWIGLU)
            mma_1cta(tmem + NB, desc_sw128(sa + C::A_BYTES + k * 32, 16, 1024), db, idesc, accum);
        }
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
      commit_1cta(accf);   // the epilogue sees s_abort if the tile is incomplete
    }
  } else {
    // epilogue: this warp's 32 weight rows (output features) x NB tokens
    const int quad = warp & 3;
    const int feat0 = n0 + quad * 32;
    bool ok = mbar_wait(accf, 0);
    if (!ok) {
      set_err(a.err, 43);
      s_abort = 1;
    }
    fence_after();
    ok = ok && !s_abort;
    const uint32_t tacc = tmem + ((uint32_t)(quad * 32) << 16);
    if (S == 1) {
      uint8_t* stg = smem + C::STG_OFF + (warp - 2) * 2 * STG_BYTES;
      int next = 0;
      const float bias =
          (ACT == ACT_NONE && a.bias != nullptr && feat0 + lane < a.N) ? __bfloat162float(a.bias[feat0 + lane]) : 0.f;
#pragma unroll 1
      for (int c = 0; c < NB / 32; ++c) {
        uint32_t r[32], ru[ACT == ACT_SWIGLU ? 32 : 1];
        tmem_ld32(tacc + c * 32, r);
        if constexpr (ACT == ACT_SWIGLU) tmem_ld32(tacc + NB + c * 32, ru);
        tmem_wait_ld();
        if (!ok || c * 32 >= a.B) continue;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        bf16* t = reinterpret_cast<bf16*>(stg + next * STG_BYTES);   // [32 tokens][32 features]
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v;
          if constexpr (ACT == ACT_SWIGLU) v = silu_mul(__uint_as_float(r[i]), __uint_as_float(ru[i]));
          else v = __uint_as_float(r[i]) + bias;
          t[i * 32 + lane] = __float2bfloat16(v);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmY, smem_u32(t), feat0, c * 32);
          bulk_commit();
        }
        next ^= 1;
      }
      if (lane == 0) bulk_wait_all();
    } else if constexpr (C::CAN_SPLIT) {
      // fp32 partial [acc][token][feature] in the drained TMA ring
      float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
      for (int c = 0; c < NB / 32; ++c) {
        uint32_t r[32], ru[ACT == ACT_SWIGLU ? 32 : 1];
        tmem_ld32(tacc + c * 32, r);
        if constexpr (ACT == ACT_SWIGLU) tmem_ld32(tacc + NB + c * 32, ru);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int o = (c * 32 + i) * BM + quad * 32 + lane;
          part[o] = ok ? __uint_as_float(r[i]) : 0.f;
          if constexpr (ACT == ACT_SWIGLU) part[NB * BM + o] = ok ? __uint_as_float(ru[i]) : 0.f;
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if constexpr (C::CAN_SPLIT) {
    if (S > 1) {
      cluster_sync();   // every CTA's partial is complete and visible to the cluster
      // this CTA's share of the tokens, all 128 features, summed over the cluster
      const int t_lo = rank * NB / S, t_hi = min((rank + 1) * NB / S, a.B);
      const int total = (t_hi > t_lo ? t_hi - t_lo : 0) * (BM / 4);
      const uint32_t base = smem_u32(smem);
      for (int idx = threadIdx.x; idx < total; idx += NTHREADS) {
        const int t = t_lo + idx / (BM / 4), f = (idx % (BM / 4)) * 4;
        if (n0 + f >= a.N) continue;
        const uint32_t off = (uint32_t)((t * BM + f) * 4);
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
        for (int q = 0; q < S; ++q) {
          const uint32_t pa = mapa(base + off, (uint32_t)q);
          const float4 v = ld_cluster_f4(pa);
          g.x += v.x; g.y += v.y; g.z += v.z; g.w += v.w;
          if constexpr (ACT == ACT_SWIGLU) {
            const float4 w = ld_cluster_f4(pa + NB * BM * 4);
            u.x += w.x; u.y += w.y; u.z += w.z; u.w += w.w;
          }
        }
        float o[4] = {g.x, g.y, g.z, g.w};
        if constexpr (ACT == ACT_SWIGLU) {
          o[0] = silu_mul(o[0], u.x);
          o[1] = silu_mul(o[1], u.y);
          o[2] = silu_mul(o[2], u.z);
          o[3] = silu_mul(o[3], u.w);
        } else if (a.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] += __bfloat162float(a.bias[n0 + f + j]);
        }
        bf162 pk[2] = {__floats2bfloat162_rn(o[0], o[1]), __floats2bfloat162_rn(o[2], o[3])};
        *reinterpret_cast<uint2*>(a.y + (int64_t)t * a.N + n0 + f) = *reinterpret_cast<const uint2*>(pk);
      }
      cluster_sync();   // no CTA leaves while a peer still reads its shared memory
    }
  }
  if (warp == 0) {
    fence_after();
    tmem_free_1cta(tmem, C::TMEM_COLS);
  }
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

template <int NB, int ACT>
static void skinny_launch(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty, const Args& a,
                          int tiles) {
  ensure_smem_attr(skinny_kernel<NB, ACT>, Cfg<NB, ACT>::SMEM_BYTES);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(tiles * a.S), 1, 1);
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg<NB, ACT>::SMEM_BYTES;
  cfg.stream = stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PSRL_CHECK_CUDA(cudaLaunchKernelEx(&cfg, skinny_kernel<NB, ACT>, tw, tx, ty, a));
}

template <int ACT>
static void skinny_dispatch(int nb, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty,
                            const Args& a, int tiles) {
  switch (nb) {
    case 32: skinny_launch<32, ACT>(tw, tx, ty, a, tiles); break;
    case 64: skinny_launch<64, ACT>(tw, tx, ty, a, tiles); break;
    case 128: skinny_launch<128, ACT>(tw, tx, ty, a, tiles); break;
    default: skinny_launch<256, ACT>(tw, tx, ty, a, tiles); break;
  }
}

static bool can_split(int nb, bool swiglu) {
  switch (nb) {
    case 32: return swiglu ? Cfg<32, ACT_SWIGLU>::CAN_SPLIT : Cfg<32, ACT_NONE>::CAN_SPLIT;
    case 64: return swiglu ? Cfg<64, ACT_SWIGLU>::CAN_SPLIT : Cfg<64, ACT_NONE>::CAN_SPLIT;
    case 128: return swiglu ? Cfg<128, ACT_SWIGLU>::CAN_SPLIT : Cfg<128, ACT_NONE>::CAN_SPLIT;
    default: return swiglu ? Cfg<256, ACT_SWIGLU>::CAN_SPLIT : Cfg<256, ACT_NONE>::CAN_SPLIT;
  }
}

// Decode GEMM, one launch: x [B, K] bf16 (B <= 256), w [R, K] bf16.
//   swiglu = false: y [B, R] = x w^T (+ bias [R]);
//   swiglu = true:  w holds gate rows [0, I) then up rows [I, 2I) (R = 2I,
//                   I % 128 == 0): y [B, I] = silu(x w_gate^T) * (x w_up^T).
// split: CTAs per 128-row tile sharing its K loop (1, 2, 4 or 8; <= 0: the
// largest that keeps tiles x split within one wave of the SMs and at least two
// 64-deep k blocks per CTA).
at::Tensor tc_gemm_skinny(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, bool swiglu, int64_t split,
                          at::Tensor err) {
  CHECK_CUDA_TENSOR(x);
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "x [B, K] and w [R, K]");
  const int64_t B = x.size(0), R = w.size(0), K = x.size(1);
  TORCH_CHECK(B <= 256, "at most 256 rows");
  TORCH_CHECK(R % 8 == 0 && K % 8 == 0, "R and K must be multiples of 8");
  TORCH_CHECK(!swiglu || (R % 256 == 0 && !bias.has_value()), "swiglu needs I = R / 2 a multiple of 128, no bias");
  const int64_t N = swiglu ? R / 2 : R;
  at::cuda::CUDAGuard g(x.device());
  auto y = at::empty({B, N}, x.options());
  if (B == 0 || N == 0) return y;
  const int nb = B <= 32 ? 32 : B <= 64 ? 64 : B <= 128 ? 128 : 256;
  const int tiles = (int)((N + BM - 1) / BM);
  Args a{};
  a.B = (int)B;
  a.N = (int)N;
  a.K = (int)K;
  a.up_off = swiglu ? (int)N : 0;
  a.kblocks = (int)((K + BK - 1) / BK);
  int S = (int)split;
  if (S <= 0) {
    S = 1;
    for (int c : {8, 4, 2})
      if ((int64_t)tiles * c <= num_sms() && a.kblocks >= 2 * c) {
        S = c;
        break;
      }
  }
  TORCH_CHECK(S == 1 || S == 2 || S == 4 || S == 8, "split must be 1, 2, 4 or 8");
  if (!can_split(nb, swiglu) || S > a.kblocks) S = 1;
  a.S = S;
  a.err = err.data_ptr<int>();
  a.y = reinterpret_cast<bf16*>(y.data_ptr());
  if (bias.has_value()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "bias must be a contiguous bf16 [N]");
    a.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  TORCH_CHECK(y.stride(0) == N, "y must be contiguous");
  const CUtensorMap tw = skinny_map(w, 64, BM, true), tx = skinny_map(x, 64, (uint32_t)nb, true);
  const CUtensorMap ty = skinny_map(y, 32, 32, false);
  if (swiglu) skinny_dispatch<ACT_SWIGLU>(nb, tw, tx, ty, a, tiles);
  else skinny_dispatch<ACT_NONE>(nb, tw, tx, ty, a, tiles);
  return y;
}

}  // namespace psrl
