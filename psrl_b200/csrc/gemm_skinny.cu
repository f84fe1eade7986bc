// Weight-streaming tcgen05 GEMM for decode (few rows, large weights), stream-K:
//   Y[b, n] = sum_k X[b, k] W[n, k] (+ bias[n])                        (ACT_NONE)
//   H[b, i] = silu(G[b, i]) * U[b, i],  G / U = X W[i] / X W[I + i]     (ACT_SWIGLU)
// for b < B <= 256.
//
// The roles of the operands are swapped so that the weight fills the MMA's M
// dimension: a tile is 128 weight rows (output features) x NB tokens, computed
// as D = W_tile X^T with tcgen05.mma (M = 128, N = NB, K = 16) into NB fp32 TMEM
// columns (two accumulators, gate and up, for ACT_SWIGLU).  A decode step's
// GEMMs have too few tiles to occupy 148 SMs with one CTA per tile (QKV of a
// 3B model: 20 tiles; gate_up: 86 tile pairs) and, with whole tiles per CTA,
// leave a partial last wave, so the kernel is persistent and stream-K: the
// (tile, 64-wide k block) units are dealt out in equal contiguous ranges to
// one CTA per SM.  A CTA whose range covers a whole tile finishes it in its
// epilogue (bias or SwiGLU, bf16 TMA store); a tile shared by several CTAs is
// accumulated in an fp32 workspace with TMA reduce-add, and the CTA that
// arrives last on the tile's ticket (an atomic counter, reset by that CTA)
// reads the sum back, applies the epilogue, stores bf16 and zeroes the
// workspace, so no second launch is needed.
//
// Per CTA: 192 threads: warp 0 TMA producer, warp 1 MMA issuer (one thread),
// warps 2..5 epilogue (TMEM lane quadrant = 32 weight rows each; tiles are
// transposed through shared memory so every store is a [tokens, features]
// box).  Accumulators are double-buffered in TMEM when they fit, so the
// epilogue of one tile overlaps the MMAs of the next.  Waits are bounded; a
// timeout records an error code and the kernel leaves after releasing its
// TMEM.  Tile loads are plain per-CTA TMA copies.
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"
#include "tcgen05.cuh"

namespace psrl {
namespace gsk {

using namespace tc5;

constexpr int BM = 128, BK = 64;
constexpr int NTHREADS = 192;
constexpr int STG_BYTES = 4096;  // per warp and buffer: 32 tokens x 32 fp32 (or bf16) features
constexpr int RING_BUDGET = 193 * 1024;  // 3 x 64 KB stages of the widest (NB 256, SwiGLU) case fit
enum { ACT_NONE = 0, ACT_SWIGLU = 1 };

template <int NB, int ACT>
struct Cfg {
  static constexpr int NACC = ACT == ACT_SWIGLU ? 2 : 1;            // accumulators per tile
  static constexpr int A_BYTES = BM * BK * 2;                        // one 128-row weight slab
  static constexpr int B_BYTES = NB * BK * 2;
  static constexpr int STAGE_BYTES = NACC * A_BYTES + B_BYTES;
  static constexpr int STAGES = RING_BUDGET / STAGE_BYTES > 8 ? 8 : RING_BUDGET / STAGE_BYTES;
  static constexpr int ACC_COLS = NACC * NB;                         // TMEM columns per tile
  static constexpr int ACC_STAGES = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = ACC_STAGES * ACC_COLS < 32 ? 32 : ACC_STAGES * ACC_COLS;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STG_OFF + 4 * 2 * STG_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
};

struct Args {
  int B, N, K;          // N: output features (I for ACT_SWIGLU)
  int up_off;           // ACT_SWIGLU: row of W where the up half starts (= I)
  int tiles, kblocks;   // work units = tiles * kblocks
  int grid;
  const bf16* bias;     // ACT_NONE only (may be null)
  float* ws;            // fp32 [B, ws_cols] accumulator of shared tiles (zero between calls)
  int ws_cols;
  int* tickets;         // [tiles] arrival counters (zero between calls)
  bf16* y;              // [B, N]
  int* err;
};

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// CTA whose unit range [c U / G, (c + 1) U / G) holds unit u
__device__ __forceinline__ int owner_of(int64_t u, int64_t U, int G) { return (int)(((u + 1) * G + U - 1) / U) - 1; }

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The last CTA on a shared tile: y = epilogue(ws) for the tile's 128 features,
// then ws = 0.  Run by the 128 epilogue threads, eight independent 16-byte
// loads in flight per thread (a load-store-load chain would pay the L2
// latency once per vector).
template <int ACT>
__device__ __forceinline__ void finalize_tile(const Args& a, int tile) {
  constexpr int V = 8;
  const int tid = threadIdx.x - 64;
  const int f0 = tile * BM;
  const int total = a.B * (BM / 4);
  for (int base = tid; base < total; base += 128 * V) {
    float4 g[V], u[V];
    int off[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const int idx = base + j * 128;
      const int t = idx / (BM / 4), f = f0 + (idx % (BM / 4)) * 4;
      off[j] = (idx < total && f < a.N) ? t * a.ws_cols + f : -1;
      g[j] = off[j] >= 0 ? __ldcg(reinterpret_cast<const float4*>(a.ws + off[j])) : make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (ACT == ACT_SWIGLU)
        u[j] = off[j] >= 0 ? __ldcg(reinterpret_cast<const float4*>(a.ws + off[j] + a.up_off))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if (off[j] < 0) continue;
      const int idx = base + j * 128;
      const int t = idx / (BM / 4), f = f0 + (idx % (BM / 4)) * 4;
      float o[4] = {g[j].x, g[j].y, g[j].z, g[j].w};
      if constexpr (ACT == ACT_SWIGLU) {
        o[0] = silu_mul(o[0], u[j].x);
        o[1] = silu_mul(o[1], u[j].y);
        o[2] = silu_mul(o[2], u[j].z);
        o[3] = silu_mul(o[3], u[j].w);
        __stcg(reinterpret_cast<float4*>(a.ws + off[j] + a.up_off), make_float4(0.f, 0.f, 0.f, 0.f));
      } else if (a.bias != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] += __bfloat162float(a.bias[f + q]);
      }
      __stcg(reinterpret_cast<float4*>(a.ws + off[j]), make_float4(0.f, 0.f, 0.f, 0.f));
      bf162 p[2] = {__floats2bfloat162_rn(o[0], o[1]), __floats2bfloat162_rn(o[2], o[3])};
      *reinterpret_cast<uint2*>(a.y + (int64_t)t * a.N + f) = *reinterpret_cast<const uint2*>(p);
    }
  }
}

template <int NB, int ACT>
__global__ void __launch_bounds__(NTHREADS, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmWS, Args a) {
  using C = Cfg<NB, ACT>;
  constexpr int STAGES = C::STAGES, ACCS = C::ACC_STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * ACCS);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES;
  const uint32_t accf0 = empty0 + 8 * STAGES, acce0 = accf0 + 8 * ACCS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.kblocks, G = a.grid;
  const int64_t U = (int64_t)a.tiles * KB;
  const int64_t u0 = (int64_t)blockIdx.x * U / G, u1 = (int64_t)(blockIdx.x + 1) * U / G;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_last;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    for (int i = 0; i < ACCS; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 4);   // one arrival per epilogue warp
    }
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
      for (int64_t u = u0; u < u1 && !s_abort;) {
        const int tile = (int)(u / KB);
        const int kb_lo = (int)(u - (int64_t)tile * KB);
        const int64_t end = u1 < (int64_t)(tile + 1) * KB ? u1 : (int64_t)(tile + 1) * KB;
        const int kb_hi = kb_lo + (int)(end - u);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1)) {
            set_err(a.err, 41);
            s_abort = 1;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          mbar_expect_tx(fb, C::STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          tma_load_2d(sa, &tmW, kb * BK, tile * BM, fb);
          if constexpr (ACT == ACT_SWIGLU) tma_load_2d(sa + C::A_BYTES, &tmW, kb * BK, a.up_off + tile * BM, fb);
          tma_load_2d(sa + C::NACC * C::A_BYTES, &tmX, kb * BK, 0, fb);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        u = end;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, NB, false, false);
      int stage = 0, s = 0;
      uint32_t phase = 0;
      for (int64_t u = u0; u < u1; ++s) {
        const int tile = (int)(u / KB);
        const int kb_lo = (int)(u - (int64_t)tile * KB);
        const int64_t end = u1 < (int64_t)(tile + 1) * KB ? u1 : (int64_t)(tile + 1) * KB;
        const int kb_hi = kb_lo + (int)(end - u);
        u = end;
        const int acc = s % ACCS;
        const uint32_t tacc = tmem + acc * C::ACC_COLS;
        bool ok = !s_abort && mbar_wait(acce0 + 8 * acc, ((s / ACCS) & 1) ^ 1);
        fence_after();
        for (int kb = kb_lo; ok && kb < kb_hi; ++kb) {
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
            mma_1cta(tacc, desc_sw128(sa + k * 32, 16, 1024), db, idesc, accum);
            if constexpr (ACT == ACT_SWIGLU)
              mma_1cta(tacc + NB, desc_sw128(sa + C::A_BYTES + k * 32, 16, 1024), db, idesc, accum);
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
        commit_1cta(accf0 + 8 * acc);   // the epilogue sees s_abort if the tile is incomplete
        if (!ok) break;
      }
    }
  } else {
    // epilogue: this warp's 32 weight rows (output features) x NB tokens
    const int quad = warp & 3;
    uint8_t* stg = smem + C::STG_OFF + (warp - 2) * 2 * STG_BYTES;
    int next = 0, s = 0;
    for (int64_t u = u0; u < u1; ++s) {
      const int tile = (int)(u / KB);
      const int kb_lo = (int)(u - (int64_t)tile * KB);
      const int64_t end = u1 < (int64_t)(tile + 1) * KB ? u1 : (int64_t)(tile + 1) * KB;
      const int kb_hi = kb_lo + (int)(end - u);
      u = end;
      const int acc = s % ACCS;
      bool ok = mbar_wait(accf0 + 8 * acc, (s / ACCS) & 1);
      if (!ok) {
        set_err(a.err, 43);
        s_abort = 1;
      }
      fence_after();
      ok = ok && !s_abort;
      const bool whole = kb_lo == 0 && kb_hi == KB;
      const int feat0 = tile * BM + quad * 32;
      const uint32_t tacc = tmem + ((uint32_t)(quad * 32) << 16) + acc * C::ACC_COLS;
      float bias = 0.f;
      if constexpr (ACT == ACT_NONE)
        if (whole && a.bias != nullptr && feat0 + lane < a.N) bias = __bfloat162float(a.bias[feat0 + lane]);
#pragma unroll 1
      for (int c = 0; c < NB / 32; ++c) {
        uint32_t r[32], ru[ACT == ACT_SWIGLU ? 32 : 1];
        tmem_ld32(tacc + c * 32, r);
        if constexpr (ACT == ACT_SWIGLU) tmem_ld32(tacc + NB + c * 32, ru);
        tmem_wait_ld();
        if (!ok || c * 32 >= a.B) continue;
        if (whole) {
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
        } else {
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          float* t0 = reinterpret_cast<float*>(stg);
#pragma unroll
          for (int i = 0; i < 32; ++i) t0[i * 32 + lane] = __uint_as_float(r[i]);
          if constexpr (ACT == ACT_SWIGLU) {
            float* t1 = reinterpret_cast<float*>(stg + STG_BYTES);
#pragma unroll
            for (int i = 0; i < 32; ++i) t1[i * 32 + lane] = __uint_as_float(ru[i]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&tmWS, smem_u32(t0), feat0, c * 32);
            if constexpr (ACT == ACT_SWIGLU) tma_reduce_add_2d(&tmWS, smem_u32(stg + STG_BYTES), a.up_off + feat0, c * 32);
            bulk_commit();
          }
        }
      }
      // the accumulator is free for the tile after next
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * acc);
      if (!whole) {
        // tile shared with other CTAs: the last to arrive finishes it
        if (lane == 0) {
          bulk_wait_all();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          __threadfence();
        }
        __syncwarp();
        epi_bar();
        if (threadIdx.x == 64) {
          int last = 0;
          if (!s_abort) {
            const int parts = owner_of((int64_t)(tile + 1) * KB - 1, U, G) - owner_of((int64_t)tile * KB, U, G) + 1;
            const int old = atomicAdd(&a.tickets[tile], 1);
            last = old == parts - 1;
            if (last) a.tickets[tile] = 0;
          }
          s_last = last;
        }
        epi_bar();
        if (s_last) {
          __threadfence();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          finalize_tile<ACT>(a, tile);
        }
        epi_bar();   // s_last is rewritten for the next shared tile
      }
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
static void skinny_launch(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty, const CUtensorMap& tws,
                          const Args& a) {
  ensure_smem_attr(skinny_kernel<NB, ACT>, Cfg<NB, ACT>::SMEM_BYTES);
  skinny_kernel<NB, ACT><<<a.grid, NTHREADS, Cfg<NB, ACT>::SMEM_BYTES, stream()>>>(tw, tx, ty, tws, a);
  PSRL_CHECK_LAUNCH();
}

template <int ACT>
static void skinny_dispatch(int nb, const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& ty,
                            const CUtensorMap& tws, const Args& a) {
  switch (nb) {
    case 32: skinny_launch<32, ACT>(tw, tx, ty, tws, a); break;
    case 64: skinny_launch<64, ACT>(tw, tx, ty, tws, a); break;
    case 128: skinny_launch<128, ACT>(tw, tx, ty, tws, a); break;
    default: skinny_launch<256, ACT>(tw, tx, ty, tws, a); break;
  }
}

// Decode GEMM, one launch: x [B, K] bf16 (B <= 256), w [R, K] bf16.
//   swiglu = false: y [B, R] = x w^T (+ bias [R]);
//   swiglu = true:  w holds gate rows [0, I) then up rows [I, 2I) (R = 2I,
//                   I % 128 == 0): y [B, I] = silu(x w_gate^T) * (x w_up^T).
// ws: fp32 workspace of at least B * R elements and tickets: int32 of at least
// ceil(R / 128) elements, both all zero on entry and zero again on return
// (after an error report their contents are undefined: zero them).
// grid: CTAs (<= 0: one per SM).
at::Tensor tc_gemm_skinny(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, bool swiglu, at::Tensor ws,
                          at::Tensor tickets, int64_t grid, at::Tensor err) {
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
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.is_contiguous() && ws.numel() >= B * R,
              "ws must be a zeroed contiguous fp32 workspace of at least B * R elements");
  const int64_t tiles = (N + BM - 1) / BM;
  TORCH_CHECK(tickets.scalar_type() == at::kInt && tickets.is_contiguous() && tickets.numel() >= tiles,
              "tickets must be a zeroed int32 tensor of at least ceil(N / 128) elements");
  const int nb = B <= 32 ? 32 : B <= 64 ? 64 : B <= 128 ? 128 : 256;
  Args a{};
  a.B = (int)B;
  a.N = (int)N;
  a.K = (int)K;
  a.up_off = swiglu ? (int)N : 0;
  a.tiles = (int)tiles;
  a.kblocks = (int)((K + BK - 1) / BK);
  const int64_t units = tiles * a.kblocks;
  a.grid = (int)std::min<int64_t>(grid > 0 ? grid : num_sms(), units);
  a.err = err.data_ptr<int>();
  a.ws = ws.data_ptr<float>();
  a.ws_cols = (int)R;
  a.tickets = tickets.data_ptr<int>();
  a.y = reinterpret_cast<bf16*>(y.data_ptr());
  if (bias.has_value()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "bias must be a contiguous bf16 [N]");
    a.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  auto acc = ws.narrow(0, 0, B * R).view({B, R});
  const CUtensorMap tw = skinny_map(w, 64, BM, true), tx = skinny_map(x, 64, (uint32_t)nb, true);
  const CUtensorMap ty = skinny_map(y, 32, 32, false), tws = skinny_map(acc, 32, 32, false);
  if (swiglu) skinny_dispatch<ACT_SWIGLU>(nb, tw, tx, ty, tws, a);
  else skinny_dispatch<ACT_NONE>(nb, tw, tx, ty, tws, a);
  return y;
}

}  // namespace psrl
