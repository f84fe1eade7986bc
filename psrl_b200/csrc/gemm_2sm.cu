// Paired-CTA persistent tcgen05 GEMM for sm_100a (the projection GEMMs of
// training and prefill):  C[M, N] = A[M, K] * B[N, K]^T, bf16 operands, fp32
// accumulation in tensor memory.
//
// A cluster of two CTAs on two SMs computes one 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r of the pair loads
// rows [128 r, 128 r + 128) of the A tile and of the B tile into its own
// shared memory, the even CTA issues the MMAs, and each CTA's tensor memory
// receives its 128 rows of the 256 x 256 accumulator.  Per SM that is 32 KB
// of operand tiles per 64-deep k-block for 2 x 2^21 FLOP, a third less
// shared-memory traffic per FLOP than one CTA on a 128 x 256 tile.
//
// Operand layouts: each operand is K-major (stored [rows, K]: activations,
// nn.Linear weights) or MN-major (stored [K, rows]: the transposed operand of
// the backward GEMMs), so forward (x W^T), data gradient (dy W) and weight
// gradient (dy^T x) are the same kernel with different template flags.
//
// Per CTA: 192 threads.
//   warp 0      TMA producer (both CTAs): a 6-stage ring of A and B halves
//               (128-byte swizzle); completion bytes of both CTAs' copies are
//               counted on the even CTA's "full" barrier.
//   warp 1      MMA issuer (even CTA, one thread): 4 MMAs per k-block into
//               one of two 256-column TMEM accumulators; tcgen05.commit frees
//               the ring slot in both CTAs and, after the last k-block, hands
//               the accumulator to both CTAs' epilogues.
//   warps 2..5  epilogue (both CTAs): tcgen05.ld of its 32-lane quadrant,
//               overlapping the next tile's MMAs, into a swizzled two-buffer
//               staging ring and out with TMA tile stores; then an arrive on
//               the even CTA's "accumulator empty" barrier.
// Epilogues:
//   OUT_BF16    C (bf16) = acc.
//   OUT_F32_ADD C (fp32) += acc with TMA reduce-add tiles: split-K partial
//               sums and accumulation into an existing fp32 buffer.
//   OUT_F32_ADD2 the same tile added into two fp32 buffers, this GPU's and the
//               tensor-parallel peer's (a mapping of its memory over NVLink):
//               a row-parallel GEMM whose all-reduce happens in the epilogue,
//               tile by tile, while later tiles are still being computed.
//   OUT_SWIGLU  gate_up projection: the B half of CTA 0 is gate rows
//               [128 j, 128 j + 128) and that of CTA 1 the matching up rows
//               I + 128 j ..., so every accumulator row holds gate and up side
//               by side; the epilogue writes both (bf16, for the backward) and
//               h = silu(gate) * up.
// Tiles are visited in groups of `group_m` tile rows so that the tiles in
// flight share A and B panels in L2.  Every wait is bounded; on a timeout the
// kernel records an error code, stops issuing work, releases its tensor
// memory and returns.
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"
#include "tcgen05.cuh"

namespace psrl {
namespace g2 {

using namespace tc5;

constexpr int TM = 256, TN = 256;   // cluster tile
constexpr int HM = 128, HN = 128;   // per-CTA halves
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_BYTES = HM * BK * 2;  // 16 KB
constexpr int B_BYTES = HN * BK * 2;  // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
// epilogue staging: per epilogue warp two 4 KB buffers (32 rows x 128 B,
// 128-byte swizzle) that feed TMA stores
constexpr int STG_BYTES = 4096;
constexpr int STG_OFF = STAGES * STAGE_BYTES;
constexpr int BAR_OFF = STG_OFF + 4 * 2 * STG_BYTES;
constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
constexpr int NTHREADS = 192;
constexpr int TMEM_COLS = 512;

enum { OUT_BF16 = 0, OUT_F32_ADD = 1, OUT_SWIGLU = 2, OUT_F32_ADD2 = 3 };

struct Args {
  int M, N, K;
  int tiles_m, tiles_n, kblocks, splits, num_tiles, num_units, group_m;
  int inter;        // OUT_SWIGLU: I (up rows start at I in B; h has I columns)
  const bf16* bias; // OUT_BF16: optional bias [N] added to every row
  int* err;
};

struct Unit {
  int tm, tn, kb_lo, kb_hi;
};

__device__ __forceinline__ Unit decode_unit(const Args& a, int u) {
  Unit w;
  const int s = u / a.num_tiles, t = u - s * a.num_tiles;
  const int span = a.group_m * a.tiles_n;
  const int g = t / span, first = g * a.group_m;
  const int gm = min(a.group_m, a.tiles_m - first);
  const int l = t - g * span;
  w.tm = first + l % gm;
  w.tn = l / gm;
  w.kb_lo = (int)((int64_t)s * a.kblocks / a.splits);
  w.kb_hi = (int)((int64_t)(s + 1) * a.kblocks / a.splits);
  return w;
}

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

// Row `r` of a 32-row staging tile in the TMA 128-byte swizzle: 16-byte chunk
// c of the row lives at chunk c ^ (r % 8).
__device__ __forceinline__ void stage_row_bf16(uint8_t* buf, int r, const float* v /* 64 */) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) *reinterpret_cast<bf16x8*>(row + ((c ^ (r & 7)) << 4)) = pack8(v + 8 * c);
}
__device__ __forceinline__ void stage_row_f32(uint8_t* buf, int r, const uint32_t* v /* 32 */) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// One warp's TMA-store pipeline: two staging buffers used in turn.
struct StoreRing {
  uint8_t* base;  // 2 x STG_BYTES, 1024-byte aligned
  int next;
  // wait until the buffer about to be filled is no longer read by an older store
  __device__ __forceinline__ uint8_t* acquire(int lane) {
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    return base + next * STG_BYTES;
  }
  __device__ __forceinline__ void store(int lane, const CUtensorMap* map, int x, int y, bool reduce_add) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      const uint32_t src = smem_u32(base + next * STG_BYTES);
      if (reduce_add) tma_reduce_add_2d(map, src, x, y);
      else tma_store_2d(map, src, x, y);
      bulk_commit();
    }
    next ^= 1;
  }
  // the same staged tile added into two tensors (this GPU's and a peer's)
  __device__ __forceinline__ void reduce2(int lane, const CUtensorMap* m0, const CUtensorMap* m1, int x, int y) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      const uint32_t src = smem_u32(base + next * STG_BYTES);
      tma_reduce_add_2d(m0, src, x, y);
      tma_reduce_add_2d(m1, src, x, y);
      bulk_commit();
    }
    next ^= 1;
  }
};

template <int OUT, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH, Args args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2]; then the TMEM slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * STAGES;
  const uint32_t accf0 = empty0 + 8 * STAGES, acce0 = accf0 + 16;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 8);  // 4 epilogue warps in each of the two CTAs
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc_2cta(smem_u32(tmem_slot), TMEM_COLS);
  fence_before();
  cluster_sync();  // both CTAs' barriers initialised and the pair's TMEM allocated
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      const uint32_t full_lead0 = mapa(full0, 0);
      int stage = 0;
      uint32_t phase = 0;
      for (int u = cid; u < args.num_units && !s_abort; u += ncl) {
        const Unit w = decode_unit(args, u);
        const int a_row = w.tm * TM + (int)rank * HM;
        int b_row;
        if constexpr (OUT == OUT_SWIGLU) b_row = (rank == 0 ? 0 : args.inter) + w.tn * HN;
        else b_row = w.tn * TN + (int)rank * HN;
        for (int kb = w.kb_lo; kb < w.kb_hi; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1)) {
            set_err(args.err, 1);
            s_abort = 1;
            break;
          }
          if (rank == 0) mbar_expect_tx(full0 + 8 * stage, 2 * STAGE_BYTES);
          const uint32_t fb = full_lead0 + 8 * stage;
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d_pair(sa, &tmA, kb * BK, a_row, fb);
          } else {
            tma_load_2d_pair(sa, &tmA, a_row, kb * BK, fb);
            tma_load_2d_pair(sa + A_BYTES / 2, &tmA, a_row + 64, kb * BK, fb);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(sb, &tmB, kb * BK, b_row, fb);
          } else {
            tma_load_2d_pair(sb, &tmB, b_row, kb * BK, fb);
            tma_load_2d_pair(sb + B_BYTES / 2, &tmB, b_row + 64, kb * BK, fb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      constexpr uint32_t idesc = idesc_bf16_f32(TM, TN, A_MN, B_MN);
      for (int u = cid; u < args.num_units && !s_abort; u += ncl) {
        const Unit w = decode_unit(args, u);
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1)) {
          set_err(args.err, 2);
          s_abort = 1;
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + acc * TN;
        bool ok = true;
        for (int kb = w.kb_lo; kb < w.kb_hi; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase)) {
            set_err(args.err, 3);
            s_abort = 1;
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = A_MN ? desc_sw128(sa + k * 2048, A_BYTES / 2, 1024) : desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t db = B_MN ? desc_sw128(sb + k * 2048, B_BYTES / 2, 1024) : desc_sw128(sb + k * 32, 16, 1024);
            mma_2cta(d_tmem, da, db, idesc, (kb > w.kb_lo || k > 0) ? 1u : 0u);
          }
          commit_2cta_mask(empty0 + 8 * stage, 0x3);  // ring slot free in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        commit_2cta_mask(accf0 + 8 * acc, 0x3);  // accumulator ready in both CTAs
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    // TMEM -> registers -> swizzled staging -> TMA store (or TMA reduce-add):
    // every global write is a whole 32-row box, out-of-range rows and
    // columns are clipped by the tensor map.
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t acce_lead0 = mapa(acce0, 0);
    if (lane == 0) tma_prefetch_desc(&tmC);
    StoreRing ring{smem + STG_OFF + (warp - 2) * 2 * STG_BYTES, 0};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = cid; u < args.num_units; u += ncl) {
      if (!mbar_wait(accf0 + 8 * acc, acc_phase)) {
        set_err(args.err, 4);
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      fence_after();
      const Unit w = decode_unit(args, u);
      const int row0 = w.tm * TM + (int)rank * HM + quad * 32;  // this warp's 32 output rows
      const uint32_t taddr = tmem_base + acc * TN + ((uint32_t)(quad * 32) << 16);
      if constexpr (OUT == OUT_SWIGLU) {
#pragma unroll 1
        for (int c = 0; c < HN / 64; ++c) {
          uint32_t r[128];
          tmem_ld32(taddr + c * 64, r);
          tmem_ld32(taddr + c * 64 + 32, r + 32);
          tmem_ld32(taddr + HN + c * 64, r + 64);
          tmem_ld32(taddr + HN + c * 64 + 32, r + 96);
          tmem_wait_ld();
          float g[64], up[64];
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            g[j] = __uint_as_float(r[j]);
            up[j] = __uint_as_float(r[64 + j]);
          }
          const int col = w.tn * HN + c * 64;
          stage_row_bf16(ring.acquire(lane), lane, g);
          ring.store(lane, &tmC, col, row0, false);
          stage_row_bf16(ring.acquire(lane), lane, up);
          ring.store(lane, &tmC, args.inter + col, row0, false);
#pragma unroll
          for (int j = 0; j < 64; ++j) g[j] = silu(g[j]) * up[j];
          stage_row_bf16(ring.acquire(lane), lane, g);
          ring.store(lane, &tmH, col, row0, false);
        }
      } else if constexpr (OUT == OUT_BF16) {
#pragma unroll 1
        for (int c = 0; c < TN / 64; ++c) {
          const int cb = w.tn * TN + c * 64;
          if (cb >= args.N) break;
          uint32_t r[64];
          tmem_ld32(taddr + c * 64, r);
          tmem_ld32(taddr + c * 64 + 32, r + 32);
          tmem_wait_ld();
          float v[64];
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j]);
          if (args.bias != nullptr) {
            if (cb + 64 <= args.N) {
#pragma unroll
              for (int j = 0; j < 64; j += 8) {
                float bv[8];
                unpack8(*reinterpret_cast<const bf16x8*>(args.bias + cb + j), bv);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[j + i] += bv[i];
              }
            } else {
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (cb + j < args.N) v[j] += __bfloat162float(args.bias[cb + j]);
            }
          }
          stage_row_bf16(ring.acquire(lane), lane, v);
          ring.store(lane, &tmC, cb, row0, false);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < TN / 32; ++c) {
          const int cb = w.tn * TN + c * 32;
          if (cb >= args.N) break;
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_wait_ld();
          stage_row_f32(ring.acquire(lane), lane, r);
          if constexpr (OUT == OUT_F32_ADD2) ring.reduce2(lane, &tmC, &tmH, cb, row0);
          else ring.store(lane, &tmC, cb, row0, true);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_lead0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  if (warp >= 2 && lane == 0) bulk_wait_all();  // this warp's stores have landed
  fence_before();
  __syncwarp();
  cluster_sync();  // no MMA, commit or copy of the pair is still outstanding
  if (warp == 0) {
    fence_after();
    tmem_free_2cta(tmem_base, TMEM_COLS);
  }
}

}  // namespace g2

using namespace g2;

// Tensor map over a row-major bf16 matrix [rows, cols] (unit inner stride),
// box {64 columns, box_rows rows}, 128-byte swizzle, zero fill out of bounds.
static CUtensorMap make_map_2d(const at::Tensor& t, uint32_t box_rows) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "operand must be 2-D with unit inner stride");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "operand rows must start on 16-byte boundaries");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * 2};
  cuuint32_t box[2] = {64u, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = PSRL_DRV(cuTensorMapEncodeTiled)(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides,
                                                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

// Tensor map for the epilogue's TMA stores into a row-major [rows, cols]
// matrix (bf16: boxes of 64 x 32, fp32: 32 x 32; 128 B per box row, 128-byte
// swizzle matching the staging layout).
static CUtensorMap make_store_map(const at::Tensor& t) {
  const bool f32 = t.scalar_type() == at::kFloat;
  const int esz = f32 ? 4 : 2;
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "output must be 2-D with unit inner stride");
  TORCH_CHECK((t.stride(0) * esz) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "output rows must start on 16-byte boundaries");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * esz};
  cuuint32_t box[2] = {f32 ? 32u : 64u, 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = PSRL_DRV(cuTensorMapEncodeTiled)(
      &m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides,
      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store) failed (", (int)r, ")");
  return m;
}

// Clusters of two that can be resident at once (one CTA per SM), per device.
static int max_pairs() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  PSRL_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = num_sms() / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * n);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm2_kernel<OUT_BF16, false, false>, &cfg) == cudaSuccess &&
      clusters > 0)
    n = std::min(n, clusters);
  (void)cudaGetLastError();
  if (dev < 64) cache[dev] = n;
  return n;
}

template <int OUT, bool A_MN, bool B_MN>
static void launch2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& th,
                    const Args& args) {
  ensure_smem_attr(gemm2_kernel<OUT, A_MN, B_MN>, SMEM_BYTES);
  const int pairs = std::max(1, std::min(args.num_units, max_pairs()));
  gemm2_kernel<OUT, A_MN, B_MN><<<2 * pairs, NTHREADS, SMEM_BYTES, stream()>>>(ta, tb, tc, th, args);
  PSRL_CHECK_LAUNCH();
}

template <int OUT>
static void dispatch2(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                      const Args& args) {
  if (!a_mn && !b_mn) launch2<OUT, false, false>(ta, tb, tc, tc, args);
  else if (!a_mn && b_mn) launch2<OUT, false, true>(ta, tb, tc, tc, args);
  else if (a_mn && !b_mn) launch2<OUT, true, false>(ta, tb, tc, tc, args);
  else launch2<OUT, true, true>(ta, tb, tc, tc, args);
}

// C = A B^T with A logically [M, K] and B logically [N, K].
//  a_mn = false: `a` is stored [M, K];  a_mn = true: `a` is stored [K, M].
//  b_mn = false: `b` is stored [N, K];  b_mn = true: `b` is stored [K, N].
// Without `out`: returns a new bf16 [M, N] (splits must be 1).  With `out`
// (fp32 [M, N], unit inner stride): C is added into it, K split `splits` ways.
// `bias` (bf16 [N], bf16 output only) is added to every row.
// `err` (int32 [1], zero) receives a nonzero code if a bounded wait expired.
at::Tensor tc_gemm2(at::Tensor a, at::Tensor b, bool a_mn, bool b_mn, c10::optional<at::Tensor> out, int64_t splits,
                    int64_t group_m, c10::optional<at::Tensor> bias, at::Tensor err) {
  CHECK_CUDA_TENSOR(a);
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(b, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "operands must be 2-D");
  const int64_t M = a_mn ? a.size(1) : a.size(0), K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0), Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "K mismatch (", K, " vs ", Kb, ")");
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "dimension too large");
  at::cuda::CUDAGuard g(a.device());
  Args args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + TM - 1) / TM);
  args.tiles_n = (int)((N + TN - 1) / TN);
  args.kblocks = (int)((K + BK - 1) / BK);
  args.num_tiles = args.tiles_m * args.tiles_n;
  args.group_m = (int)std::max<int64_t>(1, group_m);
  args.err = err.data_ptr<int>();
  at::Tensor c;
  if (out.has_value()) {
    c = *out;
    CHECK_DTYPE(c, at::kFloat);
    TORCH_CHECK(c.dim() == 2 && c.size(0) == M && c.size(1) == N, "out must be fp32 [M, N]");
    args.splits = (int)std::max<int64_t>(1, std::min<int64_t>(splits, args.kblocks));
  } else {
    TORCH_CHECK(splits <= 1, "split-K needs an fp32 output to accumulate into");
    TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
    c = at::empty({M, N}, a.options());
    args.splits = 1;
  }
  if (bias.has_value()) {
    TORCH_CHECK(!out.has_value(), "bias is added only with a bf16 output");
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous() &&
                    reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
                "bias must be a contiguous, 16-byte aligned bf16 [N]");
    args.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  if (M == 0 || N == 0) return c;
  TORCH_CHECK(K > 0, "K must be positive");
  args.num_units = args.num_tiles * args.splits;
  const CUtensorMap ta = make_map_2d(a, a_mn ? 64 : HM), tb = make_map_2d(b, b_mn ? 64 : HN);
  const CUtensorMap tc = make_store_map(c);
  if (out.has_value()) dispatch2<OUT_F32_ADD>(a_mn, b_mn, ta, tb, tc, args);
  else dispatch2<OUT_BF16>(a_mn, b_mn, ta, tb, tc, args);
  return c;
}

// Tensor-parallel row-parallel GEMM with the all-reduce in the epilogue (two
// ranks): every output tile of A B^T is added, with TMA reduce-add, into
// `acc_local` (this GPU) and `acc_peer` (the peer's accumulator, mapped into
// this process over NVLink).  Both accumulators are fp32 [M, N] and zero on
// entry on both ranks; once both ranks' kernels have finished (the caller's
// cross-GPU barrier) each holds the full sum.  The two fp32 additions into a
// zero commute exactly, so both ranks hold bit-identical sums.
void tc_gemm2_allreduce2(at::Tensor a, at::Tensor b, bool b_mn, at::Tensor acc_local, at::Tensor acc_peer,
                         int64_t group_m, at::Tensor err) {
  CHECK_CUDA_TENSOR(a);
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(b, at::kBFloat16);
  CHECK_DTYPE(acc_local, at::kFloat);
  CHECK_DTYPE(acc_peer, at::kFloat);
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0), Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "K mismatch");
  TORCH_CHECK(acc_local.dim() == 2 && acc_local.size(0) == M && acc_local.size(1) == N &&
                  acc_peer.dim() == 2 && acc_peer.size(0) == M && acc_peer.size(1) == N,
              "accumulators must be fp32 [M, N]");
  at::cuda::CUDAGuard g(a.device());
  if (M == 0 || N == 0) return;
  Args args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles_m = (int)((M + TM - 1) / TM);
  args.tiles_n = (int)((N + TN - 1) / TN);
  args.kblocks = (int)((K + BK - 1) / BK);
  args.splits = 1;
  args.num_tiles = args.tiles_m * args.tiles_n;
  args.num_units = args.num_tiles;
  args.group_m = (int)std::max<int64_t>(1, group_m);
  args.err = err.data_ptr<int>();
  const CUtensorMap ta = make_map_2d(a, HM), tb = make_map_2d(b, b_mn ? 64 : HN);
  const CUtensorMap tl = make_store_map(acc_local), tp = make_store_map(acc_peer);
  if (b_mn) launch2<OUT_F32_ADD2, false, true>(ta, tb, tl, tp, args);
  else launch2<OUT_F32_ADD2, false, false>(ta, tb, tl, tp, args);
}

// Fused gate_up projection + SwiGLU: x [M, K] (bf16), w [2 I, K] (gate rows
// then up rows).  Returns {gate_up [M, 2 I], h = silu(gate) * up [M, I]}.
std::vector<at::Tensor> tc_gemm2_swiglu(at::Tensor x, at::Tensor w, int64_t group_m, at::Tensor err) {
  CHECK_CUDA_TENSOR(x);
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "x [M, K] and w [2I, K]");
  const int64_t M = x.size(0), K = x.size(1), I = w.size(0) / 2;
  TORCH_CHECK(w.size(0) == 2 * I && I % HN == 0, "intermediate size must be a multiple of 128");
  at::cuda::CUDAGuard g(x.device());
  auto gu = at::empty({M, 2 * I}, x.options());
  auto h = at::empty({M, I}, x.options());
  if (M == 0) return {gu, h};
  Args args{};
  args.M = (int)M;
  args.N = (int)(2 * I);
  args.K = (int)K;
  args.tiles_m = (int)((M + TM - 1) / TM);
  args.tiles_n = (int)(I / HN);
  args.kblocks = (int)((K + BK - 1) / BK);
  args.splits = 1;
  args.num_tiles = args.tiles_m * args.tiles_n;
  args.num_units = args.num_tiles;
  args.group_m = (int)std::max<int64_t>(1, group_m);
  args.inter = (int)I;
  args.err = err.data_ptr<int>();
  const CUtensorMap ta = make_map_2d(x, HM), tb = make_map_2d(w, HN);
  const CUtensorMap tgu = make_store_map(gu), th = make_store_map(h);
  launch2<OUT_SWIGLU, false, false>(ta, tb, tgu, th, args);
  return {gu, h};
}

}  // namespace psrl
