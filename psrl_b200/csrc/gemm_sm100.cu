// Persistent tcgen05 / TMEM GEMM for sm_100a:  C[M, N] = A[M, K] * B[N, K]^T
// (A and B bf16, both K-major, i.e. row-major activations times an nn.Linear
// weight), fp32 accumulation in tensor memory.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 A tile + 256x64 B tile per k-block into a
//               4-stage shared-memory ring (128-byte swizzle), completion via
//               mbarrier transaction counts.
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128,
//               N=256, K=16, kind::f16) into one of two TMEM accumulators
//               (2 x 256 fp32 columns = the whole 512-column TMEM) and signals
//               ring slots / finished accumulators with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld 32x32b rows out of TMEM (warp w owns TMEM
//               lane quadrant w % 4), overlapping the next tile's MMAs.
// Epilogues:
//   EPI_STORE   bf16 store of C (bounds-masked).
//   EPI_LSE     fused LM-head statistics: per row and 256-column tile the
//               running max / sum exp / sum exp*z of z = acc / T plus the
//               label's logit; a second tiny kernel merges the tiles into
//               log p(label), entropy and log-sum-exp — the [M, V] logits are
//               never written to memory.
// Every mbarrier wait is bounded; on timeout the kernel records an error code,
// skips the remaining work, frees its TMEM and returns.
// TMA loads here are plain (no cluster multicast): A/B are local tensors.
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"

namespace psrl {
namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;     // 16 KB
constexpr int B_BYTES = BN * BK * 2;     // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int NTHREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr uint64_t WAIT_NS = 2000000000ull;  // bound of every barrier wait (global timer ns)

enum { EPI_STORE = 0, EPI_LSE = 1 };

struct Args {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  // EPI_STORE
  bf16* C;
  int64_t ldc;
  // EPI_LSE
  const int64_t* labels;
  float inv_temp;
  float* part;        // [M, tiles_n, 3]
  float* label_logit; // [M]
  int* err;           // error flag (0 = ok)
  // grouped mode (MoE experts): A rows are expert-sorted segments seg[e]..seg[e+1],
  // B is [E * N, K] (expert e's weight rows e*N..e*N+N-1), tiles are numbered
  // expert-major from tile_off (device arrays, so the launch needs no host sync)
  int grouped;
  int E;
  const int* seg;      // [E + 1]
  const int* tile_off; // [E + 1]
};

struct TileCoord {
  int a_row, b_row, col0, row_lo, row_hi;
};

__device__ __forceinline__ int total_tiles(const Args& a) { return a.grouped ? a.tile_off[a.E] : a.num_tiles; }

__device__ __forceinline__ TileCoord tile_coord(const Args& a, int tile) {
  TileCoord c;
  if (!a.grouped) {
    const int tm = tile % a.tiles_m, tn = tile / a.tiles_m;
    c.a_row = tm * BM;
    c.b_row = tn * BN;
    c.col0 = tn * BN;
    c.row_lo = tm * BM;
    c.row_hi = a.M;
    return c;
  }
  // expert e with tile_off[e] <= tile < tile_off[e + 1] (empty experts have no tiles)
  int lo = 0, hi = a.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (a.tile_off[mid] <= tile) lo = mid;
    else hi = mid;
  }
  const int e = lo;
  const int s0 = a.seg[e], s1 = a.seg[e + 1];
  const int tms = (s1 - s0 + BM - 1) / BM;
  const int local = tile - a.tile_off[e];
  const int tm = local % tms, tn = local / tms;
  c.a_row = s0 + tm * BM;
  c.b_row = e * a.N + tn * BN;
  c.col0 = tn * BN;
  c.row_lo = s0 + tm * BM;
  c.row_hi = s1;
  return c;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}
// Bounded wait for the phase with the given parity (at most WAIT_NS); false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 63) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0) t0 = t;
      else if (t - t0 > WAIT_NS) return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// UMMA shared-memory descriptor, K-major operand with 128-byte swizzle:
// start address >> 4 in bits [0,14), leading byte offset (16 B units) = 1 in
// bits [16,30), stride byte offset = 1024 B (8 rows x 128 B) >> 4 in bits
// [32,46), descriptor version 1 in bits [46,48), layout SWIZZLE_128B (2) in
// bits [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor (kind::f16): fp32 accumulator (bits 4-5 = 1), A/B
// bf16 (bits 7-9 / 10-12 = 1), both K-major, N >> 3 in bits 17-22, M >> 4 in
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

template <int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Args args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2]; then tmem slot
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_addr(bars), empty0 = full0 + 8 * STAGES;
  const uint32_t accf0 = empty0 + 8 * STAGES, acce0 = accf0 + 16;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int KB = args.K / BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const int ntiles = total_tiles(args);
      for (int tile = blockIdx.x; tile < ntiles && !s_abort; tile += gridDim.x) {
        const TileCoord tc = tile_coord(args, tile);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1)) {
            set_err(args.err, 1);
            s_abort = 1;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          mbar_expect_tx(fb, STAGE_BYTES);
          const uint32_t sa = smem_addr(smem + stage * STAGE_BYTES);
          tma_load_2d(sa, &tmA, kb * BK, tc.a_row, fb);
          tma_load_2d(sa + A_BYTES, &tmB, kb * BK, tc.b_row, fb);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint32_t idesc = idesc_bf16(BM, BN);
      const int ntiles = total_tiles(args);
      for (int tile = blockIdx.x; tile < ntiles && !s_abort; tile += gridDim.x) {
        if (!mbar_wait(acce0 + 8 * acc, acc_phase ^ 1)) {
          set_err(args.err, 2);
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(full0 + 8 * stage, phase)) {
            set_err(args.err, 3);
            s_abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + stage * STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma(d_tmem, sw128_desc(sa + k * 32), sw128_desc(sa + A_BYTES + k * 32), idesc,
                 (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty0 + 8 * stage);   // slot free once these MMAs complete
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * acc);        // accumulator ready
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quad = warp & 3;                // TMEM lane quadrant of this warp
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int ntiles = total_tiles(args);
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      if (!mbar_wait(accf0 + 8 * acc, acc_phase)) {
        set_err(args.err, 4);
        s_abort = 1;
        break;
      }
      if (s_abort) break;
      tc_fence_after();
      const TileCoord tc = tile_coord(args, tile);
      const int tn = tc.col0 / BN;
      const int row = tc.row_lo + row_in_tile;
      const int row_end = tc.row_hi;
      const int col0 = tc.col0;
      const uint32_t taddr = tmem_base + acc * BN + ((uint32_t)(quad * 32) << 16);
      if constexpr (EPI == EPI_STORE) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          const int cb = col0 + c * 32;
          if (row < row_end) {
            bf16* dst = args.C + (int64_t)row * args.ldc + cb;
            if (cb + 32 <= args.N) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                bf16x8 p = pack8(v + j);
                *reinterpret_cast<bf16x8*>(dst + j) = p;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (cb + j < args.N) dst[j] = __float2bfloat16(v[j]);
            }
          }
        }
      } else {
        // online (max, sum exp, sum exp*z) over this tile's columns of the row
        float m = -INFINITY, s = 0.f, t = 0.f;
        const int64_t lab = row < row_end ? args.labels[row] : -1;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          const int cb = col0 + c * 32;
          float cm = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = (cb + j < args.N) ? v[j] * args.inv_temp : -INFINITY;
            cm = fmaxf(cm, v[j]);
          }
          if (lab >= cb && lab < cb + 32 && row < row_end) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cb + j == lab) args.label_logit[row] = v[j];
          }
          if (cm == -INFINITY) continue;
          const float nm = fmaxf(m, cm);
          const float sc = (m == -INFINITY) ? 0.f : __expf(m - nm);
          s *= sc;
          t *= sc;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (v[j] != -INFINITY) {
              const float e = __expf(v[j] - nm);
              s += e;
              t += e * v[j];
            }
          }
          m = nm;
        }
        if (row < row_end) {
          float* p = args.part + ((int64_t)row * args.tiles_n + tn) * 3;
          p[0] = m;
          p[1] = s;
          p[2] = t;
        }
      }
      tc_fence_before();
      mbar_arrive(acce0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// merge per-tile (max, sumexp, sum exp*z) into lse, entropy, log p(label)
__global__ void lse_combine_kernel(const float* __restrict__ part, const float* __restrict__ label_logit,
                                   const int64_t* __restrict__ labels, int M, int tiles_n, int V,
                                   float* __restrict__ lp, float* __restrict__ ent, float* __restrict__ lse_out) {
  const int row = blockIdx.x * blockDim.y + threadIdx.y;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f, t = 0.f;
  for (int i = threadIdx.x; i < tiles_n; i += 32) {
    const float* p = part + ((int64_t)row * tiles_n + i) * 3;
    float pm = p[0], ps = p[1], pt = p[2];
    if (pm == -INFINITY) continue;
    const float nm = fmaxf(m, pm);
    const float a = (m == -INFINITY) ? 0.f : __expf(m - nm), b = __expf(pm - nm);
    s = s * a + ps * b;
    t = t * a + pt * b;
    m = nm;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o), os = __shfl_xor_sync(0xffffffffu, s, o),
          ot = __shfl_xor_sync(0xffffffffu, t, o);
    if (om == -INFINITY) continue;
    const float nm = fmaxf(m, om);
    const float a = (m == -INFINITY) ? 0.f : __expf(m - nm), b = __expf(om - nm);
    s = s * a + os * b;
    t = t * a + ot * b;
    m = nm;
  }
  if (threadIdx.x == 0) {
    const float lse = m + __logf(s);
    lse_out[row] = lse;
    ent[row] = lse - t / s;
    const int64_t lab = labels[row];
    lp[row] = (lab >= 0 && lab < V) ? label_logit[row] - lse : 0.f;
  }
}

}  // namespace tc

using namespace tc;

static CUtensorMap make_tmap(const at::Tensor& t, uint32_t box_rows) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "operand must be 2-D with unit inner stride");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "operand rows must be 16-byte aligned");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = PSRL_DRV(cuTensorMapEncodeTiled)(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

template <int EPI>
static void launch(const at::Tensor& a, const at::Tensor& b, Args& args) {
  ensure_smem_attr(tc_gemm_kernel<EPI>, SMEM_BYTES);
  CUtensorMap ta = make_tmap(a, BM), tb = make_tmap(b, BN);
  // grouped: the tile count lives on the device; one persistent CTA per SM
  const int grid = args.grouped ? num_sms() : std::min(args.num_tiles, num_sms());
  tc_gemm_kernel<EPI><<<grid, NTHREADS, SMEM_BYTES, stream()>>>(ta, tb, args);
  PSRL_CHECK_LAUNCH();
}

static Args make_args(const at::Tensor& a, const at::Tensor& b) {
  CHECK_CUDA_TENSOR(a);
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(b, at::kBFloat16);
  TORCH_CHECK(a.size(1) == b.size(1), "K mismatch");
  TORCH_CHECK(a.size(1) % BK == 0, "K must be a multiple of 64");
  Args args{};
  args.M = a.size(0);
  args.N = b.size(0);
  args.K = a.size(1);
  args.tiles_m = (args.M + BM - 1) / BM;
  args.tiles_n = (args.N + BN - 1) / BN;
  args.num_tiles = args.tiles_m * args.tiles_n;
  return args;
}

// C = A @ B^T (bf16 out). `err` (int32 [1], zeroed by the caller) receives a nonzero code on timeout.
at::Tensor tc_gemm(at::Tensor a, at::Tensor b, at::Tensor err) {
  Args args = make_args(a, b);
  at::cuda::CUDAGuard g(a.device());
  auto c = at::empty({args.M, args.N}, a.options());
  if (args.M == 0 || args.N == 0) return c;
  TORCH_CHECK(args.N % 8 == 0, "N must be a multiple of 8");
  args.C = reinterpret_cast<bf16*>(c.data_ptr());
  args.ldc = args.N;
  args.err = err.data_ptr<int>();
  launch<EPI_STORE>(a, b, args);
  return c;
}

// tile_off[e + 1] = sum over experts <= e of ceil(rows_e / BM) * tiles_n (one CTA, E <= 1024)
__global__ void grouped_tile_offsets_kernel(const int* __restrict__ seg, int E, int tiles_n, int* __restrict__ tile_off) {
  __shared__ int st[1024];
  const int e = threadIdx.x;
  st[e] = e < E ? (seg[e + 1] - seg[e] + BM - 1) / BM * tiles_n : 0;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int v = e >= o ? st[e - o] : 0;
    __syncthreads();
    st[e] += v;
    __syncthreads();
  }
  if (e < E) tile_off[e + 1] = st[e];
  if (e == 0) tile_off[0] = 0;
}

// Grouped GEMM for expert MLPs: C[r, :] = A[r, :] @ W[e]^T for the rows r of
// expert e's segment seg[e]..seg[e+1] (A rows sorted by expert).  A: bf16
// [R, K]; W: bf16 [E, N, K]; seg: int32 [E + 1] on the device.  No host sync:
// the tile schedule is derived on the device from seg.
at::Tensor tc_grouped_gemm(at::Tensor a, at::Tensor w, at::Tensor seg, at::Tensor err) {
  CHECK_CUDA_TENSOR(a);
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(w, at::kBFloat16);
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous(), "w must be contiguous [E, N, K]");
  TORCH_CHECK(seg.scalar_type() == at::kInt && seg.numel() == w.size(0) + 1, "seg must be int32 [E + 1]");
  const int E = w.size(0), N = w.size(1), K = w.size(2);
  TORCH_CHECK(a.size(1) == K && K % BK == 0, "K must match and be a multiple of 64");
  TORCH_CHECK(N % 8 == 0 && E <= 1024, "N % 8 == 0 and E <= 1024");
  at::cuda::CUDAGuard g(a.device());
  auto c = at::empty({a.size(0), N}, a.options());
  if (a.size(0) == 0) return c;
  Args args{};
  args.M = a.size(0);
  args.N = N;
  args.K = K;
  args.tiles_n = (N + BN - 1) / BN;
  args.grouped = 1;
  args.E = E;
  auto tile_off = at::empty({E + 1}, seg.options());
  grouped_tile_offsets_kernel<<<1, 1024, 0, stream()>>>(seg.data_ptr<int>(), E, args.tiles_n, tile_off.data_ptr<int>());
  PSRL_CHECK_LAUNCH();
  args.seg = seg.data_ptr<int>();
  args.tile_off = tile_off.data_ptr<int>();
  args.C = reinterpret_cast<bf16*>(c.data_ptr());
  args.ldc = N;
  args.err = err.data_ptr<int>();
  launch<EPI_STORE>(a, w.view({(int64_t)E * N, K}), args);
  return c;
}

// Fused LM-head log-prob: returns {logprob, entropy, lse} (fp32 [M]) without
// materialising the logits.
std::vector<at::Tensor> tc_linear_logprob(at::Tensor h, at::Tensor w, at::Tensor labels, double temperature,
                                          at::Tensor err) {
  Args args = make_args(h, w);
  at::cuda::CUDAGuard g(h.device());
  CHECK_DTYPE(labels, at::kLong);
  auto opts = h.options().dtype(at::kFloat);
  auto lp = at::empty({args.M}, opts), ent = at::empty({args.M}, opts), lse = at::empty({args.M}, opts);
  if (args.M == 0) return {lp, ent, lse};
  auto part = at::empty({args.M, args.tiles_n, 3}, opts);
  auto lab_logit = at::zeros({args.M}, opts);
  args.labels = labels.data_ptr<int64_t>();
  args.inv_temp = (float)(1.0 / temperature);
  args.part = part.data_ptr<float>();
  args.label_logit = lab_logit.data_ptr<float>();
  args.err = err.data_ptr<int>();
  launch<EPI_LSE>(h, w, args);
  dim3 blk(32, 8);
  lse_combine_kernel<<<(args.M + 7) / 8, blk, 0, stream()>>>(part.data_ptr<float>(), lab_logit.data_ptr<float>(),
                                                             args.labels, args.M, args.tiles_n, args.N,
                                                             lp.data_ptr<float>(), ent.data_ptr<float>(),
                                                             lse.data_ptr<float>());
  PSRL_CHECK_LAUNCH();
  return {lp, ent, lse};
}

}  // namespace psrl
