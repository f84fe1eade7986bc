// Causal varlen attention forward for sm_100a on the 5th-generation tensor
// cores (head_dim 128, bf16 in, fp32 softmax and accumulation).
//
// One CTA per (query head, sequence, 256-row query block).  The block is two
// 128-row query tiles A and B that share every K/V tile, so each K/V byte
// loaded by TMA serves two MMAs, and the tensor core alternates between the
// tiles while the softmax of the other one runs ("ping-pong"):
//
//   TMEM (512 columns): S_A | S_B | O_A | O_B, 128 fp32 columns each; P (bf16
//   probabilities, two per 32-bit column) overwrites the first 64 columns of
//   its S once S has been read.
//
//   warp 0      TMA producer: Q_A, Q_B once, then K_j and V_j per 128-key tile
//               into a 2-stage ring (128-byte swizzle).
//   warp 1      MMA issuer (one thread): S_g = Q_g K_j^T (both operands from
//               shared memory), O_g += P_g V_j (P from tensor memory, V read
//               MN-major from shared memory); tcgen05.commit signals S ready,
//               the K/V slot free, and O final.
//   warps 2..5  softmax of tile A, warps 6..9 of tile B: one thread per row,
//               online softmax in base 2 with lazy rescaling (O in TMEM is
//               rescaled only when the running maximum grows by more than 2^8),
//               P written back to TMEM with tcgen05.st; at the end O / l and the
//               row's log-sum-exp.
//
// Queries and keys may come from different tensors with their own row
// offsets (cu_q / cu_k): sequence b's queries are the LAST Lq of its Lk key
// positions (Lk >= Lq; self-attention has Lk = Lq), so query row p sees keys
// 0 .. p + Lk - Lq.  Context-parallel attention uses this for a rank's query
// chunks against the gathered keys of the sequence prefix.
//
// Work per block: tile A needs the key tiles up to its last row's limit,
// tile B one more or two; only tiles that cross a row's limit are masked.  Blocks are launched
// largest first.  Every wait is bounded; on timeout the kernel records an
// error code and leaves.  TMA loads are plain per-CTA copies.
#include <cuda.h>

#include "driver_api.h"

#include "common.cuh"
#include "tcgen05.cuh"

namespace psrl {
namespace fa5 {

using namespace tc5;

constexpr int D = 128;
constexpr int BQ = 128, BKV = 128;
constexpr int NS = 2;                    // K/V ring depth
constexpr int ATOM = 128 * 64 * 2;       // 128 rows x 64 bf16 (one 128-byte swizzle atom column)
constexpr int Q_BYTES = 2 * ATOM;        // 32 KB
constexpr int KV_TILE = 2 * ATOM;        // 32 KB
constexpr int STAGE = 2 * KV_TILE;       // K + V
constexpr int OFF_KV = 2 * Q_BYTES;
constexpr int OFF_BAR = OFF_KV + NS * STAGE;  // 192 KB
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr int NTHREADS = 320;
constexpr float RESCALE_LOG2 = 8.0f;

struct FwdArgs {
  const int* cu;     // [B + 1] query rows
  const int* cu_k;   // [B + 1] key / value rows
  int q_col, k_col, v_col;  // column of head 0 in the query / key / value tensors
  int nq, nkv, T;
  int blocks_z;      // grid.z = max 256-row blocks per sequence
  float scale_log2;  // softmax scale * log2(e)
  bf16* o;           // [T, nq * D]
  int64_t o_row;
  float* lse;        // [nq, T] natural log, or null
  int* err;
};

// First failure of the launch: code, then (block x, y, z, warp, iteration) in err[1..5].
__device__ __forceinline__ void set_err(int* err, int code, int it = -1) {
  if (err && atomicCAS(err, 0, code) == 0) {
    err[1] = blockIdx.x;
    err[2] = blockIdx.y;
    err[3] = blockIdx.z;
    err[4] = threadIdx.x >> 5;
    err[5] = it;
  }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV, FwdArgs a) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int blk = a.blocks_z - 1 - (int)blockIdx.z;  // largest blocks first
  const int s0 = a.cu[b], L = a.cu[b + 1] - s0;
  const int sk0 = a.cu_k[b], Lk = a.cu_k[b + 1] - sk0;
  const int off = Lk - L;  // query row p sees keys 0 .. p + off
  const int q0 = blk * 2 * BQ;
  if (q0 >= L) return;  // uniform for the whole CTA, before any barrier
  const int rowsB = max(0, min(BQ, L - q0 - BQ));
  const int nKt = (Lk + BKV - 1) / BKV;
  const int nA = min(nKt, (min(q0 + BQ, L) - 1 + off) / BKV + 1);
  const int nB = rowsB > 0 ? min(nKt, (q0 + BQ + rowsB - 1 + off) / BKV + 1) : 0;
  const int nK = max(nA, nB);
  const int hk = h / (a.nq / a.nkv);
  const int xq = a.q_col + h * D, xk = a.k_col + hk * D, xv = a.v_col + hk * D;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  // bars: q_full, kv_full[NS], kv_empty[NS], s_full[2], p_full[2], o_full; then the TMEM slot
  const uint32_t bq = smem_u32(bars), bkf = bq + 8, bke = bkf + 8 * NS, bsf = bke + 8 * NS, bpf = bsf + 16,
                 bof = bpf + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 + 2 * NS + 4 + 1);
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bq, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(bkf + 8 * i, 1);
      mbar_init(bke + 8 * i, 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(bsf + 8 * g, 1);
      mbar_init(bpf + 8 * g, 4);  // one arrive per softmax warp
    }
    mbar_init(bof, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc_1cta(smem_u32(tmem_slot), 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_A 0..127, S_B 128..255, O_A 256..383, O_B 384..511
  auto tS = [&](int g) { return tmem + 128u * (uint32_t)g; };
  auto tO = [&](int g) { return tmem + 256u + 128u * (uint32_t)g; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmKV);
      mbar_expect_tx(bq, (nB ? 2 : 1) * Q_BYTES);
      const uint32_t sq = smem_u32(smem);
      tma_load_2d(sq, &tmQ, xq, s0 + q0, bq);
      tma_load_2d(sq + ATOM, &tmQ, xq + 64, s0 + q0, bq);
      if (nB) {
        tma_load_2d(sq + Q_BYTES, &tmQ, xq, s0 + q0 + BQ, bq);
        tma_load_2d(sq + Q_BYTES + ATOM, &tmQ, xq + 64, s0 + q0 + BQ, bq);
      }
      for (int j = 0; j < nK && !s_abort; ++j) {
        const int st = j % NS;
        const uint32_t ph = (j / NS) & 1;
        if (!mbar_wait(bke + 8 * st, ph ^ 1)) {
          set_err(a.err, 11);
          s_abort = 1;
          break;
        }
        const uint32_t fb = bkf + 8 * st;
        mbar_expect_tx(fb, STAGE);
        const uint32_t sk = smem_u32(smem + OFF_KV + st * STAGE), sv = sk + KV_TILE;
        const int y = sk0 + j * BKV;
        tma_load_2d(sk, &tmKV, xk, y, fb);
        tma_load_2d(sk + ATOM, &tmKV, xk + 64, y, fb);
        tma_load_2d(sv, &tmKV, xv, y, fb);
        tma_load_2d(sv + ATOM, &tmKV, xv + 64, y, fb);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(BQ, BKV, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(BQ, D, false, true);
      bool ok = mbar_wait(bq, 0);
      int kv_ready = -1;
      auto wait_kv = [&](int j) {
        if (!ok || j <= kv_ready) return;
        if (!mbar_wait(bkf + 8 * (j % NS), (j / NS) & 1)) {
          ok = false;
          return;
        }
        kv_ready = j;
      };
      auto issue_s = [&](int g, int j) {
        fence_after();
        const uint32_t sq = smem_u32(smem + g * Q_BYTES), sk = smem_u32(smem + OFF_KV + (j % NS) * STAGE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * ATOM + (k & 3) * 32;
          mma_1cta(tS(g), desc_sw128(sq + off, 16, 1024), desc_sw128(sk + off, 16, 1024), idesc_qk, k > 0);
        }
        commit_1cta(bsf + 8 * g);
      };
      auto issue_pv = [&](int g, int j) {
        fence_after();
        const uint32_t sv = smem_u32(smem + OFF_KV + (j % NS) * STAGE + KV_TILE);
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)
          mma_1cta_ts(tO(g), tS(g) + k * 8, desc_sw128(sv + k * 2048, ATOM, 1024), idesc_pv, (j > 0 || k > 0));
      };
      wait_kv(0);
      if (ok) {
        issue_s(0, 0);
        if (nB) issue_s(1, 0);
      }
      int where = ok ? 0 : 120;
      for (int j = 0; j < nK && ok && !s_abort; ++j) {
        if (j < nA) {
          if (!mbar_wait(bpf, j & 1)) { ok = false; where = 121 + 1000 * j; break; }
          issue_pv(0, j);
        }
        if (j + 1 < nA) {
          wait_kv(j + 1);
          if (!ok) { where = 122 + 1000 * j; break; }
          issue_s(0, j + 1);
        }
        if (j < nB) {
          if (!mbar_wait(bpf + 8, j & 1)) { ok = false; where = 123 + 1000 * j; break; }
          issue_pv(1, j);
        }
        commit_1cta(bke + 8 * (j % NS));  // K_j / V_j no longer read
        if (j + 1 < nB) {
          wait_kv(j + 1);
          if (!ok) { where = 124 + 1000 * j; break; }
          issue_s(1, j + 1);
        }
      }
      if (!ok) {
        set_err(a.err, 12, where);
        s_abort = 1;
      }
      commit_1cta(bof);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int g = (warp - 2) >> 2;  // 0: tile A (warps 2..5), 1: tile B (warps 6..9)
    const int n = g == 0 ? nA : nB;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;           // row within the tile
    const int row_pos = q0 + g * BQ + r;      // position within the sequence
    const uint32_t ts = tS(g) + ((uint32_t)(quad * 32) << 16), to = tO(g) + ((uint32_t)(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(bsf + 8 * g, j & 1) || s_abort) {
        if (!s_abort) set_err(a.err, 14, j);
        ok = false;
        break;
      }
      fence_after();
      const int lim = row_pos + off - j * BKV;  // last key column of tile j this row sees
      const bool masked_tile = __any_sync(0xffffffffu, lim < BKV - 1);
      // the whole S row (128 fp32 columns) comes out of TMEM in four loads
      // behind one wait and stays in registers for both passes
      uint32_t v[128];
      tmem_ld32(ts, v);
      tmem_ld32(ts + 32, v + 32);
      tmem_ld32(ts + 64, v + 64);
      tmem_ld32(ts + 96, v + 96);
      tmem_wait_ld();
      if (masked_tile) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > lim) v[i] = 0xff800000u;  // -inf: key past this row's causal limit
      }
      // pass 1: row maximum of the raw scores; the scale is positive, so it is
      // applied once, to the maximum
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < 128; ++i) mq[i & 3] = fmaxf(mq[i & 3], __uint_as_float(v[i]));
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      const float m_new = fmaxf(m, mx * a.scale_log2);
      // tcgen05.ld / st are warp-collective (.sync.aligned): the decision to
      // rescale O is taken for the whole warp, every lane moves to its m_new
      const bool grow = __any_sync(0xffffffffu, j > 0 && m != -INFINITY && m_new > m + RESCALE_LOG2);
      float alpha = 1.f;
      if (j == 0 || (!grow && m == -INFINITY)) {
        m = m_new;
      } else if (grow) {
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        m = m_new;
      }
      const float ref = (m == -INFINITY) ? 0.f : m;
      // pass 2: P = 2^(x - ref) in bf16, packed two per column over S's first 64 columns
      float ls0 = 0.f, ls1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int c0 = c * 32 + 2 * i;
          const float x0 = fmaf(__uint_as_float(v[c0]), a.scale_log2, -ref);
          const float x1 = fmaf(__uint_as_float(v[c0 + 1]), a.scale_log2, -ref);
          const float p0 = ex2(x0), p1 = ex2(x1);
          ls0 += p0;
          ls1 += p1;
          const bf162 pp = __floats2bfloat162_rn(p0, p1);
          pk[i] = *reinterpret_cast<const uint32_t*>(&pp);
        }
        tmem_st16(ts + c * 16, pk);
      }
      if (grow) {
        // grow the reference maximum: O (complete up to P_{j-1} V_{j-1}) and l by
        // 2^(m_old - m_new); the PV MMA of tile j waits for this warp's arrive
        // below, so nothing writes O meanwhile
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(to + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st32(to + c * 32, ov);
        }
      }
      l = l * alpha + (ls0 + ls1);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bpf + 8 * g);
    }
    if (n > 0) {
      if (!mbar_wait(bof, 0)) ok = false;
      fence_after();
      if (ok && !s_abort) {
        const bool valid = row_pos < L;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        bf16* orow = a.o + (int64_t)(s0 + row_pos) * a.o_row + (int64_t)h * D;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(to + c * 32, v);
          tmem_wait_ld();
          if (valid) {
            float f[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]) * inv;
#pragma unroll
            for (int i = 0; i < 32; i += 8) *reinterpret_cast<bf16x8*>(orow + c * 32 + i) = pack8(f + i);
          }
        }
        if (valid && a.lse != nullptr)
          a.lse[(int64_t)h * a.T + s0 + row_pos] = (m + __log2f(l)) * 0.69314718055994531f;
      } else {
        set_err(a.err, 13);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_free_1cta(tmem, 512);
  }
}


// ---------------------------------------------------------------- backward
//
// Two kernels, no atomics:
//   fa_bwd_dkdv  one CTA per (kv head, sequence, 128-key tile j): K_j and V_j
//                stay in shared memory; for every query head of the GQA
//                group and every query tile i >= j it recomputes
//                S^T = K_j Q_i^T and dP^T = V_j dO_i^T into TMEM, forms
//                P^T = exp(S^T - lse) and dS^T = P^T (dP^T - D) (bf16, back
//                into TMEM) and accumulates dV += P^T dO_i and
//                dK += dS^T Q_i in TMEM (A operands from TMEM, B read MN-major).
//   fa_bwd_dq    one CTA per (query head, sequence, 128-row tile i): Q_i and
//                dO_i stay in shared memory; for every key tile j <= i it
//                recomputes S = Q_i K_j^T and dP = dO_i V_j^T, forms dS and
//                accumulates dQ += dS K_j.
// D = rowsum(dO * O) comes from fa_bwd_dot.  Softmax work uses eight warps,
// two per TMEM lane quadrant, each on one 64-column half of the tile; the
// bf16 results of half h are packed into columns [64 h, 64 h + 32) of the
// tile they were computed from, so no warp overwrites columns another warp
// still reads.
constexpr int NT_BWD = 320;

struct BwdArgs {
  const int* cu;     // [B + 1] query rows
  const int* cu_k;   // [B + 1] key / value rows
  int q_col, k_col, v_col;
  int nq, nkv, T;
  int blocks_z;      // query tiles of the longest sequence (dQ grid)
  float scale, scale_log2;
  const float* lse;  // [nq, T] natural log
  const float* dd;   // [nq, T] rowsum(dO * O)
  bf16* dq;          // query-gradient rows (dq_row apart), head 0 at column dq_col
  int64_t dq_row;
  int dq_col;
  bf16* dkv;         // key / value-gradient rows (dkv_row apart), heads at dk_col / dv_col
  int64_t dkv_row;
  int dk_col, dv_col;
  // dK/dV head split: hsplit CTAs share a key tile, each over nq / nkv / hsplit
  // query heads; with hsplit > 1 they write fp32 partial sums, part[p][key row]
  // [kv head][dK (unscaled) | dV], which fa_bwd_dkdv_reduce adds up
  int hsplit;
  float* part;
  int64_t part_rows;
  int* err;
};

__global__ void fa_bwd_dot(const bf16* __restrict__ o, const bf16* __restrict__ dout, int64_t T, int nq,
                           float* __restrict__ dd) {
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * nq) return;
  const int64_t t = w / nq;
  const int h = (int)(w - t * nq);
  const bf16* po = o + w * D + lane * 4;
  const bf16* pd = dout + w * D + lane * 4;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) s += __bfloat162float(po[i]) * __bfloat162float(pd[i]);
  s = warp_sum(s);
  if (lane == 0) dd[(int64_t)h * T + t] = s;
}

// Adds the hsplit fp32 partial dK / dV rows of fa_bwd_dkdv and writes bf16
// (dK times the softmax scale).  One thread per 8 columns of one key row and kv
// head; rows outside every sequence (at or past cu_k[B]) are left alone.
__global__ void fa_bwd_dkdv_reduce(const float* __restrict__ part, int hsplit, int64_t rows, int nkv,
                                   const int* __restrict__ cu_k, int B, float scale, bf16* __restrict__ dkv,
                                   int64_t dkv_row, int dk_col, int dv_col) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = nkv * 2 * D / 8;
  const int64_t row = t / per_row;
  if (row >= rows || row >= cu_k[B]) return;
  const int c8 = (int)(t - row * per_row) * 8;  // column within [kv head][dK | dV]
  const int hk = c8 / (2 * D), w = c8 - hk * 2 * D;
  const bool is_k = w < D;
  float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int p = 0; p < hsplit; ++p) {
    const float4* src = reinterpret_cast<const float4*>(part + ((int64_t)p * rows + row) * (2 * nkv * D) + c8);
    const float4 x = src[0], y = src[1];
    f[0] += x.x; f[1] += x.y; f[2] += x.z; f[3] += x.w;
    f[4] += y.x; f[5] += y.y; f[6] += y.z; f[7] += y.w;
  }
  if (is_k) {
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] *= scale;
  }
  bf16* dst = dkv + row * dkv_row + (is_k ? dk_col + hk * D + w : dv_col + hk * D + (w - D));
  *reinterpret_cast<bf16x8*>(dst) = pack8(f);
}

// dQ kernel tiles: 64 keys per step, so two S / dP buffers (64 TMEM columns
// each) fit beside the 128-column dQ accumulator and the tensor core computes
// S and dP of key tile jj+1 while the elementwise warps turn tile jj into dS.
constexpr int BK2 = 64;
constexpr int ATOM64 = 64 * 64 * 2;          // 64 rows x 64 bf16 (one 128-byte swizzle atom column)
constexpr int KV64_TILE = 2 * ATOM64;        // 16 KB
constexpr int NSQ = 4;                       // K/V ring depth of the dQ kernel
constexpr int DQ_STAGE = 2 * KV64_TILE;      // K + V
constexpr int OFF_DQ_KV = 2 * KV_TILE;       // after the resident Q and dO tiles
constexpr int OFF_DQ_BAR = OFF_DQ_KV + NSQ * DQ_STAGE;
constexpr int SMEM_DQ = OFF_DQ_BAR + 256 + 1024;

// dK/dV kernel tiles: 64 queries per step, so two S^T / dP^T buffers (64 TMEM
// columns each) fit beside the dV and dK accumulators and the tensor core
// computes S^T and dP^T of step it+1 while the elementwise warps work on step it.
constexpr int BQ2 = 64;
constexpr int NSK = 4;                                  // Q / dO ring depth
constexpr int DKV_STAGE = 2 * KV64_TILE + 1024;          // Q + dO (64 rows each) + 64 lse + 64 D, 1 KB aligned
constexpr int OFF_DKV_STAGE = 2 * KV_TILE;               // after the resident K and V tiles
constexpr int OFF_DKV_BAR = OFF_DKV_STAGE + NSK * DKV_STAGE;
constexpr int SMEM_DKV = OFF_DKV_BAR + 256 + 1024;

__global__ void __launch_bounds__(NT_BWD, 1)
    fa_bwd_dkdv(const __grid_constant__ CUtensorMap tmQ64, const __grid_constant__ CUtensorMap tmKV,
                const __grid_constant__ CUtensorMap tm_do64, BwdArgs a) {
  // small j: most work, launched first; the hsplit CTAs of one key tile are adjacent
  const int hk = blockIdx.x, b = blockIdx.y, j = (int)blockIdx.z / a.hsplit, part = (int)blockIdx.z % a.hsplit;
  const int s0 = a.cu[b], L = a.cu[b + 1] - s0;
  const int sk0 = a.cu_k[b], Lk = a.cu_k[b + 1] - sk0;
  const int off = Lk - L;
  if (j * BKV >= Lk) return;
  const int G = a.nq / a.nkv, Gc = G / a.hsplit;
  const int nqt = (L + BQ2 - 1) / BQ2;
  const int i0 = max(0, j * BKV - off) / BQ2;  // first 64-row query tile that sees key tile j
  const int per_head = nqt - i0;
  const int iters = Gc * per_head;
  const int xk = a.k_col + hk * D, xv = a.v_col + hk * D;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_DKV_BAR);
  // kv_full, st_full[NSK] (count 2: TMA bytes + the lse/D copy), st_empty[NSK],
  // s_full[2], p_full[2], done; then the TMEM slot
  const uint32_t bkv = smem_u32(bars), bsf0 = bkv + 8, bse0 = bsf0 + 8 * NSK, bs0 = bse0 + 8 * NSK, bp0 = bs0 + 16,
                 bdone = bp0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1 + 2 * NSK + 5);
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bkv, 1);
    for (int k = 0; k < NSK; ++k) {
      mbar_init(bsf0 + 8 * k, 2);
      mbar_init(bse0 + 8 * k, 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bs0 + 8 * k, 1);
      mbar_init(bp0 + 8 * k, 8);  // one arrive per elementwise warp
    }
    mbar_init(bdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc_1cta(smem_u32(tmem_slot), 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S^T_0 0..63, dP^T_0 64..127, S^T_1 128..191, dP^T_1 192..255, dV 256..383, dK 384..511
  auto tS = [&](int bb) { return tmem + 128u * (uint32_t)bb; };
  auto tP = [&](int bb) { return tmem + 128u * (uint32_t)bb + 64u; };
  const uint32_t tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 0) {
    // producer: K_j, V_j once; then per step Q, dO (64 rows, TMA) and lse, D (warp copy)
    const uint32_t sk = smem_u32(smem), sv = sk + KV_TILE;
    if (lane == 0) {
      tma_prefetch_desc(&tmQ64);
      tma_prefetch_desc(&tmKV);
      tma_prefetch_desc(&tm_do64);
      mbar_expect_tx(bkv, 2 * KV_TILE);
      tma_load_2d(sk, &tmKV, xk, sk0 + j * BKV, bkv);
      tma_load_2d(sk + ATOM, &tmKV, xk + 64, sk0 + j * BKV, bkv);
      tma_load_2d(sv, &tmKV, xv, sk0 + j * BKV, bkv);
      tma_load_2d(sv + ATOM, &tmKV, xv + 64, sk0 + j * BKV, bkv);
    }
    for (int it = 0; it < iters && !s_abort; ++it) {
      const int hq = hk * G + part * Gc + it / per_head, i = i0 + it % per_head;
      const int st = it % NSK;
      const uint32_t ph = (it / NSK) & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(bse0 + 8 * st, ph ^ 1);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) {
          set_err(a.err, 21);
          s_abort = 1;
        }
        break;
      }
      uint8_t* stg = smem + OFF_DKV_STAGE + st * DKV_STAGE;
      const uint32_t sq = smem_u32(stg), sdo = sq + KV64_TILE;
      const uint32_t fb = bsf0 + 8 * st;
      if (lane == 0) {
        mbar_expect_tx(fb, 2 * KV64_TILE);
        const int y = s0 + i * BQ2;
        tma_load_2d(sq, &tmQ64, a.q_col + hq * D, y, fb);
        tma_load_2d(sq + ATOM64, &tmQ64, a.q_col + hq * D + 64, y, fb);
        tma_load_2d(sdo, &tm_do64, hq * D, y, fb);
        tma_load_2d(sdo + ATOM64, &tm_do64, hq * D + 64, y, fb);
      }
      float* lse_s = reinterpret_cast<float*>(stg + 2 * KV64_TILE);
      float* dd_s = lse_s + BQ2;
#pragma unroll
      for (int c = lane; c < BQ2; c += 32) {
        const int q = i * BQ2 + c;
        const bool in = q < L;
        lse_s[c] = in ? a.lse[(int64_t)hq * a.T + s0 + q] * 1.4426950408889634f : 0.f;
        dd_s[c] = in ? a.dd[(int64_t)hq * a.T + s0 + q] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(fb);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_ss = idesc_bf16_f32(BKV, BQ2, false, false);  // M = keys, N = 64 queries
      constexpr uint32_t id_ts = idesc_bf16_f32(BKV, D, false, true);     // M = keys, N = d, K = 64 queries
      const uint32_t sk = smem_u32(smem), sv = sk + KV_TILE;
      // S^T = K Q^T and dP^T = V dO^T of step it into buffer it & 1
      auto issue_s = [&](int it) -> bool {
        const int st = it % NSK;
        if (!mbar_wait(bsf0 + 8 * st, (it / NSK) & 1)) return false;
        fence_after();
        const uint32_t sq = smem_u32(smem + OFF_DKV_STAGE + st * DKV_STAGE), sdo = sq + KV64_TILE;
        const int bb = it & 1;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t oa = (k >> 2) * ATOM + (k & 3) * 32, ob = (k >> 2) * ATOM64 + (k & 3) * 32;
          mma_1cta(tS(bb), desc_sw128(sk + oa, 16, 1024), desc_sw128(sq + ob, 16, 1024), id_ss, k > 0);
        }
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t oa = (k >> 2) * ATOM + (k & 3) * 32, ob = (k >> 2) * ATOM64 + (k & 3) * 32;
          mma_1cta(tP(bb), desc_sw128(sv + oa, 16, 1024), desc_sw128(sdo + ob, 16, 1024), id_ss, k > 0);
        }
        commit_1cta(bs0 + 8 * bb);
        return true;
      };
      bool ok = mbar_wait(bkv, 0);
      int where = 0;
      if (ok && iters > 0) {
        ok = issue_s(0);
        where = 1;
      }
      for (int it = 0; it < iters && ok && !s_abort; ++it) {
        // buffer (it + 1) & 1 was last read by the dV / dK MMAs of step it - 1,
        // issued before (tcgen05 MMAs of one thread run in order)
        if (it + 1 < iters && !issue_s(it + 1)) {
          ok = false;
          where = 2 + 10 * it;
          break;
        }
        const int bb = it & 1;
        if (!mbar_wait(bp0 + 8 * bb, (it >> 1) & 1)) {
          ok = false;
          where = 3 + 10 * it;
          break;
        }
        fence_after();
        const int st = it % NSK;
        const uint32_t sq = smem_u32(smem + OFF_DKV_STAGE + st * DKV_STAGE), sdo = sq + KV64_TILE;
        // P^T and dS^T (bf16) sit packed in columns [0, 16) and [32, 48) of S^T_bb and dP^T_bb
#pragma unroll
        for (int k = 0; k < BQ2 / 16; ++k) {
          const uint32_t acol = (k < 2) ? k * 8 : 32 + (k - 2) * 8;
          const uint32_t acc = (it > 0 || k > 0) ? 1u : 0u;
          mma_1cta_ts(tdV, tS(bb) + acol, desc_sw128(sdo + k * 2048, ATOM64, 1024), id_ts, acc);  // dV += P^T dO
          mma_1cta_ts(tdK, tP(bb) + acol, desc_sw128(sq + k * 2048, ATOM64, 1024), id_ts, acc);   // dK += dS^T Q
        }
        commit_1cta(bse0 + 8 * st);  // Q / dO of this step no longer read
      }
      if (!ok) {
        set_err(a.err, 22, where);
        s_abort = 1;
      }
      commit_1cta(bdone);
    }
  } else {
    // elementwise warps: thread = key row r, half = which 32 of the step's 64 queries
    const int quad = warp & 3, half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int key = j * BKV + r;
    const int col0 = half * 32;
    bool ok = true;
    for (int it = 0; it < iters; ++it) {
      const int i = i0 + it % per_head;
      const int st = it % NSK, bb = it & 1;
      if (!mbar_wait(bs0 + 8 * bb, (it >> 1) & 1) || s_abort) {
        ok = false;
        break;
      }
      fence_after();
      const float* lse_s = reinterpret_cast<const float*>(smem + OFF_DKV_STAGE + st * DKV_STAGE + 2 * KV64_TILE);
      const float* dd_s = lse_s + BQ2;
      // every query of tile i is in the sequence and sees every key of tile j:
      // no per-element mask
      const bool full = (i + 1) * BQ2 <= L && (j + 1) * BKV - 1 <= i * BQ2 + off;
      uint32_t vs[32], vp[32], pk[16], dk[16];
      tmem_ld32(tS(bb) + lane_off + col0, vs);
      tmem_ld32(tP(bb) + lane_off + col0, vp);
      tmem_wait_ld();
      if (!full) {
        // masked scores become -inf: P = 0 and dS = P (dP - D) = 0 (dP and D
        // are finite; rows past the sequence were loaded as zeros)
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int q = i * BQ2 + col0 + e;
          if (!(q < L && key <= q + off)) vs[e] = 0xff800000u;
        }
      }
#pragma unroll
      for (int e4 = 0; e4 < 8; ++e4) {
        const float4 l4 = *reinterpret_cast<const float4*>(lse_s + col0 + 4 * e4);
        const float4 d4 = *reinterpret_cast<const float4*>(dd_s + col0 + 4 * e4);
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
        float pv[4], dv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          pv[u] = ex2(fmaf(__uint_as_float(vs[4 * e4 + u]), a.scale_log2, -lv[u]));
          dv[u] = pv[u] * (__uint_as_float(vp[4 * e4 + u]) - dv4[u]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const bf162 pp = __floats2bfloat162_rn(pv[2 * u], pv[2 * u + 1]);
          const bf162 dp = __floats2bfloat162_rn(dv[2 * u], dv[2 * u + 1]);
          pk[2 * e4 + u] = *reinterpret_cast<const uint32_t*>(&pp);
          dk[2 * e4 + u] = *reinterpret_cast<const uint32_t*>(&dp);
        }
      }
      // P^T and dS^T of this half's 32 queries, packed into the first 16 of the 32 columns it read
      tmem_st16(tS(bb) + lane_off + col0, pk);
      tmem_st16(tP(bb) + lane_off + col0, dk);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bp0 + 8 * bb);
    }
    // epilogue: dV and dK (x scale) rows of this thread's key, half the columns each
    if (!mbar_wait(bdone, 0)) ok = false;
    fence_after();
    if (ok && !s_abort) {
      const int key = j * BKV + r;
      const bool valid = key < Lk;
      bf16* rowp = a.dkv + (int64_t)(sk0 + key) * a.dkv_row;
      const int ok_col = a.dk_col + hk * D, ov_col = a.dv_col + hk * D;
      float* prow = a.part + ((int64_t)part * a.part_rows + sk0 + key) * (2 * a.nkv * D) + hk * 2 * D;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int col0 = half * 64 + c * 32;
        uint32_t vdv[32], vdk[32];
        tmem_ld32(tdV + lane_off + col0, vdv);
        tmem_ld32(tdK + lane_off + col0, vdk);
        tmem_wait_ld();
        if (valid && a.hsplit > 1) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            *reinterpret_cast<uint4*>(prow + col0 + e) = make_uint4(vdk[e], vdk[e + 1], vdk[e + 2], vdk[e + 3]);
            *reinterpret_cast<uint4*>(prow + D + col0 + e) = make_uint4(vdv[e], vdv[e + 1], vdv[e + 2], vdv[e + 3]);
          }
        } else if (valid) {
          float f[32], g[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            f[e] = __uint_as_float(vdv[e]);
            g[e] = __uint_as_float(vdk[e]) * a.scale;
          }
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            *reinterpret_cast<bf16x8*>(rowp + ov_col + col0 + e) = pack8(f + e);
            *reinterpret_cast<bf16x8*>(rowp + ok_col + col0 + e) = pack8(g + e);
          }
        }
      }
    } else {
      set_err(a.err, 23);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_free_1cta(tmem, 512);
  }
}


__global__ void __launch_bounds__(NT_BWD, 1)
    fa_bwd_dq(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV64,
              const __grid_constant__ CUtensorMap tm_do, BwdArgs a) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int i = a.blocks_z - 1 - (int)blockIdx.z;  // large query tiles (most key tiles) first
  const int s0 = a.cu[b], L = a.cu[b + 1] - s0;
  const int sk0 = a.cu_k[b], Lk = a.cu_k[b + 1] - sk0;
  const int off = Lk - L;
  if (i * BQ >= L) return;
  const int n = min((Lk + BK2 - 1) / BK2, (min((i + 1) * BQ, L) - 1 + off) / BK2 + 1);
  const int hk = h / (a.nq / a.nkv);
  const int xk = a.k_col + hk * D, xv = a.v_col + hk * D;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_DQ_BAR);
  // q_full, kv_full[NSQ], kv_empty[NSQ], s_full[2], ds_full[2], done; then the TMEM slot
  const uint32_t bqd = smem_u32(bars), bkf0 = bqd + 8, bke0 = bkf0 + 8 * NSQ, bs0 = bke0 + 8 * NSQ, bp0 = bs0 + 16,
                 bdone = bp0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1 + 2 * NSQ + 5);
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(bqd, 1);
    for (int k = 0; k < NSQ; ++k) {
      mbar_init(bkf0 + 8 * k, 1);
      mbar_init(bke0 + 8 * k, 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bs0 + 8 * k, 1);
      mbar_init(bp0 + 8 * k, 8);  // one arrive per elementwise warp
    }
    mbar_init(bdone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tmem_alloc_1cta(smem_u32(tmem_slot), 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_0 0..63, dP_0 64..127, S_1 128..191, dP_1 192..255, dQ 256..383
  auto tS = [&](int bb) { return tmem + 128u * (uint32_t)bb; };
  auto tP = [&](int bb) { return tmem + 128u * (uint32_t)bb + 64u; };
  const uint32_t tdQ = tmem + 256;
  const uint32_t sq = smem_u32(smem), sdo = sq + KV_TILE;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmKV64);
      tma_prefetch_desc(&tm_do);
      mbar_expect_tx(bqd, 2 * KV_TILE);
      const int y = s0 + i * BQ;
      tma_load_2d(sq, &tmQ, a.q_col + h * D, y, bqd);
      tma_load_2d(sq + ATOM, &tmQ, a.q_col + h * D + 64, y, bqd);
      tma_load_2d(sdo, &tm_do, h * D, y, bqd);
      tma_load_2d(sdo + ATOM, &tm_do, h * D + 64, y, bqd);
      for (int jj = 0; jj < n && !s_abort; ++jj) {
        const int st = jj % NSQ;
        const uint32_t ph = (jj / NSQ) & 1;
        if (!mbar_wait(bke0 + 8 * st, ph ^ 1)) {
          set_err(a.err, 31);
          s_abort = 1;
          break;
        }
        const uint32_t fb = bkf0 + 8 * st;
        mbar_expect_tx(fb, DQ_STAGE);
        const uint32_t sk = smem_u32(smem + OFF_DQ_KV + st * DQ_STAGE), sv = sk + KV64_TILE;
        const int y2 = sk0 + jj * BK2;
        tma_load_2d(sk, &tmKV64, xk, y2, fb);
        tma_load_2d(sk + ATOM64, &tmKV64, xk + 64, y2, fb);
        tma_load_2d(sv, &tmKV64, xv, y2, fb);
        tma_load_2d(sv + ATOM64, &tmKV64, xv + 64, y2, fb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(BQ, BK2, false, false);  // M = queries, N = 64 keys
      constexpr uint32_t id_dq = idesc_bf16_f32(BQ, D, false, true);    // M = queries, N = d, K = 64 keys
      // S = Q K^T and dP = dO V^T of key tile jj into buffer jj & 1
      auto issue_sdp = [&](int jj) -> bool {
        const int st = jj % NSQ;
        if (!mbar_wait(bkf0 + 8 * st, (jj / NSQ) & 1)) return false;
        fence_after();
        const uint32_t sk = smem_u32(smem + OFF_DQ_KV + st * DQ_STAGE), sv = sk + KV64_TILE;
        const int bb = jj & 1;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t oa = (k >> 2) * ATOM + (k & 3) * 32, ob = (k >> 2) * ATOM64 + (k & 3) * 32;
          mma_1cta(tS(bb), desc_sw128(sq + oa, 16, 1024), desc_sw128(sk + ob, 16, 1024), id_s, k > 0);
        }
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t oa = (k >> 2) * ATOM + (k & 3) * 32, ob = (k >> 2) * ATOM64 + (k & 3) * 32;
          mma_1cta(tP(bb), desc_sw128(sdo + oa, 16, 1024), desc_sw128(sv + ob, 16, 1024), id_s, k > 0);
        }
        commit_1cta(bs0 + 8 * bb);
        return true;
      };
      bool ok = mbar_wait(bqd, 0);
      int where = 0;
      if (ok && n > 0) {
        ok = issue_sdp(0);
        where = 1;
      }
      for (int jj = 0; jj < n && ok && !s_abort; ++jj) {
        // buffer (jj + 1) & 1 was last read by dQ of tile jj - 1, issued before
        // (tcgen05 MMAs of one thread run in order)
        if (jj + 1 < n && !issue_sdp(jj + 1)) {
          ok = false;
          where = 2 + 10 * jj;
          break;
        }
        const int bb = jj & 1;
        if (!mbar_wait(bp0 + 8 * bb, (jj >> 1) & 1)) {
          ok = false;
          where = 3 + 10 * jj;
          break;
        }
        fence_after();
        const uint32_t sk = smem_u32(smem + OFF_DQ_KV + (jj % NSQ) * DQ_STAGE);
        // dQ += dS K: dS (bf16) sits packed in columns [0, 16) and [32, 48) of S_bb
#pragma unroll
        for (int k = 0; k < BK2 / 16; ++k) {
          const uint32_t acol = (k < 2) ? k * 8 : 32 + (k - 2) * 8;
          mma_1cta_ts(tdQ, tS(bb) + acol, desc_sw128(sk + k * 2048, ATOM64, 1024), id_dq, (jj > 0 || k > 0) ? 1u : 0u);
        }
        commit_1cta(bke0 + 8 * (jj % NSQ));  // K_jj / V_jj no longer read
      }
      if (!ok) {
        set_err(a.err, 32, where);
        s_abort = 1;
      }
      commit_1cta(bdone);
    }
  } else {
    // elementwise warps: thread = query row r, half = which 32 of the tile's 64 keys
    const int quad = warp & 3, half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int q = i * BQ + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const bool qin = q < L;
    const float lse2 = qin ? a.lse[(int64_t)h * a.T + s0 + q] * 1.4426950408889634f : 0.f;
    const float dd = qin ? a.dd[(int64_t)h * a.T + s0 + q] : 0.f;
    const int col0 = half * 32;
    bool ok = true;
    for (int jj = 0; jj < n; ++jj) {
      const int bb = jj & 1;
      if (!mbar_wait(bs0 + 8 * bb, (jj >> 1) & 1) || s_abort) {
        ok = false;
        break;
      }
      fence_after();
      // every query of tile i is in the sequence and sees every key of tile jj
      const bool full = (i + 1) * BQ <= L && (jj + 1) * BK2 - 1 <= i * BQ + off;
      uint32_t vs[32], vp[32], dk[16];
      tmem_ld32(tS(bb) + lane_off + col0, vs);
      tmem_ld32(tP(bb) + lane_off + col0, vp);
      tmem_wait_ld();
      if (!full) {
        // masked scores become -inf, so P = 0 and dS = P (dP - D) = 0
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = jj * BK2 + col0 + e;
          if (!(qin && key <= q + off)) vs[e] = 0xff800000u;
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        float dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float p = ex2(fmaf(__uint_as_float(vs[2 * e + u]), a.scale_log2, -lse2));
          dv[u] = p * (__uint_as_float(vp[2 * e + u]) - dd);
        }
        const bf162 dp = __floats2bfloat162_rn(dv[0], dv[1]);
        dk[e] = *reinterpret_cast<const uint32_t*>(&dp);
      }
      // dS of this half's 32 keys, packed into the first 16 of the 32 columns it read
      tmem_st16(tS(bb) + lane_off + col0, dk);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bp0 + 8 * bb);
    }
    if (!mbar_wait(bdone, 0)) ok = false;
    fence_after();
    if (ok && !s_abort) {
      bf16* rowp = a.dq + (int64_t)(s0 + q) * a.dq_row + a.dq_col + (int64_t)h * D;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        const int dc = half * 64 + c * 32;
        uint32_t v[32];
        tmem_ld32(tdQ + lane_off + dc, v);
        tmem_wait_ld();
        if (qin) {
          float f[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(v[e]) * a.scale;
#pragma unroll
          for (int e = 0; e < 32; e += 8) *reinterpret_cast<bf16x8*>(rowp + dc + e) = pack8(f + e);
        }
      }
    } else {
      set_err(a.err, 33);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_free_1cta(tmem, 512);
  }
}

}  // namespace fa5

using namespace fa5;

static CUtensorMap map_rows_64xR(const at::Tensor& t, uint32_t rows) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && (t.stride(0) * 2) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "operand rows must start on 16-byte boundaries with unit inner stride");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)t.size(1), (cuuint64_t)t.size(0)};
  cuuint64_t strides[1] = {(cuuint64_t)t.stride(0) * 2};
  cuuint32_t box[2] = {64u, rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = PSRL_DRV(cuTensorMapEncodeTiled)(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, t.data_ptr(), dims, strides,
                                                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}
static CUtensorMap map_rows_64x128(const at::Tensor& t) { return map_rows_64xR(t, 128u); }

// Shared launcher: queries in q (columns q_col + h * 128), keys and values in
// kv (k_col / v_col + hk * 128); sequence b's query rows [cu_q[b], cu_q[b+1])
// are the last of its key rows [cu_k[b], cu_k[b+1]).
static std::vector<at::Tensor> fwd_launch(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& cu_q,
                                          const at::Tensor& cu_k, int64_t max_q, int64_t nq, int64_t nkv, int q_col,
                                          int k_col, int v_col, double scale, bool want_lse, const at::Tensor& err) {
  CHECK_DTYPE(q, at::kBFloat16);
  CHECK_DTYPE(kv, at::kBFloat16);
  TORCH_CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && cu_q.is_contiguous() && cu_k.scalar_type() == at::kInt &&
                  cu_k.is_contiguous() && cu_q.numel() == cu_k.numel(),
              "cu_q / cu_k: int32 [B + 1]");
  const int64_t T = q.size(0);
  const int B = (int)cu_q.numel() - 1;
  at::cuda::CUDAGuard g(q.device());
  auto o = at::empty({T, nq * D}, q.options());
  auto lse = want_lse ? at::empty({nq, T}, q.options().dtype(at::kFloat)) : at::Tensor();
  if (T == 0 || B <= 0 || max_q <= 0) return {o, lse};
  const CUtensorMap tq = map_rows_64x128(q), tkv = map_rows_64x128(kv);
  FwdArgs a{};
  a.cu = cu_q.data_ptr<int>();
  a.cu_k = cu_k.data_ptr<int>();
  a.q_col = q_col;
  a.k_col = k_col;
  a.v_col = v_col;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.T = (int)T;
  a.blocks_z = (int)((max_q + 2 * BQ - 1) / (2 * BQ));
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.o = reinterpret_cast<bf16*>(o.data_ptr());
  a.o_row = nq * D;
  a.lse = want_lse ? lse.data_ptr<float>() : nullptr;
  a.err = err.data_ptr<int>();
  ensure_smem_attr(fa_fwd_kernel, SMEM_BYTES);
  dim3 grid((unsigned)nq, (unsigned)B, (unsigned)a.blocks_z);
  fa_fwd_kernel<<<grid, NTHREADS, SMEM_BYTES, stream()>>>(tq, tkv, a);
  PSRL_CHECK_LAUNCH();
  return {o, lse};
}

// qkv: [T, (nq + 2 nkv) * 128] bf16 (q heads, then k heads, then v heads per
// token, unit inner stride, rows on 16-byte boundaries).  Returns
// {o [T, nq * 128] bf16, lse [nq, T] fp32 (natural log; empty unless want_lse)}.
std::vector<at::Tensor> attn_fwd_sm100(at::Tensor qkv, at::Tensor cu_seqlens, int64_t max_seqlen, int64_t nq,
                                       int64_t nkv, double scale, bool want_lse, at::Tensor err) {
  CHECK_CUDA_TENSOR(qkv);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) == (nq + 2 * nkv) * D,
              "qkv must be [T, (nq + 2 nkv) * 128] with unit inner stride");
  return fwd_launch(qkv, qkv, cu_seqlens, cu_seqlens, max_seqlen, nq, nkv, 0, (int)(nq * D), (int)((nq + nkv) * D),
                    scale, want_lse, err);
}

// Queries against separately stored keys / values (context parallelism):
// q [Tq, >= nq * 128] (a row-strided view is fine), kv [Tk, 2 nkv * 128]
// (k heads then v heads); sequence b has cu_q[b+1] - cu_q[b] queries that are
// the last of its cu_k[b+1] - cu_k[b] (>=) key positions.
std::vector<at::Tensor> attn_fwd_sm100_kv(at::Tensor q, at::Tensor kv, at::Tensor cu_q, at::Tensor cu_k,
                                          int64_t max_q, int64_t nq, int64_t nkv, double scale, bool want_lse,
                                          at::Tensor err) {
  CHECK_CUDA_TENSOR(q);
  TORCH_CHECK(q.dim() == 2 && q.size(1) >= nq * D && kv.dim() == 2 && kv.size(1) == 2 * nkv * D,
              "q [Tq, nq * 128], kv [Tk, 2 nkv * 128]");
  return fwd_launch(q, kv, cu_q, cu_k, max_q, nq, nkv, 0, 0, (int)(nkv * D), scale, want_lse, err);
}

// Shared backward launcher (see fwd_launch); writes dq rows into `dq` and dk /
// dv rows into `dkv` (which may be the same tensor as dq).
static void bwd_launch(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& o, const at::Tensor& dout,
                       const at::Tensor& lse, const at::Tensor& cu_q, const at::Tensor& cu_k, int64_t max_q,
                       int64_t max_k, int64_t nq, int64_t nkv, int q_col, int k_col, int v_col, double scale,
                       at::Tensor& dq, int dq_col, at::Tensor& dkv, int dk_col, int dv_col, const at::Tensor& err) {
  CHECK_DTYPE(q, at::kBFloat16);
  CHECK_DTYPE(kv, at::kBFloat16);
  CHECK_DTYPE(o, at::kBFloat16);
  CHECK_DTYPE(dout, at::kBFloat16);
  CHECK_DTYPE(lse, at::kFloat);
  const int64_t T = q.size(0);
  TORCH_CHECK(o.is_contiguous() && dout.is_contiguous() && o.numel() == T * nq * D && dout.numel() == T * nq * D,
              "o / dout must be contiguous [Tq, nq * 128]");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == nq * T, "lse must be contiguous [nq, Tq]");
  const int B = (int)cu_q.numel() - 1;
  if (T == 0 || B <= 0 || max_q <= 0) return;
  auto dd = at::empty({nq, T}, q.options().dtype(at::kFloat));
  {
    const int64_t warps = T * nq;
    fa_bwd_dot<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream()>>>(
        reinterpret_cast<const bf16*>(o.data_ptr()), reinterpret_cast<const bf16*>(dout.data_ptr()), T, (int)nq,
        dd.data_ptr<float>());
    PSRL_CHECK_LAUNCH();
  }
  const CUtensorMap tq = map_rows_64x128(q), tkv = map_rows_64x128(kv), tdo = map_rows_64x128(dout.view({T, nq * D}));
  BwdArgs a{};
  a.cu = cu_q.data_ptr<int>();
  a.cu_k = cu_k.data_ptr<int>();
  a.q_col = q_col;
  a.k_col = k_col;
  a.v_col = v_col;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.T = (int)T;
  a.blocks_z = (int)((max_q + BQ - 1) / BQ);
  a.scale = (float)scale;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.lse = lse.data_ptr<float>();
  a.dd = dd.data_ptr<float>();
  a.dq = reinterpret_cast<bf16*>(dq.data_ptr());
  a.dq_row = dq.stride(0);
  a.dq_col = dq_col;
  a.dkv = reinterpret_cast<bf16*>(dkv.data_ptr());
  a.dkv_row = dkv.stride(0);
  a.dk_col = dk_col;
  a.dv_col = dv_col;
  a.err = err.data_ptr<int>();
  ensure_smem_attr(fa_bwd_dkdv, SMEM_DKV);
  ensure_smem_attr(fa_bwd_dq, SMEM_DQ);
  const unsigned kz = (unsigned)((max_k + BKV - 1) / BKV);
  // Causal balance: the CTA of key tile 0 loops over every query tile of all
  // G = nq / nkv heads, the last key tile over one.  Split the heads of each
  // key tile over hsplit CTAs until the longest CTA holds at most half of an
  // SM's average share (estimated for B sequences of the longest length),
  // at the price of fp32 partials summed by a small second kernel.
  const int G = (int)(nq / nkv);
  const int64_t nqt = (max_q + BQ - 1) / BQ;
  const int64_t total = (int64_t)B * nkv * G * nqt * (nqt + 1) / 2;
  const int64_t share = total / std::max(1, num_sms());
  int hsplit = 1;
  while (hsplit < 4 && G % (2 * hsplit) == 0 && 2 * (int64_t)G * nqt / hsplit > share) hsplit *= 2;
  a.hsplit = hsplit;
  at::Tensor part;
  if (hsplit > 1) {
    part = at::empty({hsplit, kv.size(0), 2 * nkv * D}, q.options().dtype(at::kFloat));
    a.part = part.data_ptr<float>();
    a.part_rows = kv.size(0);
  }
  const CUtensorMap tq64 = map_rows_64xR(q, 64u), tdo64 = map_rows_64xR(dout.view({T, nq * D}), 64u);
  fa_bwd_dkdv<<<dim3((unsigned)nkv, (unsigned)B, kz * (unsigned)hsplit), NT_BWD, SMEM_DKV, stream()>>>(tq64, tkv,
                                                                                                       tdo64, a);
  PSRL_CHECK_LAUNCH();
  if (hsplit > 1) {
    const int64_t threads = kv.size(0) * nkv * 2 * D / 8;
    fa_bwd_dkdv_reduce<<<(unsigned)((threads + 255) / 256), 256, 0, stream()>>>(
        a.part, hsplit, kv.size(0), (int)nkv, a.cu_k, B, a.scale, a.dkv, a.dkv_row, dk_col, dv_col);
    PSRL_CHECK_LAUNCH();
  }
  const CUtensorMap tkv64 = map_rows_64xR(kv, 64u);
  fa_bwd_dq<<<dim3((unsigned)nq, (unsigned)B, (unsigned)a.blocks_z), NT_BWD, SMEM_DQ, stream()>>>(tq, tkv64, tdo, a);
  PSRL_CHECK_LAUNCH();
}

// Backward of attn_fwd_sm100: qkv [T, (nq + 2 nkv) * 128], o and dout
// [T, nq * 128] (bf16), lse [nq, T].  Returns dqkv [T, (nq + 2 nkv) * 128] bf16.
at::Tensor attn_bwd_sm100(at::Tensor qkv, at::Tensor o, at::Tensor dout, at::Tensor lse, at::Tensor cu_seqlens,
                          int64_t max_seqlen, int64_t nq, int64_t nkv, double scale, at::Tensor err) {
  CHECK_CUDA_TENSOR(qkv);
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(1) == (nq + 2 * nkv) * D && nq % nkv == 0, "qkv layout");
  at::cuda::CUDAGuard g(qkv.device());
  auto dqkv = at::empty({qkv.size(0), (nq + 2 * nkv) * D}, qkv.options());
  if (qkv.size(0) == 0 || cu_seqlens.numel() < 2 || max_seqlen <= 0) return dqkv.zero_();
  const int kc = (int)(nq * D), vc = (int)((nq + nkv) * D);
  bwd_launch(qkv, qkv, o, dout, lse, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen, nq, nkv, 0, kc, vc, scale, dqkv,
             0, dqkv, kc, vc, err);
  return dqkv;
}

// Backward of attn_fwd_sm100_kv.  Returns {dq [Tq, nq * 128], dkv [Tk, 2 nkv * 128]}
// (bf16; key rows that no query sees get zero gradients).
std::vector<at::Tensor> attn_bwd_sm100_kv(at::Tensor q, at::Tensor kv, at::Tensor o, at::Tensor dout, at::Tensor lse,
                                          at::Tensor cu_q, at::Tensor cu_k, int64_t max_q, int64_t max_k, int64_t nq,
                                          int64_t nkv, double scale, at::Tensor err) {
  CHECK_CUDA_TENSOR(q);
  TORCH_CHECK(q.dim() == 2 && q.size(1) >= nq * D && kv.dim() == 2 && kv.size(1) == 2 * nkv * D && nq % nkv == 0,
              "q [Tq, nq * 128], kv [Tk, 2 nkv * 128]");
  at::cuda::CUDAGuard g(q.device());
  auto dq = at::empty({q.size(0), nq * D}, q.options());
  auto dkv = at::zeros({kv.size(0), 2 * nkv * D}, q.options());
  if (q.size(0) == 0 || cu_q.numel() < 2 || max_q <= 0) return {dq.zero_(), dkv};
  bwd_launch(q, kv, o, dout, lse, cu_q, cu_k, max_q, max_k, nq, nkv, 0, 0, (int)(nkv * D), scale, dq, 0, dkv, 0,
             (int)(nkv * D), err);
  return {dq, dkv};
}

}  // namespace psrl
