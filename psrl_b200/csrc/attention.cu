// Attention kernels (head_dim 128, bf16 in, fp32 accumulate):
//
//  attn_fwd   causal varlen attention for packed training batches and for
//             chunked prefill over a paged KV cache (queries are the last
//             q_len positions of a context of length kv_len).
//  attn_bwd   FlashAttention-2 style backward: one CTA per (key tile, kv head,
//             sequence) loops over the GQA group's query heads and query tiles,
//             accumulating dK/dV in registers; dQ is accumulated in fp32 with
//             atomics.
//  decode     split-KV paged decode: one CTA per (sequence, kv head, split)
//             processes all g = nq/nkv query heads of the group as the rows of
//             one 16-row MMA tile, so every KV byte is read once per group.
//             Partial results of the splits are merged by a combine kernel.
//
// Tiles are staged in shared memory with cp.async (16 B chunks, XOR-swizzled so
// ldmatrix is bank-conflict free) and double-buffered; the math uses
// mma.sync.m16n8k16 bf16 tensor-core instructions.
#include "checks.cuh"
#include "common.cuh"

namespace psrl {
namespace attn {

constexpr int D = 128;
constexpr int BM = 64;   // query rows per CTA (fwd) / per iteration (bwd)
constexpr int BN = 64;   // keys per tile
constexpr int NWARPS = 4;
constexpr int NTHREADS = NWARPS * 32;
constexpr float LOG2E = 1.4426950408889634f;

// ---------------------------------------------------------------- PTX utils
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x via the hardware approximation (PTX ex2.approx.ftz.f32); -inf -> 0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  bf162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Swizzled element offset of (row, col) in a [rows][128] bf16 tile; col % 8 == 0.
__device__ __forceinline__ int swz(int row, int col) { return row * D + ((((col >> 3) ^ (row & 7))) << 3); }

// Load `rows` x 128 tile rows given per-row global pointers (nullptr = zero fill).
// `fb` is any valid global address, used as the (unread) source of zero-filled chunks.
template <int ROWS>
__device__ __forceinline__ void load_tile(bf16* sm, const bf16* const* rowptr, const bf16* fb) {
  // ROWS * 16 chunks of 16 B
#pragma unroll
  for (int i = 0; i < ROWS * 16 / NTHREADS; ++i) {
    const int idx = threadIdx.x + i * NTHREADS;
    const int r = idx >> 4, c = idx & 15;
    const bf16* src = rowptr[r];
    cp_async16(sm + swz(r, c * 8), src ? src + c * 8 : fb, src != nullptr);
  }
}

// Load rows [0, ROWS) of a row-strided matrix starting at `base` (rows past
// `n_valid` are zero-filled); each thread computes its chunk addresses directly.
template <int ROWS>
__device__ __forceinline__ void load_rows(bf16* sm, const bf16* base, int64_t stride, int n_valid) {
#pragma unroll
  for (int i = 0; i < ROWS * 16 / NTHREADS; ++i) {
    const int idx = threadIdx.x + i * NTHREADS;
    const int r = idx >> 4, c = idx & 15;
    const bool ok = r < n_valid;
    cp_async16(sm + swz(r, c * 8), ok ? base + (int64_t)r * stride + c * 8 : base, ok);
  }
}

struct Params {
  const bf16* q;
  int64_t q_row;      // element stride between tokens
  int64_t q_head;     // element stride between heads
  const bf16* k;
  const bf16* v;
  int64_t k_row, v_row;  // contiguous mode: token strides
  int64_t kv_head;       // contiguous mode: head strides
  bf16* o;
  int64_t o_row, o_head;
  float* lse;            // [nq, total_q] natural-log LSE (may be null)
  const int* cu_q;       // [B+1]
  const int* cu_k;       // contiguous mode: [B+1]
  const int* kv_lens;    // paged mode: [B]
  const int* block_table;  // paged mode: [B, max_blocks]
  int max_blocks;
  int num_blocks;        // paged mode: blocks in the cache (bounds checks)
  int block_size;
  int nq, nkv;
  float scale;
  int64_t lse_stride;    // = total_q
};

// Row pointer for key `key` of sequence b / kv head kvh.
template <bool PAGED>
__device__ __forceinline__ const bf16* krow(const Params& p, const bf16* base, int64_t row_stride, int b, int kvh,
                                            int key) {
  if constexpr (PAGED) {
    const int blk = p.block_table[(int64_t)b * p.max_blocks + key / p.block_size];
    if (!chk::in_range(blk, p.num_blocks, 62, b, key / p.block_size)) return nullptr;
    return base + (((int64_t)blk * p.nkv + kvh) * p.block_size + key % p.block_size) * D;
  } else {
    return base + ((int64_t)p.cu_k[b] + key) * row_stride + (int64_t)kvh * p.kv_head;
  }
}

// ---------------------------------------------------------------- forward
template <bool PAGED>
__global__ void __launch_bounds__(NTHREADS) attn_fwd_kernel(Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sK = sQ + BM * D;           // [2][BN][D]
  bf16* sV = sK + 2 * BN * D;       // [2][BN][D]
  __shared__ const bf16* rowp[BN];

  const int mb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = p.cu_q[b];
  const int q_len = p.cu_q[b + 1] - q0;
  if (mb * BM >= q_len) return;
  const int kv_len =
      PAGED ? chk::clamp_to(p.kv_lens[b], p.max_blocks * p.block_size, 61, b) : (p.cu_k[b + 1] - p.cu_k[b]);
  const int kvh = h / (p.nq / p.nkv);
  const int ctx_off = kv_len - q_len;  // absolute position of query 0
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Q tile
  load_rows<BM>(sQ, p.q + (int64_t)(q0 + mb * BM) * p.q_row + (int64_t)h * p.q_head, p.q_row,
                min(BM, q_len - mb * BM));
  cp_async_commit();

  const int q_hi = min(q_len, (mb + 1) * BM);           // exclusive
  const int k_end = min(kv_len, ctx_off + q_hi);        // keys needed
  const int n_tiles = (k_end + BN - 1) / BN;

  auto load_kv = [&](int t, int stage) {
    // the stage being refilled was last read before the previous iteration's
    // closing barrier
    if constexpr (!PAGED) {
      const int nk = min(BN, k_end - t * BN);
      const int64_t r0 = (int64_t)p.cu_k[b] + t * BN;
      load_rows<BN>(sK + stage * BN * D, p.k + r0 * p.k_row + (int64_t)kvh * p.kv_head, p.k_row, nk);
      load_rows<BN>(sV + stage * BN * D, p.v + r0 * p.v_row + (int64_t)kvh * p.kv_head, p.v_row, nk);
      return;
    } else {
      if (p.block_size % BN == 0) {
        // the tile sits in one cache block: one block-table lookup
        const int key0 = t * BN;
        int blk = p.block_table[(int64_t)b * p.max_blocks + key0 / p.block_size];
        int nk = min(BN, k_end - key0);
        if (!chk::in_range(blk, p.num_blocks, 62, b, key0 / p.block_size)) blk = nk = 0;
        const int64_t off = (((int64_t)blk * p.nkv + kvh) * p.block_size + key0 % p.block_size) * D;
        load_rows<BN>(sK + stage * BN * D, p.k + off, D, nk);
        load_rows<BN>(sV + stage * BN * D, p.v + off, D, nk);
        return;
      }
    }
    __syncthreads();
    if (threadIdx.x < BN) {
      const int key = t * BN + threadIdx.x;
      rowp[threadIdx.x] = key < k_end ? krow<PAGED>(p, p.k, p.k_row, b, kvh, key) : nullptr;
    }
    __syncthreads();
    load_tile<BN>(sK + stage * BN * D, rowp, p.k);
    __syncthreads();
    if (threadIdx.x < BN) {
      const int key = t * BN + threadIdx.x;
      rowp[threadIdx.x] = key < k_end ? krow<PAGED>(p, p.v, p.v_row, b, kvh, key) : nullptr;
    }
    __syncthreads();
    load_tile<BN>(sV + stage * BN * D, rowp, p.v);
  };

  if (n_tiles > 0) load_kv(0, 0);
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  // Q fragments: 8 k-steps x 4 regs
  uint32_t qf[8][4];
  {
    const int r = warp * 16 + (lane & 15);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = ks * 16 + (lane >> 4) * 8;
      ldsm_x4(qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], sQ + swz(r, c));
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
  const int qrow0 = mb * BM + warp * 16 + (lane >> 2);  // this thread's rows: qrow0, qrow0 + 8

  for (int t = 0; t < n_tiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < n_tiles) load_kv(t + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const bf16* k_s = sK + stage * BN * D;
    const bf16* v_s = sV + stage * BN * D;

    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(b0, b1, b2, b3, k_s + swz(r, c));
        mma16816(s[2 * np], qf[ks], b0, b1);
        mma16816(s[2 * np + 1], qf[ks], b2, b3);
      }
    }
    // mask + online softmax (base 2)
    const bool need_mask = (t + 1) * BN > ctx_off + mb * BM + warp * 16 || (t + 1) * BN > k_end;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[nt][e] * sl2;
        if (need_mask) {
          const int key = t * BN + nt * 8 + (lane & 3) * 2 + (e & 1);
          const int qpos = ctx_off + qrow0 + (e >> 1) * 8;
          if (key > qpos || key >= k_end) v = -INFINITY;
        }
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      corr[r] = (mx[r] == -INFINITY) ? 1.f : ex2(m_r[r] - mx[r]);
      m_r[r] = mx[r];
      l_r[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        pv[e] = (mm == -INFINITY) ? 0.f : ex2(s[nt][e] - mm);
        l_r[e >> 1] += pv[e];
      }
      const int ks = nt >> 1, hi = nt & 1;
      pf[ks][hi * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pf[ks][hi * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        const int r = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(b0, b1, b2, b3, v_s + swz(r, c));
        mma16816(o[2 * dp], pf[ks], b0, b1);
        mma16816(o[2 * dp + 1], pf[ks], b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = qrow0 + r * 8;
    if (row >= q_len) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    bf16* orow = p.o + (int64_t)(q0 + row) * p.o_row + (int64_t)h * p.o_head;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      const int c = dt * 8 + (lane & 3) * 2;
      *reinterpret_cast<bf162*>(orow + c) = __floats2bfloat162_rn(o[dt][r * 2] * inv, o[dt][r * 2 + 1] * inv);
    }
    if (p.lse && (lane & 3) == 0)
      p.lse[(int64_t)h * p.lse_stride + q0 + row] = (l_r[r] > 0.f) ? (m_r[r] + log2f(l_r[r])) / LOG2E : -INFINITY;
  }
}

// ---------------------------------------------------------------- backward
// D[t, h] = sum_d dO * O
__global__ void bwd_dot_kernel(const bf16* __restrict__ o, int64_t o_row, int64_t o_head, const bf16* __restrict__ dO,
                               int64_t do_row, int64_t do_head, float* __restrict__ Dout, int T, int nq) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= (int64_t)T * nq) return;
  const int t = warp / nq, h = warp % nq;
  const bf16* a = o + t * o_row + (int64_t)h * o_head;
  const bf16* g = dO + t * do_row + (int64_t)h * do_head;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) acc += to_f(a[lane * 4 + k]) * to_f(g[lane * 4 + k]);
  acc = warp_sum(acc);
  if (lane == 0) Dout[(int64_t)h * T + t] = acc;
}

struct BwdParams {
  Params f;            // q/k/v/cu as in forward (contiguous mode)
  const bf16* dO;
  int64_t do_row, do_head;
  const float* lse;    // [nq, T]
  const float* Dd;     // [nq, T]
  float* dq;           // [T, nq, D] fp32 accumulators
  float* dk;           // [T, nkv, D] fp32 accumulators (the GQA group is split over CTAs)
  float* dv;
  int B;               // sequences
  int64_t dkv_row;     // = nkv * D
  int T;
};

// One CTA = (key tile, half of the GQA group, kv head, sequence), numbered so
// that the longest CTAs (first key tiles: most causal query tiles) start first.
// It loops over its query heads and the causal query tiles; the next query
// tile's Q / dO / lse / D loads are issued as soon as the current tile's last
// reader of them is done (before the dQ product and its atomics), so the copy
// overlaps that work.  dK / dV of the two group halves meet in fp32 atomics.
constexpr int BWD_HSPLIT = 2;

__global__ void __launch_bounds__(NTHREADS) attn_bwd_kernel(BwdParams bp) {
  const Params& p = bp.f;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sK = reinterpret_cast<bf16*>(smem_raw);  // [BN][D]
  bf16* sV = sK + BN * D;                         // [BN][D]
  bf16* sQ = sV + BN * D;                         // [BM][D]
  bf16* sdO = sQ + BM * D;                        // [BM][D]
  bf16* sdS = sdO + BM * D;                       // [BN][BM] (keys x queries), swizzled as 64-wide rows
  __shared__ float sLse[BM], sDd[BM];

  int idx = blockIdx.x;
  const int b = idx % bp.B;
  idx /= bp.B;
  const int kvh = idx % p.nkv;
  idx /= p.nkv;
  const int hs = idx % BWD_HSPLIT;
  const int nb = idx / BWD_HSPLIT;
  const int s0 = p.cu_q[b];
  const int len = p.cu_q[b + 1] - s0;
  if (nb * BN >= len) return;
  const int grp_all = p.nq / p.nkv;
  const int per_split = (grp_all + BWD_HSPLIT - 1) / BWD_HSPLIT;
  const int h_first = kvh * grp_all + hs * per_split;
  const int grp = max(0, min(per_split, grp_all - hs * per_split));   // query heads of this CTA
  if (grp == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float sl2 = p.scale * LOG2E;

  // K, V tiles of this CTA
  const int nk = min(BN, len - nb * BN);
  load_rows<BN>(sK, p.k + (int64_t)(s0 + nb * BN) * p.k_row + (int64_t)kvh * p.kv_head, p.k_row, nk);
  load_rows<BN>(sV, p.v + (int64_t)(s0 + nb * BN) * p.v_row + (int64_t)kvh * p.kv_head, p.v_row, nk);
  cp_async_commit();

  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int key_row0 = nb * BN + warp * 16 + (lane >> 2);  // this thread's keys: key_row0, +8
  const int m_start = (nb * BN) / BM;                       // causal: first query tile touching this key tile
  const int m_tiles = (len + BM - 1) / BM;
  const int per_head = m_tiles - m_start;
  const int n_iter = grp * per_head;

  // issue the loads of iteration `it` (query head, query tile) into the single buffer
  auto issue = [&](int it) {
    const int h = h_first + it / per_head;
    const int mt = m_start + it % per_head;
    const int nq_valid = min(BM, len - mt * BM);
    load_rows<BM>(sQ, p.q + (int64_t)(s0 + mt * BM) * p.q_row + (int64_t)h * p.q_head, p.q_row, nq_valid);
    load_rows<BM>(sdO, bp.dO + (int64_t)(s0 + mt * BM) * bp.do_row + (int64_t)h * bp.do_head, bp.do_row,
                  nq_valid);
    cp_async_commit();
    if (threadIdx.x < BM) {
      const int q = mt * BM + threadIdx.x;
      sLse[threadIdx.x] = q < len ? bp.lse[(int64_t)h * bp.T + s0 + q] * LOG2E : INFINITY;
      sDd[threadIdx.x] = q < len ? bp.Dd[(int64_t)h * bp.T + s0 + q] : 0.f;
    }
  };
  if (n_iter > 0) issue(0);

  for (int it = 0; it < n_iter; ++it) {
    const int h = h_first + it / per_head;
    const int mt = m_start + it % per_head;
    cp_async_wait<0>();
    __syncthreads();   // Q / dO / lse / D of this iteration visible; sdS of the previous one consumed

    // S^T (16 keys x 64 queries per warp) = K Q^T
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], sK + swz(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, sQ + swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 16 + ((lane >> 3) & 1) * 8));
        mma16816(s[2 * np], a, b0, b1);
        mma16816(s[2 * np + 1], a, b2, b3);
      }
    }
    // P^T = exp2(S*scale*log2e - lse*log2e), causal mask (query >= key)
    uint32_t pf[4][4];
    float (&pval)[8][4] = s;  // P^T overwrites S^T
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + (lane & 3) * 2 + (e & 1);
        const int q = mt * BM + qi;
        const int key = key_row0 + (e >> 1) * 8;
        float pv = ex2(s[nt][e] * sl2 - sLse[qi]);
        if (q < key || q >= len || key >= len) pv = 0.f;
        pval[nt][e] = pv;
      }
      pf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(pval[nt][0], pval[nt][1]);
      pf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(pval[nt][2], pval[nt][3]);
    }
    // dV += P^T dO  (k = queries, n = d)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, sdO + swz(ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
        mma16816(dv[2 * dp], pf[ks], b0, b1);
        mma16816(dv[2 * dp + 1], pf[ks], b2, b3);
      }
    }
    // dP^T = V dO^T
    float dp_[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) dp_[i][0] = dp_[i][1] = dp_[i][2] = dp_[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      ldsm_x4(a[0], a[1], a[2], a[3], sV + swz(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b0, b1, b2, b3, sdO + swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 16 + ((lane >> 3) & 1) * 8));
        mma16816(dp_[2 * np], a, b0, b1);
        mma16816(dp_[2 * np + 1], a, b2, b3);
      }
    }
    // dS^T = P^T * (dP^T - D) * scale ; stage to smem as [keys][queries]
    uint32_t dsf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + (lane & 3) * 2 + (e & 1);
        ds[e] = pval[nt][e] * (dp_[nt][e] - sDd[qi]) * p.scale;
      }
      dsf[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(ds[0], ds[1]);
      dsf[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(ds[2], ds[3]);
      const int kr = warp * 16 + (lane >> 2);
      const int qc = nt * 8 + (lane & 3) * 2;
      // sdS rows are 64 wide (128 B): swizzle with 8 chunks
      const int o0 = kr * BM + ((((qc >> 3) ^ (kr & 7))) << 3) + (qc & 7);
      const int o1 = (kr + 8) * BM + ((((qc >> 3) ^ ((kr + 8) & 7))) << 3) + (qc & 7);
      *reinterpret_cast<uint32_t*>(sdS + o0) = dsf[nt >> 1][(nt & 1) * 2 + 0];
      *reinterpret_cast<uint32_t*>(sdS + o1) = dsf[nt >> 1][(nt & 1) * 2 + 1];
    }
    // dK += dS^T Q  (k = queries, n = d)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(b0, b1, b2, b3, sQ + swz(ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
        mma16816(dk[2 * dp], dsf[ks], b0, b1);
        mma16816(dk[2 * dp + 1], dsf[ks], b2, b3);
      }
    }
    __syncthreads();   // sQ / sdO / lse / D no longer read; sdS complete
    if (it + 1 < n_iter) issue(it + 1);
    // dQ (warp: 16 queries x 128 d) += dS K, with dS = (dS^T)^T read transposed from smem
    // two halves of the head dimension keep the dQ accumulator at 32 registers
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float dq[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // keys in steps of 16
        uint32_t a[4];
        // A = dS[q][key] (16 q x 16 keys) = transpose of sdS[key][q]
        {
          const int kr = ks * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int qc = warp * 16 + ((lane >> 3) & 1) * 8;
          const int off = kr * BM + ((((qc >> 3) ^ (kr & 7))) << 3);
          ldsm_x4_t(a[0], a[1], a[2], a[3], sdS + off);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int dp = half * 4 + j;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(b0, b1, b2, b3, sK + swz(ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
          mma16816(dq[2 * j], a, b0, b1);
          mma16816(dq[2 * j + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int q = mt * BM + warp * 16 + (lane >> 2) + r * 8;
        if (q >= len) continue;
        float* dst = bp.dq + ((int64_t)(s0 + q) * p.nq + h) * D + half * 64;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          const int c = dt * 8 + (lane & 3) * 2;
          atomicAdd(reinterpret_cast<float2*>(dst + c), make_float2(dq[dt][r * 2], dq[dt][r * 2 + 1]));
        }
      }
    }
  }
  // add this CTA's share of dK, dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key_row0 + r * 8;
    if (key >= len) continue;
    float* dkr = bp.dk + (int64_t)(s0 + key) * bp.dkv_row + (int64_t)kvh * D;
    float* dvr = bp.dv + (int64_t)(s0 + key) * bp.dkv_row + (int64_t)kvh * D;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      const int c = dt * 8 + (lane & 3) * 2;
      atomicAdd(reinterpret_cast<float2*>(dkr + c), make_float2(dk[dt][r * 2], dk[dt][r * 2 + 1]));
      atomicAdd(reinterpret_cast<float2*>(dvr + c), make_float2(dv[dt][r * 2], dv[dt][r * 2 + 1]));
    }
  }
}

// ---------------------------------------------------------------- decode
struct DecodeParams {
  const bf16* q;      // [B, nq, D], rows q_row elements apart (heads contiguous)
  int64_t q_row;
  const bf16* kc;     // [blocks, nkv, bs, D]
  const bf16* vc;
  const int* block_table;
  const int* kv_lens;
  int max_blocks, block_size, nq, nkv, splits;
  int num_blocks;     // blocks in the cache (bounds checks)
  float scale;
  bf16* o;            // [B, nq, D]
  float* part_o;      // [B, nq, splits, D]  (splits > 1)
  float* part_lse;    // [B, nq, splits]
};

// One CTA = (sequence, kv head, split). Warp w handles keys w*16..w*16+15 of each
// 64-key tile with its own online softmax; warps are merged at the end.
// K/V tiles stream through a DEC_STAGES-deep cp.async ring; every thread
// computes the paged address of the chunks it copies directly (no row table),
// so a tile costs one barrier.  The warp-merge area aliases the ring.
constexpr int DEC_STAGES = 2;   // default ring depth (x 3 resident CTAs per SM)

__device__ __forceinline__ void dec_load_tile(bf16* sm, const bf16* cache, const int* bt_row, int block_size,
                                              int nkv, int kvh, int key0, int k_end, int b, int num_blocks) {
  // BN rows x 16 chunks of 16 B; 128 threads -> 8 chunks each
  if (block_size % BN == 0) {
    // tiles start on multiples of BN, so the whole tile sits in one cache
    // block: one block-table lookup and no per-chunk division
    int blk = bt_row[key0 / block_size];
    if (!chk::in_range(blk, num_blocks, 64, b, key0 / block_size)) blk = -1;
    const bf16* base = cache + (((int64_t)(blk < 0 ? 0 : blk) * nkv + kvh) * block_size + key0 % block_size) * D;
#pragma unroll
    for (int i = 0; i < BN * 16 / NTHREADS; ++i) {
      const int idx = threadIdx.x + i * NTHREADS;
      const int r = idx >> 4, c = idx & 15;
      const bool ok = key0 + r < k_end && blk >= 0;
      cp_async16(sm + swz(r, c * 8), ok ? base + r * D + c * 8 : cache, ok);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < BN * 16 / NTHREADS; ++i) {
    const int idx = threadIdx.x + i * NTHREADS;
    const int r = idx >> 4, c = idx & 15;
    const int key = key0 + r;
    bool ok = key < k_end;
    const bf16* src = cache;
    if (ok) {
      const int blk = bt_row[key / block_size];
      ok = chk::in_range(blk, num_blocks, 64, b, key / block_size);
      if (ok) src = cache + (((int64_t)blk * nkv + kvh) * block_size + key % block_size) * D + c * 8;
    }
    cp_async16(sm + swz(r, c * 8), src, ok);
  }
}

template <int STAGES>
__device__ __forceinline__ void decode_body(const DecodeParams& p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);  // [16][D]
  bf16* sK = sQ + 16 * D;                         // [STAGES][BN][D]
  bf16* sV = sK + STAGES * BN * D;            // [STAGES][BN][D]
  float* sO = reinterpret_cast<float*>(sK);       // [NWARPS][16][D] merge area (after the loop)
  __shared__ float sM[NWARPS][16], sL[NWARPS][16];

  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int grp = p.nq / p.nkv;
  const int kv_len = chk::clamp_to(p.kv_lens[b], p.max_blocks * p.block_size, 63, b);
  const int per = (((kv_len + p.splits - 1) / p.splits) + BN - 1) / BN * BN;
  const int k_begin = split * per;
  const int k_end = min(kv_len, k_begin + per);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int* bt_row = p.block_table + (int64_t)b * p.max_blocks;

  // Q rows (grp <= 16), zero padded
#pragma unroll
  for (int i = 0; i < 16 * 16 / NTHREADS; ++i) {
    const int idx = threadIdx.x + i * NTHREADS;
    const int r = idx >> 4, c = idx & 15;
    const bool ok = r < grp;
    const bf16* src = ok ? p.q + (int64_t)b * p.q_row + (int64_t)(kvh * grp + r) * D + c * 8 : p.q;
    cp_async16(sQ + swz(r, c * 8), src, ok);
  }
  cp_async_commit();

  const int n_tiles = k_end > k_begin ? (k_end - k_begin + BN - 1) / BN : 0;
#pragma unroll
  for (int st = 0; st < STAGES - 1; ++st) {
    if (st < n_tiles) {
      dec_load_tile(sK + st * BN * D, p.kc, bt_row, p.block_size, p.nkv, kvh, k_begin + st * BN, k_end, b,
                    p.num_blocks);
      dec_load_tile(sV + st * BN * D, p.vc, bt_row, p.block_size, p.nkv, kvh, k_begin + st * BN, k_end, b,
                    p.num_blocks);
    }
    cp_async_commit();
  }
  cp_async_wait<STAGES - 1>();   // Q landed
  __syncthreads();

  uint32_t qf[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
    ldsm_x4(qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], sQ + swz(lane & 15, ks * 16 + (lane >> 4) * 8));

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;

  for (int t = 0; t < n_tiles; ++t) {
    const int stage = t % STAGES;
    cp_async_wait<STAGES - 2>();   // tile t landed (this thread's copies)
    __syncthreads();                   // ... and everyone's; stage (t-1) is free to refill
    {
      const int tn = t + STAGES - 1;
      if (tn < n_tiles) {
        const int sn = tn % STAGES;
        dec_load_tile(sK + sn * BN * D, p.kc, bt_row, p.block_size, p.nkv, kvh, k_begin + tn * BN, k_end, b,
                      p.num_blocks);
        dec_load_tile(sV + sn * BN * D, p.vc, bt_row, p.block_size, p.nkv, kvh, k_begin + tn * BN, k_end, b,
                      p.num_blocks);
      }
      cp_async_commit();
    }
    const bf16* k_s = sK + stage * BN * D;
    const bf16* v_s = sV + stage * BN * D;
    float s[2][4];
    s[0][0] = s[0][1] = s[0][2] = s[0][3] = 0.f;
    s[1][0] = s[1][1] = s[1][2] = s[1][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b0, b1, b2, b3;
      const int ar = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int c = ks * 16 + ((lane >> 3) & 1) * 8;
      ldsm_x4(b0, b1, b2, b3, k_s + swz(ar, c));
      mma16816(s[0], qf[ks], b0, b1);
      mma16816(s[1], qf[ks], b2, b3);
    }
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k_begin + t * BN + warp * 16 + nt * 8 + (lane & 3) * 2 + (e & 1);
        float v = key < k_end ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      corr[r] = (mx[r] == -INFINITY) ? 1.f : ex2(m_r[r] - mx[r]);
      m_r[r] = mx[r];
      l_r[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
    uint32_t pf[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        pv[e] = (mm == -INFINITY) ? 0.f : ex2(s[nt][e] - mm);
        l_r[e >> 1] += pv[e];
      }
      pf[nt * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pf[nt * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      uint32_t b0, b1, b2, b3;
      const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = dp * 16 + (lane >> 4) * 8;
      ldsm_x4_t(b0, b1, b2, b3, v_s + swz(r, c));
      mma16816(o[2 * dp], pf, b0, b1);
      mma16816(o[2 * dp + 1], pf, b2, b3);
    }
  }
  cp_async_wait<0>();
  __syncthreads();                     // ring no longer read: reuse it as the merge area
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  if ((lane & 3) == 0) {
    sM[warp][lane >> 2] = m_r[0];
    sM[warp][(lane >> 2) + 8] = m_r[1];
    sL[warp][lane >> 2] = l_r[0];
    sL[warp][(lane >> 2) + 8] = l_r[1];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = (lane >> 2) + r * 8;
    float mg = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) mg = fmaxf(mg, sM[w][row]);
    const float c = (m_r[r] == -INFINITY) ? 0.f : ex2(m_r[r] - mg);
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      const int col = dt * 8 + (lane & 3) * 2;
      sO[(warp * 16 + row) * D + col] = o[dt][r * 2] * c;
      sO[(warp * 16 + row) * D + col + 1] = o[dt][r * 2 + 1] * c;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < grp * D; idx += NTHREADS) {
    const int row = idx / D, col = idx % D;
    float mg = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) mg = fmaxf(mg, sM[w][row]);
    float lsum = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) {
      const float mw = sM[w][row];
      lsum += (mw == -INFINITY) ? 0.f : sL[w][row] * ex2(mw - mg);
      acc += sO[(w * 16 + row) * D + col];
    }
    const int hq = kvh * grp + row;
    if (p.splits == 1) {
      p.o[((int64_t)b * p.nq + hq) * D + col] = __float2bfloat16(lsum > 0.f ? acc / lsum : 0.f);
    } else {
      p.part_o[(((int64_t)b * p.nq + hq) * p.splits + split) * D + col] = lsum > 0.f ? acc / lsum : 0.f;
      if (col == 0)
        p.part_lse[((int64_t)b * p.nq + hq) * p.splits + split] = lsum > 0.f ? mg + log2f(lsum) : -INFINITY;
    }
  }
}

__global__ void __launch_bounds__(NTHREADS, 3) decode_kernel(DecodeParams p) { decode_body<DEC_STAGES>(p); }
// deeper ring (3 x 32 KB in flight per CTA) at 2 resident CTAs per SM
__global__ void __launch_bounds__(NTHREADS, 2) decode_kernel_s3(DecodeParams p) { decode_body<3>(p); }

__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                      bf16* __restrict__ o, int splits) {
  // one CTA (128 threads) per (b, head); lse in base 2
  const int64_t bh = blockIdx.x;
  const float* lse = part_lse + bh * splits;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, lse[s]);
  float den = 0.f, acc = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float w = (lse[s] == -INFINITY) ? 0.f : ex2(lse[s] - mx);
    den += w;
    acc += w * part_o[(bh * splits + s) * D + threadIdx.x];
  }
  o[bh * D + threadIdx.x] = __float2bfloat16(den > 0.f ? acc / den : 0.f);
}

}  // namespace attn

using namespace attn;

static size_t fwd_smem() { return (size_t)(BM * D + 4 * BN * D) * sizeof(bf16); }
static size_t bwd_smem() { return (size_t)(2 * BN * D + 2 * BM * D + BN * BM) * sizeof(bf16); }
static size_t dec_smem(int stages = DEC_STAGES) {
  // Q + K/V ring; the fp32 warp-merge area (NWARPS x 16 x D) aliases the ring
  const size_t ring = (size_t)(16 * D + 2 * stages * BN * D) * sizeof(bf16);
  const size_t merge = (size_t)16 * D * sizeof(bf16) + (size_t)NWARPS * 16 * D * sizeof(float);
  return ring > merge ? ring : merge;
}

// Varlen causal attention forward over contiguous q/k/v views.
// q: [T, nq, D] view, k/v: [T, nkv, D] views (token stride arbitrary, unit stride on D)
std::vector<at::Tensor> attn_varlen_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                        int64_t max_seqlen, double scale, bool want_lse) {
  CHECK_CUDA_TENSOR(q);
  TORCH_CHECK(q.size(-1) == D && q.stride(-1) == 1, "head_dim must be 128 with unit stride");
  const int T = q.size(0), nq = q.size(1), nkv = k.size(1);
  const int B = cu_seqlens.numel() - 1;
  at::cuda::CUDAGuard g(q.device());
  auto o = at::empty({T, nq, D}, q.options());
  auto lse = want_lse ? at::empty({nq, T}, q.options().dtype(at::kFloat)) : at::Tensor();
  if (T == 0 || B == 0) return {o, lse};
  for (const at::Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->stride(0) % 8 == 0 && t->stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "q/k/v rows and heads must start on 16-byte boundaries");
  Params p{};
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.q_row = q.stride(0);
  p.q_head = q.stride(1);
  p.k = reinterpret_cast<const bf16*>(k.data_ptr());
  p.v = reinterpret_cast<const bf16*>(v.data_ptr());
  p.k_row = k.stride(0);
  p.v_row = v.stride(0);
  TORCH_CHECK(k.stride(1) == v.stride(1), "k/v head strides must match");
  p.kv_head = k.stride(1);
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.o_row = nq * D;
  p.o_head = D;
  p.lse = want_lse ? lse.data_ptr<float>() : nullptr;
  p.lse_stride = T;
  p.cu_q = cu_seqlens.data_ptr<int>();
  p.cu_k = cu_seqlens.data_ptr<int>();
  p.nq = nq;
  p.nkv = nkv;
  p.scale = scale;
  const size_t sm = fwd_smem();
  ensure_smem_attr(attn_fwd_kernel<false>, (int)sm);
  dim3 grid((max_seqlen + BM - 1) / BM, nq, B);
  attn_fwd_kernel<false><<<grid, NTHREADS, sm, stream()>>>(p);
  PSRL_CHECK_LAUNCH();
  return {o, lse};
}

// Chunked prefill against the paged cache (new K/V already written to the cache).
at::Tensor attn_paged_prefill(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor cu_q,
                              at::Tensor kv_lens, at::Tensor block_table, int64_t max_q_len, double scale) {
  CHECK_CUDA_TENSOR(q);
  TORCH_CHECK(q.size(-1) == D && q.stride(-1) == 1, "head_dim must be 128");
  const int T = q.size(0), nq = q.size(1), nkv = k_cache.size(1);
  const int B = cu_q.numel() - 1;
  at::cuda::CUDAGuard g(q.device());
  auto o = at::empty({T, nq, D}, q.options());
  if (T == 0 || B == 0) return o;
  TORCH_CHECK(q.stride(0) % 8 == 0 && q.stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "q rows and heads must start on 16-byte boundaries");
  Params p{};
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.q_row = q.stride(0);
  p.q_head = q.stride(1);
  p.k = reinterpret_cast<const bf16*>(k_cache.data_ptr());
  p.v = reinterpret_cast<const bf16*>(v_cache.data_ptr());
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.o_row = nq * D;
  p.o_head = D;
  p.cu_q = cu_q.data_ptr<int>();
  p.kv_lens = kv_lens.data_ptr<int>();
  p.block_table = block_table.data_ptr<int>();
  p.max_blocks = block_table.size(1);
  p.num_blocks = k_cache.size(0);
  p.block_size = k_cache.size(2);
  p.nq = nq;
  p.nkv = nkv;
  p.scale = scale;
  const size_t sm = fwd_smem();
  ensure_smem_attr(attn_fwd_kernel<true>, (int)sm);
  dim3 grid((max_q_len + BM - 1) / BM, nq, B);
  attn_fwd_kernel<true><<<grid, NTHREADS, sm, stream()>>>(p);
  PSRL_CHECK_LAUNCH();
  return o;
}

// Backward. Returns {dq (bf16 [T,nq,D]), dk, dv ([T,nkv,D])}.
std::vector<at::Tensor> attn_varlen_bwd(at::Tensor dO, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                                        at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale) {
  const int T = q.size(0), nq = q.size(1), nkv = k.size(1);
  const int B = cu_seqlens.numel() - 1;
  at::cuda::CUDAGuard g(q.device());
  auto dq = at::zeros({T, nq, D}, q.options().dtype(at::kFloat));
  auto dk = at::zeros({T, nkv, D}, q.options().dtype(at::kFloat));
  auto dv = at::zeros({T, nkv, D}, q.options().dtype(at::kFloat));
  auto Dd = at::empty({nq, T}, q.options().dtype(at::kFloat));
  if (T == 0 || B == 0) return {dq.to(at::kBFloat16), dk.to(at::kBFloat16), dv.to(at::kBFloat16)};
  TORCH_CHECK(dO.stride(-1) == 1 && o.stride(-1) == 1, "dO/O need unit stride on D");
  // rows are copied in 16-byte chunks
  for (const at::Tensor* t : {&q, &k, &v, &dO})
    TORCH_CHECK(t->stride(0) % 8 == 0 && t->stride(1) % 8 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "q/k/v/dO rows and heads must start on 16-byte boundaries");
  {
    const int64_t warps = (int64_t)T * nq;
    bwd_dot_kernel<<<(warps * 32 + 255) / 256, 256, 0, stream()>>>(
        reinterpret_cast<const bf16*>(o.data_ptr()), o.stride(0), o.stride(1),
        reinterpret_cast<const bf16*>(dO.data_ptr()), dO.stride(0), dO.stride(1), Dd.data_ptr<float>(), T, nq);
    PSRL_CHECK_LAUNCH();
  }
  BwdParams bp{};
  Params& p = bp.f;
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.q_row = q.stride(0);
  p.q_head = q.stride(1);
  p.k = reinterpret_cast<const bf16*>(k.data_ptr());
  p.v = reinterpret_cast<const bf16*>(v.data_ptr());
  p.k_row = k.stride(0);
  p.v_row = v.stride(0);
  p.kv_head = k.stride(1);
  p.cu_q = cu_seqlens.data_ptr<int>();
  p.cu_k = cu_seqlens.data_ptr<int>();
  p.nq = nq;
  p.nkv = nkv;
  p.scale = scale;
  bp.dO = reinterpret_cast<const bf16*>(dO.data_ptr());
  bp.do_row = dO.stride(0);
  bp.do_head = dO.stride(1);
  bp.lse = lse.data_ptr<float>();
  bp.Dd = Dd.data_ptr<float>();
  bp.dq = dq.data_ptr<float>();
  bp.dk = dk.data_ptr<float>();
  bp.dv = dv.data_ptr<float>();
  bp.dkv_row = (int64_t)nkv * D;
  bp.T = T;
  bp.B = B;
  const size_t sm = bwd_smem();
  ensure_smem_attr(attn_bwd_kernel, (int)sm);
  const int64_t nblk = (int64_t)((max_seqlen + BN - 1) / BN) * BWD_HSPLIT * nkv * B;
  attn_bwd_kernel<<<(unsigned)nblk, NTHREADS, sm, stream()>>>(bp);
  PSRL_CHECK_LAUNCH();
  return {dq.to(at::kBFloat16), dk.to(at::kBFloat16), dv.to(at::kBFloat16)};
}

int64_t decode_num_splits(int64_t batch, int64_t nkv, int64_t max_ctx) {
  // Split a sequence's keys only while there is less than one CTA per SM (a
  // split adds a combine pass and partial-result traffic; measured on B200 the
  // unsplit 3-stage kernel wins from one CTA per SM on); every split keeps at
  // least 4 key tiles.
  const int64_t ctas = std::max<int64_t>(1, batch * nkv);
  const int64_t target = num_sms();
  int64_t s = (target + ctas - 1) / ctas;
  s = std::min<int64_t>(s, std::max<int64_t>(1, (max_ctx + 4 * BN - 1) / (4 * BN)));
  return std::max<int64_t>(1, std::min<int64_t>(s, 32));
}

// Paged decode. q: [B, nq, D] contiguous. `scratch` (optional) is a float buffer of
// at least B*nq*splits*(D+1) elements used when splits > 1.
at::Tensor attn_decode(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_table,
                       at::Tensor kv_lens, double scale, int64_t splits, c10::optional<at::Tensor> scratch,
                       int64_t stages) {
  CHECK_CUDA_TENSOR(q);
  TORCH_CHECK(q.dim() == 3 && q.size(-1) == D, "q must be [B, heads, 128]");
  // rows may be strided (q viewed out of the fused qkv projection); heads and
  // head dims must be contiguous and every row 16-byte aligned
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == D && q.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "q rows must hold contiguous heads and start 16-byte aligned");
  const int B = q.size(0), nq = q.size(1), nkv = k_cache.size(1);
  TORCH_CHECK(nq % nkv == 0 && nq / nkv <= 16, "GQA group must be <= 16");
  at::cuda::CUDAGuard g(q.device());
  auto o = at::empty({B, nq, D}, q.options());
  if (B == 0) return o;
  DecodeParams p{};
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.q_row = q.stride(0);
  p.kc = reinterpret_cast<const bf16*>(k_cache.data_ptr());
  p.vc = reinterpret_cast<const bf16*>(v_cache.data_ptr());
  p.block_table = block_table.data_ptr<int>();
  p.kv_lens = kv_lens.data_ptr<int>();
  p.max_blocks = block_table.size(1);
  p.num_blocks = k_cache.size(0);
  p.block_size = k_cache.size(2);
  p.nq = nq;
  p.nkv = nkv;
  p.splits = (int)splits;
  p.scale = scale;
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  at::Tensor buf;
  if (splits > 1) {
    const int64_t need = (int64_t)B * nq * splits * (D + 1);
    if (scratch.has_value() && scratch->numel() >= need) {
      buf = scratch.value();
    } else {
      buf = at::empty({need}, q.options().dtype(at::kFloat));
    }
    p.part_o = buf.data_ptr<float>();
    p.part_lse = p.part_o + (int64_t)B * nq * splits * D;
  }
  // ring depth: 3 stages x 2 CTAs/SM (default; 0.86-0.92 of copy bandwidth at
  // rollout shapes) or 2 stages x 3 CTAs/SM (stages == 2)
  const int st = stages == 2 ? 2 : 3;
  const size_t sm = dec_smem(st);
  ensure_smem_attr(st == 3 ? decode_kernel_s3 : decode_kernel, (int)sm);
  dim3 grid(B, nkv, splits);
  if (st == 3)
    decode_kernel_s3<<<grid, NTHREADS, sm, stream()>>>(p);
  else
    decode_kernel<<<grid, NTHREADS, sm, stream()>>>(p);
  PSRL_CHECK_LAUNCH();
  if (splits > 1) {
    decode_combine_kernel<<<B * nq, D, 0, stream()>>>(p.part_o, p.part_lse, p.o, (int)splits);
    PSRL_CHECK_LAUNCH();
  }
  return o;
}

}  // namespace psrl

// ------------------------------------------------------------------------------
// Allocation-free variant of the paged decode entry point (declared in
// noalloc.h, which documents the contract).  It has no counterpart in the
// reference.  It reuses decode_kernel / decode_combine_kernel unchanged; only the
// split scratch comes from the file-scope array below instead of a caller-
// or torch-allocated buffer.
#include <mutex>

#include "noalloc.h"

namespace psrl {
namespace attn {

constexpr long long NOALLOC_SCRATCH_FLOATS = PSRL_NOALLOC_SCRATCH_BYTES / 4;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];

constexpr int NOALLOC_MAX_DEVICES = 64;
static float* g_noalloc_ptr[NOALLOC_MAX_DEVICES];  // device address of the scratch, per device
static std::mutex g_noalloc_mu;

// Once per device, with that device current: resolve the scratch array's device
// address (in host code its name is only a host-side stand-in) and allow the
// decode kernel its dynamic shared memory.
static int noalloc_setup(int dev, float** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return PSRL_NOALLOC_ECUDA;
    if (cudaFuncSetAttribute(decode_kernel_s3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec_smem(3)) !=
        cudaSuccess)
      return PSRL_NOALLOC_ECUDA;
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PSRL_NOALLOC_OK;
}

}  // namespace attn
}  // namespace psrl

extern "C" __attribute__((visibility("default"))) int psrl_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_table, const int* kv_lens, void* out,
    int batch, int num_heads, int num_kv_heads, int head_dim, int block_size, int max_blocks, int splits,
    float scale, void* stream) {
  using namespace psrl;
  using namespace psrl::attn;
  if (!q || !k_cache || !v_cache || !block_table || !kv_lens || !out) return PSRL_NOALLOC_EBADARG;
  // the kernel moves q, K, V and out in 16-byte vectors
  const uintptr_t misalign = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
                             reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out);
  if (misalign % 16 != 0) return PSRL_NOALLOC_EBADARG;
  if (head_dim != D || batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0 ||
      num_heads / num_kv_heads > 16 || block_size <= 0 || max_blocks <= 0 || splits < 1 || splits > 32)
    return PSRL_NOALLOC_EBADARG;
  const long long need = splits > 1 ? (long long)batch * num_heads * splits * (D + 1) : 0;
  if (need > NOALLOC_SCRATCH_FLOATS) return PSRL_NOALLOC_ETOOBIG;
  if (batch == 0) return PSRL_NOALLOC_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES) return PSRL_NOALLOC_ECUDA;
  float* scratch = nullptr;
  int rc = noalloc_setup(dev, &scratch);
  if (rc != PSRL_NOALLOC_OK) return rc;
  DecodeParams p{};
  p.q = static_cast<const bf16*>(q);
  p.q_row = (int64_t)num_heads * D;
  p.kc = static_cast<const bf16*>(k_cache);
  p.vc = static_cast<const bf16*>(v_cache);
  p.block_table = block_table;
  p.kv_lens = kv_lens;
  p.max_blocks = max_blocks;
  p.num_blocks = 0x7fffffff;  // the C entry point does not take the cache's size
  p.block_size = block_size;
  p.nq = num_heads;
  p.nkv = num_kv_heads;
  p.splits = splits;
  p.scale = scale;
  p.o = static_cast<bf16*>(out);
  if (splits > 1) {
    p.part_o = scratch;
    p.part_lse = scratch + (long long)batch * num_heads * splits * D;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  decode_kernel_s3<<<dim3(batch, num_kv_heads, splits), NTHREADS, dec_smem(3), st>>>(p);
  if (cudaPeekAtLastError() != cudaSuccess) return PSRL_NOALLOC_ECUDA;
  if (splits > 1) {
    decode_combine_kernel<<<batch * num_heads, D, 0, st>>>(p.part_o, p.part_lse, p.o, splits);
    if (cudaPeekAtLastError() != cudaSuccess) return PSRL_NOALLOC_ECUDA;
  }
  return PSRL_NOALLOC_OK;
}
