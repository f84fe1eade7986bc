// Debug-build bounds checks for indices that kernels take from their inputs.
//
// A build with PSRL_KERNEL_CHECKS=1 (setup.py passes -DPSRL_KERNEL_CHECKS=1
// when the variable is set) compiles range checks into the kernels that
// index memory through caller-supplied tables: paged-KV block tables and
// sequence lengths (attention.cu), copy segments (ipc.cu), optimizer shard
// offsets (peer_optim.cu) and KV block moves (kv_copy.cu).  A failing check
// records (code, four ints of context, count) in a device-side record and
// SKIPS the access it guards — nothing traps, so the context stays usable and
// the host reads the record with kernel_check_status().  In a regular build
// the checks compile to nothing.
//
// Error codes, with the record's four context ints:
//   61  paged prefill: kv_len above max_blocks * block_size   (b, kv_len, cap, 0)
//   62  paged prefill: block id out of range                  (b, slot, blk, num_blocks)
//   63  decode: kv_len above max_blocks * block_size          (b, kv_len, cap, 0)
//   64  decode: block id out of range                         (b, slot, blk, num_blocks)
//   65  peer copies: destination out of range                 (segment, 0 copy_segments | 1 scatter_segments
//                                                              | 2 copy_rows, index, bound)
//   66  peer optimizer: shard offset out of range             (bucket, 0 reduce | 1 update, off, numel)
//   67  kv_copy_blocks: block id out of range                 (pair, 0 src | 1 dst, blk, blocks)
// (values above 2^31 - 1 are reported truncated)
#pragma once

#include <vector>

#include "common.cuh"

namespace psrl {
namespace chk {

#if defined(PSRL_KERNEL_CHECKS) && PSRL_KERNEL_CHECKS
constexpr bool kOn = true;
#else
constexpr bool kOn = false;
#endif

constexpr int REC = 6;  // code, a, b, c, d, number of failed checks

// One record per translation unit (no relocatable device code); the host
// reads every unit's record through the registered readers below.
static __device__ int g_rec[REC];

static __device__ __noinline__ void record(int code, int a, int b, int c, int d) {
  atomicAdd(&g_rec[5], 1);
  if (atomicCAS(&g_rec[0], 0, code) == 0) {
    g_rec[1] = a;
    g_rec[2] = b;
    g_rec[3] = c;
    g_rec[4] = d;
  }
}

// true when 0 <= v < n (always true in a regular build); otherwise records
// (code, a, b, v, n) and returns false so the caller skips the access.
static __device__ __forceinline__ bool in_range(long long v, long long n, int code, int a, int b) {
  if constexpr (!kOn) {
    return true;
  } else {
    if (v >= 0 && v < n) return true;
    record(code, a, b, (int)v, (int)(n > 0x7fffffffLL ? 0x7fffffff : n));
    return false;
  }
}

// clamps v to cap (a checks build records the overflow first)
static __device__ __forceinline__ int clamp_to(int v, int cap, int code, int a) {
  if constexpr (!kOn) {
    return v;
  } else {
    if (v <= cap) return v;
    record(code, a, v, cap, 0);
    return cap;
  }
}

using Reader = void (*)(int* out, bool clear);
inline std::vector<Reader>& readers() {
  static std::vector<Reader> r;
  return r;
}
inline bool add_reader(Reader r) {
  readers().push_back(r);
  return true;
}

static void read_unit(int* out, bool clear) {
  PSRL_CHECK_CUDA(cudaMemcpyFromSymbol(out, g_rec, sizeof(int) * REC));
  if (clear) {
    const int zero[REC] = {0, 0, 0, 0, 0, 0};
    PSRL_CHECK_CUDA(cudaMemcpyToSymbol(g_rec, zero, sizeof(zero)));
  }
}
static const bool unit_registered = kOn && add_reader(&read_unit);

}  // namespace chk
}  // namespace psrl
