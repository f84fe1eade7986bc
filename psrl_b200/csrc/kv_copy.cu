// Paged KV-cache block moves (K18): gather/scatter blocks between two paged
// layouts whose per-layer base pointers may live in this GPU's HBM, in another
// GPU's HBM (an IPC mapping, read over NVLink) or in pinned host memory (UVA
// mapped, moved over the host link).  One CTA copies one (layer, block) pair
// with 16-byte vector accesses.
#include "checks.cuh"
#include "common.cuh"

namespace psrl {

__global__ void kv_copy_blocks_kernel(const uint64_t* __restrict__ src_layers, const uint64_t* __restrict__ dst_layers,
                                      const int* __restrict__ src_blk, const int* __restrict__ dst_blk, int n_pairs,
                                      int64_t block_vecs, int64_t src_blocks, int64_t dst_blocks) {
  const int pair = blockIdx.x % n_pairs;
  const int layer = blockIdx.x / n_pairs;
  if (!chk::in_range(src_blk[pair], src_blocks, 67, pair, 0) || !chk::in_range(dst_blk[pair], dst_blocks, 67, pair, 1))
    return;
  const uint4* src = reinterpret_cast<const uint4*>(src_layers[layer]) + (int64_t)src_blk[pair] * block_vecs;
  uint4* dst = reinterpret_cast<uint4*>(dst_layers[layer]) + (int64_t)dst_blk[pair] * block_vecs;
  for (int64_t i = threadIdx.x; i < block_vecs; i += blockDim.x) dst[i] = src[i];
}

// src_layers / dst_layers: int64 tensors (on this device) of base addresses, one per
// layer-tensor (K and V of every layer); src_blk / dst_blk: int32 block ids;
// src_blocks / dst_blocks: blocks per layer-tensor on each side (0 = unknown),
// used by the bounds checks of a checks build.
void kv_copy_blocks(at::Tensor src_layers, at::Tensor dst_layers, at::Tensor src_blk, at::Tensor dst_blk,
                    int64_t block_bytes, int64_t src_blocks, int64_t dst_blocks) {
  CHECK_CUDA_TENSOR(src_layers);
  TORCH_CHECK(src_layers.numel() == dst_layers.numel(), "layer lists differ");
  TORCH_CHECK(src_blk.numel() == dst_blk.numel(), "block lists differ");
  TORCH_CHECK(block_bytes % 16 == 0, "block bytes must be a multiple of 16");
  const int n_pairs = src_blk.numel();
  const int n_layers = src_layers.numel();
  if (n_pairs == 0 || n_layers == 0) return;
  at::cuda::CUDAGuard g(src_layers.device());
  kv_copy_blocks_kernel<<<n_pairs * n_layers, 256, 0, stream()>>>(
      reinterpret_cast<const uint64_t*>(src_layers.data_ptr<int64_t>()),
      reinterpret_cast<const uint64_t*>(dst_layers.data_ptr<int64_t>()), src_blk.data_ptr<int>(),
      dst_blk.data_ptr<int>(), n_pairs, block_bytes / 16, src_blocks > 0 ? src_blocks : INT64_MAX,
      dst_blocks > 0 ? dst_blocks : INT64_MAX);
  PSRL_CHECK_LAUNCH();
}

}  // namespace psrl
