// Allocation-free paged decode attention: C entry point.
//
// This entry point has no counterpart in the reference; it exists for callers
// of this library that cannot allocate GPU memory while they run.  Examples:
// an inference server or plugin embedded in another runtime that reserves all
// device memory up front and forbids cudaMalloc from foreign code, and
// latency-critical loops where a cudaMalloc/cudaFree (which may synchronise the
// device) is not acceptable.  Such callers pass only their own input and output
// buffers; the intermediate per-split results live in a fixed scratch array
// compiled into the library (PSRL_NOALLOC_SCRATCH_BYTES, 16 MiB) that every GPU
// loading the library holds until the process exits.
//
// Contract:
//  * q, k_cache, v_cache and out start on 16-byte boundaries (the kernel moves
//    them in 16-byte vectors); a misaligned pointer is rejected with
//    PSRL_NOALLOC_EBADARG.  num_heads > 0, num_kv_heads > 0 and divides it, at
//    most 16 query heads per KV head.
//  * q          [batch, num_heads, 128] bf16, contiguous
//  * k_cache,
//    v_cache    [num_blocks, num_kv_heads, block_size, 128] bf16
//  * block_table[batch, max_blocks] int32;  kv_lens [batch] int32 (context length
//               including the current token)
//  * The caller guarantees, for every b, 1 <= kv_lens[b] <= max_blocks * block_size
//    and that the first ceil(kv_lens[b] / block_size) entries of block_table row b
//    are valid block indices of the caches.  These arrays live on the device and
//    are not read by the host, so the call cannot check them; a longer context
//    or a bad block index reads outside the caches.
//  * out        [batch, num_heads, 128] bf16 (written)
//  * splits     number of KV splits (1..32); with splits > 1 the call needs
//               batch * num_heads * splits * 129 floats of scratch, which must
//               not exceed PSRL_NOALLOC_SCRATCH_BYTES / 4; larger requests are
//               rejected with PSRL_NOALLOC_ETOOBIG before anything is launched.
//  * stream     cudaStream_t to launch on (may be 0).
//  * The first call on a device looks up the scratch array's device address
//    (cudaGetSymbolAddress) and sets the kernel's shared-memory limit, with that
//    device current; make that first call before any stream capture.
//  * Every call on a device shares the one scratch array and leaves the last
//    call's partial results in it.  Each call overwrites every scratch element it
//    reads, so nothing has to start at zero, but calls that overlap on the GPU
//    (concurrent streams, or another thread's launches) race on the scratch:
//    serialise them.
//  * The function calls no cudaMalloc, cudaFree or allocating library routine.
//  * Returns PSRL_NOALLOC_OK (0) or one of the error codes below.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define PSRL_NOALLOC_SCRATCH_BYTES (16ll * 1024 * 1024)
#define PSRL_NOALLOC_OK 0
#define PSRL_NOALLOC_EBADARG 1
#define PSRL_NOALLOC_ETOOBIG 2
#define PSRL_NOALLOC_ECUDA 3

__attribute__((visibility("default"))) int psrl_decode_attention_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_table, const int* kv_lens, void* out,
    int batch, int num_heads, int num_kv_heads, int head_dim, int block_size, int max_blocks, int splits,
    float scale, void* stream);

#ifdef __cplusplus
}
#endif
