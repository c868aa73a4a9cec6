// Allocation-free C entry point for the paged split-K attention kernel.
//
// This entry point has no counterpart in the reference engine; it exists for callers that
// cannot allocate GPU memory themselves: code running inside a CUDA-graph-captured region that
// must not touch an allocator, plugins embedded in a host framework that owns every device
// allocation, and C callers that link this library without PyTorch's caching allocator.
// Those callers pass their inputs and outputs; the kernel's split-K scratch (partial maxima,
// sums and value accumulators of every split) lives in a file-scope device array inside the
// library instead of coming from cudaMalloc or PyTorch.
//
// Limits and behaviour:
//   * The scratch array is QB_ATTN_NOALLOC_SCRATCH_BYTES (16 MiB) per device. Every GPU that
//     loads the library holds it until the process exits. A call needing more,
//     num_rows * nq * splits * (head_dim + 2) * 4 bytes, is rejected with
//     QB_NOALLOC_ERR_TOO_LARGE before anything is launched.
//   * The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current). Make that first call before any stream
//     capture begins.
//   * All calls on a device share the one array, and it keeps whatever the last call wrote.
//     Calls whose kernels can overlap on the GPU (different streams without ordering between
//     them) race on the scratch and must be serialised by the caller.
//   * Nothing in this path calls cudaMalloc, cudaFree or any allocating library routine.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#define QB_ATTN_NOALLOC_SCRATCH_BYTES (16u << 20)
#define QB_NOALLOC_OK 0
#define QB_NOALLOC_ERR_TOO_LARGE (-2)
#define QB_NOALLOC_ERR_ARGS (-3)
#define QB_NOALLOC_ERR_SYMBOL (-4)
// Query heads per KV head handled by one CTA of the split kernel (4 warps x 4 heads).
#define QB_NOALLOC_MAX_GQA_GROUP 16

#ifdef __cplusplus
extern "C" {
#endif

// Causal GQA attention of `num_rows` query rows over a paged bf16 KV cache, split over the
// context in `splits` parts that are combined in a second kernel. Arguments match
// qb::attention_varlen: q [rows, nq, head_dim] bf16; k_cache/v_cache [pool_rows, nkv, head_dim]
// bf16; block_table [lanes, max_blocks] int32; positions [rows] int32 (absolute position of each
// query row, causal context is 0..position); seg_lane [segments] and cu [segments + 1] int32
// describe which lane each row belongs to; out [rows, nq, head_dim] bf16.
// Returns one of:
//   QB_NOALLOC_OK             launched (or nothing to do when num_rows == 0);
//   QB_NOALLOC_ERR_TOO_LARGE  splits > 1 and the scratch the call needs exceeds the array;
//   QB_NOALLOC_ERR_ARGS       a bad argument: num_rows < 0, num_segments <= 0, nq or nkv <= 0,
//                             nq % nkv != 0, nq / nkv > QB_NOALLOC_MAX_GQA_GROUP (16),
//                             head_dim not 64, 128 or 256, block_size <= 0, splits outside 1..64,
//                             or a current device index >= 64;
//   QB_NOALLOC_ERR_SYMBOL     the scratch array's device address could not be looked up;
//   a positive cudaError_t    the launch failed (the value of cudaGetLastError()).
// Nothing is launched on any of the negative codes.
int qb_attention_varlen_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                                int max_blocks, const int* positions, const int* seg_lane, const int* cu,
                                int num_segments, int num_rows, int nq, int nkv, int head_dim, int block_size,
                                int splits, void* out, cudaStream_t stream);

// Size of the per-device scratch array, in bytes.
size_t qb_attention_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
