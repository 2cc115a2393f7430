// An entry point for callers that cannot allocate device memory.
//
// This has no counterpart in the reference: its runtime allocates through its device library
// wherever it likes. It exists for hosts of this library that run under a fixed memory plan:
// code inside a CUDA-graph capture or a pre-sized arena, plug-ins of a serving process whose
// memory pool is owned by somebody else, and processes whose device memory is already handed
// out in full, where a cudaMalloc (by this library, or by torch on its behalf) either fails or
// breaks the owner's accounting.
//
// ttb_paged_attention_decode_noalloc is the split-KV decode attention of attention_mma.cu (one
// new token per request, keys and values read from cache pages through a block table) with its
// scratch memory (the float32 partial results of the key splits) taken from a fixed array that
// lives in the library image instead of from the caller or an allocator. It calls no cudaMalloc,
// no cudaFree and no allocating library routine. The caller passes inputs and outputs, as for
// ttb_paged_attention_mma.
//
// The array holds TTB_NOALLOC_SCRATCH_BYTES (16 MiB) on every GPU whose context loads this
// library, until the process ends. A call needs
//     segments * heads * num_splits * (head_dim + 2) * 4   bytes
// of it and is refused with TTB_ERR_SCRATCH (-4) if that is more; ttb_noalloc_scratch_bytes()
// returns the limit. (64 requests x 32 heads x 16 splits x head size 64 need 8.25 MiB.)
//
// The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
// that device current) and sets the kernel's shared-memory limit; make that first call outside
// any stream capture. Later calls only launch kernels on `stream`.
//
// All calls on a device share the one array: two calls whose kernels may overlap on the GPU
// (different streams, no dependency between them) race on it and give wrong results; order them.
// The array keeps whatever the last call left. Nothing in it has to start at zero: every slot
// that the merge step reads was written by the split kernels of the same call.
#pragma once
#include <cuda_runtime.h>

#define TTB_NOALLOC_SCRATCH_BYTES (16u << 20)
#define TTB_ERR_SCRATCH (-4)

#ifdef __cplusplus
extern "C" {
#endif

// qkv: bfloat16 [segments, q_row_stride], queries first; out: bfloat16 [segments, heads * head_dim];
// cu_seqlens: int32 [segments + 1] = 0, 1, 2, ...; seg_pos0: int32 [segments], the position of each
// request's new token (= keys already cached); pages: bfloat16 [num_pages, kv_heads, page_size, head_dim];
// block_table: int32 [segments, table_width]. head_dim 64 or 128, heads / kv_heads <= 16.
// Returns 0, a negative TTB_ERR_* code, or a positive cudaError_t.
int ttb_paged_attention_decode_noalloc(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                       const int* seg_pos0, const void* key_pages, const void* value_pages,
                                       const int* block_table, int table_width, int page_size, int segments,
                                       int heads, int kv_heads, int head_dim, float scale, int window,
                                       int num_splits, cudaStream_t stream);

unsigned int ttb_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
