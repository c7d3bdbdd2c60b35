// C entry point of the paged-attention decode that allocates no device memory.
//
// It has no counterpart in the reference, whose attention always obtains its
// workspaces from PyTorch.  It exists for callers that cannot allocate:
//   * host code outside PyTorch (a C or C++ runtime embedding this library's
//     kernels), which has no caching allocator to ask;
//   * a serving process that handed all free HBM to its KV cache at start-up,
//     where a cudaMalloc in the middle of a decode step can fail or stall.
// Its split-KV partials live in one fixed device array compiled into the
// library (ISB_NOALLOC_SCRATCH_BYTES); shapes that need more are rejected.
//
// Sharing: every call on a device uses that same array.  Calls whose GPU work
// overlaps (unordered streams, several host threads) race on it; issue them on
// one stream or order them.  No byte of the array has to start at zero: each
// call writes every partial it later reads.
//
// Set-up: the first call on each device (with that device current) looks up
// the array's address with cudaGetSymbolAddress and sets the kernels' shared
// memory attributes.  Make that first call, or call isb_noalloc_setup(), before
// any CUDA stream capture begins.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ISB_NOALLOC_SCRATCH_BYTES (16u << 20)
// Block-table width limit: one grid slice per 64-token chunk, at most 65535 slices.
#define ISB_NOALLOC_MAX_BLOCKS (65535 / 4)

enum {
  ISB_NOALLOC_OK = 0,
  ISB_NOALLOC_ETOOBIG = 1,      // partials need more than ISB_NOALLOC_SCRATCH_BYTES
  ISB_NOALLOC_EUNSUPPORTED = 2, // (head_dim, q heads per kv head) without a kernel
  ISB_NOALLOC_EINVAL = 3,       // null pointer or non-positive size
  ISB_NOALLOC_ESETUP = 4,       // symbol lookup or kernel attribute call failed
  ISB_NOALLOC_ELAUNCH = 5,      // kernel launch reported an error
  ISB_NOALLOC_EPENDING = 6,     // a CUDA error from the caller's earlier work was pending (left
                                // for the caller to read); nothing was launched
};

// Bytes of scratch one call with these sizes uses (partial outputs + softmax stats).
size_t isb_attention_decode_noalloc_scratch_bytes(int batch, int num_q_heads, int head_dim, int max_blocks);

// Per-device set-up; runs on the current device.  Returns ISB_NOALLOC_OK or ISB_NOALLOC_ESETUP.
int isb_noalloc_setup(void);

// Decode attention of one new token per sequence over the paged KV cache.
//   q            [batch, num_q_heads, head_dim] bf16 (normed, rotated)
//   gate         [batch, num_q_heads * head_dim] bf16 sigmoid output gate, or NULL
//   k_cache/v_cache [num_blocks, num_kv_heads, 256, head_dim] bf16
//   ctx_lens     [batch] int32 tokens visible to each sequence (new token included);
//                each must be <= max_blocks * 256.  A longer context is cut to the
//                block table's pages and sets 0x2 in the error word below.
//                max_blocks <= ISB_NOALLOC_MAX_BLOCKS and batch <= 65535.
//   block_tables [batch, max_blocks] int32 page ids
//   out          [batch, num_q_heads * head_dim] bf16
// head_dim 256 with 1, 2, 3, 4, 6 or 8 q heads per kv head, or head_dim 128
// with 1, 2 or 4.  Returns one of the ISB_NOALLOC_* codes.
int isb_attention_decode_noalloc(const void* q, const void* gate, const void* k_cache, const void* v_cache,
                                 const int* ctx_lens, const int* block_tables, int max_blocks, int batch,
                                 int num_q_heads, int num_kv_heads, int head_dim, float scale, void* out,
                                 cudaStream_t stream);

// Device error word of the attention kernels, read and cleared (a synchronous copy on the
// current device; it allocates nothing).  0x1: a bounded wait for a key/value copy ran
// out; 0x2: a context was longer than its block table.  A nonzero word means the output
// of the calls made since the last read is not valid.  The word is shared with the
// library's PyTorch-facing attention ops on the same device.  0xFFFFFFFF: the read failed.
unsigned int isb_noalloc_error_word(void);

// Text for an ISB_NOALLOC_* code.
const char* isb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
