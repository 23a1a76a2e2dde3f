// Allocation-free split-KV decode attention: a plain C entry point.
//
// This entry point has no counterpart in the reference; it exists for callers
// that must not allocate device memory while they run: a runtime that owns
// every byte of the GPU up front (a fixed arena, a serving process that sized
// its KV cache to the last block), an embedding application that is not
// linked against PyTorch's caching allocator, or code running where an
// allocation would synchronise the device at a bad time. The regular
// `paged_attention` op needs two caller-allocated fp32 workspaces when the key
// range is split across CTAs (flash-decoding); this variant keeps those
// partial results in a fixed-size scratch array that is compiled into the
// library as a `static __device__` global, so neither it nor the caller
// allocates anything per call.
//
// Contract:
// * Inputs and outputs are caller-owned device pointers on the current device;
//   the call only enqueues kernels on `stream` and returns.
// * Set-up: the first call on each device (with that device current) looks up
//   the scratch array's device address (cudaGetSymbolAddress) and raises the
//   kernels' dynamic shared-memory limit. Make that first call before any
//   stream capture begins on the device.
// * Scratch limit: nsplit * num_tokens * num_q_heads * (head_dim + 1) fp32
//   values, plus 64 for alignment, must fit in GSB_NOALLOC_SCRATCH_FLOATS
//   (1,048,576 = 4 MiB). Larger requests are rejected with
//   GSB_NOALLOC_ETOOBIG and a message; nothing is launched. nsplit == 1 needs
//   no scratch.
// * Every call on a device shares the one scratch array and leaves its last
//   contents there. The log-sum-exp part is reset to -inf at the start of each
//   call; the partial outputs are written before they are read. Two calls that
//   overlap in time on one device (different streams, or different host
//   threads without ordering) race on the scratch array and give wrong results:
//   serialise them.
// * Layout (as for the `paged_attention` op with rows_per_tile = 16):
//   q [num_tokens, >= Hq*D] bf16 with row stride q_stride (elements, multiple
//   of 8, base 16-byte aligned); k_cache / v_cache [num_blocks, Hkv, 16, D]
//   bf16 contiguous; block_table [S, block_table_stride] int32; q_start [S+1],
//   kv_len [S] int32; work_seq / work_row0 [num_work] int32 (one decode tile of
//   16 rows each); out [num_tokens, Hq*D] bf16 with row stride out_stride;
//   err: the library's device error word (uint32, nonzero after a bounded
//   wait ran out).
// * Returns GSB_NOALLOC_OK or an error code; `msg` (may be NULL) receives a
//   one-line reason.
#pragma once

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#define GSB_NOALLOC_SCRATCH_FLOATS (1 << 20)

#ifdef __cplusplus
extern "C" {
#endif

enum {
  GSB_NOALLOC_OK = 0,
  GSB_NOALLOC_EINVAL = 1,   // bad argument (null pointer, head_dim, alignment, ...)
  GSB_NOALLOC_ETOOBIG = 2,  // split partials exceed the fixed scratch array
  GSB_NOALLOC_ECUDA = 3,    // a CUDA runtime call or launch failed
};

__attribute__((visibility("default"))) int gsb_decode_attention_noalloc(
    const void* q, int64_t q_stride, const void* k_cache, const void* v_cache, int64_t num_blocks,
    int num_kv_heads, int head_dim, const int32_t* block_table, int64_t block_table_stride,
    const int32_t* q_start, const int32_t* kv_len, const int32_t* work_seq, const int32_t* work_row0,
    int num_work, int num_tokens, int num_q_heads, float scale, int nsplit, void* out, int64_t out_stride,
    uint32_t* err, cudaStream_t stream, char* msg, size_t msg_len);

#ifdef __cplusplus
}
#endif
