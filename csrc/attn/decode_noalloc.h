// Allocation-free entry point for split-KV decode attention.
//
// This entry point has no counterpart in the reference; it is an addition of
// this library.
//
// Who needs it: code that runs attention from inside a host runtime that owns
// all device memory and forbids allocation while it executes - for example a
// plugin called from another inference runtime's enqueue hook, or a C/C++
// service that links this library without PyTorch and its caching allocator.
// In those places cudaMalloc/cudaFree is either not allowed (it can block on
// the whole device and break the host runtime's timing guarantees) or there is
// simply no allocator to ask for temporary buffers.
//
// What it does: the same decode-attention kernels as the regular entry point,
// but the split-KV partial results live in a fixed, file-scope device array
// (one per GPU that loads the library, kept until the process exits) instead
// of caller-provided scratch. The caller still provides every input and the
// output.
//
// Limits: the scratch holds at most MBX_NOALLOC_MAX_PARTIAL_ROWS rows of
// partial results, i.e. batch * q_heads * splits <= 16384 when splits > 1
// (8 MiB of fp32 partial outputs plus 64 KiB of log-sum-exps per GPU). With
// splits == 1 the kernel writes the output directly, uses no scratch and has
// no such limit. Larger split requests are rejected with error code 2 and a
// message from mbx_noalloc_last_error().
//
// Rules for callers:
//  * The first call on each device looks up the array's device address (with
//    that device current). Make that first call before any stream capture.
//  * Every call shares the one array. Calls whose kernels overlap on the GPU
//    (different streams, or different host threads on the same device) race
//    on it; serialise them. Each call overwrites every partial it reads, so
//    nothing has to be cleared between calls.
//  * Return value: 0 on success, non-zero on error (see mbx_noalloc_last_error):
//    1 null pointer or bad size, 2 scratch too small for the split count,
//    3 CUDA runtime error while looking up the scratch, 4 launch refused
//    (e.g. q_heads not a multiple of kv_heads, or a group above 16 heads).
#pragma once
#include <stddef.h>
#include <stdint.h>

#define MBX_NOALLOC_MAX_PARTIAL_ROWS 16384

#ifdef __cplusplus
extern "C" {
#endif

// q [B, nq, 128] bf16, k_cache/v_cache [blocks, nkv, 16, 128] bf16,
// out [B, nq, 128] bf16, kv_len [B] int32, block_table [B, max_blocks] int32,
// all device pointers; stream is a cudaStream_t (NULL = default stream).
int mbx_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                                 const int32_t* kv_len, const int32_t* block_table, int max_blocks, int batch,
                                 int q_heads, int kv_heads, int splits, float scale, void* stream);

// Largest batch * q_heads * splits the scratch array holds.
size_t mbx_decode_attention_noalloc_max_rows(void);

// Message of the last failed call on this host thread ("" if none).
const char* mbx_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
