// C entry point of the paged decode attention that allocates no device memory.
//
// This entry point has no counterpart in the reference project: it exists for
// callers that cannot allocate device memory themselves. Examples are plugin
// hosts that own every device buffer and forbid a plugin from calling
// cudaMalloc while it executes, and latency-critical loops that cannot accept
// cudaMalloc's implicit device-wide synchronisation and unbounded run time.
// The caller passes device pointers for every input and output; the split-KV
// partial results live in a fixed array compiled into the library.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest scratch the entry point can use, in floats: partial accumulators
// (B * kv_heads * splits * group * head_dim) and partial max/sum pairs
// (B * kv_heads * splits * group * 2). 4 MiB + 256 KiB of device memory that
// every GPU which loads this library holds until the process exits.
#define B200_NOALLOC_MAX_ACC_FLOATS (1u << 20)
#define B200_NOALLOC_MAX_ML_FLOATS (1u << 16)

// One new query token per sequence against a paged bf16 KV cache.
//   q            [B, nq, head_dim] bf16          k_cache, v_cache [blocks, nkv, 16, head_dim] bf16
//   block_tables [B, max_blocks] int32            seq_lens [B] int32 (tokens incl. the new one)
//   out          [B, nq, head_dim] bf16 (written)
//   tokens_per_split: multiple of 16; nsplit: number of KV splits (grid size)
// Caller preconditions (seq_lens lives on the device, so the entry point cannot check them):
//   * seq_lens[b] <= max_blocks * 16 for every b: keys past the block table are never read;
//   * seq_lens[b] <= nsplit * tokens_per_split: split s covers keys [s*tps, (s+1)*tps), so keys
//     past the last split are dropped and the result is wrong although the call returns 0.
// With nsplit == 1 the kernel writes `out` directly and uses no scratch (no size limit).
// Returns 0 on success, otherwise a nonzero code with a message available from
// b200_noalloc_last_error(). Every call on a device shares the same scratch
// array and leaves its contents behind; no state is carried between calls
// (each call writes every scratch slot it later reads), but two calls that
// overlap on the GPU, e.g. on two streams, race on that array.
// The first call on each device looks up the array's device address with that
// device current (cudaGetSymbolAddress) and caches it; make that first call
// before any stream capture.
int b200_paged_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                        const int* block_tables, const int* seq_lens, void* out, int B, int nq,
                                        int nkv, int head_dim, int max_blocks, float scale, int tokens_per_split,
                                        int nsplit, cudaStream_t stream);

// Human-readable reason of the last failing call on this thread ("" if none).
const char* b200_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
