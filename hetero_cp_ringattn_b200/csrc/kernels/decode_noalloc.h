// Allocation-free single-rank decode attention (C ABI).
//
// This entry point has no counterpart in the reference: it exists for callers that cannot
// allocate device memory themselves, such as plug-ins hosted by a runtime that owns the device
// allocator (an allocation behind its back would escape its memory accounting) and embedders
// that only hand this library input and output buffers. Such a caller cannot provide the split-KV
// scratch (partial outputs, partial log-sum-exps, completion counters) that the regular entry
// point takes as arguments, so this variant keeps that scratch, and a device status word, in a
// fixed-size array that is part of the loaded library (`static __device__`), sized
// HCP_DECODE_NOALLOC_SCRATCH_BYTES (4 MiB) on every device that loads the library.
//
// Contract:
//   * inputs: q [B, H, D] bf16; the paged KV arena (bf16 [layers][pages][2][Hkv][page][D]);
//     page tables [B, pt_stride] int32 and per-row KV lengths [B] int32 (all device memory);
//   * output: out [B, H * D] bf16, the attention of each row's query over its first n_tokens[b]
//     keys / values of `layer` (no causal mask: every stored row is in the past);
//   * a row's KV length is bounded by its page-table row: n_tokens[b] <= pt_stride * page. A
//     longer (or negative) length is clamped to that bound and reported through the status word,
//     so the kernel never reads page ids past the caller's row;
//   * nothing is allocated: no cudaMalloc / cudaFree / allocating library routine is called;
//   * the first call on a device (and the first after that device's context was reset) looks up
//     the device address of the scratch array (cudaGetSymbolAddress) with that device current;
//     make that first call outside any stream capture;
//   * every call on a device shares the one scratch array and it keeps the previous call's
//     contents; the entry point clears the parts that must start at zero (the completion
//     counters, the live status words) at the start of each call. Calls that overlap on the GPU
//     (different streams, no ordering between them) race on the scratch array and must be
//     avoided by the caller;
//   * problems that need more scratch than HCP_DECODE_NOALLOC_SCRATCH_BYTES are rejected with an
//     error code and a message (hcp_decode_attention_noalloc_error());
//   * device-side failures (a bounded wait that ran out, an out-of-range KV length) do not fail
//     the call itself, which returns once the kernels are queued: they are kept in the status
//     word until hcp_decode_attention_noalloc_status() reads them.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Size of the static scratch array (bytes) each device holds while the library is loaded.
#define HCP_DECODE_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u)

// Returns 0 on success, a negative value on a rejected argument, or a positive cudaError_t.
int hcp_decode_attention_noalloc(const void* q, const void* arena, int layers, int pages,
                                 int page, int hkv, int d, int layer, const int* page_tables,
                                 int pt_stride, const int* n_tokens, int batch, int heads,
                                 float scale, int splits, void* out, cudaStream_t stream);

// Message of the last rejected call on this host thread ("" if none).
const char* hcp_decode_attention_noalloc_error(void);

// Device status of the calls made on the current device since the last read: synchronises
// `stream`, writes 4 words (code, site, info, info; code 0 = no error, otherwise the first error
// seen) and resets them. Returns 0, or an error code as hcp_decode_attention_noalloc does.
int hcp_decode_attention_noalloc_status(int* words, cudaStream_t stream);

// Bytes of scratch a problem needs (to check against HCP_DECODE_NOALLOC_SCRATCH_BYTES);
// ULLONG_MAX for non-positive sizes.
unsigned long long hcp_decode_attention_noalloc_scratch_bytes(int batch, int heads, int hkv,
                                                              int d, int splits);

#ifdef __cplusplus
}
#endif
