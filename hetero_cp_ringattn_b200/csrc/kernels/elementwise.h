// Host interface of the memory-bound model kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kv_layout.h"

namespace hcp {
namespace ew {

struct QkvPrefillArgs {
  const __nv_bfloat16* qkv;   // [T, ld_qkv] (q | k | v) after bias
  long ld_qkv;
  const int* pos;             // [T] global positions
  const float* cos_t;         // [max_pos, D/2]
  const float* sin_t;
  int max_pos;
  int T, H, Hkv, D;
  __nv_bfloat16* q_out;       // [T, H, D]
  // local arena (may be null)
  __nv_bfloat16* arena;
  ArenaGeom geom;
  int layer;
  const int* page_table;      // pages of this request
  int slot_base;              // first slot of this chunk
  int slot_cap;               // slots available in the page table
  // staging destinations (own staging first or in rank order; peers via P2P mappings)
  void* const* stage_ptrs;    // device array [n_stage] of staging K base (current parity)
  int n_stage;
  int stage_cap;              // Lcap
  // completion signalling (may be null for single-rank runs)
  unsigned int* done_counter;
  unsigned long long* const* ready_ptrs;  // device array [n_stage]: &kv_ready[my_rank] per rank
  unsigned long long epoch;
  int* status;
};

struct QkvDecodeArgs {
  const float* qkv;           // [B, (H + 2Hkv) D] fp32
  const int* pos;             // [B]
  const float* cos_t;
  const float* sin_t;
  int max_pos;
  int B, H, Hkv, D;
  __nv_bfloat16* q_out;       // [B, H, D]
  __nv_bfloat16* arena;
  ArenaGeom geom;
  int layer;
  const int* page_tables;     // [B, pt_stride]
  int pt_stride;
  int slot_cap;
  const int* owner;           // [B, owner_stride] 1 if this rank stores (b, layer)
  const int* slot;            // [B, owner_stride] slot to write on the owner
  int owner_stride;
  int* status;
};

struct StagePushArgs {
  const __nv_bfloat16* arena;
  ArenaGeom geom;
  int layer;
  const int* page_table;
  const int* slot_pos;        // [n] global position of each stored slot
  int n;
  void* const* stage_ptrs;
  int n_stage;
  int stage_cap;
};

const char* embedding(const int* ids, const __nv_bfloat16* W, __nv_bfloat16* out, int T,
                      int hidden, int vocab, int* status, cudaStream_t s);
const char* rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int T,
                    int hidden, long ldx, long ldy, float eps, cudaStream_t s);
const char* qkv_prefill(const QkvPrefillArgs& a, cudaStream_t s);
const char* qkv_decode(const QkvDecodeArgs& a, cudaStream_t s);
const char* stage_push(const StagePushArgs& a, cudaStream_t s);
const char* wait_consumed(const unsigned long long* consumed, int n, unsigned long long need,
                          unsigned long long budget_ns, int* status, cudaStream_t s);
const char* signal_peers(unsigned long long* const* ptrs, int n, unsigned long long epoch,
                         cudaStream_t s);
// tflag_ptrs[r][push_tiles[k][0] * world + my_rank] = epoch for every own tile k and rank r.
const char* publish_tiles(const int* push_tiles, int n_push, unsigned long long* const* tflag_ptrs,
                          int world, int my_rank, unsigned long long epoch, cudaStream_t s);
// ptrs[r][base + i] = epoch for every rank r and i < n (release stores after a system fence).
const char* publish_range(unsigned long long* const* ptrs, int world, long base, int n,
                          unsigned long long epoch, cudaStream_t s);
// Source: slots[r][2 p] = *tok, release slots[r][2 p + 1] = epoch (p = epoch & 1) for every rank;
// others: bounded wait for own_slot[2 p + 1] >= epoch, then *tok = own_slot[2 p].
const char* token_bcast(long long* tok, unsigned long long* const* slots,
                        const unsigned long long* own_slot, int world, bool is_src,
                        unsigned long long epoch, unsigned long long budget_ns, int* status,
                        cudaStream_t s);

}  // namespace ew
}  // namespace hcp
