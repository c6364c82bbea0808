// Host interface of the sm_100a ring flash-attention kernel (K1).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hcp {
namespace attn {

// The in-kernel KV ring of one layer step (context-parallel prefill, overlapped mode). Every
// rank's attention kernel stores this rank's own K/V rows into every peer's staging buffer
// (NVLink peer stores issued by warps that the attention does not otherwise use, tile by tile,
// claimed from a work counter so resident CTAs always finish them) and publishes a per-(tile,
// source) epoch flag for each; the TMA producer waits (bounded) for the flags of the remote
// tiles it is about to read, starting with this rank's own rows. The last CTA then tells every
// rank that this rank is done reading its staging parity.
struct RingArgs {
  int world = 1, my_rank = 0;
  unsigned long long epoch = 0;
  const unsigned long long* tile_src = nullptr;  // [kv tiles] bitmask of ranks with rows in tile
  const unsigned long long* tile_flags = nullptr;  // local flags of this parity [tiles][world]
  // push of this rank's rows (n_push = 0: nothing to push)
  const int* push_tiles = nullptr;   // [n_push][3]: (tile, first row, end row) of q_pos
  int n_push = 0;
  const __nv_bfloat16* own_stage = nullptr;       // this rank's staging parity (K then V)
  void* const* stage_ptrs = nullptr;              // [world] staging parity on every rank
  unsigned long long* const* tflag_ptrs = nullptr;  // [world] tile-flag parity on every rank
  const unsigned long long* consumed = nullptr;   // local consumed[src]
  unsigned long long* const* consumed_ptrs = nullptr;  // [world] &consumed[my_rank] on each rank
  unsigned int* counters = nullptr;               // [2]: push items claimed, CTAs finished
  int stage_cap = 0;
};

struct AttnArgs {
  const __nv_bfloat16* Q;   // [T, H, D]
  const __nv_bfloat16* K;   // [Hkv, kv_head_stride / D, D], row p = global position p
  const __nv_bfloat16* V;   // same layout as K
  __nv_bfloat16* O;         // [T, H, D]
  float* lse;               // [H, T] natural-log LSE (may be null)
  const int* q_pos;         // [T] global positions of the q rows
  int T, H, Hkv, D;
  int L;                    // number of valid KV positions (0..L-1)
  long kv_head_stride;      // elements between consecutive KV heads (>= L * D)
  float scale;
  int causal;
  RingArgs ring;            // ring.tile_src == nullptr: every KV row is already in place
  unsigned long long wait_budget_ns;
  int* status;
  // head_dim 64 kernel variant: 0 = the build's default (HCP_ATTN_HV), 1 = one softmax stream
  // per q tile, 2 = two 64-column streams per tile, 3 = one stream with P in its own TMEM
  // columns (pipelined Q K^T); head_dim 128 always runs one stream per tile
  int variant;
  // CTA order: -1 = the build's choice (pair major for grids of at most 8 waves, else KV-head
  // major; HCP_ATTN_ORDER overrides), 0 = KV-head major, 1 = pair major
  int order = -1;
};

const char* attn_fwd(const AttnArgs& args, cudaStream_t stream);

}  // namespace attn
}  // namespace hcp
