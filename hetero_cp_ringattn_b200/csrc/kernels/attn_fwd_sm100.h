// Host interface of the sm_100a ring flash-attention kernel (K1).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hcp {
namespace attn {

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
  int kv_start_tile;        // first kv tile in processing order (this rank's own chunk)
  const unsigned long long* kv_ready;  // optional [Hkv][ceil(L/128)] ready epochs
  unsigned long long kv_epoch;
  unsigned long long wait_budget_ns;
  int* status;
};

const char* attn_fwd(const AttnArgs& args, cudaStream_t stream);

}  // namespace attn
}  // namespace hcp
