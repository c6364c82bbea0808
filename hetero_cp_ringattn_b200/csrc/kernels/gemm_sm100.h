// Host interface of the sm_100a tcgen05 GEMM (K3/K6) and the TMA descriptor helpers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kv_layout.h"

namespace hcp {
namespace gemm {

enum Epilogue : int {
  kEpiStore = 0,     // C = A B^T
  kEpiBias = 1,      // C = A B^T + bias[n]
  kEpiResidual = 2,  // C = bf16(A B^T) + R   (R may alias C)
  kEpiSwiGLU = 3,    // C[:, j] = silu(G_j) * U_j with B rows interleaved [128 gate | 128 up]
  kEpiQkvPush = 4,   // QKV projection fused with RoPE and the K/V push (QkvPushArgs)
};

// The QKV projection's epilogue: the row of q | k | v heads is never stored. +bias (Qwen2),
// rotate-half RoPE of the q and k heads at the row's global position, q -> q_out [M, H, D];
// k and v -> the row's slot in the local paged KV arena and row `pos` of every rank's staging
// buffer (peer stores over NVLink); finally the last CTA publishes `epoch` to every rank's
// kv_ready slot (release stores after a system-scope fence).
struct QkvPushArgs {
  const int* pos;                 // [M] global positions
  const float* cos_t;             // [max_pos, D/2]
  const float* sin_t;
  int max_pos;
  int H, Hkv, D;
  __nv_bfloat16* q_out;           // [M, H, D]
  __nv_bfloat16* arena;           // local paged arena (null: no arena write)
  ArenaGeom geom;
  int layer;
  const int* page_table;
  int slot_base, slot_cap;
  void* const* stage_ptrs;        // device array [n_stage]: every rank's staging buffer
  int n_stage, stage_cap;
  unsigned int* done_counter;     // null: no kv_ready publish (single rank)
  unsigned long long* const* ready_ptrs;
  unsigned long long epoch;
};

struct GemmArgs {
  const __nv_bfloat16* A;  // [M, K] row-major (K contiguous)
  long lda;
  const __nv_bfloat16* B;  // [N, K] row-major (nn.Linear weight layout)
  long ldb;
  __nv_bfloat16* C;        // [M, N] (SwiGLU: [M, N/2])
  long ldc;
  int M, N, K;
  int epi;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  long ldr;
  int* status;             // device status words (may be null)
  int num_sms;
  int variant;             // 0: the build's default (HCP_GEMM_PAIR), 1: one CTA per 128x256
                           // tile, 2: CTA pairs on 256x256 tiles (tcgen05 cta_group::2)
  int group = -1;          // tile order: bands of this many m-blocks (0: n fastest; -1: by the
                           // weight's size, HCP_GEMM_GROUP overrides)
};

// Returns nullptr on success, otherwise a static error string.
const char* gemm_bf16(const GemmArgs& args, cudaStream_t stream);
// args.epi is ignored (kEpiQkvPush); args.C / ldc / R are unused; args.bias optional.
const char* gemm_qkv_push(const GemmArgs& args, const QkvPushArgs& q, cudaStream_t stream);

bool make_tma_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);
bool make_tma_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                      uint32_t b2);

}  // namespace gemm
}  // namespace hcp
